"""render_b200_head: the decoder head's raw outputs rendered with the head's activation fused into
the projection, against the reference's GaussianParameterHeads.forward + dense renderer + loss
(fixtures: tests/golden/make_golden_head.py).  Image within 1e-4, gradients with respect to the
raw head outputs within 1e-3 of scale and per element."""
import numpy as np
import pytest
import torch

from conftest import grad_close, grad_close_elementwise, load_golden
from dynaworld_b200.losses import reconstruction_loss_per_image
from dynaworld_b200.renderer import HeadActivation, render_b200_head
from gpu_helpers import DEV

pytestmark = pytest.mark.gpu

RAW = ("xyz", "scale", "rot", "opacity", "rgb")


@pytest.mark.parametrize("name", ["head_static", "head_clips"])
def test_head_render_matches_reference(name):
    g = load_golden("head")
    n_sets, G, vps, H, W = (int(v) for v in g[f"{name}_shape"])
    ext, z0, z1, si = (float(v) for v in g[f"{name}_head"])
    leaves = {k: g.t(f"{name}_raw_{k}", DEV).requires_grad_(True) for k in RAW}
    image, alpha, _ = render_b200_head(
        leaves["xyz"], leaves["scale"], leaves["rot"], leaves["opacity"], leaves["rgb"],
        head=HeadActivation(ext, z0, z1, si), intrinsics=g.t(f"{name}_intrinsics", DEV),
        camera_to_world=g.t(f"{name}_camera_to_world", DEV), height=H, width=W, views_per_set=vps)
    assert (image.detach().cpu() - g.t(f"{name}_image")).abs().max().item() <= 1e-4
    loss = reconstruction_loss_per_image(image, g.t(f"{name}_target", DEV))
    np.testing.assert_allclose(loss.detach().cpu().numpy(), g[f"{name}_loss"], rtol=0, atol=1e-5)
    loss.sum().backward()
    for k in RAW:
        got = leaves[k].grad.cpu()
        ok, err, scale = grad_close(got, g.t(f"{name}_grad_{k}"))
        assert ok, f"{k}: {err:.3e} vs {scale:.3e}"
        ok, ratio, scale = grad_close_elementwise(got, g.t(f"{name}_grad_{k}"))
        assert ok, f"{k}: per-element {ratio:.2f}x the bound (scale {scale:.3e})"


def test_head_from_module_attributes():
    class Heads:  # the attributes GaussianParameterHeads keeps (blocks.py:119-123)
        xy_extent, z_min, z_extent, scale_init = 1.5, 0.5, 2.0, 0.05

    assert HeadActivation.from_heads(Heads()) == HeadActivation(1.5, 0.5, 2.5, 0.05)
