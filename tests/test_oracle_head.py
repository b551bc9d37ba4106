"""The decoder-head activation restatement (oracle.splat_oracle.activate_head) against the
reference's GaussianParameterHeads.forward (fixtures: tests/golden/make_golden_head.py)."""
import pytest
import torch

from conftest import grad_close, grad_close_elementwise, load_golden
from oracle import splat_oracle as so

CASES = ["head_static", "head_clips"]
RAW = ("xyz", "scale", "rot", "opacity", "rgb")


def head_inputs(g, name):
    n_sets, G, vps, H, W = (int(v) for v in g[f"{name}_shape"])
    ext, z0, z1, si = (float(v) for v in g[f"{name}_head"])
    return n_sets, G, vps, H, W, (ext, z0, z1, si)


@pytest.mark.parametrize("name", CASES)
def test_head_activation_matches_reference(name):
    g = load_golden("head")
    *_, consts = head_inputs(g, name)
    act = so.activate_head(*(g.t(f"{name}_raw_{k}") for k in RAW), *consts)
    for k, v in zip(("xyz", "scales", "quats", "opacities", "rgbs"), act):
        torch.testing.assert_close(v, g.t(f"{name}_act_{k}"), rtol=0, atol=1e-6)


@pytest.mark.parametrize("name", CASES)
def test_head_render_gradients_match_reference(name):
    g = load_golden("head")
    n_sets, G, vps, H, W, consts = head_inputs(g, name)
    leaves = {k: g.t(f"{name}_raw_{k}").clone().requires_grad_(True) for k in RAW}
    act = so.activate_head(*(leaves[k] for k in RAW), *consts)
    B = n_sets * vps
    idx = torch.arange(B) // vps
    intr = g.t(f"{name}_intrinsics")
    c2w = g.t(f"{name}_camera_to_world")
    m, s, q, o, rgb = (a[idx] for a in act)
    img, _, _ = so.render_dense(m, s, q, o, rgb, H, W, intr[:, 0], intr[:, 1], intr[:, 2], intr[:, 3], c2w,
                                sort_key=so.camera_depth_fp32(m.detach(), c2w))
    assert (img.detach() - g.t(f"{name}_image")).abs().max().item() <= 2e-6
    so.reconstruction_loss_per_image(img, g.t(f"{name}_target")).sum().backward()
    for k in RAW:
        ok, err, scale = grad_close(leaves[k].grad, g.t(f"{name}_grad_{k}"))
        assert ok, f"{k}: {err:.3e} vs {scale:.3e}"
        ok, ratio, scale = grad_close_elementwise(leaves[k].grad, g.t(f"{name}_grad_{k}"))
        assert ok, f"{k}: per-element {ratio:.2f}x the bound"
