"""The tiled-renderer restatement (oracle/tiled_oracle.py) against the reference's tiled.py.

Fixtures: tests/golden/make_golden.py ran render_pytorch_3dgs_tiled (tiled.py:74-198) on the five
golden scenes with tile sizes 8 and 16: images, tile lists (tiled.py:31-71) and, under the
standard_gs loss, gradients with respect to the raw parameters (tiled_grads.npz).
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, grad_close, grad_close_elementwise, load_golden
from oracle import splat_oracle as so
from oracle import tiled_oracle as to

RAW = ("means", "log_scales", "quats", "opacity_logits", "sh")


def _render(wl, leaves, vel, tile):
    raw = so.RawGaussians(*(leaves[k] for k in RAW), vel)
    m, s, q, o, rgb = so.activate(raw, wl.times, wl.camera_to_world, wl.views_per_set)
    return torch.stack([to.render_tiled_view(m[b], s[b], q[b], o[b], rgb[b], wl.height, wl.width, wl.fx[b], wl.fy[b],
                                             wl.cx[b], wl.cy[b], wl.camera_to_world[b], tile_size=tile)
                        for b in range(wl.n_views)])


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("tile", [8, 16])
def test_tiled_oracle_image_and_lists(case, tile):
    g = load_golden(case)
    wl = g.workload()
    leaves = {k: getattr(wl, k) for k in RAW}
    img = _render(wl, leaves, wl.velocity, tile)
    assert (img - g.t(f"ref_tiled{tile}_image")).abs().max().item() <= 2e-6
    # lists of view 0 from the reference's projected Gaussians (its depth order)
    H, W = wl.height, wl.width
    bounds = to.gaussian_bounds(g.t("ref_means2d")[0], g.t("ref_cov2d")[0], g.t("ref_proj_opacity")[0], H, W)
    tiles_x = -(-W // tile)
    lists = to.tile_lists(*bounds, tile, tiles_x)
    sel = g["ref_tiled%d_view" % tile] == 0
    ref_tile, ref_rank = g["ref_tiled%d_tile" % tile][sel], g["ref_tiled%d_rank" % tile][sel]
    got_tile = np.concatenate([np.full(len(v), t) for t, v in sorted(lists.items())]) if lists else np.zeros(0)
    got_rank = np.concatenate([v.numpy() for _t, v in sorted(lists.items())]) if lists else np.zeros(0)
    np.testing.assert_array_equal(got_tile, ref_tile)
    np.testing.assert_array_equal(got_rank, ref_rank)
    only = sorted(lists)[:: max(1, len(lists) // 5)]
    sub = to.tile_lists(*bounds, tile, tiles_x, only=only)
    for t in only:
        np.testing.assert_array_equal(sub[t].numpy(), lists[t].numpy())


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("tile", [8, 16])
def test_tiled_oracle_gradients(case, tile):
    g = load_golden(case)
    t = load_golden("tiled_grads")
    wl = g.workload()
    key = f"{case}_t{tile}"
    leaves = {k: getattr(wl, k).clone().requires_grad_(True) for k in RAW}
    vel = wl.velocity.clone().requires_grad_(True) if wl.velocity is not None else None
    img = _render(wl, leaves, vel, tile)
    assert (img.detach() - t.t(f"{key}_image")).abs().max().item() <= 2e-6
    so.reconstruction_loss_per_image(img, wl.target).sum().backward()
    grads = {k: v.grad for k, v in leaves.items()}
    if vel is not None:
        grads["velocity"] = vel.grad
    for k, v in grads.items():
        ok, err, scale = grad_close(v, t.t(f"{key}_grad_{k}"))
        assert ok, f"{k}: {err:.3e} vs {scale:.3e}"
        ok, ratio, scale = grad_close_elementwise(v, t.t(f"{key}_grad_{k}"))
        assert ok, f"{k}: per-element {ratio:.2f}x the bound"
