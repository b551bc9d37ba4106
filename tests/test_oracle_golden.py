"""The oracle against the reference's own outputs (golden fixtures): this pins the oracle.

CPU only.  Tolerances: the reference and the float32 oracle differ only in summation order.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, grad_close, load_golden
from oracle import culled_oracle as co
from oracle import splat_oracle as so
from oracle import tiles_oracle as to


def activated(g, dtype=torch.float32):
    wl = g.workload()
    raw = so.RawGaussians(*(t.to(dtype) for t in (wl.means, wl.log_scales, wl.quats, wl.opacity_logits, wl.sh)),
                          None if wl.velocity is None else wl.velocity.to(dtype))
    return wl, so.activate(raw, wl.times, wl.camera_to_world, wl.views_per_set)


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_depth_keys_bit_exact(case):
    g = load_golden(case)
    wl, (m, s, q, o, rgb) = activated(g)
    z = so.camera_depth_fp32(m, wl.camera_to_world)
    assert torch.equal(z, g.t("ref_cam_z")), "depth keys differ from the reference's float32 z"
    order = torch.argsort(z, dim=1, stable=True)
    assert torch.equal(order, g.t("ref_depth_order"))


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_projection_matches_reference(case):
    g = load_golden(case)
    wl, (m, s, q, o, rgb) = activated(g)
    m2, inv, cov, op, rgbo, z, order = so.project_batch(m, s, q, o, rgb, wl.fx, wl.fy, wl.cx, wl.cy,
                                                        wl.camera_to_world,
                                                        sort_key=so.camera_depth_fp32(m, wl.camera_to_world))
    torch.testing.assert_close(m2, g.t("ref_means2d"), rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(cov, g.t("ref_cov2d"), rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(op, g.t("ref_proj_opacity"), rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(rgbo, g.t("ref_proj_rgb"), rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_dense_image_and_loss(case, dtype):
    g = load_golden(case)
    wl, (m, s, q, o, rgb) = activated(g, dtype)
    img, alpha, _ = so.render_dense(m, s, q, o, rgb, wl.height, wl.width, wl.fx, wl.fy, wl.cx, wl.cy,
                                    wl.camera_to_world, sort_key=so.camera_depth_fp32(m, wl.camera_to_world))
    assert (img.float() - g.t("ref_image")).abs().max().item() < 5e-6
    loss = so.reconstruction_loss_per_image(img, wl.target.to(dtype))
    torch.testing.assert_close(loss.float(), g.t("ref_loss"), rtol=1e-5, atol=1e-6)
    assert alpha.min().item() >= 0.0


@pytest.mark.parametrize("case", ["static64", "dynamic128_small", "edge"])
def test_raw_gradients_match_reference(case):
    g = load_golden(case)
    wl = g.workload()
    leaves = {k: getattr(wl, k).double().requires_grad_(True) for k in ("means", "log_scales", "quats",
                                                                        "opacity_logits", "sh")}
    vel = wl.velocity.double().requires_grad_(True) if wl.velocity is not None else None
    raw = so.RawGaussians(leaves["means"], leaves["log_scales"], leaves["quats"], leaves["opacity_logits"],
                          leaves["sh"], vel)
    m, s, q, o, rgb = so.activate(raw, wl.times.double(), wl.camera_to_world, wl.views_per_set)
    key = so.camera_depth_fp32(m.float(), wl.camera_to_world)
    img, _, _ = so.render_dense(m, s, q, o, rgb, wl.height, wl.width, wl.fx, wl.fy, wl.cx, wl.cy,
                                wl.camera_to_world, sort_key=key)
    so.reconstruction_loss_per_image(img, wl.target.double()).sum().backward()
    for k, leaf in leaves.items():
        ok, err, scale = grad_close(leaf.grad, g.t(f"ref_grad_{k}"))
        assert ok, f"{k}: max err {err:.3e} vs scale {scale:.3e}"
    if vel is not None:
        ok, err, scale = grad_close(vel.grad, g.t("ref_grad_velocity"))
        assert ok, f"velocity: max err {err:.3e} vs scale {scale:.3e}"


def test_losses_match_reference():
    g = load_golden("losses")
    for i in range(3):
        pred, tgt = g.t(f"loss{i}_pred"), g.t(f"loss{i}_target")
        B = pred.shape[0]
        for kind in ("standard_gs", "l1", "mse", "l1_mse"):
            p = pred.double().clone().requires_grad_(True)
            loss = so.reconstruction_loss_per_image(p, tgt.double(), {"type": kind})
            (loss * torch.arange(1, B + 1, dtype=torch.float64)).sum().backward()
            torch.testing.assert_close(loss.float(), g.t(f"loss{i}_{kind}_value"), rtol=1e-5, atol=1e-6)
            ok, err, scale = grad_close(p.grad, g.t(f"loss{i}_{kind}_grad"), rel=1e-4)
            assert ok, f"loss{i} {kind}: {err:.3e} vs {scale:.3e}"


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("tile", [8, 16])
def test_tiled_compat_lists_bit_exact(case, tile):
    """tiles_oracle's restatement of tiled.py:7-71 gives the reference's lists and order exactly."""
    g = load_golden(case)
    H, W = int(g["height"]), int(g["width"])
    m2, cov, op = g["ref_means2d"], g["ref_cov2d"], g["ref_proj_opacity"]
    for b in range(m2.shape[0]):
        tiles, ranks = to.compat_pairs_one_view(m2[b], cov[b], op[b, :, 0], H, W, tile)
        order = np.lexsort((ranks, tiles))  # stable sort by tile keeps rank order
        sel = g[f"ref_tiled{tile}_view"] == b
        np.testing.assert_array_equal(tiles[order], g[f"ref_tiled{tile}_tile"][sel])
        np.testing.assert_array_equal(ranks[order], g[f"ref_tiled{tile}_rank"][sel])


@pytest.mark.parametrize("case", ["static64", "multiview384_small", "edge"])
def test_culled_blend_matches_dense(case):
    """The rank-corrected, tile-culled recurrence the CUDA raster implements reproduces dense.py."""
    g = load_golden(case)
    H, W = int(g["height"]), int(g["width"])
    m2 = g.t("ref_means2d", dtype=torch.float64)
    inv = g.t("ref_inv_cov", dtype=torch.float64)
    op = g.t("ref_proj_opacity", dtype=torch.float64)
    rgb = g.t("ref_proj_rgb", dtype=torch.float64)
    ref = g.t("ref_image")
    for b in range(m2.shape[0]):
        inv3 = torch.stack([inv[b, :, 0, 0], inv[b, :, 0, 1] + inv[b, :, 1, 0], inv[b, :, 1, 1]], -1)
        f = lambda t: t.float().numpy()  # noqa: E731
        tiles, ranks = to.exact_pairs_one_view(f(m2[b, :, 0]), f(m2[b, :, 1]), f(inv3[:, 0]), f(inv3[:, 1]),
                                               f(inv3[:, 2]), f(op[b, :, 0]), H, W, 16, 2.0 ** -25)
        img, alpha, _, n, te = co.blend_culled_view(m2[b], inv3, op[b, :, 0], rgb[b], None,
                                                    co.ranks_by_tile(tiles, ranks), H, W, 16,
                                                    alpha_cutoff=2.0 ** -25, transmittance_threshold=1e-7)
        assert (img.float() - ref[b]).abs().max().item() < 2e-6


def test_culled_tiled_compat_matches_reference_tiled():
    """tile_local eps over tiled.py's lists reproduces render_pytorch_3dgs_tiled."""
    g = load_golden("static64")
    H, W = int(g["height"]), int(g["width"])
    m2 = g.t("ref_means2d", dtype=torch.float64)[0]
    inv = g.t("ref_inv_cov", dtype=torch.float64)[0]
    op = g.t("ref_proj_opacity", dtype=torch.float64)[0, :, 0]
    rgb = g.t("ref_proj_rgb", dtype=torch.float64)[0]
    inv3 = torch.stack([inv[:, 0, 0], inv[:, 0, 1] + inv[:, 1, 0], inv[:, 1, 1]], -1)
    for tile in (8, 16):
        rpt = co.ranks_by_tile(g[f"ref_tiled{tile}_tile"], g[f"ref_tiled{tile}_rank"])
        img, *_ = co.blend_culled_view(m2, inv3, op, rgb, None, rpt, H, W, tile, alpha_cutoff=0.0,
                                       transmittance_threshold=0.0, eps_mode="tile_local")
        assert (img.float() - g.t(f"ref_tiled{tile}_image")[0]).abs().max().item() < 2e-6


@pytest.mark.parametrize("case", ["static64", "dynamic128_small", "multiview384_small"])
def test_activated_input_gradients_match_reference(case):
    """Gradients w.r.t. the reference render call's own inputs (xyz, scales, quats, opacities, rgbs)."""
    g = load_golden(case)
    wl = g.workload()
    act = {k: g.t(f"ref_act_{k}").double().requires_grad_(True) for k in ("xyz", "scales", "quats", "opacities",
                                                                            "rgbs")}
    key = so.camera_depth_fp32(act["xyz"].float(), wl.camera_to_world)
    img, _, _ = so.render_dense(act["xyz"], act["scales"], act["quats"], act["opacities"], act["rgbs"], wl.height,
                                wl.width, wl.fx, wl.fy, wl.cx, wl.cy, wl.camera_to_world, sort_key=key)
    so.reconstruction_loss_per_image(img, wl.target.double()).sum().backward()
    for k, v in act.items():
        ok, err, scale = grad_close(v.grad, g.t(f"ref_grad_act_{k}"))
        assert ok, f"{k}: {err:.3e} vs {scale:.3e}"


def test_flip_clamp_takes_the_other_side_of_the_kink():
    x = torch.tensor([0.5, 1.0 + 1e-7, 1.0 - 1e-7, -1e-7], dtype=torch.float64, requires_grad=True)
    c = x.clamp(0, 1)
    f = so.flip_clamp(x, c)
    torch.testing.assert_close(f[[0, 2]], c[[0, 2]])
    f.sum().backward()
    # torch.clamp passes the gradient at 0.5 and 1 - 1e-7 and blocks it outside; flipped, the reverse
    assert x.grad.tolist() == [0.0, 1.0, 0.0, 1.0]


def test_clips256_small_has_a_weight_sum_at_the_kink():
    """The golden clips256_small scene holds pixels whose weight sum is within 3e-7 of 1, where the
    reference's gradient jumps with the last bit of that sum (tests/kinks.py)."""
    g = load_golden("clips256_small")
    wl = g.workload()
    raw = so.RawGaussians(*(getattr(wl, k).double() for k in ("means", "log_scales", "quats", "opacity_logits",
                                                             "sh")), wl.velocity.double())
    m, s, q, o, rgb = so.activate(raw, wl.times.double(), wl.camera_to_world, wl.views_per_set)
    key = so.camera_depth_fp32(m.float(), wl.camera_to_world)
    _img, wsum, _ = so.render_dense(m, s, q, o, rgb, wl.height, wl.width, wl.fx, wl.fy, wl.cx, wl.cy,
                                    wl.camera_to_world, sort_key=key)
    assert (wsum - 1.0).abs().min().item() < 3e-7
