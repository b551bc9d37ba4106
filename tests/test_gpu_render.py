"""CUDA render + loss against the reference's outputs (golden fixtures) and the oracle.

Tolerances: image and alpha within 1e-4 absolute; gradients within 1e-3 of each tensor's largest
magnitude (max |g - g_ref| <= 1e-3 * max |g_ref|) and, per element,
|g - g_ref| <= 1e-3 * |g_ref| + 1e-4 * max |g_ref| up to the side of a clamp's kink taken at pixels
within rounding of it (kinks.check_gradients); tile lists and sorted key order bit-exact.
"""
import numpy as np
import pytest
import torch

import kinks
from conftest import GOLDEN_CASES, grad_close, load_golden
from dynaworld_b200 import synthetic
from dynaworld_b200.config import B200RendererConfig
from dynaworld_b200.renderer import render_b200_3dgs, render_b200_3dgs_batch
from gpu_helpers import DEV, keys_np, records_np, render_raw, sorted_ids_from_rank, stages
from oracle import splat_oracle as so
from oracle import tiled_oracle
from oracle import tiles_oracle as to

pytestmark = pytest.mark.gpu

IMAGE_TOL = 1e-4
GRAD_REL = 1e-3


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_depth_order_bit_exact(case):
    g = load_golden(case)
    wl = g.workload()
    _, _, _, st = stages(wl)
    ids = sorted_ids_from_rank(st.rank_of, wl.n_views, wl.n_gaussians)
    np.testing.assert_array_equal(ids, g["ref_depth_order"])


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_projected_records_match_reference(case):
    g = load_golden(case)
    wl = g.workload()
    _, _, _, st = stages(wl)
    rec = records_np(st, wl.n_views, wl.n_gaussians)
    m2, inv = g["ref_means2d"], g["ref_inv_cov"]
    np.testing.assert_allclose(rec[..., 0:2], m2, rtol=1e-5, atol=1e-3)
    scale = np.abs(inv).max()
    np.testing.assert_allclose(rec[..., 2], inv[..., 0, 0], rtol=1e-4, atol=1e-6 * scale)
    np.testing.assert_allclose(rec[..., 3], inv[..., 0, 1] + inv[..., 1, 0], rtol=1e-4, atol=1e-6 * scale)
    np.testing.assert_allclose(rec[..., 4], inv[..., 1, 1], rtol=1e-4, atol=1e-6 * scale)
    np.testing.assert_allclose(rec[..., 5], g["ref_proj_opacity"][..., 0], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(rec[..., 8:11], g["ref_proj_rgb"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("ellipse", [True, False])
def test_exact_mode_lists_bit_exact(case, ellipse):
    """Pair keys from the GPU equal the numpy restatement of the exact-mode rule applied to the
    GPU's own projected records (same float64 operation order)."""
    g = load_golden(case)
    wl = g.workload()
    cfg = B200RendererConfig(ellipse_culling=ellipse)
    _, _, _, st = stages(wl, cfg)
    rec = records_np(st, wl.n_views, wl.n_gaussians)
    per_view = []
    for b in range(wl.n_views):
        r = rec[b]
        per_view.append(to.exact_pairs_one_view(r[:, 0], r[:, 1], r[:, 2], r[:, 3], r[:, 4], r[:, 5], wl.height,
                                                wl.width, 16, np.float32(cfg.alpha_cutoff), ellipse_test=ellipse))
    ref = to.sort_pairs(per_view, to.n_tiles_for(wl.height, wl.width, 16))
    np.testing.assert_array_equal(keys_np(st), ref)


def _large_splat_scene():
    """2 views of 192x192 from the multiview384 generator (2000 Gaussians) with a quarter of them
    grown 4-12x: many Gaussians span more than 32 tiles (long emission runs, many rows) next to
    small ones."""
    wl = synthetic.multiview384(scale=0.01, image_scale=0.5, views=2)
    g = torch.Generator().manual_seed(17)
    grow = torch.rand(wl.n_gaussians, generator=g) < 0.25
    wl.log_scales[:, grow] += torch.log(4.0 + 8.0 * torch.rand(int(grow.sum()), 1, generator=g))
    return wl


@pytest.mark.parametrize("tile", [8, 16])
@pytest.mark.parametrize("ellipse", [True, False])
def test_lists_of_large_splats(tile, ellipse):
    """Keys of Gaussians listed in more than 32 tiles equal the numpy restatement."""
    wl = _large_splat_scene()
    cfg = B200RendererConfig(tile_size=tile, ellipse_culling=ellipse)
    _, _, _, st = stages(wl, cfg)
    rec = records_np(st, wl.n_views, wl.n_gaussians)
    per_view = [to.exact_pairs_one_view(rec[b][:, 0], rec[b][:, 1], rec[b][:, 2], rec[b][:, 3], rec[b][:, 4],
                                        rec[b][:, 5], wl.height, wl.width, tile, np.float32(cfg.alpha_cutoff),
                                        ellipse_test=ellipse) for b in range(wl.n_views)]
    ref = to.sort_pairs(per_view, to.n_tiles_for(wl.height, wl.width, tile))
    np.testing.assert_array_equal(keys_np(st), ref)
    ranks = (ref & np.uint64(0xFFFFFFFF)).astype(np.int64) + (ref >> np.uint64(32)).astype(np.int64) // \
        to.n_tiles_for(wl.height, wl.width, tile) * wl.n_gaussians
    assert np.bincount(ranks).max() > 32  # some Gaussians span more than 32 tiles


@pytest.mark.parametrize("tile", [8, 16])
def test_tiled_compat_large_splats_match_tiled_oracle(tile):
    """tiled_compat lists of large Gaussians (long emission runs, edge-clamped rectangles): the image equals
    the tiled renderer restated (oracle/tiled_oracle.py)."""
    wl = _large_splat_scene()
    out = render_raw(wl, B200RendererConfig(mode="tiled_compat", tile_size=tile), grads=False, loss=False)
    raw = so.RawGaussians(wl.means, wl.log_scales, wl.quats, wl.opacity_logits, wl.sh, wl.velocity)
    m, s, q, o, rgb = so.activate(raw, wl.times, wl.camera_to_world, wl.views_per_set)
    for b in range(wl.n_views):
        ref = tiled_oracle.render_tiled_view(m[b], s[b], q[b], o[b], rgb[b], wl.height, wl.width, wl.fx[b], wl.fy[b],
                                             wl.cx[b], wl.cy[b], wl.camera_to_world[b], tile_size=tile)
        assert (out["image"][b] - ref).abs().max().item() <= IMAGE_TOL


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("tile", [8, 16])
def test_tiled_compat_lists_match_reference(case, tile):
    """tiled_compat mode reproduces tiled.py's tile lists and their order exactly."""
    g = load_golden(case)
    wl = g.workload()
    _, _, _, st = stages(wl, B200RendererConfig(mode="tiled_compat", tile_size=tile))
    k = keys_np(st)
    n_tiles = to.n_tiles_for(wl.height, wl.width, tile)
    view_tile = (k >> np.uint64(32)).astype(np.int64)
    rank = (k & np.uint64(0xFFFFFFFF)).astype(np.int64)
    np.testing.assert_array_equal(view_tile // n_tiles, g[f"ref_tiled{tile}_view"])
    np.testing.assert_array_equal(view_tile % n_tiles, g[f"ref_tiled{tile}_tile"])
    np.testing.assert_array_equal(rank, g[f"ref_tiled{tile}_rank"])


@pytest.mark.parametrize("case", ["dynamic128_small", "multiview384_small"])
def test_tile_launch_order_is_a_permutation_by_descending_length(case):
    wl = load_golden(case).workload()
    _, _, _, st = stages(wl)
    order = st.order.cpu().numpy().astype(np.int64)
    np.testing.assert_array_equal(np.sort(order), np.arange(order.size))
    r = st.ranges.cpu().numpy().astype(np.int64).reshape(-1, 2)
    lengths = r[:, 1] - r[:, 0]
    # 8-bit log-scale length class (exact below 16, 8 steps per power of two), longest first, ties
    # in (view, tile) order
    e = np.array([max(int(n).bit_length() - 1, 0) for n in lengths], dtype=np.int64)
    cls = np.where(lengths < 8, lengths, (e - 2) * 8 + ((lengths >> np.maximum(e - 3, 0)) & 7))
    np.testing.assert_array_equal(order, np.argsort(255 - cls, kind="stable"))


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_image_loss_and_gradients_match_reference(case):
    g = load_golden(case)
    wl = g.workload()
    out = render_raw(wl)
    err = (out["image"] - g.t("ref_image")).abs().max().item()
    assert err <= IMAGE_TOL, f"image max abs err {err:.3e}"
    torch.testing.assert_close(out["loss"], g.t("ref_loss"), rtol=1e-4, atol=2e-6)
    keys = ("means", "log_scales", "quats", "opacity_logits", "sh") + (("velocity",) if wl.velocity is not None
                                                                          else ())
    for k in keys:
        ok, e, s = grad_close(out[f"grad_{k}"], g.t(f"ref_grad_{k}"), GRAD_REL)
        assert ok, f"{case} {k}: max err {e:.3e} vs scale {s:.3e}"
    # per element, up to the side a clamp's kink is taken at pixels within rounding of it (kinks.py)
    kinks.check_gradients(wl, {k: out[f"grad_{k}"] for k in keys}, {k: g.t(f"ref_grad_{k}") for k in keys})


@pytest.mark.parametrize("case", ["static64", "dynamic128_small", "edge"])
def test_alpha_and_depth_match_oracle(case):
    g = load_golden(case)
    wl = g.workload()
    out = render_raw(wl, B200RendererConfig(depth=True), grads=False, loss=False)
    raw = so.RawGaussians(*(t.double() for t in (wl.means, wl.log_scales, wl.quats, wl.opacity_logits, wl.sh)),
                          None if wl.velocity is None else wl.velocity.double())
    m, s, q, o, rgb = so.activate(raw, wl.times.double(), wl.camera_to_world, wl.views_per_set)
    img, alpha, depth = so.render_dense(m, s, q, o, rgb, wl.height, wl.width, wl.fx, wl.fy, wl.cx, wl.cy,
                                        wl.camera_to_world, sort_key=so.camera_depth_fp32(m.float(),
                                                                                           wl.camera_to_world))
    assert (out["alpha"].double() - alpha).abs().max().item() <= IMAGE_TOL
    assert (out["depth"].double() - depth).abs().max().item() <= IMAGE_TOL * max(1.0, depth.abs().max().item())


@pytest.mark.parametrize("case", ["static64", "dynamic128_small", "multiview384_small"])
def test_dropin_activated_batch_api(case):
    """render_b200_3dgs_batch takes the reference's activated [K,G,C] payload (dense.py:170)."""
    g = load_golden(case)
    wl = g.workload()
    act = {k: g.t(f"ref_act_{k}", DEV).requires_grad_(True) for k in ("xyz", "scales", "quats", "opacities",
                                                                        "rgbs")}
    img = render_b200_3dgs_batch(act["xyz"], act["scales"], act["quats"], act["opacities"], act["rgbs"],
                                 wl.height, wl.width, wl.fx.to(DEV), wl.fy.to(DEV), wl.cx.to(DEV), wl.cy.to(DEV),
                                 camera_to_world=wl.camera_to_world.to(DEV))
    assert (img.detach().cpu() - g.t("ref_image")).abs().max().item() <= IMAGE_TOL
    from dynaworld_b200.losses import reconstruction_loss_per_image

    reconstruction_loss_per_image(img, wl.target.to(DEV)).sum().backward()
    for k, v in act.items():
        ok, e, s = grad_close(v.grad, g.t(f"ref_grad_act_{k}"), GRAD_REL)
        assert ok, f"{case} {k}: {e:.3e} vs {s:.3e}"


def test_dropin_single_frame_api():
    g = load_golden("static64")
    a = {k: g.t(f"ref_act_{k}", DEV)[0] for k in ("xyz", "scales", "quats", "opacities", "rgbs")}
    img = render_b200_3dgs(a["xyz"], a["scales"], a["quats"], a["opacities"], a["rgbs"], 64, 64, 64.0, 64.0, 32.0,
                           32.0, camera_to_world=torch.eye(4, device=DEV))
    assert img.shape == (3, 64, 64)
    assert (img.cpu() - g.t("ref_image")[0]).abs().max().item() <= IMAGE_TOL


@pytest.mark.parametrize("tile", [8, 16])
@pytest.mark.parametrize("case", ["static64", "dynamic128_small", "edge"])
def test_tiled_compat_image_matches_reference_tiled(case, tile):
    g = load_golden(case)
    wl = g.workload()
    out = render_raw(wl, B200RendererConfig(mode="tiled_compat", tile_size=tile), grads=False, loss=False)
    err = (out["image"] - g.t(f"ref_tiled{tile}_image")).abs().max().item()
    assert err <= IMAGE_TOL, f"{err:.3e}"


def test_full_size_dynamic128_window():
    """G=32768 at 128x128: frame 5's 32x32 window against the reference's dense render of it."""
    g = load_golden("dynamic128_crop")
    wl = synthetic.dynamic128().views(5, 6)
    from tests.golden.make_golden import workload_arrays  # noqa: F401  (checksum layout)

    for k, v in workload_arrays(wl).items():
        assert float(v.double().sum()) == pytest.approx(float(g[f"checksum_{k}"]), rel=1e-12, abs=1e-9), k
    out = render_raw(wl, grads=False, loss=False)
    x0, y0, w, h = (int(v) for v in g["crop"])
    err = (out["image"][:, :, y0:y0 + h, x0:x0 + w] - g.t("ref_image")).abs().max().item()
    assert err <= IMAGE_TOL, f"{err:.3e}"


def test_forward_is_deterministic_and_backward_is_stable():
    wl = load_golden("dynamic128_small").workload()
    a = render_raw(wl)
    b = render_raw(wl)
    assert torch.equal(a["image"], b["image"])
    for k in ("means", "sh"):
        ok, e, s = grad_close(a[f"grad_{k}"], b[f"grad_{k}"], 1e-5)
        assert ok, (k, e, s)


def test_empty_and_invisible_scenes():
    """All Gaussians behind the camera: white image, zero alpha, zero gradients (no pairs)."""
    wl = synthetic.static64(scale=0.01)
    wl.means[..., 2] = -5.0
    out = render_raw(wl)
    assert torch.all(out["image"] == 1.0) and torch.all(out["alpha"] == 0.0)
    for k in ("means", "log_scales", "quats", "opacity_logits", "sh"):
        assert torch.all(out[f"grad_{k}"] == 0.0)


def test_ragged_image_sizes():
    """Images that are not a multiple of the tile: matches the dense oracle on every pixel."""
    wl = synthetic.static64(scale=0.25)
    for H, W in [(37, 45), (16, 17), (9, 70)]:
        wl2 = synthetic.Workload(**{**wl.__dict__, "height": H, "width": W,
                                    "target": torch.rand(1, 3, H, W, generator=torch.Generator().manual_seed(H))})
        out = render_raw(wl2, grads=False, loss=False)
        raw = so.RawGaussians(wl.means.double(), wl.log_scales.double(), wl.quats.double(),
                              wl.opacity_logits.double(), wl.sh.double(), None)
        m, s, q, o, rgb = so.activate(raw, wl.times.double(), wl.camera_to_world, 1)
        img, _, _ = so.render_dense(m, s, q, o, rgb, H, W, wl.fx, wl.fy, wl.cx, wl.cy, wl.camera_to_world,
                                    sort_key=so.camera_depth_fp32(m.float(), wl.camera_to_world))
        assert (out["image"].double() - img).abs().max().item() <= IMAGE_TOL


@pytest.mark.parametrize("tile", [8, 16])
@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_tiled_compat_gradients_match_reference_tiled(case, tile):
    """tiled_compat backward (tile-local (1 + eps) products, no power clamp) against autograd
    through the reference's tiled renderer (tiled.py:74-198) under the standard_gs loss."""
    g = load_golden(case)
    t = load_golden("tiled_grads")
    key = f"{case}_t{tile}"
    wl = g.workload()
    out = render_raw(wl, B200RendererConfig(mode="tiled_compat", tile_size=tile))
    assert (out["image"] - t.t(f"{key}_image")).abs().max().item() <= IMAGE_TOL
    np.testing.assert_allclose(out["loss"].numpy(), t[f"{key}_loss"], rtol=0, atol=1e-5)
    keys = [k for k in ("means", "log_scales", "quats", "opacity_logits", "sh", "velocity") if f"{key}_grad_{k}" in t]
    for k in keys:
        ok, e, s = grad_close(out[f"grad_{k}"], t.t(f"{key}_grad_{k}"), GRAD_REL)
        assert ok, f"{key} {k}: {e:.3e} vs {s:.3e}"
    kinks.check_gradients(wl, {k: out[f"grad_{k}"] for k in keys}, {k: t.t(f"{key}_grad_{k}") for k in keys},
                          tiled_tile=tile)


@pytest.mark.parametrize("tile", [8, 16])
@pytest.mark.parametrize("case", ["static64", "dynamic128_small", "edge"])
def test_tiled_compat_activated_api_gradients(case, tile):
    """The drop-in activated payload in tiled_compat mode: gradients w.r.t. the render call's own
    inputs against the reference's tiled renderer."""
    from dynaworld_b200.losses import reconstruction_loss_per_image

    g = load_golden(case)
    t = load_golden("tiled_grads")
    key = f"{case}_t{tile}"
    wl = g.workload()
    act = {k: g.t(f"ref_act_{k}", DEV).requires_grad_(True) for k in ("xyz", "scales", "quats", "opacities",
                                                                        "rgbs")}
    img = render_b200_3dgs_batch(act["xyz"], act["scales"], act["quats"], act["opacities"], act["rgbs"],
                                 wl.height, wl.width, wl.fx.to(DEV), wl.fy.to(DEV), wl.cx.to(DEV), wl.cy.to(DEV),
                                 camera_to_world=wl.camera_to_world.to(DEV),
                                 config=B200RendererConfig(mode="tiled_compat", tile_size=tile))
    assert (img.detach().cpu() - t.t(f"{key}_image")).abs().max().item() <= IMAGE_TOL
    reconstruction_loss_per_image(img, wl.target.to(DEV)).sum().backward()
    for k, v in act.items():
        ok, e, s = grad_close(v.grad, t.t(f"{key}_grad_act_{k}"), GRAD_REL)
        assert ok, f"{key} {k}: {e:.3e} vs {s:.3e}"
