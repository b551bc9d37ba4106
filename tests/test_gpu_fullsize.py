"""Full-size workloads on the GPU: whole views rendered by the CUDA path, windows of them checked
against the dense oracle (the reference's all-pairs blend restated; a window is exact because
pixels are independent given the Gaussians), plus size-independent properties of the full step."""
import pytest
import torch

from dynaworld_b200 import synthetic
from dynaworld_b200.config import B200RendererConfig
from gpu_helpers import render_raw, stages
from oracle import splat_oracle as so

pytestmark = pytest.mark.gpu

IMAGE_TOL = 1e-4


def oracle_window(wl, view, x0, y0, w, h):
    """Dense oracle (float32, as the reference computes) of a window of one view."""
    s = view // wl.views_per_set if wl.views_per_set < wl.n_views else 0
    raw = so.RawGaussians(wl.means[s:s + 1], wl.log_scales[s:s + 1], wl.quats[s:s + 1],
                          wl.opacity_logits[s:s + 1], wl.sh[s:s + 1],
                          None if wl.velocity is None else wl.velocity[s:s + 1])
    sl = slice(view, view + 1)
    m, sc, q, o, rgb = so.activate(raw, wl.times[sl], wl.camera_to_world[sl], 1)
    img, alpha, _ = so.render_dense(m, sc, q, o, rgb, h, w, wl.fx[sl], wl.fy[sl], wl.cx[sl], wl.cy[sl],
                                    wl.camera_to_world[sl], sort_key=so.camera_depth_fp32(m, wl.camera_to_world[sl]),
                                    x0=x0, y0=y0)
    return img[0], alpha[0]


def check_windows(wl, out, windows):
    for view, x0, y0, w, h in windows:
        ref, ref_alpha = oracle_window(wl, view, x0, y0, w, h)
        got = out["image"][view, :, y0:y0 + h, x0:x0 + w]
        err = (got - ref).abs().max().item()
        assert err <= IMAGE_TOL, f"view {view} window ({x0},{y0}): {err:.3e}"
        aerr = (out["alpha"][view, y0:y0 + h, x0:x0 + w] - ref_alpha).abs().max().item()
        assert aerr <= IMAGE_TOL, f"alpha view {view} window ({x0},{y0}): {aerr:.3e}"


def check_step_properties(out):
    assert torch.isfinite(out["image"]).all() and out["image"].min() >= 0 and out["image"].max() <= 1
    assert torch.isfinite(out["alpha"]).all() and out["alpha"].min() >= 0
    assert torch.isfinite(out["loss"]).all()
    for k, v in out.items():
        if k.startswith("grad_"):
            assert torch.isfinite(v).all(), k


def test_multiview384_full():
    """8 views at 384x384, 200k Gaussians with 5% anisotropic outliers, SH degree 3."""
    wl = synthetic.multiview384()
    out = render_raw(wl)
    check_step_properties(out)
    check_windows(wl, out, [(0, 184, 184, 16, 16), (3, 100, 250, 16, 16), (7, 300, 40, 16, 16)])


def test_large1080_views():
    """1M Gaussians at 1920x1080 (4 of the 32 views), windows against the dense oracle."""
    wl = synthetic.large1080().views(0, 4)
    out = render_raw(wl)
    check_step_properties(out)
    check_windows(wl, out, [(0, 952, 532, 8, 8), (2, 100, 900, 8, 8), (3, 1900, 10, 8, 8)])


def test_clips256_per_clip_gradients_are_independent():
    """Per-clip Gaussian sets: a clip's gradients depend only on its own frames."""
    wl = synthetic.clips256(clips=3)
    out = render_raw(wl)
    check_step_properties(out)
    check_windows(wl, out, [(0, 120, 120, 16, 16), (13, 10, 200, 16, 16)])
    wl2 = synthetic.clips256(clips=3)
    wl2.target[0:8] = 1.0 - wl2.target[0:8]  # change clip 0's targets only
    out2 = render_raw(wl2)
    for k in ("means", "sh", "velocity"):
        a, b = out[f"grad_{k}"], out2[f"grad_{k}"]
        assert not torch.allclose(a[0], b[0]), k
        scale = a[1:].abs().max().item()
        assert (a[1:] - b[1:]).abs().max().item() <= 1e-5 * scale, k


def test_pair_counts_fit_and_tile_lists_are_sorted():
    wl = synthetic.large1080().views(0, 2)
    _, _, _, st = stages(wl)
    assert 0 < st.n_pairs < 2**30
    keys = st.keys[: st.n_pairs]
    assert bool((keys[1:] >= keys[:-1]).all())


def test_tiled_compat_runs_at_full_size():
    wl = synthetic.multiview384().views(0, 2)
    out = render_raw(wl, B200RendererConfig(mode="tiled_compat", tile_size=16), grads=False, loss=False)
    assert torch.isfinite(out["image"]).all()
