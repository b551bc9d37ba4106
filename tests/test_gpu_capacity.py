"""Binning queued with a pair capacity instead of the pair count.

gsb_bin reads the count (pair_offsets[B*G]) on the device: a capacity above it gives the same
keys and ranges, one below it records GSB_ERR_CAPACITY without writing past the capacity.  The
render path guesses the capacity from earlier frames of the same shape and re-runs binning and
the blend when the guess was short.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import grad_close, load_golden
from dynaworld_b200 import _lib, render
from dynaworld_b200.config import B200RendererConfig
from gpu_helpers import DEV, render_raw, stages

pytestmark = pytest.mark.gpu

GRAD_KEYS = ("means", "log_scales", "quats", "opacity_logits", "sh", "velocity")


def _bin(capacity: int):
    """Three Gaussians on a 32x32 frame of 16x16 tiles, tile rectangles given directly (ellipse
    culling off): 4 + 2 + 1 = 7 pairs."""
    L = _lib.lib()
    B, G, H, W = 1, 3, 32, 32
    v = _lib.Views()
    v.n_views, v.views_per_set, v.height, v.width = B, 1, H, W
    o = B200RendererConfig(ellipse_culling=False).options(1e-4)
    records = torch.zeros(B * G * _lib.RECORD_FLOATS, dtype=torch.float32, device=DEV)
    rects = torch.tensor([[0, 0, 1, 1], [1, 0, 1, 1], [0, 1, 0, 1]], dtype=torch.int32, device=DEV)
    offsets = torch.tensor([0, 4, 6, 7], dtype=torch.int32, device=DEV)
    keys = torch.full((max(capacity, 1),), -1, dtype=torch.int64, device=DEV)
    ranges = torch.empty(4 * 2, dtype=torch.int32, device=DEV)
    order = torch.empty(4, dtype=torch.int32, device=DEV)
    ws = torch.empty(L.gsb_bin_workspace(v, o, G, capacity), dtype=torch.uint8, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check("gsb_bin", L.gsb_bin(v, o, G, records.data_ptr(), rects.data_ptr(), offsets.data_ptr(), capacity,
                                    keys.data_ptr(), ranges.data_ptr(), order.data_ptr(), ws.data_ptr(),
                                    ws.numel(), st))
    status = ctypes.c_int(0)
    _lib.check("gsb_read_status", L.gsb_read_status(ws.data_ptr(), ctypes.byref(status), st))
    torch.cuda.synchronize()
    return status.value, keys.cpu().numpy().view(np.uint64), ranges.cpu().numpy()


@pytest.mark.parametrize("capacity", [7, 8, 1000])
def test_bin_capacity_at_or_above_the_count(capacity):
    status, keys, ranges = _bin(capacity)
    assert status == 0
    tiles_and_ranks = [(0, 0), (1, 0), (1, 1), (2, 0), (2, 2), (3, 0), (3, 1)]
    np.testing.assert_array_equal(keys[:7], [(t << 32) | r for t, r in tiles_and_ranks])
    np.testing.assert_array_equal(ranges, [0, 1, 1, 3, 3, 5, 5, 7])
    if capacity > 7:
        assert (keys[7:] == np.uint64(2**64 - 1)).all()  # untouched past the count


@pytest.mark.parametrize("capacity", [0, 5])
def test_bin_capacity_below_the_count_is_reported(capacity):
    status, keys, ranges = _bin(capacity)
    assert _lib.STATUS_NAMES[status] == "GSB_ERR_CAPACITY"
    assert ranges.max() <= capacity


@pytest.mark.parametrize("guess", ["short", "generous"])
def test_render_with_a_capacity_guess(guess):
    g = load_golden("dynamic128_small")
    wl = g.workload()
    cfg = B200RendererConfig()
    render._PAIR_CAPACITY.clear()
    _, _, _, state = stages(wl, cfg)
    (shape,) = render._PAIR_CAPACITY.keys()
    n = state.n_pairs
    render._PAIR_CAPACITY[shape] = 64 if guess == "short" else 3 * n + 7
    out = render_raw(wl, cfg)
    assert render._PAIR_CAPACITY[shape] >= n
    assert (out["image"] - g.t("ref_image")).abs().max().item() <= 1e-4
    torch.testing.assert_close(out["loss"], g.t("ref_loss"), rtol=1e-4, atol=2e-6)
    for k in GRAD_KEYS:
        if f"grad_{k}" not in out:
            continue
        ok, e, s = grad_close(out[f"grad_{k}"], g.t(f"ref_grad_{k}"), 1e-3)
        assert ok, f"{guess} {k}: max err {e:.3e} vs scale {s:.3e}"
