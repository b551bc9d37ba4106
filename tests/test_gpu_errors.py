"""Error paths on the GPU, made without faulting or hanging it.

* A bounded look-back wait that runs out: the radix sort's test hook runs one pass in which the
  first partition never runs, so its successor waits for a publication that never comes.  The wait
  gives up after a short spin limit; the status word reads GSB_ERR_TIMEOUT, every kernel returns,
  nothing is written past the output, and the context stays usable.
* Non-finite inputs: NaN / inf parameters made on the host are counted by the projection and the
  render call raises FloatingPointError, as the reference's trainers do on a non-finite render
  (src/train/dynamicTokenGS.py:559-590); with check_finite off the frame renders without them.
* Launch-shape limits: the loss over more than 65,535 image planes (grid.z limit of one launch).
"""
import ctypes

import numpy as np
import pytest
import torch

from dynaworld_b200 import _lib, synthetic
from dynaworld_b200.config import B200RendererConfig
from dynaworld_b200.losses import reconstruction_loss_per_image
from gpu_helpers import DEV, render_raw

pytestmark = pytest.mark.gpu


def _status(L, ws) -> int:
    out = ctypes.c_int(-1)
    _lib.check("gsb_read_status", L.gsb_read_status(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(out),
                                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return out.value


@pytest.mark.parametrize("spin_limit", [1, 64])
def test_lookback_wait_gives_up_with_timeout_status(spin_limit):
    L = _lib.load()
    n = 3 * 2048 + 517  # four partitions of 2048 keys; the first never runs
    g = torch.Generator().manual_seed(7)
    keys = torch.randint(0, 2**31 - 1, (n,), generator=g, dtype=torch.int64).to(torch.int32).to(DEV)
    guard = 4096
    canary = 0x5A5A5A5A
    out = torch.full((n + guard,), canary, dtype=torch.int32, device=DEV)
    ws = torch.zeros(L.gsb_radix_sort_workspace(n, 4, 0), dtype=torch.uint8, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check("gsb_debug_sort_lookback_timeout",
               L.gsb_debug_sort_lookback_timeout(keys.data_ptr(), out.data_ptr(), n, spin_limit, ws.data_ptr(),
                                                 ws.numel(), st))
    torch.cuda.synchronize()  # every kernel returned
    assert _status(L, ws) == _lib.GSB_ERR_TIMEOUT
    assert bool((out[n:] == canary).all()), "a write landed past the output"
    # the first partition's 2048 keys were never scattered: the output is not the sorted input
    assert not torch.equal(out[:n].sort().values, keys.sort().values)
    # the context is still usable: a normal sort on the same workspace gives the sorted order
    ws2 = torch.zeros(L.gsb_radix_sort_workspace(n, 4, 0), dtype=torch.uint8, device=DEV)
    sorted_out = torch.empty(n, dtype=torch.int32, device=DEV)
    _lib.check("gsb_radix_sort", L.gsb_radix_sort(keys.data_ptr(), sorted_out.data_ptr(), None, None, n, 4, 0, 32,
                                                  ws2.data_ptr(), ws2.numel(), st))
    torch.cuda.synchronize()
    assert _status(L, ws2) == _lib.GSB_OK
    ref = np.sort(keys.cpu().numpy().view(np.uint32))
    np.testing.assert_array_equal(sorted_out.cpu().numpy().view(np.uint32), ref)


def test_lookback_hook_rejects_single_partition_inputs():
    L = _lib.load()
    keys = torch.zeros(1000, dtype=torch.int32, device=DEV)
    ws = torch.zeros(L.gsb_radix_sort_workspace(1000, 4, 0), dtype=torch.uint8, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    assert L.gsb_debug_sort_lookback_timeout(keys.data_ptr(), keys.data_ptr(), 1000, 1, ws.data_ptr(), ws.numel(),
                                             st) == 1  # GSB_ERR_SHAPE


def _poisoned(kind):
    wl = synthetic.static64(scale=0.25, image_scale=0.5)
    if kind == "nan_mean":
        wl.means[0, 7, 0] = float("nan")
    elif kind == "inf_scale":
        wl.log_scales[0, 11, 1] = float("inf")
    elif kind == "nan_sh":
        wl.sh[0, 3, 0, 2] = float("nan")
    elif kind == "nan_opacity":
        wl.opacity_logits[0, 5, 0] = float("nan")
    return wl


@pytest.mark.parametrize("kind", ["nan_mean", "inf_scale", "nan_sh", "nan_opacity"])
def test_nonfinite_inputs_raise(kind):
    wl = _poisoned(kind)
    with pytest.raises(FloatingPointError, match="Non-finite render input: 1 projected"):
        render_raw(wl, grads=False, loss=False)


def test_nonfinite_inputs_skipped_when_unchecked():
    """With check_finite off the poisoned Gaussian is left out of the frame, which then equals the
    frame rendered without it (its (1 + eps) factor aside: it would multiply every later pixel's
    transmittance by 1 + 2^-20, below the 1e-4 image bar)."""
    wl = _poisoned("nan_sh")
    out = render_raw(wl, B200RendererConfig(check_finite=False), grads=False, loss=False)
    assert torch.isfinite(out["image"]).all()
    keep = torch.ones(wl.n_gaussians, dtype=torch.bool)
    keep[3] = False
    clean = synthetic.static64(scale=0.25, image_scale=0.5)
    for k in ("means", "log_scales", "quats", "opacity_logits", "sh"):
        setattr(clean, k, getattr(clean, k)[:, keep])
    ref = render_raw(clean, grads=False, loss=False)
    assert (out["image"] - ref["image"]).abs().max().item() <= 1e-4


def test_finite_scene_reports_nothing():
    wl = synthetic.static64(scale=0.25, image_scale=0.5)
    out = render_raw(wl)
    assert torch.isfinite(out["image"]).all()


def test_loss_over_more_than_65535_planes():
    """21,846 three-channel images (65,538 planes) go to two launches; every per-image loss and
    gradient equals the one computed over a slice of the batch."""
    g = torch.Generator().manual_seed(3)
    B, H, W = 21846, 16, 16
    pred = torch.rand(B, 3, H, W, generator=g).to(DEV).requires_grad_(True)
    tgt = torch.rand(B, 3, H, W, generator=g).to(DEV)
    loss = reconstruction_loss_per_image(pred, tgt)
    loss.sum().backward()
    for lo, hi in ((0, 8), (21840, 21846)):
        p2 = pred.detach()[lo:hi].clone().requires_grad_(True)
        l2 = reconstruction_loss_per_image(p2, tgt[lo:hi])
        l2.sum().backward()
        assert torch.allclose(loss.detach()[lo:hi], l2.detach(), rtol=0, atol=1e-6)
        assert torch.allclose(pred.grad[lo:hi], p2.grad, rtol=0, atol=1e-9)
