"""The allocation-free loss entry point, gsb_loss_fwd_bwd_noalloc, through the C ABI.

It serves callers that cannot allocate device memory themselves (for instance a binding that only
receives input and output buffers from a host framework that owns the allocator): its scratch is a
fixed array inside libgsb200.so instead of a caller-provided workspace.  Its results must equal
those of gsb_loss_fwd_bwd, on repeated calls too, since every call reuses that one array.

Collected last (file name) so that a run stopping at the first failure has run everything else.
"""
import ctypes

import pytest
import torch

from dynaworld_b200 import _lib, build
from dynaworld_b200.config import LossConfig

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
MAX_IMAGES = 4096  # GSB_LOSS_NOALLOC_MAX_IMAGES in include/gsb200.h


def _inputs(B=3, H=40, W=52, seed=7):
    g = torch.Generator().manual_seed(seed)
    pred = torch.rand(B, 3, H, W, generator=g).to(DEV)
    target = torch.rand(B, 3, H, W, generator=g).to(DEV)
    return pred, target


def _with_workspace(L, opts, pred, target):
    B, C, H, W = pred.shape
    loss = torch.empty(B, device=DEV)
    dpred = torch.empty_like(pred)
    ws = torch.empty(L.gsb_loss_workspace(B), dtype=torch.uint8, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check("gsb_loss_fwd_bwd", L.gsb_loss_fwd_bwd(ctypes.byref(opts), B, C, H, W, pred.data_ptr(),
                                                      target.data_ptr(), loss.data_ptr(), dpred.data_ptr(),
                                                      ws.data_ptr(), ws.numel(), st))
    torch.cuda.synchronize()
    return loss, dpred


def _no_alloc(L, opts, pred, target):
    B, C, H, W = pred.shape
    loss = torch.full((B,), float("nan"), device=DEV)
    dpred = torch.full_like(pred, float("nan"))
    st = torch.cuda.current_stream().cuda_stream
    _lib.check("gsb_loss_fwd_bwd_noalloc", L.gsb_loss_fwd_bwd_noalloc(ctypes.byref(opts), B, C, H, W,
                                                                      pred.data_ptr(), target.data_ptr(),
                                                                      loss.data_ptr(), dpred.data_ptr(), st))
    torch.cuda.synchronize()
    return loss, dpred


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


@pytest.mark.parametrize("kind", ["standard_gs", "l1_mse"])
def test_no_alloc_matches_workspace_entry_on_consecutive_calls(lib, kind):
    opts = LossConfig.from_mapping({"type": kind}).options()
    pred, target = _inputs()
    ref_loss, ref_dpred = _with_workspace(lib, opts, pred, target)
    scale = ref_dpred.abs().max().item()
    for _ in range(2):  # the second call reuses the array the first one left behind
        loss, dpred = _no_alloc(lib, opts, pred, target)
        torch.testing.assert_close(loss, ref_loss, rtol=1e-5, atol=1e-6)
        assert (dpred - ref_dpred).abs().max().item() <= 1e-4 * scale


def test_no_alloc_other_batch_after_a_larger_one(lib):
    """A smaller batch right after a larger one: stale sums of the larger call must not leak in."""
    opts = LossConfig().options()
    big_p, big_t = _inputs(B=5, seed=1)
    _no_alloc(lib, opts, big_p, big_t)
    pred, target = _inputs(B=2, seed=2)
    ref_loss, ref_dpred = _with_workspace(lib, opts, pred, target)
    loss, dpred = _no_alloc(lib, opts, pred, target)
    torch.testing.assert_close(loss, ref_loss, rtol=1e-5, atol=1e-6)
    assert (dpred - ref_dpred).abs().max().item() <= 1e-4 * ref_dpred.abs().max().item()


def test_no_alloc_rejects_batches_beyond_its_array(lib):
    opts = LossConfig().options()
    dummy = torch.zeros(1, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    status = lib.gsb_loss_fwd_bwd_noalloc(ctypes.byref(opts), MAX_IMAGES + 1, 3, 16, 16, dummy.data_ptr(),
                                          dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), st)
    assert status == 1  # GSB_ERR_SHAPE, returned before any launch
