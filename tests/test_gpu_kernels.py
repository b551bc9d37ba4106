"""CUDA loss kernel and radix sort against the reference / numpy, through the C ABI."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import grad_close, load_golden
from dynaworld_b200 import _lib
from dynaworld_b200.config import LossConfig
from dynaworld_b200.losses import reconstruction_loss_per_image
from gpu_helpers import DEV
from oracle import splat_oracle as so

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["standard_gs", "l1", "mse", "l1_mse"])
def test_loss_matches_reference(kind):
    g = load_golden("losses")
    for i in range(3):
        pred = g.t(f"loss{i}_pred", DEV).requires_grad_(True)
        tgt = g.t(f"loss{i}_target", DEV)
        B = pred.shape[0]
        loss = reconstruction_loss_per_image(pred, tgt, {"type": kind})
        (loss * torch.arange(1, B + 1, device=DEV, dtype=torch.float32)).sum().backward()
        torch.testing.assert_close(loss.cpu(), g.t(f"loss{i}_{kind}_value"), rtol=1e-5, atol=1e-6)
        ok, e, s = grad_close(pred.grad, g.t(f"loss{i}_{kind}_grad"), 1e-4)
        assert ok, f"loss{i} {kind}: {e:.3e} vs {s:.3e}"


@pytest.mark.parametrize("window,half", [("gaussian", True), ("box", False), ("gaussian", False)])
def test_loss_variants_match_oracle(window, half):
    gen = torch.Generator().manual_seed(3)
    pred = torch.rand(2, 3, 40, 52, generator=gen)
    tgt = torch.rand(2, 3, 40, 52, generator=gen)
    cfg = {"ssim_window": window, "dssim_half": half}
    p = pred.double().requires_grad_(True)
    ref = so.reconstruction_loss_per_image(p, tgt.double(), cfg)
    ref.sum().backward()
    q = pred.to(DEV).requires_grad_(True)
    got = reconstruction_loss_per_image(q, tgt.to(DEV), cfg)
    got.sum().backward()
    torch.testing.assert_close(got.double().cpu(), ref.detach(), rtol=1e-5, atol=1e-6)
    ok, e, s = grad_close(q.grad, p.grad, 1e-4)
    assert ok, (e, s)


def test_loss_window_sizes():
    gen = torch.Generator().manual_seed(4)
    pred, tgt = torch.rand(1, 3, 33, 33, generator=gen), torch.rand(1, 3, 33, 33, generator=gen)
    for ws in (3, 7, 15):
        cfg = {"ssim_window_size": ws}
        p = pred.double().requires_grad_(True)
        ref = so.reconstruction_loss_per_image(p, tgt.double(), cfg)
        ref.sum().backward()
        q = pred.to(DEV).requires_grad_(True)
        got = reconstruction_loss_per_image(q, tgt.to(DEV), cfg)
        got.sum().backward()
        torch.testing.assert_close(got.double().cpu(), ref.detach(), rtol=1e-5, atol=1e-6)
        assert grad_close(q.grad, p.grad, 1e-4)[0]


def _sort(keys: torch.Tensor, vals: torch.Tensor | None, bit_lo: int, bit_hi: int):
    L = _lib.lib()
    n = keys.numel()
    kb = keys.element_size()
    out_k = torch.empty_like(keys)
    out_v = torch.empty_like(vals) if vals is not None else None
    ws = torch.empty(L.gsb_radix_sort_workspace(n, kb, int(vals is not None)), dtype=torch.uint8, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check("gsb_radix_sort", L.gsb_radix_sort(keys.data_ptr(), out_k.data_ptr(), _lib.ptr(vals),
                                                  _lib.ptr(out_v), n, kb, bit_lo, bit_hi, ws.data_ptr(),
                                                  ws.numel(), st))
    status = ctypes.c_int(0)
    _lib.check("gsb_read_status", L.gsb_read_status(ws.data_ptr(), ctypes.byref(status), st))
    assert status.value == 0
    return out_k, out_v


@pytest.mark.parametrize("n", [1, 31, 3072, 100_003, 1_500_001])
@pytest.mark.parametrize("kbits,bits", [(32, (0, 32)), (64, (0, 40)), (64, (32, 50)), (32, (3, 13))])
def test_radix_sort_stable_vs_numpy(n, kbits, bits):
    rng = np.random.default_rng(n + bits[1])
    dtype = np.uint32 if kbits == 32 else np.uint64
    hi = np.iinfo(dtype).max
    keys = rng.integers(0, hi, size=n, dtype=dtype, endpoint=True)
    keys[: n // 3] = keys[n // 2] if n > 2 else keys[: n // 3]  # many duplicates: stability matters
    vals = np.arange(n, dtype=np.uint32)
    lo, hib = bits
    mask = ((1 << (hib - lo)) - 1)
    digit = (keys >> dtype(lo)) & dtype(mask)
    order = np.argsort(digit, kind="stable")
    tk = torch.from_numpy(keys.view(np.int32 if kbits == 32 else np.int64)).to(DEV)
    tv = torch.from_numpy(vals.view(np.int32)).to(DEV)
    ok, ov = _sort(tk, tv, lo, hib)
    np.testing.assert_array_equal(ok.cpu().numpy().view(dtype), keys[order])
    np.testing.assert_array_equal(ov.cpu().numpy().view(np.uint32), vals[order])


def test_radix_sort_keys_only_and_empty():
    rng = np.random.default_rng(0)
    keys = rng.integers(0, 2**63, size=50_000, dtype=np.uint64)
    tk = torch.from_numpy(keys.view(np.int64)).to(DEV)
    ok, _ = _sort(tk, None, 0, 64)
    np.testing.assert_array_equal(ok.cpu().numpy().view(np.uint64), np.sort(keys))
    empty = torch.empty(0, dtype=torch.int64, device=DEV)
    ok, _ = _sort(empty, None, 0, 64)
    assert ok.numel() == 0
