"""Reconstruction loss on the fused CUDA kernel.

``reconstruction_loss_per_image(prediction, target, loss_cfg)`` is a drop-in for the reference's
function of the same name (src/train/losses.py:58-85): [B,C,H,W] images -> loss [B], with
types standard_gs (L1 + box-window D-SSIM), l1, mse and l1_mse.  The forward kernel also writes
d loss[b] / d prediction; the backward scales it by the upstream gradient.
"""
from __future__ import annotations

from typing import Any

import torch

from . import _lib
from .config import LossConfig
from .render import _stage, _stream


def loss_forward(pred: torch.Tensor, target: torch.Tensor, cfg: LossConfig, need_grad: bool = True):
    """loss [B] and d loss[b] / d pred ([B,C,H,W], unit upstream gradient; None if not needed)."""
    L = _lib.lib()
    B, Cc, H, W = (int(s) for s in pred.shape)
    dev = pred.device
    p = pred.detach().to(torch.float32).contiguous()
    t = target.detach().to(device=dev, dtype=torch.float32).contiguous()
    loss = torch.empty(B, dtype=torch.float32, device=dev)
    dpred = torch.empty_like(p) if need_grad else None
    ws = torch.empty(max(int(L.gsb_loss_workspace(B)), 256), dtype=torch.uint8, device=dev)
    opts = cfg.options()
    with _stage("loss"):
        _lib.check("gsb_loss_fwd_bwd", L.gsb_loss_fwd_bwd(opts, B, Cc, H, W, p.data_ptr(), t.data_ptr(),
                                                          loss.data_ptr(), _lib.ptr(dpred), ws.data_ptr(), ws.numel(),
                                                          _stream(dev)))
    return loss, dpred


def scale_planes(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """out[b] = scale[b] * x[b] on the library's kernel."""
    L = _lib.lib()
    B = int(x.shape[0])
    out = torch.empty_like(x)
    s = scale.detach().to(device=x.device, dtype=torch.float32).contiguous()
    with _stage("loss_scale"):
        _lib.check("gsb_scale_planes", L.gsb_scale_planes(x.data_ptr(), s.data_ptr(), out.data_ptr(), B,
                                                          x.numel() // max(B, 1), _stream(x.device)))
    return out


class _LossFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, cfg, pred, target):
        loss, dpred = loss_forward(pred, target, cfg, need_grad=pred.requires_grad)
        ctx.dpred = dpred
        ctx.dtype = pred.dtype
        return loss

    @staticmethod
    def backward(ctx, grad_loss):
        dpred = ctx.dpred
        ctx.dpred = None
        if dpred is None:
            return None, None, None
        g = scale_planes(dpred, grad_loss.contiguous())
        return None, g.to(ctx.dtype), None


def reconstruction_loss_per_image(prediction: torch.Tensor, target: torch.Tensor,
                                  loss_cfg: dict[str, Any] | LossConfig | None = None) -> torch.Tensor:
    """Per-image loss [B] (losses.py:58-85).  Gradients flow to ``prediction`` only."""
    cfg = loss_cfg if isinstance(loss_cfg, LossConfig) else LossConfig.from_mapping(loss_cfg)
    if not prediction.is_cuda:
        raise RuntimeError("the b200 loss runs on CUDA devices only (got a tensor on %s)" % prediction.device)
    if target.requires_grad:
        raise NotImplementedError("the b200 loss does not differentiate the target; detach it.")
    if prediction.shape != target.shape or prediction.ndim != 4:
        raise ValueError(f"prediction and target must both be [B,C,H,W], got {tuple(prediction.shape)} and "
                         f"{tuple(target.shape)}")
    return _LossFunction.apply(cfg, prediction, target)


def reconstruction_loss(prediction, target, loss_cfg=None) -> torch.Tensor:
    """Mean over images (losses.py:88-93)."""
    return reconstruction_loss_per_image(prediction, target, loss_cfg).mean()
