"""Helpers shared by the GPU tests: run the render + loss through the public API on cuda:0."""
from __future__ import annotations

import numpy as np
import torch

from dynaworld_b200 import _lib
from dynaworld_b200.config import B200RendererConfig
from dynaworld_b200.losses import reconstruction_loss_per_image
from dynaworld_b200.render import SceneSpec, ViewSpec, forward_stages
from dynaworld_b200.renderer import render_b200

DEV = "cuda:0"


def intrinsics_of(wl, device=DEV):
    return torch.stack([wl.fx, wl.fy, wl.cx, wl.cy], -1).to(device)


def render_raw(wl, cfg: B200RendererConfig | None = None, *, grads=True, loss=True, device=DEV, lens_models=None,
               distortion=None, depth_loss=False):
    """render_b200 + reconstruction_loss_per_image on the GPU; returns a dict of CPU tensors.
    ``depth_loss``: also back-propagate through the alpha and depth outputs (needs cfg.depth)."""
    cfg = cfg or B200RendererConfig()
    leaves = {k: getattr(wl, k).to(device).requires_grad_(grads) for k in
              ("means", "log_scales", "quats", "opacity_logits", "sh")}
    vel = wl.velocity.to(device).requires_grad_(grads) if wl.velocity is not None else None
    image, alpha, depth = render_b200(
        leaves["means"], leaves["log_scales"], leaves["quats"], leaves["opacity_logits"], leaves["sh"],
        intrinsics=intrinsics_of(wl, device), camera_to_world=wl.camera_to_world.to(device),
        height=wl.height, width=wl.width, velocity=vel, times=wl.times.to(device),
        views_per_set=wl.views_per_set, config=cfg, lens_models=lens_models, distortion=distortion,
    )
    out = {"image": image.detach().cpu(), "alpha": alpha.detach().cpu(),
           "depth": None if depth is None else depth.detach().cpu()}
    if loss:
        l = reconstruction_loss_per_image(image, wl.target.to(device))
        out["loss"] = l.detach().cpu()
        if grads:
            total = l.sum()
            if depth_loss:
                total = total + 1e-3 * (depth * torch.cos(depth)).sum() + 0.05 * (alpha * alpha).sum()
            total.backward()
            for k, v in leaves.items():
                out[f"grad_{k}"] = v.grad.detach().cpu()
            if vel is not None:
                out["grad_velocity"] = vel.grad.detach().cpu()
    torch.cuda.synchronize()
    return out


def render_vjp(wl, cotangent: torch.Tensor, cfg: B200RendererConfig | None = None, device=DEV):
    """render_b200 on the GPU, then the backward of sum(cotangent * image) ([B,3,H,W] cotangent);
    returns the image and the raw-parameter gradients as CPU tensors."""
    cfg = cfg or B200RendererConfig()
    leaves = {k: getattr(wl, k).to(device).requires_grad_(True) for k in
              ("means", "log_scales", "quats", "opacity_logits", "sh")}
    if wl.velocity is not None:
        leaves["velocity"] = wl.velocity.to(device).requires_grad_(True)
    image, _alpha, _depth = render_b200(
        leaves["means"], leaves["log_scales"], leaves["quats"], leaves["opacity_logits"], leaves["sh"],
        intrinsics=intrinsics_of(wl, device), camera_to_world=wl.camera_to_world.to(device),
        height=wl.height, width=wl.width, velocity=leaves.get("velocity"), times=wl.times.to(device),
        views_per_set=wl.views_per_set, config=cfg,
    )
    image.backward(cotangent.to(device))
    out = {"image": image.detach().cpu()}
    out.update({f"grad_{k}": v.grad.detach().cpu() for k, v in leaves.items()})
    torch.cuda.synchronize()
    return out


def stages(wl, cfg: B200RendererConfig | None = None, device=DEV, lens=None):
    """Forward stages only; returns the FrameState and the outputs.  ``lens``: the pair
    render.lens_tensors returns (None: pinhole views)."""
    cfg = cfg or B200RendererConfig()
    S, G = wl.n_sets, wl.n_gaussians
    sspec = SceneSpec(S, G, True, wl.sh_degree, wl.velocity is not None, cfg.sh_clamp)
    vspec = ViewSpec(wl.n_views, wl.views_per_set, wl.height, wl.width)
    t = {
        "means": wl.means.to(device).contiguous(), "scales": wl.log_scales.to(device).contiguous(),
        "quats": wl.quats.to(device).contiguous(), "opacities": wl.opacity_logits.reshape(S, G).to(device).contiguous(),
        "colors": wl.sh.to(device).contiguous(),
        "velocity": None if wl.velocity is None else wl.velocity.to(device).contiguous(),
        "intrinsics": intrinsics_of(wl, device).contiguous(),
        "camera_to_world": wl.camera_to_world.to(device).contiguous(), "times": wl.times.to(device).contiguous(),
    }
    if lens is not None:
        t["lens_models"], t["distortion"] = lens
    image, alpha, depth, state = forward_stages(sspec, vspec, cfg, 1e-4, t)
    torch.cuda.synchronize()
    return image, alpha, depth, state


def sorted_ids_from_rank(rank_of: torch.Tensor, B: int, G: int) -> np.ndarray:
    r = rank_of.view(B, G).cpu().long()
    ids = torch.empty_like(r)
    ids.scatter_(1, r, torch.arange(G).expand(B, G))
    return ids.numpy()


def records_np(state, B: int, G: int) -> np.ndarray:
    return state.records.view(B, G, _lib.RECORD_FLOATS).cpu().numpy()


def keys_np(state) -> np.ndarray:
    return state.keys[: state.n_pairs].cpu().numpy().view(np.uint64)
