"""Dynamic Gaussian bank, evaluated and rendered in one call.

The reference's dynamic video-token model decodes a bank once per clip
(gs_models/dynamic_video_token_gs_implicit_camera.py:855-952, DynamicResidualGaussianBankHead) and
then, for every decode time, evaluates it in torch (:1206-1224, _eval_dynamic_bank):

    phi       = temporal basis of the time (:806-825)                         [M]
    xyz_t     = xyz0 + sum_m phi_m A_mu[:, m]
    quats_t   = normalize(quats0 (x) axis_angle_quat(sum_m phi_m A_rot[:, m]))  (:828-852)
    opacity_t = sigmoid(logit(clamp(opacities0, 1e-6, 1 - 1e-6)) + sum_m phi_m A_alpha[:, m])
    scales, rgbs unchanged

puts the static Gaussians in front (:1256-1275, _decode_static_dynamic_split) and renders the
frames (rendering.py:230-351).  ``render_dynamic_bank`` does the evaluation inside the
projection kernel for every (frame, Gaussian), so the per-frame [K, G, *] tensors are never
written, and its backward sums the coefficient gradients over the frames in registers.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib
from .config import B200RendererConfig
from .render import MIN_RENDER_DEPTH, SceneSpec, ViewSpec, render_scene
from .renderer import _intrinsics, _lens_of


@dataclass(frozen=True)
class DynamicGaussianBank:
    """The reference's bank (:795-803).  A leading clip dimension of 1 is accepted and dropped:
    xyz0 [G,3], scales [G,3], quats0 [G,4], opacities0 [G,1], rgbs [G,3], A_mu [G,M,3],
    A_rot [G,M,3] (axis-angle, radians), A_alpha [G,M,1]."""

    xyz0: torch.Tensor
    scales: torch.Tensor
    quats0: torch.Tensor
    opacities0: torch.Tensor
    rgbs: torch.Tensor
    A_mu: torch.Tensor
    A_rot: torch.Tensor
    A_alpha: torch.Tensor


def temporal_basis(decode_time: torch.Tensor, basis_count: int, max_frequency: float) -> torch.Tensor:
    """[K] times -> [K, M] basis (:806-825): sines of 2 pi t f for M // 2 frequencies
    f = 2^linspace(0, log2 max_frequency), then the cosines, then 2t - 1 when M is odd.  Same
    float32 operations as the reference, so the basis is the reference's to the bit on one
    device."""
    if basis_count < 1:
        raise ValueError(f"basis_count must be >= 1, got {basis_count}.")
    if max_frequency <= 0:
        raise ValueError(f"max_frequency must be positive, got {max_frequency}.")
    t = decode_time.reshape(-1, 1)
    n_freq = basis_count // 2
    columns = []
    if n_freq:
        exponents = torch.linspace(0.0, math.log2(float(max_frequency)), n_freq, device=t.device, dtype=t.dtype)
        freqs = torch.pow(torch.tensor(2.0, device=t.device, dtype=t.dtype), exponents)
        angles = (2.0 * math.pi) * t * freqs[None, :]
        columns += [torch.sin(angles), torch.cos(angles)]
    if basis_count % 2:
        columns.append(2.0 * t - 1.0)
    return torch.cat(columns, dim=-1)[:, :basis_count]


def _rows(t: torch.Tensor, width: int, name: str) -> torch.Tensor:
    if t.ndim == 3 and t.shape[0] == 1:
        t = t[0]
    if t.ndim != 2 or t.shape[-1] != width:
        raise ValueError(f"{name} must be [G, {width}] (or [1, G, {width}]), got {tuple(t.shape)}")
    return t


def _coefficients(t: torch.Tensor, channels: int, name: str) -> torch.Tensor:
    if t.ndim == 4 and t.shape[0] == 1:
        t = t[0]
    if channels == 1 and t.ndim == 2:
        t = t[..., None]
    if t.ndim != 3 or t.shape[-1] != channels:
        raise ValueError(f"{name} must be [G, M, {channels}], got {tuple(t.shape)}")
    return t


def render_dynamic_bank(
    bank: DynamicGaussianBank,
    decode_times: torch.Tensor,
    height: int,
    width: int,
    fx,
    fy,
    cx,
    cy,
    *,
    camera_to_world: torch.Tensor | None = None,
    static: tuple | None = None,
    max_frequency: float = 8.0,
    cameras=None,
    projection_mode: str = "legacy_pinhole",
    near_plane: float = MIN_RENDER_DEPTH,
    config: B200RendererConfig | None = None,
):
    """Renders frame k of a clip at decode time ``decode_times[k]`` with camera k: the static
    Gaussians ``static`` = (xyz, scales, quats, opacities, rgbs) (or None) followed by the bank
    evaluated at that time.  Intrinsics are scalars or [K] tensors, camera_to_world [K,4,4] (or
    one [4,4] for every frame).  The temporal basis has as many functions as the bank's
    coefficients (``dynamic_time_basis_count``) and ``max_frequency``
    (``dynamic_time_max_frequency``, the model's default 8).

    Returns (image [K,3,H,W], alpha [K,H,W], depth [K,H,W] or None with config.depth off), all
    differentiable: gradients reach every bank and static tensor and, when they require them,
    the cameras (not the decode times)."""
    config = config or B200RendererConfig()
    if decode_times.requires_grad:
        raise NotImplementedError("the b200 renderer does not differentiate the decode times; detach them.")
    times = decode_times.reshape(-1)
    K = int(times.numel())
    dev = bank.xyz0.device
    if not bank.xyz0.is_cuda:
        raise RuntimeError("the b200 renderer runs on CUDA devices only (got a tensor on %s)" % dev)
    xyz0 = _rows(bank.xyz0, 3, "xyz0")
    Gd = int(xyz0.shape[0])
    mu = _coefficients(bank.A_mu, 3, "A_mu")
    rot = _coefficients(bank.A_rot, 3, "A_rot")
    alpha = _coefficients(bank.A_alpha, 1, "A_alpha")
    M = int(mu.shape[1])
    if not (1 <= M <= _lib.BANK_MAX_BASIS):
        raise ValueError(f"the bank needs 1 to {_lib.BANK_MAX_BASIS} basis functions, got {M}")
    for name, t in (("A_rot", rot), ("A_alpha", alpha)):
        if t.shape[0] != Gd or t.shape[1] != M:
            raise ValueError(f"{name} must be [{Gd}, {M}, *], got {tuple(t.shape)}")
    parts = [(xyz0, _rows(bank.scales, 3, "scales"), _rows(bank.quats0, 4, "quats0"),
              bank.opacities0.reshape(-1), _rows(bank.rgbs, 3, "rgbs"))]
    Gs = 0
    if static is not None:
        s_xyz, s_scales, s_quats, s_opac, s_rgbs = static
        s_xyz = _rows(s_xyz, 3, "static xyz")
        Gs = int(s_xyz.shape[0])
        parts.insert(0, (s_xyz, _rows(s_scales, 3, "static scales"), _rows(s_quats, 4, "static quats"),
                         s_opac.reshape(-1), _rows(s_rgbs, 3, "static rgbs")))
    means, scales, quats, opacities, rgbs = (torch.cat(cols, 0) if len(parts) > 1 else cols[0]
                                             for cols in zip(*parts))
    G = Gs + Gd
    for name, t in (("scales", scales), ("quats", quats), ("opacities", opacities), ("rgbs", rgbs)):
        if t.shape[0] != G:
            raise ValueError(f"{name} has {t.shape[0]} Gaussians, the means {G}")
    intr = _intrinsics(fx, fy, cx, cy, K, dev)
    if camera_to_world is None:
        c2w = torch.eye(4, device=dev, dtype=torch.float32).expand(K, 4, 4).contiguous()
    else:
        c2w = camera_to_world.to(device=dev, dtype=torch.float32)
        c2w = (c2w.unsqueeze(0).expand(K, 4, 4) if c2w.ndim == 2 else c2w).contiguous()
    lens = _lens_of(projection_mode, cameras, K, dev)
    with_bank = Gd > 0
    sspec = SceneSpec(n_sets=1, n_gaussians=G, raw=False, sh_degree=0, velocity=False, sh_clamp=False,
                      bank_basis=M if with_bank else 0, bank_first=Gs)
    vspec = ViewSpec(n_views=K, views_per_set=K, height=int(height), width=int(width))
    basis = temporal_basis(times.to(device=dev, dtype=torch.float32), M, max_frequency).contiguous()
    image, alpha_out, depth = render_scene(
        sspec, vspec, config, near_plane, means=means[None], scales=scales[None], quats=quats[None],
        opacities=opacities[None], colors=rgbs[None], velocity=None, intrinsics=intr, camera_to_world=c2w,
        times=None, lens=lens, bank=(mu, rot, alpha[..., 0]) if with_bank else None,
        basis=basis if with_bank else None,
    )
    return image, alpha_out, (depth if config.depth else None)
