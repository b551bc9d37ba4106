"""Torch restatement of the reference's dynamic Gaussian bank evaluation.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the tests compare the bank path of the CUDA
preprocess with it; never imported by the product.  Differentiable through torch autograd, usable in
float32 or float64.  Citations are to src/train/gs_models/dynamic_video_token_gs_implicit_camera.py
of nbardy/dynaworld:

  * temporal basis        :806-825  (_temporal_basis)
  * axis-angle quaternion :828-838  (_axis_angle_to_quat)
  * quaternion product    :841-852  (_quat_multiply)
  * bank evaluation       :1206-1224 (_eval_dynamic_bank)
  * static + dynamic      :1256-1275 (_decode_static_dynamic_split: static Gaussians first)

The frames it returns feed splat_oracle.render_dense (dense.py restated) like any per-frame
Gaussian sequence.
"""
from __future__ import annotations

import math

import torch


def temporal_basis(t: torch.Tensor, basis_count: int, max_frequency: float) -> torch.Tensor:
    """[K] -> [K, M]: sin(2 pi t f_j), j < M // 2, then cos(2 pi t f_j), then 2t - 1 for odd M,
    with f_j = 2^(j log2(max_frequency) / (M // 2 - 1)) (f_0 = 1)."""
    t = t.reshape(-1, 1)
    n = basis_count // 2
    cols = []
    if n:
        if n == 1:
            expo = torch.zeros(1, dtype=t.dtype)
        else:
            expo = torch.arange(n, dtype=t.dtype) * (math.log2(max_frequency) / (n - 1))
        ang = 2.0 * math.pi * t * torch.pow(torch.tensor(2.0, dtype=t.dtype), expo)[None]
        cols += [torch.sin(ang), torch.cos(ang)]
    if basis_count % 2:
        cols.append(2.0 * t - 1.0)
    return torch.cat(cols, -1)[:, :basis_count]


def axis_angle_to_quat(r: torch.Tensor) -> torch.Tensor:
    """(cos(a/2), r sin(a/2)/a) normalised, a = |r|; below a = 1e-6 the factor is the series
    0.5 - a^2/48."""
    a = torch.sqrt((r * r).sum(-1, keepdim=True))
    small = a < 1e-6
    factor = torch.where(small, 0.5 - a * a / 48.0, torch.sin(0.5 * a) / torch.clamp(a, min=1e-12))
    q = torch.cat([torch.cos(0.5 * a), r * factor], -1)
    return q / torch.clamp(torch.sqrt((q * q).sum(-1, keepdim=True)), min=1e-12)


def quat_multiply(l: torch.Tensor, r: torch.Tensor) -> torch.Tensor:
    """Hamilton product, components (w, x, y, z)."""
    lw, lx, ly, lz = l.unbind(-1)
    rw, rx, ry, rz = r.unbind(-1)
    return torch.stack([
        lw * rw - lx * rx - ly * ry - lz * rz,
        lw * rx + lx * rw + ly * rz - lz * ry,
        lw * ry - lx * rz + ly * rw + lz * rx,
        lw * rz + lx * ry - ly * rx + lz * rw,
    ], -1)


def eval_bank(xyz0, scales, quats0, opacities0, rgbs, A_mu, A_rot, A_alpha, phi):
    """One decode time: bank [G, *] (A_* [G, M, C]) and basis phi [M] -> (xyz, scales, quats,
    opacities [G, 1], rgbs) at that time."""
    d_xyz = (phi[None, :, None] * A_mu).sum(1)
    d_rot = (phi[None, :, None] * A_rot).sum(1)
    d_alpha = (phi[None, :, None] * A_alpha.reshape(A_alpha.shape[0], -1, 1)).sum(1)
    c = torch.clamp(opacities0.reshape(-1, 1), 1e-6, 1.0 - 1e-6)
    q = quat_multiply(quats0, axis_angle_to_quat(d_rot))
    q = q / torch.clamp(torch.sqrt((q * q).sum(-1, keepdim=True)), min=1e-12)
    return xyz0 + d_xyz, scales, q, torch.sigmoid(torch.log(c / (1.0 - c)) + d_alpha), rgbs


def frames(bank: dict, times: torch.Tensor, max_frequency: float, static: dict | None = None):
    """Per-frame Gaussians [K, Gs + Gd, *] (static first) for decode times [K]; ``bank`` and
    ``static`` map the reference's field names (xyz0/xyz, scales, quats0/quats,
    opacities0/opacities, rgbs, A_mu, A_rot, A_alpha) to tensors."""
    M = bank["A_mu"].shape[1]
    phi = temporal_basis(times, M, max_frequency)
    out = [[] for _ in range(5)]
    for k in range(phi.shape[0]):
        dyn = eval_bank(bank["xyz0"], bank["scales"], bank["quats0"], bank["opacities0"], bank["rgbs"],
                        bank["A_mu"], bank["A_rot"], bank["A_alpha"], phi[k])
        if static is not None:
            st = (static["xyz"], static["scales"], static["quats"], static["opacities"].reshape(-1, 1),
                  static["rgbs"])
            dyn = tuple(torch.cat([a, b], 0) for a, b in zip(st, dyn))
        for i, v in enumerate(dyn):
            out[i].append(v)
    return tuple(torch.stack(v, 0) for v in out)
