"""Torch restatement of the tile-culled, depth-rank-corrected blend.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The reference blends every Gaussian at every pixel (dense.py:208-233):
T_i = prod_{j<i} (1 - alpha_j + eps) over all G Gaussians of the view in
depth order.  A Gaussian that does not touch the pixel still multiplies T by
F0 = fl32(1 + eps) (= 1 + 2^-20 for eps = 1e-6).  The CUDA raster visits only
the Gaussians listed for the pixel's tile, so it restores those factors from
the depth ranks:

    T before list entry 0      = F0 ** rank_0
    T after  list entry i      = T_i * f_i * F0 ** (rank_{i+1} - rank_i - 1)
    f_i = fl32(fl32(1 - alpha_i) + eps)   (F0 when the entry is skipped)

A pair is skipped (alpha treated as 0) when alpha < alpha_cutoff; for
alpha < 2^-25, fl32(1 - alpha) == 1, so such a skip changes nothing at all.
A pixel stops after the first entry that leaves T below the transmittance
threshold.  ``eps_mode='tile_local'`` drops the rank factors and applies eps
only over the list, which is what tiled.py:176-185 does.

This module evaluates that recurrence per tile with a cumulative product, in
float64, differentiably (skip and stop decisions are constants, as in the
CUDA backward).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .splat_oracle import transmittance_factors


def f0_of(eps: float) -> float:
    return float(np.float32(np.float32(1.0) + np.float32(eps)))


def blend_culled_view(
    means2d, inv3, opac, rgb, depth, ranks_per_tile, H, W, tile_size,
    *, alpha_cutoff, transmittance_threshold, eps=1e-6, eps_mode="dense_rank",
    alpha_clamp=0.99, pixel_center=0.0, background=(1.0, 1.0, 1.0),
):
    """One view.  Per-Gaussian inputs are in depth-rank order; ``ranks_per_tile``
    maps tile id -> int64 array of ranks (ascending) listed for that tile.

    inv3 [G,3] = (inv00, inv01 + inv10, inv11).  Returns image [3,H,W],
    alpha [H,W], depth [H,W] or None, n_processed [H,W], T_end [H,W].
    """
    dtype = means2d.dtype
    tiles_x = (W + tile_size - 1) // tile_size
    F0 = f0_of(eps) if eps_mode != "none" else 1.0
    eps_eff = eps if eps_mode != "none" else 0.0
    log_f0 = math.log(F0)
    bg = torch.as_tensor(background, dtype=dtype)
    img = bg.view(3, 1, 1).expand(3, H, W).clone()
    alpha_out = torch.zeros(H, W, dtype=dtype)
    depth_out = torch.zeros(H, W, dtype=dtype) if depth is not None else None
    n_proc = torch.zeros(H, W, dtype=torch.int64)
    t_end = torch.ones(H, W, dtype=dtype)
    img_rows, alpha_rows, depth_rows = {}, {}, {}
    for tile, ranks in ranks_per_tile.items():
        ty, tx = divmod(int(tile), tiles_x)
        ys = torch.arange(ty * tile_size, min(ty * tile_size + tile_size, H))
        xs = torch.arange(tx * tile_size, min(tx * tile_size + tile_size, W))
        gy, gx = torch.meshgrid(ys.to(dtype) + pixel_center, xs.to(dtype) + pixel_center, indexing="ij")
        px, py = gx.reshape(1, -1), gy.reshape(1, -1)
        r = torch.as_tensor(ranks, dtype=torch.int64)
        L = r.numel()
        if L == 0:
            continue
        m = means2d[r]
        dx = px - m[:, 0:1]
        dy = py - m[:, 1:2]
        a, b, c = inv3[r, 0:1], inv3[r, 1:2], inv3[r, 2:3]
        power = torch.minimum(-0.5 * (a * dx * dx + b * dx * dy + c * dy * dy), torch.zeros((), dtype=dtype))
        alpha = torch.clamp(opac[r].view(-1, 1) * torch.exp(power), 0.0, alpha_clamp)
        skip = (alpha < alpha_cutoff).detach()
        alpha = torch.where(skip, torch.zeros_like(alpha), alpha)
        f = torch.where(skip, torch.full_like(alpha, F0), transmittance_factors(alpha, eps_eff))
        if eps_mode == "dense_rank":
            gaps = torch.zeros(L, dtype=dtype)
            gaps[:-1] = (r[1:] - r[:-1] - 1).to(dtype)
            E = torch.exp(gaps * log_f0).view(-1, 1)
            t0 = math.exp(float(r[0]) * log_f0)
        else:
            E = torch.ones(L, 1, dtype=dtype)
            t0 = 1.0
        fac = f * E
        T_after = t0 * torch.cumprod(fac, dim=0)
        T_before = torch.cat([torch.full((1, fac.shape[1]), t0, dtype=dtype), T_after[:-1]], dim=0)
        below = (T_after < transmittance_threshold).detach()
        hit = torch.cumsum(below.to(torch.int64), dim=0)
        # entry i is processed iff no earlier entry left T below the threshold
        processed = torch.cat([torch.ones(1, fac.shape[1], dtype=torch.bool), hit[:-1] == 0], dim=0)
        w = torch.where(processed, T_before * alpha, torch.zeros_like(alpha))
        col = w.t() @ rgb[r]  # [P,3]
        wsum = w.sum(0)
        out = col + (1.0 - wsum.clamp(0, 1)).unsqueeze(-1) * bg
        out = out.clamp(0.0, 1.0)
        nproc = processed.sum(0)
        last = (nproc - 1).clamp(min=0)
        tend = T_after.gather(0, last.view(1, -1)).view(-1)
        shape = (ys.numel(), xs.numel())
        y0, x0 = ty * tile_size, tx * tile_size
        img_rows[(y0, x0)] = (out.t().reshape(3, *shape), shape)
        alpha_rows[(y0, x0)] = wsum.reshape(shape)
        if depth is not None:
            depth_rows[(y0, x0)] = (w.t() @ depth[r].view(-1, 1)).reshape(shape)
        n_proc[y0:y0 + shape[0], x0:x0 + shape[1]] = nproc.reshape(shape)
        t_end[y0:y0 + shape[0], x0:x0 + shape[1]] = tend.detach().reshape(shape)
    # assemble differentiably
    if img_rows:
        img = _scatter_tiles(img, img_rows, channels=True)
        alpha_out = _scatter_tiles(alpha_out, alpha_rows, channels=False)
        if depth is not None:
            depth_out = _scatter_tiles(depth_out, depth_rows, channels=False)
    return img, alpha_out, depth_out, n_proc, t_end


def _scatter_tiles(base, pieces, channels):
    out = base.clone()
    for (y0, x0), val in pieces.items():
        if channels:
            v, shape = val
            out[:, y0:y0 + shape[0], x0:x0 + shape[1]] = v
        else:
            out[y0:y0 + val.shape[0], x0:x0 + val.shape[1]] = val
    return out


def ranks_by_tile(tiles: np.ndarray, ranks: np.ndarray) -> dict:
    """Group (tile, rank) pairs into tile -> ascending ranks."""
    order = np.lexsort((ranks, tiles))
    t, r = tiles[order], ranks[order]
    out = {}
    if t.size == 0:
        return out
    cuts = np.nonzero(np.diff(t))[0] + 1
    for seg_t, seg_r in zip(np.split(t, cuts), np.split(r, cuts)):
        out[int(seg_t[0])] = seg_r
    return out
