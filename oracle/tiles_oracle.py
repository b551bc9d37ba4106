"""Numpy restatement of tile binning: bounds, tile lists and sorted key order.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Two bound rules:

* ``tiled_compat`` restates compute_gaussian_bounds + build_tile_assignments
  of the reference (src/train/renderers/tiled.py:7-71) in float32: radius =
  min(bound_scale, sqrt(2 ln(o/thr))) * sqrt(cov_ii), pixel AABB floored /
  ceiled and clamped into the image, tile rectangle by floor division, pairs
  ordered by (tile, depth rank) -- the stable argsort of tiled.py:59 applied
  to Gaussians already in depth order (common.py:191).
* ``exact`` is this library's rule for dense-equivalent rendering: every
  tile whose pixel-centre rectangle holds a point with
  opacity * exp(-q/2) >= alpha_cutoff, i.e. min over the rectangle of
  q = d^T inv_cov d <= tau = 2 ln(opacity / alpha_cutoff).  Computed in
  float64 with the operation order of the CUDA preprocess so that both give
  the same lists bit for bit.

Keys: one 64-bit key per (view, tile, Gaussian) pair,
``(view * n_tiles + tile) << 32 | depth_rank``; the sorted order is the key
order.
"""
from __future__ import annotations

import math

import numpy as np

# Relative and absolute slack added to the exact-mode ellipse extents so that
# float32 rounding in the raster's own test never finds a pixel outside them.
EXACT_REL_MARGIN = 1e-5
EXACT_ABS_MARGIN = 1e-3


def log_f32(x: np.ndarray) -> np.ndarray:
    """float32 natural log, formed in float64 and rounded once."""
    return np.log(x.astype(np.float64)).astype(np.float32)


def tiled_compat_bounds(means2d, cov2d, opac, H, W, bound_scale=3.0, alpha_threshold=1.0 / 255.0):
    """compute_gaussian_bounds (tiled.py:7-28), float32, one view.

    means2d [G,2], cov2d [G,2,2] (or [G,3] = c00,c01,c11), opac [G].
    Returns int64 min_x, max_x, min_y, max_y and bool valid.
    """
    f32 = np.float32
    m = np.asarray(means2d, dtype=f32)
    cov = np.asarray(cov2d, dtype=f32)
    c00 = cov[:, 0, 0] if cov.ndim == 3 else cov[:, 0]
    c11 = cov[:, 1, 1] if cov.ndim == 3 else cov[:, 2]
    o = np.asarray(opac, dtype=f32).reshape(-1)
    sx = np.sqrt(np.maximum(c00, f32(1e-6)))
    sy = np.sqrt(np.maximum(c11, f32(1e-6)))
    if alpha_threshold > 0.0:
        thr = f32(alpha_threshold)
        ratio = np.maximum(o, thr) / thr
        of = np.sqrt(np.maximum(f32(2.0) * log_f32(ratio), f32(0.0)))
        rf = np.minimum(f32(bound_scale), of)
    else:
        rf = np.full_like(sx, f32(bound_scale))
    rx = rf * sx
    ry = rf * sy
    min_x = np.clip(np.floor(m[:, 0] - rx), 0, W - 1).astype(np.int64)
    max_x = np.clip(np.ceil(m[:, 0] + rx), 0, W - 1).astype(np.int64)
    min_y = np.clip(np.floor(m[:, 1] - ry), 0, H - 1).astype(np.int64)
    max_y = np.clip(np.ceil(m[:, 1] + ry), 0, H - 1).astype(np.int64)
    valid = (max_x >= min_x) & (max_y >= min_y) & (rf > 0)
    return min_x, max_x, min_y, max_y, valid


def tile_rects_from_pixel_bounds(min_x, max_x, min_y, max_y, valid, tile_size):
    """Tile rectangle [tx0, tx1] x [ty0, ty1] (inclusive) per Gaussian, tiled.py:31-41."""
    tx0, tx1 = min_x // tile_size, max_x // tile_size
    ty0, ty1 = min_y // tile_size, max_y // tile_size
    count = np.where(valid, (tx1 - tx0 + 1) * (ty1 - ty0 + 1), 0)
    return tx0, tx1, ty0, ty1, count


def _exact_min_q(a, b, c, mx, my, X0, X1, Y0, Y1):
    """Minimum of q = a dx^2 + b dx dy + c dy^2 over the box [X0,X1] x [Y0,Y1] (float64).

    dx = x - mx, dy = y - my.  Zero if the mean lies in the box, else the
    least of the four edge minima (1-D quadratic minimiser clamped to the
    edge).  Same operation order as the CUDA kernel.
    """
    inside = (X0 <= mx) & (mx <= X1) & (Y0 <= my) & (my <= Y1)

    def edge_x(xe, lo, hi):  # x fixed, minimise over dy in [lo-my, hi-my]
        dx = xe - mx
        t = -(b * dx) / (2.0 * c)
        dy = np.minimum(np.maximum(t, lo - my), hi - my)
        return (a * dx) * dx + ((b * dx) * dy + (c * dy) * dy)

    def edge_y(ye, lo, hi):  # y fixed, minimise over dx
        dy = ye - my
        t = -(b * dy) / (2.0 * a)
        dx = np.minimum(np.maximum(t, lo - mx), hi - mx)
        return (a * dx) * dx + ((b * dx) * dy + (c * dy) * dy)

    q = np.minimum(
        np.minimum(edge_x(X0, Y0, Y1), edge_x(X1, Y0, Y1)),
        np.minimum(edge_y(Y0, X0, X1), edge_y(Y1, X0, X1)),
    )
    return np.where(inside, 0.0, q)


def exact_pairs_one_view(mx, my, a, b, c, o, H, W, tile_size, alpha_cutoff, pixel_center=0.0, ellipse_test=True):
    """Exact-mode tile lists for one view; inputs are float32 per-Gaussian records in rank order.

    a = inv_cov00, b = inv_cov01 + inv_cov10, c = inv_cov11.
    Returns (tile_ids, ranks) of every pair, ordered by (rank, tile).
    """
    mx, my, a, b, c, o = (np.asarray(v, dtype=np.float32).astype(np.float64) for v in (mx, my, a, b, c, o))
    G = mx.shape[0]
    tiles_x = (W + tile_size - 1) // tile_size
    with np.errstate(divide="ignore", invalid="ignore"):
        vis = o > alpha_cutoff
        tau = np.where(vis, 2.0 * np.log(np.where(vis, o, 1.0) / alpha_cutoff), 0.0)
        det = a * c - (0.25 * b) * b
        ok = vis & (det > 0) & (a > 0) & (c > 0)
        # extents of {d : q(d) <= tau}: sqrt(tau * (A^-1)_ii), (A^-1)_00 = c/det.
        ex = np.sqrt(np.where(ok, tau * (c / det), 0.0)) * (1.0 + EXACT_REL_MARGIN) + EXACT_ABS_MARGIN
        ey = np.sqrt(np.where(ok, tau * (a / det), 0.0)) * (1.0 + EXACT_REL_MARGIN) + EXACT_ABS_MARGIN
    px0 = np.maximum(np.ceil(mx - ex - pixel_center), 0.0)
    px1 = np.minimum(np.floor(mx + ex - pixel_center), W - 1.0)
    py0 = np.maximum(np.ceil(my - ey - pixel_center), 0.0)
    py1 = np.minimum(np.floor(my + ey - pixel_center), H - 1.0)
    ok = ok & (px0 <= px1) & (py0 <= py1) & np.isfinite(mx) & np.isfinite(my)
    tiles, ranks = [], []
    for g in np.nonzero(ok)[0]:
        tx0, tx1 = int(px0[g]) // tile_size, int(px1[g]) // tile_size
        ty0, ty1 = int(py0[g]) // tile_size, int(py1[g]) // tile_size
        for ty in range(ty0, ty1 + 1):
            for tx in range(tx0, tx1 + 1):
                if ellipse_test:
                    X0 = max(tx * tile_size, 0) + pixel_center
                    X1 = min(tx * tile_size + tile_size - 1, W - 1) + pixel_center
                    Y0 = max(ty * tile_size, 0) + pixel_center
                    Y1 = min(ty * tile_size + tile_size - 1, H - 1) + pixel_center
                    q = _exact_min_q(a[g], b[g], c[g], mx[g], my[g], X0, X1, Y0, Y1)
                    if not (q <= tau[g] * (1.0 + EXACT_REL_MARGIN) + EXACT_ABS_MARGIN):
                        continue
                tiles.append(ty * tiles_x + tx)
                ranks.append(g)
    return np.asarray(tiles, dtype=np.int64), np.asarray(ranks, dtype=np.int64)


def compat_pairs_one_view(means2d, cov2d, opac, H, W, tile_size, bound_scale=3.0, alpha_threshold=1.0 / 255.0):
    """tiled_compat pairs for one view (inputs in rank order): (tile_ids, ranks) ordered by (rank, tile)."""
    bounds = tiled_compat_bounds(means2d, cov2d, opac, H, W, bound_scale, alpha_threshold)
    tx0, tx1, ty0, ty1, count = tile_rects_from_pixel_bounds(*bounds, tile_size)
    tiles_x = (W + tile_size - 1) // tile_size
    tiles, ranks = [], []
    for g in np.nonzero(count > 0)[0]:
        # tiled.py:37-45 enumerates local_ids row-major: x fastest.
        for ty in range(int(ty0[g]), int(ty1[g]) + 1):
            for tx in range(int(tx0[g]), int(tx1[g]) + 1):
                tiles.append(ty * tiles_x + tx)
                ranks.append(g)
    return np.asarray(tiles, dtype=np.int64), np.asarray(ranks, dtype=np.int64)


def sort_pairs(view_tiles_ranks, n_tiles):
    """Sorted 64-bit keys for all views: key = (view*n_tiles + tile) << 32 | rank."""
    keys = []
    for v, (tiles, ranks) in enumerate(view_tiles_ranks):
        keys.append(((v * n_tiles + tiles.astype(np.uint64)) << np.uint64(32)) | ranks.astype(np.uint64))
    if not keys:
        return np.zeros(0, dtype=np.uint64)
    k = np.concatenate(keys).astype(np.uint64)
    return np.sort(k, kind="stable")


def tile_ranges(sorted_keys, n_views, n_tiles):
    """[n_views*n_tiles, 2] start/end of each tile's run in the sorted keys."""
    tk = (sorted_keys >> np.uint64(32)).astype(np.int64)
    idx = np.arange(n_views * n_tiles)
    start = np.searchsorted(tk, idx, side="left")
    end = np.searchsorted(tk, idx, side="right")
    return np.stack([start, end], axis=1).astype(np.int64)


def reference_packed_lists(unique_tile_ids, packed_ids, valid):
    """Flatten tiled.py's packed per-tile lists into (tile, gaussian) pairs in list order."""
    u = np.asarray(unique_tile_ids)
    p = np.asarray(packed_ids)
    v = np.asarray(valid).astype(bool)
    tiles = np.repeat(u, v.sum(axis=1))
    return tiles.astype(np.int64), p[v].astype(np.int64)


def n_tiles_for(H, W, tile_size):
    return ((H + tile_size - 1) // tile_size) * ((W + tile_size - 1) // tile_size)


LOG2_F0 = math.log2(1.0 + 2.0 ** -20)
