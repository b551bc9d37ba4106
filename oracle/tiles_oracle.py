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
  tile holding a pixel centre with opacity * exp(-q/2) >= alpha_cutoff, i.e.
  q = d^T inv_cov d <= tau = 2 ln(opacity / alpha_cutoff) (plus slack),
  found row by row from the ellipse's x-interval over each tile row.
  Computed in float64 with the operation order of the CUDA preprocess so
  that both give the same lists bit for bit.

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


def _ellipse_x(a, b, det, L, u, right):
    """x offset of the ellipse boundary at row offset u: (-(b u) -/+ sqrt(4 a L - 4 det u^2)) (1 / (2 a))."""
    disc = max((4.0 * a) * L - (4.0 * det) * (u * u), 0.0)
    r = math.sqrt(disc)
    nb = -(b * u)
    return ((nb + r) if right else (nb - r)) * (1.0 / (2.0 * a))


def exact_pairs_one_view(mx, my, a, b, c, o, H, W, tile_size, alpha_cutoff, pixel_center=0.0, ellipse_test=True):
    """Exact-mode tile lists for one view; inputs are float32 per-Gaussian records in rank order.

    a = inv_cov00, b = inv_cov01 + inv_cov10, c = inv_cov11.  A tile is listed when it holds a
    pixel centre with q <= L, L = tau (1 + rel) + abs, tau = 2 ln(o / cutoff): per tile row, the
    ellipse restricted to the row band projects onto an x-interval; the row's tiles are those
    holding a pixel-column centre in it (``ellipse_test=False`` keeps the whole bounding box).
    Float64, one rounding per operation, in the order of the CUDA preprocess (tiles.cuh).
    Returns (tile_ids, ranks) of every pair, ordered by (rank, tile).
    """
    f64 = lambda v: np.asarray(v, dtype=np.float32).astype(np.float64)  # noqa: E731
    mx, my, a, b, c, o = (f64(v) for v in (mx, my, a, b, c, o))
    cut = float(np.float32(alpha_cutoff))
    tiles_x = (W + tile_size - 1) // tile_size
    pc = float(pixel_center)
    tiles, ranks = [], []
    for g in range(mx.shape[0]):
        if not (o[g] > cut):
            continue
        A, Bq, Cq, MX, MY = float(a[g]), float(b[g]), float(c[g]), float(mx[g]), float(my[g])
        tau = 2.0 * math.log(float(o[g]) / cut)
        det = A * Cq - (0.25 * Bq) * Bq
        if not (det > 0.0 and A > 0.0 and Cq > 0.0):
            continue
        L = tau * (1.0 + EXACT_REL_MARGIN) + EXACT_ABS_MARGIN
        ex = math.sqrt(L * (Cq / det))
        ey = math.sqrt(L * (A / det))
        px0 = max(math.ceil((MX - ex) - pc), 0.0)
        px1 = min(math.floor((MX + ex) - pc), W - 1.0)
        py0 = max(math.ceil((MY - ey) - pc), 0.0)
        py1 = min(math.floor((MY + ey) - pc), H - 1.0)
        if not (px0 <= px1 and py0 <= py1 and math.isfinite(MX) and math.isfinite(MY)):
            continue
        px0, px1, py0, py1 = int(px0), int(px1), int(py0), int(py1)
        for ty in range(py0 // tile_size, py1 // tile_size + 1):
            if ellipse_test:
                Y0 = float(max(ty * tile_size, py0)) + pc
                Y1 = float(min(ty * tile_size + tile_size - 1, py1)) + pc
                u0 = max(Y0 - MY, -ey)
                u1 = min(Y1 - MY, ey)
                if not (u0 <= u1):
                    continue
                ul = (Bq * ex) / (2.0 * Cq)
                ur = -ul
                xl = -ex if (u0 <= ul <= u1) else min(_ellipse_x(A, Bq, det, L, u0, False),
                                                      _ellipse_x(A, Bq, det, L, u1, False))
                xr = ex if (u0 <= ur <= u1) else max(_ellipse_x(A, Bq, det, L, u0, True),
                                                     _ellipse_x(A, Bq, det, L, u1, True))
                qx0 = max(math.ceil((MX + xl) - pc), float(px0))
                qx1 = min(math.floor((MX + xr) - pc), float(px1))
                if not (qx0 <= qx1):
                    continue
                tx0, tx1 = int(qx0) // tile_size, int(qx1) // tile_size
            else:
                tx0, tx1 = px0 // tile_size, px1 // tile_size
            for tx in range(tx0, tx1 + 1):
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
