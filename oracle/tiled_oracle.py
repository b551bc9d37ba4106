"""Torch restatement of the reference's tiled renderer, differentiable (forward and backward).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Restates
render_pytorch_3dgs_tiled (src/train/renderers/tiled.py:74-198) for the pinhole projection:

  * projection and depth order: project_gaussians_2d (common.py:54-131), here
    splat_oracle.project_batch on one view (same arithmetic, same stable z order);
  * bounds: compute_gaussian_bounds (tiled.py:7-28): radius = min(bound_scale,
    sqrt(2 ln(o / thr))) * sqrt(cov_ii), floor / ceil, clamped into the image;
  * lists: build_tile_assignments (tiled.py:31-71): per tile, the Gaussians whose tile
    rectangle holds it, in depth order (stable argsort by tile id of depth-ordered pairs);
  * blend per tile (tiled.py:162-198): no power clamp, alpha = clamp(o exp(power), 0, 0.99),
    tile-local T = prod (1 - alpha + 1e-6) over the tile's list only, white background where no
    tile is listed, the whole image clamped to [0, 1].

The tests compare the CUDA path's tiled_compat mode with it; bench.py times it as the CPU baseline
of the reference's faster CPU renderer.
"""
from __future__ import annotations

import torch

from .splat_oracle import MIN_RENDER_DEPTH, flip_clamp, project_batch


def gaussian_bounds(means2d, cov2d, opacities, H, W, bound_scale=3.0, alpha_threshold=1.0 / 255.0):
    """compute_gaussian_bounds (tiled.py:7-28) on one view: pixel AABB and validity."""
    sigma_x = torch.sqrt(torch.clamp(cov2d[:, 0, 0], min=1e-6))
    sigma_y = torch.sqrt(torch.clamp(cov2d[:, 1, 1], min=1e-6))
    if alpha_threshold > 0.0:
        o = torch.clamp(opacities.reshape(-1), min=alpha_threshold)
        factor = torch.sqrt(torch.clamp(2.0 * torch.log(o / alpha_threshold), min=0.0))
        factor = torch.minimum(torch.full_like(factor, bound_scale), factor)
    else:
        factor = torch.full_like(sigma_x, bound_scale)
    rx, ry = factor * sigma_x, factor * sigma_y
    x0 = torch.floor(means2d[:, 0] - rx).clamp(0, W - 1).to(torch.int64)
    x1 = torch.ceil(means2d[:, 0] + rx).clamp(0, W - 1).to(torch.int64)
    y0 = torch.floor(means2d[:, 1] - ry).clamp(0, H - 1).to(torch.int64)
    y1 = torch.ceil(means2d[:, 1] + ry).clamp(0, H - 1).to(torch.int64)
    valid = (x1 >= x0) & (y1 >= y0) & (factor > 0)
    return x0, x1, y0, y1, valid


def tile_lists(x0, x1, y0, y1, valid, tile: int, tiles_x: int, only=None) -> dict[int, torch.Tensor]:
    """build_tile_assignments (tiled.py:31-71) as a dict tile id -> depth-ordered Gaussian ids
    (the stable argsort by tile of pairs emitted in Gaussian = depth order).  ``only``: compute
    the lists of these tile ids alone (the same lists, without expanding every pair)."""
    tx0, tx1 = torch.div(x0, tile, rounding_mode="floor"), torch.div(x1, tile, rounding_mode="floor")
    ty0, ty1 = torch.div(y0, tile, rounding_mode="floor"), torch.div(y1, tile, rounding_mode="floor")
    if only is not None:
        out = {}
        for tid in only:
            tx, ty = tid % tiles_x, tid // tiles_x
            hit = valid & (tx0 <= tx) & (tx <= tx1) & (ty0 <= ty) & (ty <= ty1)
            ids = torch.nonzero(hit).flatten()
            if ids.numel():
                out[int(tid)] = ids
        return out
    w = tx1 - tx0 + 1
    counts = torch.where(valid, w * (ty1 - ty0 + 1), torch.zeros_like(w))
    total = int(counts.sum())
    if total == 0:
        return {}
    gid = torch.repeat_interleave(torch.arange(counts.numel()), counts)
    first = torch.cumsum(counts, 0) - counts
    local = torch.arange(total) - first[gid]
    tiles = (ty0[gid] + torch.div(local, w[gid], rounding_mode="floor")) * tiles_x + tx0[gid] + local % w[gid]
    order = torch.argsort(tiles, stable=True)
    tiles, gid = tiles[order], gid[order]
    ids, n = torch.unique_consecutive(tiles, return_counts=True)
    return {int(t): g for t, g in zip(ids.tolist(), torch.split(gid, n.tolist()))}


def project_view(means, scales, quats, opacities, rgbs, fx, fy, cx, cy, camera_to_world, near_plane=MIN_RENDER_DEPTH):
    """project_gaussians_2d (common.py:54-131) on one view: means2d, inv_cov, cov2d, opacity, rgb
    in depth order."""
    m2, inv, cov, op, rgb, _z, _order = project_batch(
        means[None], scales[None], quats[None], opacities[None], rgbs[None],
        torch.as_tensor(fx).reshape(1), torch.as_tensor(fy).reshape(1), torch.as_tensor(cx).reshape(1),
        torch.as_tensor(cy).reshape(1), camera_to_world[None], near_plane=near_plane)
    return m2[0], inv[0], cov[0], op[0], rgb[0]


def blend_tile(m2, inv, op, rgb, ids, ox: int, oy: int, tile_size: int, eps=1e-6, alpha_clamp=0.99, flip=None,
               with_wsum=False):
    """tiled.py:178-194 for one tile: [tile, tile, 3] before the image clamp.  ``flip`` [tile, tile]
    (bool, optional): pixels where the clamp of the weight sum takes the other side of its kink.
    ``with_wsum``: return (colour, weight sum)."""
    dtype = m2.dtype
    ly, lx = torch.meshgrid(torch.arange(tile_size, dtype=dtype), torch.arange(tile_size, dtype=dtype),
                            indexing="ij")
    dx = (lx + ox).view(1, tile_size, tile_size) - m2[ids, 0].view(-1, 1, 1)
    dy = (ly + oy).view(1, tile_size, tile_size) - m2[ids, 1].view(-1, 1, 1)
    # einsum("tmhwi,tmij,tmhwj") of tiled.py:185, no clamp of the power
    power = -0.5 * (dx * (inv[ids, 0, 0].view(-1, 1, 1) * dx + inv[ids, 0, 1].view(-1, 1, 1) * dy)
                    + dy * (inv[ids, 1, 0].view(-1, 1, 1) * dx + inv[ids, 1, 1].view(-1, 1, 1) * dy))
    alpha = torch.clamp(op[ids].view(-1, 1, 1) * torch.exp(power), 0.0, alpha_clamp)
    T = torch.cat([alpha.new_ones((1, tile_size, tile_size)), torch.cumprod(1.0 - alpha[:-1] + eps, dim=0)], 0)
    w = T * alpha
    col = (w.unsqueeze(-1) * rgb[ids][:, None, None, :]).sum(0)
    ws = w.sum(0)
    ws_c = ws.clamp(0, 1)
    if flip is not None:
        ws_c = torch.where(flip, flip_clamp(ws, ws_c), ws_c)
    if with_wsum:
        return col + (1.0 - ws_c.unsqueeze(-1)), ws
    return col + (1.0 - ws_c.unsqueeze(-1))


def render_tiled_view(means, scales, quats, opacities, rgbs, H, W, fx, fy, cx, cy, camera_to_world, *,
                      tile_size=8, bound_scale=3.0, alpha_threshold=1.0 / 255.0, near_plane=MIN_RENDER_DEPTH,
                      eps=1e-6, alpha_clamp=0.99, flip_wsum=None, flip_image=None, return_pre=False):
    """One view ([G,*] activated tensors, scalar intrinsics, [4,4] camera) -> image [3,H,W].
    ``flip_wsum`` [H,W] / ``flip_image`` [3,H,W] (bool, optional): pixels whose weight-sum / image
    clamp takes the other side of its kink (splat_oracle.flip_clamp).  ``return_pre``: return
    (image, weight sum [H,W], image before its clamp [3,H,W])."""
    m2, inv, cov, op, rgb = project_view(means, scales, quats, opacities, rgbs, fx, fy, cx, cy, camera_to_world,
                                         near_plane)
    bounds = gaussian_bounds(m2.detach(), cov.detach(), op.detach(), H, W, bound_scale, alpha_threshold)
    tiles_x = (W + tile_size - 1) // tile_size
    lists = tile_lists(*bounds, tile_size, tiles_x)
    Hp = -(-H // tile_size) * tile_size
    Wp = -(-W // tile_size) * tile_size
    fw = None
    if flip_wsum is not None:
        fw = torch.zeros(Hp, Wp, dtype=torch.bool)
        fw[:H, :W] = flip_wsum

    def flip_of(tid):
        if fw is None:
            return None
        ox, oy = (tid % tiles_x) * tile_size, (tid // tiles_x) * tile_size
        return fw[oy:oy + tile_size, ox:ox + tile_size]

    parts = {tid: blend_tile(m2, inv, op, rgb, ids, (tid % tiles_x) * tile_size, (tid // tiles_x) * tile_size,
                             tile_size, eps, alpha_clamp, flip_of(tid), with_wsum=True) for tid, ids in lists.items()}
    blank = torch.ones(tile_size, tile_size, 3, dtype=m2.dtype)  # tiled.py:190, unlisted tiles
    zero = torch.zeros(tile_size, tile_size, dtype=m2.dtype)
    rows = [torch.cat([parts[ty * tiles_x + tx][0] if ty * tiles_x + tx in parts else blank
                       for tx in range(Wp // tile_size)], 1) for ty in range(Hp // tile_size)]
    img = torch.cat(rows, 0)[:H, :W]
    wrows = [torch.cat([parts[ty * tiles_x + tx][1] if ty * tiles_x + tx in parts else zero
                        for tx in range(Wp // tile_size)], 1) for ty in range(Hp // tile_size)]
    wsum = torch.cat(wrows, 0)[:H, :W]
    img_c = img.clamp(0.0, 1.0)
    if flip_image is not None:
        img_c = torch.where(flip_image.permute(1, 2, 0), flip_clamp(img, img_c), img_c)
    if return_pre:
        return img_c.permute(2, 0, 1), wsum, img.permute(2, 0, 1)
    return img_c.permute(2, 0, 1)
