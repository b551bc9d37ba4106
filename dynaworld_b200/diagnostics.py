"""Per-call render statistics and NVTX ranges.

The reference logs, per rendered frame, how the splats overlap the tile grid:
summarize_overlap_counts (src/train/renderers/overlap_metrics.py:36-74) over the per-splat tile
counts and the per-tile splat counts, averaged and maximised over the frames by
aggregate_stat_dicts (:415-426), reduced to selected_overlap_summary's keys (:429-439) and logged
under "TileDiag/..." by tile_overlap_diagnostics (src/train/debug_metrics.py:233-273).  That code
recomputes the overlaps from the projected Gaussians.  Here the statistics come from the lists the
renderer actually built in the call -- per Gaussian the number of tiles it was listed in (the
preprocess's pair offsets), per tile the length of its list (the tile ranges) -- so they describe
the work the raster kernels did, and nothing is recomputed.

    from dynaworld_b200 import diagnostics
    with diagnostics.collect() as frames:
        image, alpha, depth = renderer(...)
    stats = diagnostics.overlap_summary(frames)      # {"TileDiag/B200_total_overlap_keys_mean": ...}

Collecting keeps references to two device tensors per render call (no copies, no kernels); the
summary runs torch reductions on them and reads back one scalar per statistic.

NVTX: with ``nvtx(True)`` (or GSB200_NVTX=1 in the environment) every C-ABI stage of the render
(depth_order, preprocess_fwd, bin, raster_fwd, loss, raster_bwd, preprocess_bwd, ...) is a named
NVTX range "gsb:<stage>" on the host timeline, for Nsight Systems.
"""
from __future__ import annotations

import contextlib
import math
import os
from dataclasses import dataclass

import torch

from . import render

SELECTED_KEYS = ("total_overlap_keys", "duplication_factor", "p95_tiles_per_splat", "max_tiles_per_splat",
                 "large_splat_count", "p95_splats_per_tile", "max_splats_per_tile")
LARGE_SPLAT_TILES = 64  # render.large_splat_tile_threshold's default (debug_metrics.py:238)


@dataclass
class FrameLists:
    """The lists one render call built: ``offsets`` [B*G+1] pair offsets by (view, depth rank),
    ``ranges`` [B*n_tiles*2] (start, end) of every tile's list."""

    n_views: int
    n_gaussians: int
    n_tiles: int
    tile_size: int
    mode: str
    offsets: torch.Tensor
    ranges: torch.Tensor

    def per_splat_counts(self, view: int) -> torch.Tensor:
        G = self.n_gaussians
        o = self.offsets[view * G:(view + 1) * G + 1].to(torch.int64)
        return o[1:] - o[:-1]

    def per_tile_counts(self, view: int) -> torch.Tensor:
        r = self.ranges.view(self.n_views, self.n_tiles, 2)[view].to(torch.int64)
        return r[:, 1] - r[:, 0]


@contextlib.contextmanager
def collect():
    """Within the block, every render call appends its FrameLists to the yielded list."""
    frames: list[FrameLists] = []
    previous = render.STATS_FRAMES
    render.STATS_FRAMES = frames
    try:
        yield frames
    finally:
        render.STATS_FRAMES = previous


def quantile(values: torch.Tensor, q: float) -> float:
    """torch.quantile's default (linear interpolation between the two nearest ranks), without its
    input-size limit; 0 for an empty tensor as overlap_metrics._quantile (:30-33)."""
    n = values.numel()
    if n == 0:
        return 0.0
    v = torch.sort(values.flatten().to(torch.float64)).values
    pos = q * (n - 1)
    lo = int(math.floor(pos))
    hi = min(lo + 1, n - 1)
    a, b = v[lo].item(), v[hi].item()
    return float(a + (b - a) * (pos - lo))


def summarize_counts(per_splat: torch.Tensor, per_tile: torch.Tensor, *, tile_size: int,
                     large_splat_tile_threshold: int = LARGE_SPLAT_TILES) -> dict[str, float]:
    """The statistics of overlap_metrics.summarize_overlap_counts (:36-74) for one frame."""
    splats, tiles = int(per_splat.numel()), int(per_tile.numel())
    total = int(per_splat.sum().item())
    active = per_splat[per_splat > 0]
    nonempty = per_tile[per_tile > 0]
    large = int((per_splat >= int(large_splat_tile_threshold)).sum().item())
    mean = lambda t: float(t.to(torch.float64).mean().item()) if t.numel() else 0.0  # noqa: E731
    return {
        "tile_size": float(tile_size),
        "total_overlap_keys": float(total),
        "duplication_factor": float(total / splats) if splats else 0.0,
        "active_splats": float(active.numel()),
        "zero_overlap_splats": float(splats - active.numel()),
        "mean_tiles_per_splat": mean(per_splat),
        "mean_tiles_per_active_splat": mean(active),
        "p95_tiles_per_splat": quantile(per_splat, 0.95),
        "max_tiles_per_splat": float(per_splat.max().item()) if splats else 0.0,
        "large_splat_count": float(large),
        "large_splat_fraction": float(large / splats) if splats else 0.0,
        "mean_splats_per_tile": mean(per_tile),
        "mean_splats_per_nonempty_tile": mean(nonempty),
        "p95_splats_per_tile": quantile(per_tile, 0.95),
        "max_splats_per_tile": float(per_tile.max().item()) if tiles else 0.0,
        "nonempty_tiles": float(nonempty.numel()),
        "nonempty_tile_fraction": float(nonempty.numel() / tiles) if tiles else 0.0,
    }


def frame_stats(frames: list[FrameLists], large_splat_tile_threshold: int = LARGE_SPLAT_TILES) -> list[dict]:
    """summarize_counts of every view of every collected call, in call and view order."""
    out = []
    for f in frames:
        for b in range(f.n_views):
            out.append(summarize_counts(f.per_splat_counts(b), f.per_tile_counts(b), tile_size=f.tile_size,
                                        large_splat_tile_threshold=large_splat_tile_threshold))
    return out


def aggregate(stats: list[dict], prefix: str) -> dict[str, float]:
    """overlap_metrics.aggregate_stat_dicts (:415-426): ``{prefix}_{key}_mean`` and ``_max`` over the
    frames of every finite statistic."""
    out: dict[str, float] = {}
    for key in sorted({k for s in stats for k in s}):
        values = [float(s[key]) for s in stats if key in s and math.isfinite(float(s[key]))]
        if values:
            out[f"{prefix}_{key}_mean"] = sum(values) / len(values)
            out[f"{prefix}_{key}_max"] = max(values)
    return out


def overlap_summary(frames: list[FrameLists], prefix: str = "TileDiag/B200", selected: bool = True,
                    large_splat_tile_threshold: int = LARGE_SPLAT_TILES) -> dict[str, float]:
    """Mean and max over the collected frames of the selected_overlap_summary statistics (all of
    summarize_counts' with ``selected=False``), under the reference's TileDiag naming."""
    stats = frame_stats(frames, large_splat_tile_threshold)
    if selected:
        stats = [{k: s[k] for k in SELECTED_KEYS if k in s} for s in stats]
    return aggregate(stats, prefix)


def nvtx(enabled: bool = True) -> None:
    """Named NVTX ranges around every C-ABI stage of the render (see the module docstring)."""
    render.NVTX = bool(enabled)


if os.environ.get("GSB200_NVTX", "") not in ("", "0"):
    nvtx(True)
