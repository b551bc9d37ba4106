"""Host side of the per-call render statistics (dynaworld_b200/diagnostics.py): the summary of
overlap_metrics.summarize_overlap_counts (src/train/renderers/overlap_metrics.py:36-74) and its
aggregation (:415-426), checked against numpy on fixed counts."""
import math

import numpy as np
import torch

from dynaworld_b200 import diagnostics as dg


def _counts(seed, n, hi, zeros):
    g = np.random.default_rng(seed)
    c = g.integers(0, hi, n)
    c[g.random(n) < zeros] = 0
    return c


def test_summary_matches_numpy():
    splat = _counts(0, 1001, 90, 0.3)
    tile = _counts(1, 377, 500, 0.1)
    s = dg.summarize_counts(torch.from_numpy(splat), torch.from_numpy(tile), tile_size=16)
    assert s["total_overlap_keys"] == splat.sum()
    assert math.isclose(s["duplication_factor"], splat.sum() / splat.size)
    assert s["active_splats"] == (splat > 0).sum() and s["zero_overlap_splats"] == (splat == 0).sum()
    assert math.isclose(s["mean_tiles_per_active_splat"], splat[splat > 0].mean())
    assert math.isclose(s["p95_tiles_per_splat"], np.percentile(splat, 95))  # linear, as torch.quantile
    assert math.isclose(s["p95_splats_per_tile"], np.percentile(tile, 95))
    assert s["max_tiles_per_splat"] == splat.max() and s["max_splats_per_tile"] == tile.max()
    assert s["large_splat_count"] == (splat >= 64).sum()
    assert math.isclose(s["mean_splats_per_nonempty_tile"], tile[tile > 0].mean())
    assert s["nonempty_tiles"] == (tile > 0).sum()
    assert math.isclose(s["nonempty_tile_fraction"], (tile > 0).mean())


def test_empty_counts_and_quantile_edges():
    s = dg.summarize_counts(torch.zeros(0, dtype=torch.int64), torch.zeros(0, dtype=torch.int64), tile_size=8)
    assert s["total_overlap_keys"] == 0 and s["p95_splats_per_tile"] == 0.0 and s["max_tiles_per_splat"] == 0.0
    assert dg.quantile(torch.tensor([7]), 0.95) == 7.0
    v = torch.arange(21)
    assert dg.quantile(v, 0.95) == 19.0 and dg.quantile(v, 0.5) == 10.0


def test_aggregate_means_and_maxima():
    out = dg.aggregate([{"a": 1.0, "b": float("nan")}, {"a": 3.0, "b": 2.0}], "TileDiag/X")
    assert out == {"TileDiag/X_a_mean": 2.0, "TileDiag/X_a_max": 3.0, "TileDiag/X_b_mean": 2.0,
                   "TileDiag/X_b_max": 2.0}


def test_frame_lists_slice_views():
    offsets = torch.tensor([0, 2, 2, 5, 6, 6, 9], dtype=torch.int32)  # 2 views x 3 Gaussians
    ranges = torch.tensor([0, 3, 3, 5, 5, 5, 6, 9], dtype=torch.int32)  # 2 views x 2 tiles
    f = dg.FrameLists(2, 3, 2, 16, "exact", offsets, ranges)
    assert f.per_splat_counts(0).tolist() == [2, 0, 3] and f.per_splat_counts(1).tolist() == [1, 0, 3]
    assert f.per_tile_counts(0).tolist() == [3, 2] and f.per_tile_counts(1).tolist() == [0, 3]
    keys = dg.overlap_summary([f])
    assert keys["TileDiag/B200_total_overlap_keys_mean"] == 4.5 and keys["TileDiag/B200_max_splats_per_tile_max"] == 3
