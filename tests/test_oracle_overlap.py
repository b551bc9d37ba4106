"""The exact-mode tile rule against the reference's exact-conic overlap statistic.

tests/golden/make_golden.py --only overlap recorded, per splat, the tile counts of
exact_conic_overlap_stats (src/train/renderers/overlap_metrics.py:286-408) for the projected
Gaussians of the golden scenes at threshold 1/255, pixel centres at +0.5.  That statistic lists a
tile when the ellipse q <= -2 ln(threshold / opacity) meets the tile's pixel-centre box as a
continuous rectangle.  This library's exact rule (oracle/tiles_oracle.py restates it bit for bit)
lists a tile when, over the tile row's band, the ellipse's x-extent holds a pixel-centre column
of the tile: the blend evaluates pixel centres only, so a tile that the ellipse crosses only
between two pixel columns holds no pixel to blend and is not listed.  Its ellipse level carries a
margin (tau (1 + 1e-5) + 1e-3) against float32 rounding in the blend.  So:

* every tile that holds a pixel centre inside the ellipse (brute force over the pixels) is listed,
  by this rule and by the reference's;
* per splat, this rule lists at most the reference's count plus the margin's odd tile, and at most
  a few tiles fewer (ellipses that cross a tile only between pixel columns); in total within 0.5%.
"""
import numpy as np
import pytest

from conftest import load_golden
from oracle import tiles_oracle as to

CASES = ["static64", "dynamic128_small", "multiview384_small", "clips256_small", "edge"]
THRESHOLD = 1.0 / 255.0


def exact_lists(g, case, tile):
    m, q, o = g[f"{case}_means2d"], g[f"{case}_conics"], g[f"{case}_opacities"]
    H, W = (int(v) for v in g[f"{case}_size"])
    tiles, ranks = to.exact_pairs_one_view(m[:, 0], m[:, 1], q[:, 0], 2.0 * q[:, 1], q[:, 2], o, H, W, tile,
                                           np.float32(THRESHOLD), pixel_center=0.5)
    return tiles, ranks


def brute_force_pairs(g, case, tile):
    """(splat, tile) pairs whose tile holds a pixel centre with q <= tau, float64 over every pixel."""
    m = g[f"{case}_means2d"].astype(np.float64)
    q = g[f"{case}_conics"].astype(np.float64)
    o = g[f"{case}_opacities"].astype(np.float64)
    H, W = (int(v) for v in g[f"{case}_size"])
    tiles_x = -(-W // tile)
    ys, xs = np.mgrid[0:H, 0:W]
    px, py = xs.ravel() + 0.5, ys.ravel() + 0.5
    tid = (ys.ravel() // tile) * tiles_x + xs.ravel() // tile
    pairs = set()
    for s in np.nonzero(o > THRESHOLD)[0]:
        a, b, c = q[s]
        if not (a * c - b * b > 0 and a > 0 and c > 0):
            continue
        tau = 2.0 * np.log(o[s] / THRESHOLD)
        dx, dy = px - m[s, 0], py - m[s, 1]
        hit = a * dx * dx + 2 * b * dx * dy + c * dy * dy <= tau
        pairs.update((int(s), int(t)) for t in np.unique(tid[hit]))
    return pairs


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("tile", [8, 16])
def test_exact_rule_against_reference_overlap_counts(case, tile):
    g = load_golden("overlap")
    ref = g[f"{case}_t{tile}_counts"]
    tiles, ranks = exact_lists(g, case, tile)
    got = np.bincount(ranks, minlength=ref.size)
    listed = set(zip(ranks.tolist(), tiles.tolist()))
    needed = brute_force_pairs(g, case, tile)
    assert needed <= listed, f"{len(needed - listed)} tiles with a pixel inside the ellipse are missing"
    need_counts = np.bincount(np.array([s for s, _ in needed], dtype=np.int64), minlength=ref.size)
    assert (ref >= need_counts).all()  # the reference's statistic holds them too
    assert (got <= ref + 1).all()
    assert (got >= ref - 3).all()
    assert abs(int(got.sum()) - int(ref.sum())) <= 0.005 * ref.sum() + 2
