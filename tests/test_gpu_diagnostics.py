"""Per-call render statistics (dynaworld_b200/diagnostics.py) from the lists the renderer built:
per-Gaussian tile counts and per-tile list lengths equal those of the numpy restatement of the
exact-mode lists on the same records; NVTX ranges leave the output unchanged."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, load_golden
from dynaworld_b200 import diagnostics
from dynaworld_b200.config import B200RendererConfig
from gpu_helpers import records_np, render_raw, stages
from oracle import tiles_oracle as to

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_overlap_counts_match_restated_lists(case):
    g = load_golden(case)
    wl = g.workload()
    cfg = B200RendererConfig()
    with diagnostics.collect() as frames:
        _, _, _, st = stages(wl, cfg)
    assert len(frames) == 1
    f = frames[0]
    rec = records_np(st, wl.n_views, wl.n_gaussians)
    n_tiles = to.n_tiles_for(wl.height, wl.width, cfg.tile_size)
    for b in range(wl.n_views):
        r = rec[b]
        tiles, ranks = to.exact_pairs_one_view(r[:, 0], r[:, 1], r[:, 2], r[:, 3], r[:, 4], r[:, 5], wl.height,
                                               wl.width, cfg.tile_size, np.float32(cfg.alpha_cutoff))
        np.testing.assert_array_equal(f.per_splat_counts(b).cpu().numpy(), np.bincount(ranks, minlength=wl.n_gaussians))
        np.testing.assert_array_equal(f.per_tile_counts(b).cpu().numpy(), np.bincount(tiles, minlength=n_tiles))
    s = diagnostics.overlap_summary(frames)
    assert s["TileDiag/B200_total_overlap_keys_mean"] * wl.n_views == pytest.approx(st.n_pairs)
    assert set(s) == {f"TileDiag/B200_{k}_{a}" for k in diagnostics.SELECTED_KEYS for a in ("mean", "max")}


def test_nvtx_ranges_leave_output_unchanged():
    wl = load_golden("static64").workload()
    base = render_raw(wl, grads=True, loss=True)
    diagnostics.nvtx(True)
    try:
        out = render_raw(wl, grads=True, loss=True)
    finally:
        diagnostics.nvtx(False)
    assert torch.equal(out["image"], base["image"])
    torch.testing.assert_close(out["grad_means"], base["grad_means"], rtol=1e-5, atol=1e-7)
