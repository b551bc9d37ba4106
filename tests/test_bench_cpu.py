"""bench.py's CPU legs (the dense and tiled baselines and the reference arm's sample) run on a
small slice of every seeded workload: they are part of the default bench line, and a failure there
fails the whole bench."""
import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


@pytest.mark.parametrize("name", sorted(bench.CPU_WINDOW))
def test_cpu_baselines_run(name, monkeypatch):
    monkeypatch.setitem(bench.CPU_WINDOW, name, 8)  # the same code at the smallest window the loss takes
    full, wl = bench.make_workload(name, 0, 1, 0.002, 1.0, 8 if name == "clips256" else 1)
    dense = bench.cpu_baseline(name, wl, reps=1)
    assert dense["value"] > 0 and dense["kind"] == "port"
    tiled = bench.cpu_tiled_baseline(wl, tiles=2)
    assert tiled["value"] > 0
