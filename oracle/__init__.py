"""CPU oracle for the Gaussian-splat render + L1/SSIM loss path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``dynaworld_b200`` imports this package;
only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use it, and only as the reference the CUDA results are compared with or as
the timed CPU port.

Modules:
  splat_oracle  torch restatement (float32/float64) of the reference's
                projection (src/train/renderers/common.py), dense blend
                (src/train/renderers/dense.py) and loss (src/train/losses.py),
                plus the raw-parameter front end (activation, SH, velocity).
  tiles_oracle  numpy restatement of the tile bounds / assignment rules
                (src/train/renderers/tiled.py) and of this library's exact
                tile binning, key layout and sorted order.
  culled_oracle torch restatement of the tile-culled, rank-corrected blend the
                CUDA raster kernels implement (same semantics as dense.py up to
                the alpha cutoff and transmittance threshold).

Parity is pinned: tests/golden/make_golden.py runs the reference's own
functions (imported from a checkout of nbardy/dynaworld) and stores their
outputs; tests/test_oracle_golden.py checks these restatements against them.
"""
