"""Generates tests/golden/splats2d_accuracy.npz from the reference's own 2-D accuracy harness.

    python tests/golden/make_golden_2d.py --reference PATH   (or DYNAWORLD_REFERENCE=PATH)

Imports src/benchmarks/splat_renderer_accuracy.py from a checkout of nbardy/dynaworld and, for
each case, records what the reference computes: the inputs of make_accuracy_case (:190-238; its
own seeds, sizes and value ranges from DEFAULT_CONFIG), the float64 image of
torch_reference_rasterize (:262-305), the harness loss mse_loss (:446-447) and the autograd
gradients of that loss w.r.t. the packed rows and the features -- exactly the baseline the
harness holds every 2-D renderer to (run_accuracy, :534-600).

Cases: the harness's default grid (resolutions 16 and 32, 4 / 8 / 16 splats, 3 sets each, its
seed formula), plus larger cases drawn by make_accuracy_case at other sizes so that images span
several 16x16 tiles.

Needs the reference checkout (it cannot travel to GPU machines); the .npz it writes is committed
and is all the tests read.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# larger cases: (height, width, splats, sets); seeds follow the harness's formula
EXTRA_CASES = [(48, 64, 64, 2), (96, 80, 160, 1), (128, 128, 400, 1)]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DYNAWORLD_REFERENCE"),
                    help="checkout of nbardy/dynaworld (default: $DYNAWORLD_REFERENCE)")
    ap.add_argument("--out", default=str(HERE / "splats2d_accuracy.npz"))
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("give the reference checkout with --reference PATH or DYNAWORLD_REFERENCE")
    sys.path.insert(0, str(Path(args.reference) / "src" / "benchmarks"))
    import splat_renderer_accuracy as acc  # noqa: E402

    cfg = acc.DEFAULT_CONFIG
    base_seed = int(cfg["seed"])
    grid = []
    for hw in cfg["resolutions"]:
        height, width = acc.normalize_resolution(hw)
        for g in cfg["splat_counts"]:
            grid.append((height, width, int(g), int(cfg["sets_per_case"])))
    out: dict[str, np.ndarray] = {}
    idx = 0
    for height, width, g, sets in grid + EXTRA_CASES:
        for set_index in range(sets):
            seed = base_seed + height * 1_000_003 + width * 10_007 + g * 101 + set_index
            case = acc.make_accuracy_case(height, width, g, set_index, seed, cfg["random_splats_2d"])
            ref = acc.clone_for_device(case, torch.device("cpu"), torch.float64, requires_grad=True)
            image = acc.torch_reference_rasterize(ref, cfg["taichi"])
            loss = acc.mse_loss(image, ref.target)
            loss.backward()
            p = f"c{idx}_"
            out[p + "packed"] = case.packed.numpy().astype(np.float32)
            out[p + "depths"] = case.depths.numpy().astype(np.float32)
            out[p + "features"] = case.features.numpy().astype(np.float32)
            out[p + "target"] = case.target.numpy().astype(np.float32)
            out[p + "background"] = case.background.numpy().astype(np.float32)
            out[p + "size"] = np.array([height, width, g, set_index, seed], dtype=np.int64)
            out[p + "image"] = image.detach().numpy()
            out[p + "loss"] = np.array(float(loss.detach()))
            out[p + "packed_grad"] = ref.packed.grad.numpy()
            out[p + "feature_grad"] = ref.features.grad.numpy()
            idx += 1
    out["n_cases"] = np.array(idx)
    out["taichi_cfg"] = np.array([cfg["taichi"]["alpha_threshold"], cfg["taichi"]["clamp_max_alpha"],
                                  cfg["taichi"]["saturate_threshold"]], dtype=np.float64)
    tol = cfg["tolerances"]
    out["tolerances"] = np.array([tol["image_max_abs"], tol["image_mean_abs"], tol["loss_abs"],
                                  tol["packed_grad_max_abs"], tol["packed_grad_mean_abs"],
                                  tol["feature_grad_max_abs"], tol["feature_grad_mean_abs"]], dtype=np.float64)
    np.savez_compressed(args.out, **out)
    print(f"wrote {idx} cases to {args.out}")


if __name__ == "__main__":
    main()
