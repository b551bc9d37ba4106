"""Generates tests/golden/lens_*.npz: the reference's camera_model rendering with distorted lenses.

    python tests/golden/make_golden_lens.py --reference PATH   (or DYNAWORLD_REFERENCE=PATH)

Imports the reference's src/train modules and records, for seeded synthetic scenes seen through
radial-tangential, OpenCV-fisheye and pinhole CameraSpec values (camera.py:11-31) in one batch,
what the reference computes: the image of render_pytorch_3dgs_batch(..., cameras=...,
projection_mode="camera_model") (dense.py:170-236 -> projection.py:283-330), the
reconstruction_loss_per_image loss (losses.py:58-85) and autograd gradients, and the projected
Gaussians of project_gaussians_2d_camera_batch.

As in make_golden.py, raw-parameter gradients come from autograd through
oracle.splat_oracle.activate followed by the reference's render and loss.  The .npz files are
committed and are all the tests read.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from dynaworld_b200 import synthetic as syn  # noqa: E402
from make_golden import LOSS_CFG, to_np, workload_arrays  # noqa: E402
from oracle import splat_oracle as so  # noqa: E402

# (lens model, distortion) per view
MIXED = [
    ("radial_tangential", [-0.12, 0.03, 0.001, -0.002, 0.004]),
    ("opencv_fisheye", [0.05, -0.01, 0.003, -0.0005]),
    ("pinhole", None),
    ("radial_tangential", [-0.3, 0.08, 0.004, 0.003, -0.01]),
]
WIDE = [
    ("opencv_fisheye", [-0.02, 0.004, -0.001, 0.0002]),
    ("opencv_fisheye", [0.12, -0.03, 0.01, -0.002]),
]


def wide_workload() -> syn.Workload:
    """Gaussians spread over a wide field of view (up to ~60 degrees off axis), where the fisheye
    model departs furthest from a pinhole; two static views."""
    g = torch.Generator().manual_seed(21)
    G = 2500
    z = torch.rand(G, generator=g) * 2.0 + 1.0
    xy = (torch.rand(G, 2, generator=g) * 2 - 1) * z[:, None] * 1.6
    means = torch.cat([xy, z[:, None]], -1)
    log_scales = torch.randn(G, 3, generator=g) * 0.5 - 3.2
    quats = torch.randn(G, 4, generator=g)
    logits = torch.randn(G, 1, generator=g)
    sh = torch.randn(G, 4, 3, generator=g) * 0.1
    sh[:, 0] = torch.randn(G, 3, generator=g) * 0.3
    c2w = torch.eye(4).repeat(2, 1, 1)
    c2w[1, :3, 3] = torch.tensor([0.1, -0.05, 0.0])
    target = torch.rand(2, 3, 80, 96, generator=g)
    f = torch.tensor([40.0, 42.0])
    return syn.Workload("lens_wide", means[None], log_scales[None], quats[None], logits[None], sh[None], None,
                        f, f, torch.tensor([47.5, 48.0]), torch.tensor([39.5, 40.0]), c2w, torch.zeros(2), 2, 80, 96,
                        target)


def render_case(R, CameraSpec, wl: syn.Workload, lenses) -> dict:
    raw = {k: v.clone().requires_grad_(True) for k, v in dict(
        means=wl.means, log_scales=wl.log_scales, quats=wl.quats, opacity_logits=wl.opacity_logits,
        sh=wl.sh).items()}
    vel = None if wl.velocity is None else wl.velocity.clone().requires_grad_(True)
    rg = so.RawGaussians(raw["means"], raw["log_scales"], raw["quats"], raw["opacity_logits"], raw["sh"], vel)
    m, s, q, o, rgb = so.activate(rg, wl.times, wl.camera_to_world, wl.views_per_set)
    cams = [CameraSpec(fx=float(wl.fx[b]), fy=float(wl.fy[b]), cx=float(wl.cx[b]), cy=float(wl.cy[b]),
                       camera_to_world=wl.camera_to_world[b], lens_model=lens, distortion=dist)
            for b, (lens, dist) in enumerate(lenses)]
    img = R["dense"](m, s, q, o, rgb, wl.height, wl.width, wl.fx, wl.fy, wl.cx, wl.cy, cameras=cams,
                     projection_mode="camera_model", camera_to_world=wl.camera_to_world)
    loss = R["loss"](img, wl.target, LOSS_CFG)
    loss.sum().backward()
    out = {"image": img.detach(), "loss": loss.detach()}
    for k, v in raw.items():
        out[f"grad_{k}"] = v.grad
    if vel is not None:
        out["grad_velocity"] = vel.grad
    with torch.no_grad():
        m2, inv, cov, op, _rgb = R["project_camera_batch"](m, s, q, o, rgb, cams)
    out.update(means2d=m2, inv_cov=inv, cov2d=cov, proj_opacity=op)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DYNAWORLD_REFERENCE"),
                    help="checkout of nbardy/dynaworld (default: $DYNAWORLD_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("give the reference checkout with --reference PATH or DYNAWORLD_REFERENCE")
    sys.path.insert(0, str(Path(args.reference) / "src" / "train"))
    from camera import CameraSpec  # noqa: E402
    from losses import reconstruction_loss_per_image  # noqa: E402
    from renderers.dense import render_pytorch_3dgs_batch  # noqa: E402
    from renderers.projection import project_gaussians_2d_camera_batch  # noqa: E402

    R = dict(dense=render_pytorch_3dgs_batch, loss=reconstruction_loss_per_image,
             project_camera_batch=project_gaussians_2d_camera_batch)
    cases = {
        "lens_mixed": (syn.dynamic128(scale=0.1, image_scale=0.5, frames=4), MIXED),
        "lens_wide": (wide_workload(), WIDE),
    }
    for name, (wl, lenses) in cases.items():
        res = render_case(R, CameraSpec, wl, lenses)
        arrays = to_np(workload_arrays(wl))
        arrays.update({f"ref_{k}": v for k, v in to_np(res).items()})
        arrays["lens_models"] = np.array([l for l, _ in lenses])
        arrays["distortion"] = np.array([(d or []) + [0.0] * (5 - len(d or [])) for _, d in lenses], np.float32)
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **arrays)
        print(f"wrote {path.name}: {path.stat().st_size / 1e6:.2f} MB", flush=True)


if __name__ == "__main__":
    main()
