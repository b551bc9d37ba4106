"""Generates tests/golden/bank.npz: the reference's dynamic-bank frames, image, loss and gradients.

    python tests/golden/make_golden_bank.py --reference PATH   (or DYNAWORLD_REFERENCE=PATH)

For seeded banks this runs the reference's own evaluation
(gs_models/dynamic_video_token_gs_implicit_camera.py:1206-1224, _eval_dynamic_bank, with the
DynamicGaussianBank of :795-803), puts static Gaussians first as _decode_static_dynamic_split
does (:1256-1275), renders the frames with render_pytorch_3dgs_batch (dense.py:170-236) and
back-propagates reconstruction_loss_per_image (losses.py:58-85) into every bank and static tensor.
Bank values follow DynamicResidualGaussianBankHead (:930-952): tanh-bounded coefficients times
motion_extent 0.25, rotation 10 degrees and alpha-logit extent 2.

Cases:
* ``mixed``: 250 static + 450 dynamic Gaussians, 8 basis functions, 4 frames;
* ``odd``: dynamic only, 5 basis functions (odd: the 2t - 1 column), rotation coefficients of
  1e-8 for a third of the Gaussians (the small-angle series branch of :833-837) and opacities
  at 0, 1 and 1e-7 (outside the logit clamp).

Needs the reference checkout; the .npz it writes is committed and is all the tests read.
"""
from __future__ import annotations

import argparse
import os
import math
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from dynaworld_b200 import synthetic as syn  # noqa: E402
from make_golden import LOSS_CFG  # noqa: E402

MAX_FREQUENCY = 8.0


def make_bank(g: torch.Generator, G: int, M: int, *, small_rot=False, edge_opacity=False) -> dict:
    xyz0 = torch.stack([torch.rand(G, generator=g) * 3 - 1.5, torch.rand(G, generator=g) * 3 - 1.5,
                        torch.rand(G, generator=g) * 3 + 2], -1)
    scales = torch.exp(torch.randn(G, 3, generator=g) * 0.6 - 3.3)
    q = torch.randn(G, 4, generator=g)
    quats0 = q / q.norm(dim=-1, keepdim=True)
    opacities0 = torch.sigmoid(torch.randn(G, 1, generator=g))
    rgbs = torch.sigmoid(torch.randn(G, 3, generator=g))
    A_mu = torch.tanh(torch.randn(G, M, 3, generator=g)) * 0.25
    A_rot = torch.tanh(torch.randn(G, M, 3, generator=g)) * math.radians(10.0)
    A_alpha = torch.tanh(torch.randn(G, M, 1, generator=g)) * 2.0
    if small_rot:
        A_rot[: G // 3] *= 1e-7 / math.radians(10.0)
    if edge_opacity:
        opacities0[0:5] = 0.0
        opacities0[5:10] = 1.0
        opacities0[10:15] = 1e-7
    return dict(xyz0=xyz0, scales=scales, quats0=quats0, opacities0=opacities0, rgbs=rgbs, A_mu=A_mu, A_rot=A_rot,
                A_alpha=A_alpha)


def make_static(g: torch.Generator, G: int) -> dict:
    xyz = torch.stack([torch.rand(G, generator=g) * 3 - 1.5, torch.rand(G, generator=g) * 3 - 1.5,
                       torch.rand(G, generator=g) * 3 + 2], -1)
    q = torch.randn(G, 4, generator=g)
    return dict(xyz=xyz, scales=torch.exp(torch.randn(G, 3, generator=g) * 0.6 - 3.3), quats=q / q.norm(dim=-1,
                                                                                                         keepdim=True),
                opacities=torch.sigmoid(torch.randn(G, 1, generator=g)), rgbs=torch.sigmoid(torch.randn(G, 3,
                                                                                                        generator=g)))


def case_arrays(R, bank: dict, static: dict | None, wl: syn.Workload) -> dict:
    M = bank["A_mu"].shape[1]
    leaves = {f"bank_{k}": v.clone().requires_grad_(True) for k, v in bank.items()}
    if static is not None:
        leaves.update({f"static_{k}": v.clone().requires_grad_(True) for k, v in static.items()})
    ref_bank = R["Bank"](**{k: leaves[f"bank_{k}"][None] for k in bank})
    ns = SimpleNamespace(dynamic_time_basis_count=M, dynamic_time_max_frequency=MAX_FREQUENCY)
    decode_times = wl.times[None]  # [1, K] as the model's forward takes them
    per_frame = []
    for k in range(decode_times.shape[1]):
        dyn = R["eval"](ns, ref_bank, decode_times[:, k])
        if static is not None:
            st = [leaves[f"static_{n}"][None] for n in ("xyz", "scales", "quats", "opacities", "rgbs")]
            dyn = [torch.cat([a, b], dim=1) for a, b in zip(st, dyn)]
        per_frame.append([t.squeeze(0) for t in dyn])
    xyz, scales, quats, opac, rgbs = (torch.stack([f[i] for f in per_frame]) for i in range(5))
    img = R["dense"](xyz, scales, quats, opac, rgbs, wl.height, wl.width, wl.fx, wl.fy, wl.cx, wl.cy,
                     camera_to_world=wl.camera_to_world)
    loss = R["loss"](img, wl.target, LOSS_CFG)
    loss.sum().backward()
    out = {"image": img.detach(), "loss": loss.detach(), "frame_xyz": xyz.detach(), "frame_quats": quats.detach(),
           "frame_opacities": opac.detach()}
    for k, v in leaves.items():
        out[k] = v.detach()
        out[f"grad_{k}"] = v.grad
    out.update(fx=wl.fx, fy=wl.fy, cx=wl.cx, cy=wl.cy, camera_to_world=wl.camera_to_world, target=wl.target,
               times=wl.times, height=torch.tensor(wl.height), width=torch.tensor(wl.width),
               max_frequency=torch.tensor(MAX_FREQUENCY))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DYNAWORLD_REFERENCE"),
                    help="checkout of nbardy/dynaworld (default: $DYNAWORLD_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("give the reference checkout with --reference PATH or DYNAWORLD_REFERENCE")
    sys.path.insert(0, str(Path(args.reference) / "src" / "train"))
    from gs_models.dynamic_video_token_gs_implicit_camera import (  # noqa: E402
        DynamicGaussianBank,
        DynamicVideoTokenGSImplicitCamera,
    )
    from losses import reconstruction_loss_per_image  # noqa: E402
    from renderers.dense import render_pytorch_3dgs_batch  # noqa: E402

    R = dict(dense=render_pytorch_3dgs_batch, loss=reconstruction_loss_per_image, Bank=DynamicGaussianBank,
             eval=DynamicVideoTokenGSImplicitCamera._eval_dynamic_bank)
    g = torch.Generator().manual_seed(31)
    cases = {
        "mixed": (make_bank(g, 450, 8), make_static(g, 250),
                  syn.dynamic128(scale=0.02, image_scale=0.375, frames=4, seed=11)),
        "odd": (make_bank(g, 500, 5, small_rot=True, edge_opacity=True), None,
                syn.dynamic128(scale=0.02, image_scale=0.375, frames=3, seed=12)),
    }
    arrays = {}
    for name, (bank, static, wl) in cases.items():
        for k, v in case_arrays(R, bank, static, wl).items():
            v = v.detach().numpy()
            arrays[f"{name}_{k}"] = v.astype(np.float32) if v.dtype.kind == "f" else v
    path = HERE / "bank.npz"
    np.savez_compressed(path, **arrays)
    print(f"wrote {path.name}: {path.stat().st_size / 1e6:.2f} MB", flush=True)


if __name__ == "__main__":
    main()
