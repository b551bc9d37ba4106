"""Generates tests/golden/camera_grads.npz: gradients w.r.t. the cameras from the reference.

    python tests/golden/make_golden_camera.py --reference PATH   (or DYNAWORLD_REFERENCE=PATH)

The reference's implicit-camera models predict fx, fy, cx, cy, camera_to_world and lens
distortion with networks (gs_models/implicit_camera.py:146-262) and train them through the render
call, so torch autograd through render_pytorch_3dgs_batch (dense.py:170-236) also yields
gradients for every camera tensor.  For seeded scenes this records the reference's image, loss
and the gradients w.r.t. the activated Gaussians and w.r.t. fx, fy, cx, cy [B], camera_to_world
[B,4,4] and (camera_model case) the distortion coefficients [B,5]:

* ``pin``: 3 pinhole views (legacy_pinhole batch path, common.py:149-231), tilted cameras;
* ``lens``: the lens_mixed scene of make_golden_lens.py (radial-tangential, fisheye, pinhole,
  radial-tangential; camera_model path, projection.py:283-330).

Needs the reference checkout; the .npz it writes is committed and is all the tests read.
"""
from __future__ import annotations

import argparse
import os
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from dynaworld_b200 import synthetic as syn  # noqa: E402
from make_golden import LOSS_CFG  # noqa: E402
from make_golden_lens import MIXED  # noqa: E402
from oracle import splat_oracle as so  # noqa: E402

N_COEF = {"pinhole": 0, "radial_tangential": 5, "opencv_fisheye": 4}


def tilted_views(wl: syn.Workload) -> syn.Workload:
    """Tilt and roll the cameras a little so that every rotation entry carries a gradient."""
    c2w = wl.camera_to_world.clone()
    for b in range(c2w.shape[0]):
        a, r = 0.05 * (b + 1), -0.03 * (b + 1)
        rx = torch.tensor([[1, 0, 0], [0, math.cos(a), -math.sin(a)], [0, math.sin(a), math.cos(a)]])
        rz = torch.tensor([[math.cos(r), -math.sin(r), 0], [math.sin(r), math.cos(r), 0], [0, 0, 1]])
        c2w[b, :3, :3] = c2w[b, :3, :3] @ rx @ rz
    wl.camera_to_world = c2w
    return wl


def case_arrays(R, CameraSpec, wl: syn.Workload, lenses) -> dict:
    raw = so.RawGaussians(wl.means, wl.log_scales, wl.quats, wl.opacity_logits, wl.sh, wl.velocity)
    with torch.no_grad():
        m, s, q, o, rgb = so.activate(raw, wl.times, wl.camera_to_world, wl.views_per_set)
    act = {k: v.detach().clone().requires_grad_(True) for k, v in dict(xyz=m, scales=s, quats=q, opacities=o,
                                                                          rgbs=rgb).items()}
    fx, fy, cx, cy = (v.clone().requires_grad_(True) for v in (wl.fx, wl.fy, wl.cx, wl.cy))
    c2w = wl.camera_to_world.clone().requires_grad_(True)
    dist = None
    if lenses is None:
        img = R["dense"](act["xyz"], act["scales"], act["quats"], act["opacities"], act["rgbs"], wl.height, wl.width,
                         fx, fy, cx, cy, camera_to_world=c2w)
    else:
        dist = torch.tensor([(d or []) + [0.0] * (5 - len(d or [])) for _, d in lenses]).requires_grad_(True)
        cams = [CameraSpec(fx=fx[b], fy=fy[b], cx=cx[b], cy=cy[b], camera_to_world=c2w[b], lens_model=lens,
                           distortion=None if lens == "pinhole" else dist[b, : N_COEF[lens]])
                for b, (lens, _d) in enumerate(lenses)]
        img = R["dense"](act["xyz"], act["scales"], act["quats"], act["opacities"], act["rgbs"], wl.height, wl.width,
                         fx, fy, cx, cy, cameras=cams, projection_mode="camera_model", camera_to_world=c2w)
    loss = R["loss"](img, wl.target, LOSS_CFG)
    loss.sum().backward()
    out = {"image": img.detach(), "loss": loss.detach(),
           "grad_intrinsics": torch.stack([fx.grad, fy.grad, cx.grad, cy.grad], -1), "grad_c2w": c2w.grad}
    for k, v in act.items():
        out[f"act_{k}"] = v.detach()
        out[f"grad_act_{k}"] = v.grad
    if dist is not None:
        out["grad_distortion"] = dist.grad
        out["distortion"] = dist.detach()
        out["lens_models"] = np.array([l for l, _ in lenses])
    out.update(fx=wl.fx, fy=wl.fy, cx=wl.cx, cy=wl.cy, camera_to_world=wl.camera_to_world, target=wl.target,
               height=torch.tensor(wl.height), width=torch.tensor(wl.width))
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

    R = dict(dense=render_pytorch_3dgs_batch, loss=reconstruction_loss_per_image)
    arrays = {}
    cases = {
        "pin": (tilted_views(syn.dynamic128(scale=0.06, image_scale=0.375, frames=3)), None),
        "lens": (syn.dynamic128(scale=0.1, image_scale=0.5, frames=4), MIXED),
    }
    for name, (wl, lenses) in cases.items():
        for k, v in case_arrays(R, CameraSpec, wl, lenses).items():
            if torch.is_tensor(v):
                v = v.detach().numpy()
                v = v.astype(np.float32) if v.dtype.kind == "f" else v
            arrays[f"{name}_{k}"] = v
    path = HERE / "camera_grads.npz"
    np.savez_compressed(path, **arrays)
    print(f"wrote {path.name}: {path.stat().st_size / 1e6:.2f} MB", flush=True)


if __name__ == "__main__":
    main()
