"""Generates the golden fixtures of tests/golden/ from the reference implementation itself.

    python tests/golden/make_golden.py --reference PATH [--only scenes losses tiled_grads overlap]
    (or DYNAWORLD_REFERENCE=PATH python tests/golden/make_golden.py)

Imports the reference's src/train modules (renderers.dense, renderers.common, renderers.tiled,
losses) from a checkout of nbardy/dynaworld and records, for seeded synthetic scenes, what the
reference computes: images of render_pytorch_3dgs_batch (dense.py:170-236), losses of
reconstruction_loss_per_image (losses.py:58-85) and their autograd gradients, the projected
Gaussians of project_gaussians_2d_batch (common.py:149-231) with the depth order, and the tile
lists of compute_gaussian_bounds + build_tile_assignments (tiled.py:7-71).

The reference takes activated parameters; the raw-parameter front end (exp, normalise, sigmoid,
SH, time offset) has no reference code, so raw gradients come from autograd through
oracle.splat_oracle.activate followed by the reference's render and loss.

Needs the reference checkout (it cannot travel to GPU machines); the .npz files it writes are
committed and are all the tests read.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from dynaworld_b200 import synthetic as syn  # noqa: E402
from oracle import splat_oracle as so  # noqa: E402

LOSS_CFG = dict(so.LOSS_DEFAULTS)


def ref_modules(reference: Path):
    sys.path.insert(0, str(reference / "src" / "train"))
    from losses import reconstruction_loss_per_image  # noqa: E402
    from renderers.common import project_gaussians_2d, project_gaussians_2d_batch  # noqa: E402
    from renderers.dense import render_pytorch_3dgs_batch  # noqa: E402
    from renderers.tiled import build_tile_assignments, compute_gaussian_bounds, render_pytorch_3dgs_tiled  # noqa

    return dict(loss=reconstruction_loss_per_image, project=project_gaussians_2d,
                project_batch=project_gaussians_2d_batch, dense=render_pytorch_3dgs_batch,
                bounds=compute_gaussian_bounds, assign=build_tile_assignments, tiled=render_pytorch_3dgs_tiled)


def workload_arrays(wl: syn.Workload) -> dict:
    out = dict(
        means=wl.means, log_scales=wl.log_scales, quats=wl.quats, opacity_logits=wl.opacity_logits, sh=wl.sh,
        fx=wl.fx, fy=wl.fy, cx=wl.cx, cy=wl.cy, camera_to_world=wl.camera_to_world, times=wl.times,
        target=wl.target, views_per_set=torch.tensor(wl.views_per_set), height=torch.tensor(wl.height),
        width=torch.tensor(wl.width),
    )
    if wl.velocity is not None:
        out["velocity"] = wl.velocity
    return out


def render_case(R, wl: syn.Workload, crop=None, with_grads=True, tiles=(8, 16)) -> dict:
    """Reference render + loss (+ gradients) of a workload; ``crop`` = (x0, y0, w, h) renders a window
    by shifting the principal point (pixels are independent given the Gaussians)."""
    raw = {k: v.clone().requires_grad_(with_grads) for k, v in dict(
        means=wl.means, log_scales=wl.log_scales, quats=wl.quats, opacity_logits=wl.opacity_logits,
        sh=wl.sh).items()}
    vel = None
    if wl.velocity is not None:
        vel = wl.velocity.clone().requires_grad_(with_grads)
    rg = so.RawGaussians(raw["means"], raw["log_scales"], raw["quats"], raw["opacity_logits"], raw["sh"], vel)
    m, s, q, o, rgb = so.activate(rg, wl.times, wl.camera_to_world, wl.views_per_set)
    act = {"xyz": m, "scales": s, "quats": q, "opacities": o, "rgbs": rgb}
    if with_grads:
        for t in act.values():
            t.retain_grad()
    H, W = wl.height, wl.width
    cx, cy = wl.cx, wl.cy
    target = wl.target
    if crop is not None:
        x0, y0, w, h = crop
        cx, cy, H, W = cx - x0, cy - y0, h, w
        target = target[:, :, y0:y0 + h, x0:x0 + w]
    img = R["dense"](m, s, q, o, rgb, H, W, wl.fx, wl.fy, cx, cy, camera_to_world=wl.camera_to_world)
    loss = R["loss"](img, target, LOSS_CFG)
    out = {"image": img.detach(), "loss": loss.detach()}
    if with_grads:
        loss.sum().backward()
        for k, v in raw.items():
            out[f"grad_{k}"] = v.grad
        if vel is not None:
            out["grad_velocity"] = vel.grad
        # gradients w.r.t. the reference render call's own inputs: activated tensors as independent
        # leaves (rgb no longer depends on xyz through the SH view direction)
        leaves = {k: v.detach().clone().requires_grad_(True) for k, v in act.items()}
        img2 = R["dense"](leaves["xyz"], leaves["scales"], leaves["quats"], leaves["opacities"], leaves["rgbs"], H, W,
                          wl.fx, wl.fy, cx, cy, camera_to_world=wl.camera_to_world)
        R["loss"](img2, target, LOSS_CFG).sum().backward()
        for k, v in leaves.items():
            out[f"grad_act_{k}"] = v.grad
    # projection internals of the reference, in its depth order
    with torch.no_grad():
        m2, inv, cov, op, rgbo = R["project_batch"](m, s, q, o, rgb, wl.fx, wl.fy, cx, cy,
                                                    camera_to_world=wl.camera_to_world)
        rcw = wl.camera_to_world[:, :3, :3]
        t = wl.camera_to_world[:, :3, 3]
        z = ((m - t[:, None, :]) @ rcw)[..., 2]
        order = torch.argsort(z, dim=1, stable=True)
    out.update(means2d=m2, inv_cov=inv, cov2d=cov, proj_opacity=op, proj_rgb=rgbo, depth_order=order, cam_z=z,
               act_xyz=m.detach(), act_scales=s.detach(), act_quats=q.detach(), act_opacities=o.detach(),
               act_rgbs=rgb.detach())
    # tile lists of the reference's tiled renderer, per view (tiled.py:7-71)
    if tiles and crop is None:
        for ts in tiles:
            tiles_x = (W + ts - 1) // ts
            all_t, all_g, all_v = [], [], []
            for b in range(m2.shape[0]):
                bounds = R["bounds"](m2[b], cov[b], op[b], H, W, bound_scale=3.0, alpha_threshold=1.0 / 255.0)
                a = R["assign"](*bounds, ts, tiles_x)
                if a is None:
                    continue
                u, packed, valid = a
                tl = torch.repeat_interleave(u, valid.sum(1))
                all_t.append(tl)
                all_g.append(packed[valid])
                all_v.append(torch.full_like(tl, b))
            out[f"tiled{ts}_view"] = torch.cat(all_v) if all_v else torch.zeros(0, dtype=torch.int64)
            out[f"tiled{ts}_tile"] = torch.cat(all_t) if all_t else torch.zeros(0, dtype=torch.int64)
            out[f"tiled{ts}_rank"] = torch.cat(all_g) if all_g else torch.zeros(0, dtype=torch.int64)
            imgs = [R["tiled"](m[b], s[b], q[b], o[b], rgb[b], H, W, float(wl.fx[b]), float(wl.fy[b]),
                               float(cx[b]), float(cy[b]), tile_size=ts,
                               camera_to_world=wl.camera_to_world[b]).detach() for b in range(m.shape[0])]
            out[f"tiled{ts}_image"] = torch.stack(imgs)
    return out


def to_np(d: dict) -> dict:
    out = {}
    for k, v in d.items():
        if torch.is_tensor(v):
            v = v.detach().cpu()
            v = v.numpy().astype(np.float32) if v.is_floating_point() else v.numpy()
        out[k] = v
    return out


def save(name: str, wl: syn.Workload, res: dict, extra: dict | None = None, lean: bool = False) -> None:
    """``lean``: store float64 checksums of the inputs instead of the inputs (the test regenerates
    them from dynaworld_b200.synthetic with the same seed) and only the reference image."""
    if lean:
        arrays = {f"checksum_{k}": np.float64(v.double().sum()) for k, v in workload_arrays(wl).items()}
        res = {"image": res["image"], "loss": res["loss"]}
    else:
        arrays = to_np(workload_arrays(wl))
    arrays.update({f"ref_{k}": v for k, v in to_np(res).items()})
    if extra:
        arrays.update(to_np(extra))
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, **arrays)
    print(f"wrote {path.name}: {path.stat().st_size / 1e6:.2f} MB", flush=True)


def edge_workload() -> syn.Workload:
    """Hand-made scene: near-plane and behind-camera Gaussians, off-screen ones, a saturated crowd
    of opaque Gaussians on one pixel, one splat much larger than the image, exact depth ties."""
    g = torch.Generator().manual_seed(11)
    G = 512
    means = torch.stack([torch.rand(G, generator=g) * 2 - 1, torch.rand(G, generator=g) * 2 - 1,
                         torch.rand(G, generator=g) * 2 + 2], -1)
    means[:16, 2] = torch.linspace(-1.0, 1e-4, 16)            # behind the camera / on the near plane
    means[16:32, 0] = torch.linspace(3.0, 6.0, 16)             # off-screen right
    means[32:96, :2] = 0.0                                     # crowd on the principal point
    means[32:96, 2] = 2.5 + 1e-3 * torch.arange(64)
    means[96:104, 2] = 3.0                                     # exact depth ties (index order)
    log_scales = torch.randn(G, 3, generator=g) * 0.4 - 3.0
    log_scales[104] = torch.tensor([1.0, 1.0, -2.0])           # splat larger than the image
    means[104] = torch.tensor([0.1, -0.1, 3.9])
    quats = torch.randn(G, 4, generator=g)
    logits = torch.randn(G, 1, generator=g)
    logits[32:96] = 6.0                                        # opaque crowd (alpha clamps at 0.99)
    sh = torch.randn(G, 1, 3, generator=g) * 0.3
    target = torch.rand(1, 3, 48, 40, generator=g)
    return syn.Workload("edge", means[None], log_scales[None], quats[None], logits[None], sh[None], None,
                        torch.tensor([44.0]), torch.tensor([48.0]), torch.tensor([20.5]), torch.tensor([23.0]),
                        torch.eye(4)[None], torch.zeros(1), 1, 48, 40, target)


def tiled_grad_cases(R) -> dict:
    """Gradients of the reference's tiled renderer (render_pytorch_3dgs_tiled, tiled.py:74-198,
    one call per view) under the standard_gs loss of all views, for the five golden scenes and tile
    sizes 8 and 16: with respect to the activated tensors of the render call (independent leaves per
    view; static64, dynamic128_small and edge) and, through the raw-parameter front end, to the raw
    parameters (all five)."""
    out = {}
    for case, wl in (("static64", syn.static64()), ("dynamic128_small", syn.dynamic128(scale=1 / 16, image_scale=0.5,
                                                                                        frames=2)),
                     ("multiview384_small", syn.multiview384(scale=0.01, image_scale=1 / 6, views=2)),
                     ("clips256_small", syn.clips256(scale=1 / 32, image_scale=0.25, clips=2, frames=2)),
                     ("edge", edge_workload())):
        for ts in (8, 16):
            raw = {k: getattr(wl, k).clone().requires_grad_(True)
                   for k in ("means", "log_scales", "quats", "opacity_logits", "sh")}
            vel = wl.velocity.clone().requires_grad_(True) if wl.velocity is not None else None
            rg = so.RawGaussians(raw["means"], raw["log_scales"], raw["quats"], raw["opacity_logits"], raw["sh"], vel)
            act = so.activate(rg, wl.times, wl.camera_to_world, wl.views_per_set)

            def render(m, s, q, o, rgb):
                return torch.stack([R["tiled"](m[b], s[b], q[b], o[b], rgb[b], wl.height, wl.width, float(wl.fx[b]),
                                               float(wl.fy[b]), float(wl.cx[b]), float(wl.cy[b]), tile_size=ts,
                                               camera_to_world=wl.camera_to_world[b])
                                    for b in range(wl.n_views)])

            img = render(*act)
            loss = R["loss"](img, wl.target, LOSS_CFG)
            loss.sum().backward()
            key = f"{case}_t{ts}"
            out[f"{key}_image"] = img.detach()
            out[f"{key}_loss"] = loss.detach()
            for k, v in raw.items():
                out[f"{key}_grad_{k}"] = v.grad
            if vel is not None:
                out[f"{key}_grad_velocity"] = vel.grad
            if case in ("multiview384_small", "clips256_small"):
                continue  # activated-input gradients of the three smaller scenes suffice
            leaves = [t.detach().clone().requires_grad_(True) for t in act]
            R["loss"](render(*leaves), wl.target, LOSS_CFG).sum().backward()
            for name, v in zip(("xyz", "scales", "quats", "opacities", "rgbs"), leaves):
                out[f"{key}_grad_act_{name}"] = v.grad
            print(f"tiled gradients: {key}", flush=True)
    return out


def overlap_cases(reference: Path) -> dict:
    """Per-splat tile counts of the reference's exact-conic overlap statistic
    (exact_conic_overlap_stats, renderers/overlap_metrics.py:286-408: tiles whose pixel-centre box,
    centres at +0.5, meets the ellipse q <= -2 ln(threshold / opacity)) for the projected Gaussians of
    view 0 of the five golden scenes, threshold 1/255, tiles of 8 and 16.  The statistic returns
    totals only, so each splat is counted by its own call."""
    from renderers.overlap_metrics import exact_conic_overlap_stats  # noqa: E402

    R = ref_modules(reference)
    out = {}
    for case, wl in (("static64", syn.static64()), ("dynamic128_small", syn.dynamic128(scale=1 / 16, image_scale=0.5,
                                                                                        frames=2)),
                     ("multiview384_small", syn.multiview384(scale=0.01, image_scale=1 / 6, views=2)),
                     ("clips256_small", syn.clips256(scale=1 / 32, image_scale=0.25, clips=2, frames=2)),
                     ("edge", edge_workload())):
        rg = so.RawGaussians(wl.means, wl.log_scales, wl.quats, wl.opacity_logits, wl.sh, wl.velocity)
        m, s, q, o, rgb = so.activate(rg, wl.times, wl.camera_to_world, wl.views_per_set)
        with torch.no_grad():
            m2, inv, _cov, op, _rgb = R["project_batch"](m, s, q, o, rgb, wl.fx, wl.fy, wl.cx, wl.cy,
                                                          camera_to_world=wl.camera_to_world)
        means2d = m2[0].float()
        conics = torch.stack([inv[0, :, 0, 0], 0.5 * (inv[0, :, 0, 1] + inv[0, :, 1, 0]), inv[0, :, 1, 1]], -1).float()
        opac = op[0, :, 0].float()
        out[f"{case}_means2d"], out[f"{case}_conics"], out[f"{case}_opacities"] = means2d, conics, opac
        out[f"{case}_size"] = torch.tensor([wl.height, wl.width])
        for ts in (8, 16):
            counts = [int(exact_conic_overlap_stats(means2d[g:g + 1], conics[g:g + 1], opac[g:g + 1],
                                                    (wl.height, wl.width), tile_size=ts,
                                                    alpha_threshold=1.0 / 255.0)["total_overlap_keys"])
                      for g in range(means2d.shape[0])]
            out[f"{case}_t{ts}_counts"] = torch.tensor(counts, dtype=torch.int64)
            total = exact_conic_overlap_stats(means2d, conics, opac, (wl.height, wl.width), tile_size=ts,
                                              alpha_threshold=1.0 / 255.0)["total_overlap_keys"]
            assert int(total) == sum(counts)
        print(f"overlap counts: {case}", flush=True)
    return out


def loss_cases(R) -> dict:
    g = torch.Generator().manual_seed(5)
    out = {}
    for i, (B, H, W) in enumerate([(2, 64, 64), (1, 37, 45), (3, 13, 70)]):
        pred = torch.rand(B, 3, H, W, generator=g).requires_grad_(True)
        tgt = torch.rand(B, 3, H, W, generator=g)
        if i == 0:
            tgt[1] = pred[1].detach()  # identical image: SSIM map of ones, clamp boundary
        out[f"loss{i}_pred"] = pred.detach()
        out[f"loss{i}_target"] = tgt
        for kind in ("standard_gs", "l1", "mse", "l1_mse"):
            cfg = dict(LOSS_CFG, type=kind)
            p = pred.detach().clone().requires_grad_(True)
            loss = R["loss"](p, tgt, cfg)
            (loss * torch.arange(1, B + 1, dtype=torch.float32)).sum().backward()
            out[f"loss{i}_{kind}_value"] = loss.detach()
            out[f"loss{i}_{kind}_grad"] = p.grad  # upstream gradient [1, 2, ..., B]
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DYNAWORLD_REFERENCE"),
                    help="checkout of nbardy/dynaworld (default: $DYNAWORLD_REFERENCE)")
    ap.add_argument("--only", nargs="*", default=["scenes", "losses", "tiled_grads", "overlap"],
                    choices=["scenes", "losses", "tiled_grads", "overlap"])
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("give the reference checkout with --reference PATH or DYNAWORLD_REFERENCE")
    torch.set_num_threads(8)
    R = ref_modules(Path(args.reference))

    if "scenes" in args.only:
        wl = syn.static64()
        save("static64", wl, render_case(R, wl))

        wl = syn.dynamic128(scale=1 / 16, image_scale=0.5, frames=2)
        save("dynamic128_small", wl, render_case(R, wl))

        wl = syn.multiview384(scale=0.01, image_scale=1 / 6, views=2)
        save("multiview384_small", wl, render_case(R, wl))

        wl = syn.clips256(scale=1 / 32, image_scale=0.25, clips=2, frames=2)
        save("clips256_small", wl, render_case(R, wl))

        wl = edge_workload()
        save("edge", wl, render_case(R, wl))

        # full-size dynamic128 (G=32768, 128x128): image of a 32x32 window of frame 5 only
        wl = syn.dynamic128().views(5, 6)
        save("dynamic128_crop", wl, render_case(R, wl, crop=(48, 40, 32, 32), with_grads=False, tiles=()),
             extra={"crop": torch.tensor([48, 40, 32, 32])}, lean=True)

    if "losses" in args.only:
        np.savez_compressed(HERE / "losses.npz", **to_np(loss_cases(R)))
        print("wrote losses.npz", flush=True)

    if "tiled_grads" in args.only:
        np.savez_compressed(HERE / "tiled_grads.npz", **to_np(tiled_grad_cases(R)))
        print("wrote tiled_grads.npz", flush=True)

    if "overlap" in args.only:
        np.savez_compressed(HERE / "overlap.npz", **to_np(overlap_cases(Path(args.reference))))
        print("wrote overlap.npz", flush=True)


if __name__ == "__main__":
    main()
