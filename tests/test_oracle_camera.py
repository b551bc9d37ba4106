"""The oracle's gradients w.r.t. the cameras (intrinsics, camera_to_world, lens distortion)
against the reference's own autograd (tests/golden/camera_grads.npz)."""
import numpy as np
import pytest
import torch

from conftest import grad_close, load_golden
from oracle import splat_oracle as so

CAM = load_golden("camera_grads")


def case(name):
    g = {k[len(name) + 1:]: v for k, v in CAM.items() if k.startswith(name + "_")}
    t = {k: torch.from_numpy(np.array(v)) for k, v in g.items() if np.array(v).dtype.kind in "fiu"}
    lenses = [str(s) for s in g["lens_models"]] if "lens_models" in g else None
    return t, lenses


@pytest.mark.parametrize("name", ["pin", "lens"])
def test_camera_gradients_match_reference(name):
    t, lenses = case(name)
    H, W = int(t["height"]), int(t["width"])
    act = {k: t[f"act_{k}"].double().requires_grad_(True) for k in ("xyz", "scales", "quats", "opacities", "rgbs")}
    intr = torch.stack([t["fx"], t["fy"], t["cx"], t["cy"]], -1).double().requires_grad_(True)
    c2w = t["camera_to_world"].double().requires_grad_(True)
    dist = t["distortion"].double().requires_grad_(True) if lenses else None
    key = so.camera_depth_fp32(act["xyz"].float(), t["camera_to_world"])
    img, _, _ = so.render_dense(act["xyz"], act["scales"], act["quats"], act["opacities"], act["rgbs"], H, W,
                                intr[:, 0], intr[:, 1], intr[:, 2], intr[:, 3], c2w, sort_key=key,
                                lens_models=lenses, distortion=dist)
    assert (img.float() - t["image"]).abs().max().item() <= 5e-6
    so.reconstruction_loss_per_image(img, t["target"].double()).sum().backward()
    for got, ref, label in ((intr.grad, t["grad_intrinsics"], "intrinsics"), (c2w.grad, t["grad_c2w"], "c2w"),
                            *(((dist.grad, t["grad_distortion"], "distortion"),) if lenses else ())):
        ok, e, s = grad_close(got, ref, 1e-3)
        assert ok, f"{name} {label}: {e:.3e} vs {s:.3e}"
    for k, v in act.items():
        ok, e, s = grad_close(v.grad, t[f"grad_act_{k}"], 1e-3)
        assert ok, f"{name} {k}: {e:.3e} vs {s:.3e}"
