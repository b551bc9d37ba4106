"""CUDA gradients w.r.t. the cameras against the reference's autograd (camera_grads.npz).

The reference's implicit-camera models learn fx, fy, cx, cy, camera_to_world and lens distortion
through the render call (gs_models/implicit_camera.py:146-262); render_b200_3dgs_batch must give
those tensors the same gradients.  Tolerance as the other gradient parity tests: max |g - g_ref|
<= 1e-3 * max |g_ref| per tensor.
"""
import numpy as np
import pytest
import torch

from conftest import grad_close, load_golden
from dynaworld_b200.losses import reconstruction_loss_per_image
from dynaworld_b200.renderer import render_b200, render_b200_3dgs_batch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
CAM = load_golden("camera_grads")
NCOEF = {"pinhole": 0, "radial_tangential": 5, "opencv_fisheye": 4}


class Camera:
    def __init__(self, fx, fy, cx, cy, camera_to_world, lens_model="pinhole", distortion=None):
        self.fx, self.fy, self.cx, self.cy = fx, fy, cx, cy
        self.camera_to_world = camera_to_world
        self.lens_model, self.distortion = lens_model, distortion


def case(name):
    g = {k[len(name) + 1:]: v for k, v in CAM.items() if k.startswith(name + "_")}
    t = {k: torch.from_numpy(np.array(v)) for k, v in g.items() if np.array(v).dtype.kind in "fiu"}
    lenses = [str(s) for s in g["lens_models"]] if "lens_models" in g else None
    return t, lenses


def check(got, ref, label):
    ok, e, s = grad_close(got.detach().cpu(), ref, 1e-3)
    assert ok, f"{label}: max err {e:.3e} vs scale {s:.3e}"


@pytest.mark.parametrize("name", ["pin", "lens"])
@pytest.mark.parametrize("px", ["1", "2"])
def test_camera_gradients_through_dropin_api(name, px, monkeypatch):
    monkeypatch.setenv("GSB200_RASTER_PX", px)
    t, lenses = case(name)
    H, W = int(t["height"]), int(t["width"])
    B = t["fx"].shape[0]
    act = {k: t[f"act_{k}"].to(DEV).requires_grad_(True) for k in ("xyz", "scales", "quats", "opacities", "rgbs")}
    fx, fy, cx, cy = (t[k].to(DEV).requires_grad_(True) for k in ("fx", "fy", "cx", "cy"))
    c2w = t["camera_to_world"].to(DEV).requires_grad_(True)
    dist = None
    if lenses is None:
        img = render_b200_3dgs_batch(act["xyz"], act["scales"], act["quats"], act["opacities"], act["rgbs"], H, W,
                                     fx, fy, cx, cy, camera_to_world=c2w)
    else:
        dist = t["distortion"].to(DEV).requires_grad_(True)
        cams = [Camera(fx[b], fy[b], cx[b], cy[b], c2w[b], lenses[b],
                       None if lenses[b] == "pinhole" else dist[b, : NCOEF[lenses[b]]]) for b in range(B)]
        img = render_b200_3dgs_batch(act["xyz"], act["scales"], act["quats"], act["opacities"], act["rgbs"], H, W,
                                     fx, fy, cx, cy, cameras=cams, projection_mode="camera_model",
                                     camera_to_world=c2w)
    assert (img.detach().cpu() - t["image"]).abs().max().item() <= 1e-4
    reconstruction_loss_per_image(img, t["target"].to(DEV)).sum().backward()
    check(torch.stack([fx.grad, fy.grad, cx.grad, cy.grad], -1), t["grad_intrinsics"], f"{name} intrinsics")
    check(c2w.grad, t["grad_c2w"], f"{name} camera_to_world")
    if dist is not None:
        check(dist.grad, t["grad_distortion"], f"{name} distortion")
    for k, v in act.items():
        check(v.grad, t[f"grad_act_{k}"], f"{name} {k}")


def test_raw_entry_camera_gradients_and_no_extra_work_without_them():
    """render_b200 takes intrinsics [B,4] / camera_to_world requiring grad; without them the
    camera stage is not launched."""
    from dynaworld_b200 import _lib

    t, _ = case("pin")
    G = t["act_xyz"].shape[1]
    torch.manual_seed(0)
    means = t["act_xyz"][0].to(DEV).requires_grad_(True)
    log_scales = torch.log(t["act_scales"][0]).to(DEV)
    quats = t["act_quats"][0].to(DEV)
    logits = torch.logit(t["act_opacities"][0].clamp(1e-4, 1 - 1e-4)).to(DEV)
    sh = (torch.randn(G, 4, 3) * 0.1).to(DEV)
    intr = torch.stack([t["fx"], t["fy"], t["cx"], t["cy"]], -1).to(DEV)
    c2w = t["camera_to_world"].to(DEV)
    H, W = int(t["height"]), int(t["width"])

    def run(cam_grad):
        i = intr.clone().requires_grad_(cam_grad)
        c = c2w.clone().requires_grad_(cam_grad)
        img, _a, _d = render_b200(means, log_scales, quats, logits, sh, intrinsics=i, camera_to_world=c,
                                  height=H, width=W)
        before = _lib.lib().gsb_kernel_launches()
        reconstruction_loss_per_image(img, t["target"].to(DEV)).sum().backward()
        torch.cuda.synchronize()
        return i.grad, c.grad, _lib.lib().gsb_kernel_launches() - before

    gi, gc, n_with = run(True)
    assert gi is not None and gc is not None and torch.isfinite(gc).all() and gc[:, 3].abs().sum() == 0
    assert gi.abs().sum() > 0 and gc[:, :3].abs().sum() > 0
    _gi, _gc, n_without = run(False)
    assert n_with == n_without + 1  # exactly the camera stage
