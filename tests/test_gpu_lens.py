"""CUDA camera_model projection (radial-tangential, OpenCV fisheye, pinhole views in one batch)
against the reference's camera_model render (golden fixtures) and the oracle.

Tolerances as the other parity tests: image within 1e-4 absolute, gradients within 1e-3 of each
tensor's largest magnitude.
"""
import numpy as np
import pytest
import torch

from conftest import grad_close, load_golden
from dynaworld_b200.config import B200RendererConfig
from dynaworld_b200.losses import reconstruction_loss_per_image
from dynaworld_b200.renderer import render_b200_3dgs_batch
from gpu_helpers import DEV, records_np, render_raw, stages
from oracle import splat_oracle as so

pytestmark = pytest.mark.gpu

IMAGE_TOL = 1e-4
GRAD_REL = 1e-3
LENS_CASES = ["lens_mixed", "lens_wide"]


class Camera:
    """CameraSpec's fields (camera.py:11-31)."""

    def __init__(self, fx, fy, cx, cy, camera_to_world, lens_model="pinhole", distortion=None):
        self.fx, self.fy, self.cx, self.cy = fx, fy, cx, cy
        self.camera_to_world = camera_to_world
        self.lens_model, self.distortion = lens_model, distortion


def lens_of(g):
    """CameraSpec-style lens models and coefficient lists (the fixture stores rows padded to 5)."""
    from dynaworld_b200._lib import LENS_COEFFS

    models = [str(s) for s in g["lens_models"]]
    dist = [None if m == "pinhole" else g["distortion"][b][: LENS_COEFFS[m]].tolist() for b, m in enumerate(models)]
    return models, dist


@pytest.mark.parametrize("case", LENS_CASES)
@pytest.mark.parametrize("px", ["1", "2"])
def test_lens_image_loss_and_gradients_match_reference(case, px, monkeypatch):
    monkeypatch.setenv("GSB200_RASTER_PX", px)
    g = load_golden(case)
    wl = g.workload()
    models, dist = lens_of(g)
    out = render_raw(wl, lens_models=models, distortion=dist)
    err = (out["image"] - g.t("ref_image")).abs().max().item()
    assert err <= IMAGE_TOL, f"image max abs err {err:.3e}"
    torch.testing.assert_close(out["loss"], g.t("ref_loss"), rtol=1e-4, atol=2e-6)
    for k in ("means", "log_scales", "quats", "opacity_logits", "sh") + (("velocity",) if wl.velocity is not None
                                                                          else ()):
        ok, e, s = grad_close(out[f"grad_{k}"], g.t(f"ref_grad_{k}"), GRAD_REL)
        assert ok, f"{case} {k}: max err {e:.3e} vs scale {s:.3e}"


@pytest.mark.parametrize("case", LENS_CASES)
def test_lens_records_match_reference_projection(case):
    """Projected means and inverse covariances in depth order (projection.py:253-276)."""
    from dynaworld_b200.render import lens_tensors

    g = load_golden(case)
    wl = g.workload()
    models, dist = lens_of(g)
    B, G = wl.n_views, wl.n_gaussians
    _img, _a, _d, state = stages(wl, lens=lens_tensors(models, dist, B, DEV))
    rec = records_np(state, B, G)
    ref_m2 = g["ref_means2d"]
    vis = g["ref_proj_opacity"][..., 0] > 0
    assert np.abs(rec[..., 0:2] - ref_m2)[vis].max() <= 2e-3
    ref_inv = g["ref_inv_cov"]
    A, Bc, C = rec[..., 2], rec[..., 3], rec[..., 4]
    scale = np.abs(ref_inv).reshape(B, G, 4).max(-1)
    assert (np.abs(A - ref_inv[..., 0, 0]) / scale)[vis].max() <= 1e-3
    assert (np.abs(C - ref_inv[..., 1, 1]) / scale)[vis].max() <= 1e-3
    assert (np.abs(Bc - (ref_inv[..., 0, 1] + ref_inv[..., 1, 0])) / scale)[vis].max() <= 2e-3


def test_dropin_camera_model_batch_api():
    """render_b200_3dgs_batch with CameraSpec cameras and projection_mode="camera_model", the call
    render_pytorch_3dgs_batch receives from rendering.py (dense.py:170-202)."""
    g = load_golden("lens_mixed")
    wl = g.workload()
    models, dist = lens_of(g)
    leaves = {k: getattr(wl, k).double().requires_grad_(False) for k in ("means", "log_scales", "quats",
                                                                         "opacity_logits", "sh")}
    raw = so.RawGaussians(*(leaves[k] for k in ("means", "log_scales", "quats", "opacity_logits", "sh")),
                          wl.velocity.double() if wl.velocity is not None else None)
    m, s, q, o, rgb = (t.float().to(DEV) for t in so.activate(raw, wl.times.double(), wl.camera_to_world,
                                                                 wl.views_per_set))
    cams = [Camera(float(wl.fx[b]), float(wl.fy[b]), float(wl.cx[b]), float(wl.cy[b]), wl.camera_to_world[b],
                   models[b], dist[b]) for b in range(wl.n_views)]
    img = render_b200_3dgs_batch(m, s, q, o, rgb, wl.height, wl.width, wl.fx, wl.fy, wl.cx, wl.cy, cameras=cams,
                                 projection_mode="camera_model", camera_to_world=wl.camera_to_world.to(DEV))
    assert (img.detach().cpu() - g.t("ref_image")).abs().max().item() <= IMAGE_TOL
    # legacy_pinhole on the same cameras ignores the lenses: a different image
    img2 = render_b200_3dgs_batch(m, s, q, o, rgb, wl.height, wl.width, wl.fx, wl.fy, wl.cx, wl.cy, cameras=cams,
                                  projection_mode="legacy_pinhole", camera_to_world=wl.camera_to_world.to(DEV))
    assert (img2 - img).abs().max().item() > 1e-2
    loss = reconstruction_loss_per_image(img, wl.target.to(DEV))
    torch.testing.assert_close(loss.cpu(), g.t("ref_loss"), rtol=1e-4, atol=2e-6)


def test_lens_pinhole_views_are_unchanged():
    """A camera_model batch whose views are all pinhole renders exactly as legacy_pinhole
    (projection.py:238-251 delegates to common.py)."""
    g = load_golden("dynamic128_small")
    wl = g.workload()
    a = render_raw(wl, grads=False)
    b = render_raw(wl, grads=False, lens_models=["pinhole"] * wl.n_views)
    assert torch.equal(a["image"], b["image"])
