"""The oracle's camera_model (distorted-lens) projection against the reference's own outputs."""
import pytest
import torch

from conftest import grad_close, load_golden
from oracle import splat_oracle as so

LENS_CASES = ["lens_mixed", "lens_wide"]


def lens_args(g):
    return [str(s) for s in g["lens_models"]], g.t("distortion")


@pytest.mark.parametrize("case", LENS_CASES)
def test_lens_projection_matches_reference(case):
    g = load_golden(case)
    wl = g.workload()
    lenses, dist = lens_args(g)
    raw = so.RawGaussians(wl.means, wl.log_scales, wl.quats, wl.opacity_logits, wl.sh, wl.velocity)
    m, s, q, o, rgb = so.activate(raw, wl.times, wl.camera_to_world, wl.views_per_set)
    m2, inv, cov, op, _rgb, _z, _order = so.project_batch(m, s, q, o, rgb, wl.fx, wl.fy, wl.cx, wl.cy,
                                                          wl.camera_to_world, lens_models=lenses, distortion=dist)
    torch.testing.assert_close(m2, g.t("ref_means2d"), rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(cov, g.t("ref_cov2d"), rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(op, g.t("ref_proj_opacity"), rtol=0, atol=0)
    # inverse covariances: compare relative to each Gaussian's scale
    ref_inv = g.t("ref_inv_cov")
    err = (inv - ref_inv).abs().amax(dim=(-1, -2)) / ref_inv.abs().amax(dim=(-1, -2)).clamp_min(1e-6)
    assert err.max().item() <= 1e-3


@pytest.mark.parametrize("case", LENS_CASES)
def test_lens_image_loss_and_gradients_match_reference(case):
    g = load_golden(case)
    wl = g.workload()
    lenses, dist = lens_args(g)
    leaves = {k: getattr(wl, k).double().requires_grad_(True) for k in ("means", "log_scales", "quats",
                                                                        "opacity_logits", "sh")}
    vel = wl.velocity.double().requires_grad_(True) if wl.velocity is not None else None
    raw = so.RawGaussians(leaves["means"], leaves["log_scales"], leaves["quats"], leaves["opacity_logits"],
                          leaves["sh"], vel)
    m, s, q, o, rgb = so.activate(raw, wl.times.double(), wl.camera_to_world, wl.views_per_set)
    key = so.camera_depth_fp32(m.float(), wl.camera_to_world)
    img, _, _ = so.render_dense(m, s, q, o, rgb, wl.height, wl.width, wl.fx, wl.fy, wl.cx, wl.cy,
                                wl.camera_to_world, sort_key=key, lens_models=lenses, distortion=dist)
    assert (img.float() - g.t("ref_image")).abs().max().item() <= 5e-6
    loss = so.reconstruction_loss_per_image(img, wl.target.double())
    torch.testing.assert_close(loss.float(), g.t("ref_loss"), rtol=1e-5, atol=1e-6)
    loss.sum().backward()
    for k, leaf in leaves.items():
        ok, err, scale = grad_close(leaf.grad, g.t(f"ref_grad_{k}"))
        assert ok, f"{k}: max err {err:.3e} vs scale {scale:.3e}"
    if vel is not None:
        ok, err, scale = grad_close(vel.grad, g.t("ref_grad_velocity"))
        assert ok, f"velocity: max err {err:.3e} vs scale {scale:.3e}"


def test_lens_cases_differ_from_pinhole():
    """The distortion is strong enough to matter: the pinhole projection of the same scene differs."""
    g = load_golden("lens_wide")
    wl = g.workload()
    raw = so.RawGaussians(wl.means, wl.log_scales, wl.quats, wl.opacity_logits, wl.sh, wl.velocity)
    m, s, q, o, rgb = so.activate(raw, wl.times, wl.camera_to_world, wl.views_per_set)
    m2, *_ = so.project_batch(m, s, q, o, rgb, wl.fx, wl.fy, wl.cx, wl.cy, wl.camera_to_world)
    assert (m2 - g.t("ref_means2d")).abs().max().item() > 5.0
