"""Every raster decomposition (one, two or four pixels per lane) against the reference's outputs.

The launch picks the decomposition from the grid size; GSB200_RASTER_PX forces it, so every
golden case runs through each.  Forward arithmetic per pixel does not depend on the
decomposition (images must be bit-identical); backward sums arrive in a different atomic order.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, grad_close, load_golden
from dynaworld_b200 import synthetic
from dynaworld_b200.config import B200RendererConfig
from dynaworld_b200.splats2d import PACKED, Splat2DOptions, render_splats2d
from gpu_helpers import render_raw
from oracle import splats2d_oracle as so2

pytestmark = pytest.mark.gpu

IMAGE_TOL = 1e-4
GRAD_REL = 1e-3
GRAD_KEYS = ("means", "log_scales", "quats", "opacity_logits", "sh")


@pytest.fixture(params=["1", "2", "4"])
def px(request, monkeypatch):
    monkeypatch.setenv("GSB200_RASTER_PX", request.param)
    return request.param


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("tile", [8, 16])
@pytest.mark.parametrize("segments", [1, 2, 4])
def test_golden_cases_under_each_decomposition(case, tile, segments, px):
    """Pixels per lane x backward list segments (each segment its own CTA, started from the
    forward's checkpoint)."""
    g = load_golden(case)
    wl = g.workload()
    out = render_raw(wl, B200RendererConfig(tile_size=tile, backward_segments=segments, depth=True))
    assert (out["image"] - g.t("ref_image")).abs().max().item() <= IMAGE_TOL
    torch.testing.assert_close(out["loss"], g.t("ref_loss"), rtol=1e-4, atol=2e-6)
    for k in GRAD_KEYS + (("velocity",) if wl.velocity is not None else ()):
        ok, e, s = grad_close(out[f"grad_{k}"], g.t(f"ref_grad_{k}"), GRAD_REL)
        assert ok, f"{case} px={px} segments={segments} {k}: max err {e:.3e} vs scale {s:.3e}"


@pytest.mark.parametrize("case", GOLDEN_CASES)
@pytest.mark.parametrize("cw", ["1", "4", "8"])
def test_golden_cases_under_each_cta_split(case, cw, px, monkeypatch):
    """A tile's warp blocks in one CTA or spread over 2, 4, 8 adjacent CTAs (GSB200_RASTER_CW
    warps per CTA; the default is 2 for the forward and the whole tile for the backward)."""
    monkeypatch.setenv("GSB200_RASTER_CW", cw)
    g = load_golden(case)
    wl = g.workload()
    out = render_raw(wl, B200RendererConfig(depth=True))
    assert (out["image"] - g.t("ref_image")).abs().max().item() <= IMAGE_TOL
    for k in GRAD_KEYS + (("velocity",) if wl.velocity is not None else ()):
        ok, e, s = grad_close(out[f"grad_{k}"], g.t(f"ref_grad_{k}"), GRAD_REL)
        assert ok, f"{case} px={px} cw={cw} {k}: max err {e:.3e} vs scale {s:.3e}"


def test_decompositions_agree_on_a_large_scene(monkeypatch):
    """multiview384 at a quarter of its Gaussians: 8 x 384^2 (4608 tiles), depth output and a
    depth gradient on; every (pixels per lane, segments) pair against (1, 1)."""
    wl = synthetic.multiview384(scale=0.25)
    outs = {}
    for px in ("1", "2"):
        monkeypatch.setenv("GSB200_RASTER_PX", px)
        for seg in (1, 2, 4):
            outs[(px, seg)] = render_raw(wl, B200RendererConfig(depth=True, backward_segments=seg),
                                         depth_loss=True)
    a = outs[("1", 1)]
    for key, b in outs.items():
        for k in ("image", "alpha", "depth"):
            assert torch.equal(a[k], b[k]), (key, k)
        for k in GRAD_KEYS:
            ok, e, s = grad_close(b[f"grad_{k}"], a[f"grad_{k}"], 1e-4)
            assert ok, f"{key} {k}: {e:.3e} vs {s:.3e}"


def test_packed_2d_under_each_decomposition(px):
    rng = np.random.default_rng(21)
    B, G, H, W = 2, 600, 70, 90
    packed = np.zeros((B, G, 7), np.float32)
    packed[..., 0] = rng.uniform(-5, W + 5, (B, G))
    packed[..., 1] = rng.uniform(-5, H + 5, (B, G))
    ang = rng.uniform(0, 2 * np.pi, (B, G))
    packed[..., 2], packed[..., 3] = np.cos(ang), np.sin(ang)
    packed[..., 4:6] = rng.uniform(0.8, 9.0, (B, G, 2))
    packed[..., 6] = rng.uniform(0.05, 0.9, (B, G))
    feats = rng.uniform(0, 1, (B, G, 3)).astype(np.float32)
    depths = rng.uniform(0, 1, (B, G)).astype(np.float32)
    go = rng.normal(size=(B, 3, H, W)).astype(np.float32)
    p = torch.tensor(packed, device="cuda:0", requires_grad=True)
    f = torch.tensor(feats, device="cuda:0", requires_grad=True)
    image, _w = render_splats2d(PACKED, H, W, Splat2DOptions(background=(0.2, 0.4, 0.6)), colors=f,
                                depths=torch.tensor(depths, device="cuda:0"), packed=p)
    (image * torch.tensor(go, device="cuda:0")).sum().backward()
    for b in range(B):
        ref, _ = so2.render_packed(packed[b], depths[b], feats[b], H, W, background=(0.2, 0.4, 0.6))
        assert np.abs(image[b].detach().cpu().numpy() - ref).max() <= 2e-5
        mean, A, Bc, C, o = so2.packed_to_conic(packed[b])
        g = so2.blend_2d_backward(mean, A, Bc, C, o, feats[b], depths[b], H, W, go[b],
                                  background=(0.2, 0.4, 0.6))
        pg = so2.packed_grads(packed[b], g)
        got = p.grad[b].cpu().double().numpy()
        for k in range(7):
            assert np.abs(got[:, k] - pg[:, k]).max() <= 2e-3 * np.abs(pg[:, k]).max() + 1e-7
