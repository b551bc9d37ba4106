"""The 2-D oracle against the reference's own float64 accuracy harness, and the host-side checks of
the 2-D entry (no GPU needed)."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import load_golden
from dynaworld_b200 import _lib
from oracle import splats2d_oracle as so

ACC = load_golden("splats2d_accuracy")
CASES = list(range(int(ACC["n_cases"])))


def case(i):
    p = f"c{i}_"
    H, W, G, set_index, seed = (int(v) for v in ACC[p + "size"])
    return dict(H=H, W=W, G=G, packed=ACC[p + "packed"].astype(np.float64), depths=ACC[p + "depths"],
                features=ACC[p + "features"].astype(np.float64), target=ACC[p + "target"].astype(np.float64),
                background=ACC[p + "background"], image=ACC[p + "image"], loss=float(ACC[p + "loss"]),
                packed_grad=ACC[p + "packed_grad"], feature_grad=ACC[p + "feature_grad"])


def test_fixture_covers_the_harness_grid():
    sizes = {tuple(int(v) for v in ACC[f"c{i}_size"][:3]) for i in CASES}
    for hw in (16, 32):
        for g in (4, 8, 16):
            assert (hw, hw, g) in sizes
    assert len(CASES) >= 18
    assert np.allclose(ACC["taichi_cfg"], [1.0 / 255.0, 0.99, 0.9999])


@pytest.mark.parametrize("rule", ["saturation", "transmittance"])
@pytest.mark.parametrize("i", CASES)
def test_oracle_matches_reference_harness(i, rule):
    c = case(i)
    img, _w = so.render_packed(c["packed"], c["depths"], c["features"], c["H"], c["W"], background=c["background"],
                               rule=rule)
    assert np.abs(img - c["image"]).max() <= 1e-12
    loss, d_img = so.mse_loss_and_grad(img, c["target"])
    assert abs(loss - c["loss"]) <= 1e-12
    mean, A, B, C, o = so.packed_to_conic(c["packed"])
    g = so.blend_2d_backward(mean, A, B, C, o, c["features"], c["depths"], c["H"], c["W"], d_img,
                             background=c["background"], rule=rule)
    pg = so.packed_grads(c["packed"], g)
    assert np.abs(pg - c["packed_grad"]).max() <= 1e-10 * max(1.0, np.abs(c["packed_grad"]).max())
    assert np.abs(g["colors"] - c["feature_grad"]).max() <= 1e-10 * max(1.0, np.abs(c["feature_grad"]).max())


def test_oracle_backward_matches_finite_differences_with_weight_gradient():
    """d_weight path and a clamped splat, which the harness cases do not reach."""
    rng = np.random.default_rng(3)
    G, H, W = 6, 12, 10
    packed = np.zeros((G, 7))
    packed[:, 0] = rng.uniform(2, 8, G)
    packed[:, 1] = rng.uniform(2, 10, G)
    ang = rng.uniform(0, 2 * np.pi, G)
    packed[:, 2], packed[:, 3] = np.cos(ang), np.sin(ang)
    packed[:, 4:6] = rng.uniform(1.2, 3.0, (G, 2))
    packed[:, 6] = rng.uniform(0.2, 0.9, G)
    packed[0, 6] = 1.5  # alpha clamped to 0.99 near its centre
    feats = rng.uniform(0, 1, (G, 3))
    depths = rng.permutation(G).astype(np.float64)
    go = rng.normal(size=(3, H, W))
    gw = rng.normal(size=(H, W))
    bg = (0.2, 0.3, 0.4)

    def f(p, ft):
        img, w = so.render_packed(p, depths, ft, H, W, background=bg, alpha_threshold=1e-3)
        return float(np.sum(go * img) + np.sum(gw * w))

    mean, A, B, C, o = so.packed_to_conic(packed)
    g = so.blend_2d_backward(mean, A, B, C, o, feats, depths, H, W, go, gw, background=bg, alpha_threshold=1e-3)
    pg = so.packed_grads(packed, g)
    h = 1e-6
    for gi in range(G):
        for k in range(7):
            pp, pm = packed.copy(), packed.copy()
            pp[gi, k] += h
            pm[gi, k] -= h
            fd = (f(pp, feats) - f(pm, feats)) / (2 * h)
            assert abs(fd - pg[gi, k]) <= 1e-4 * max(1.0, abs(fd)), (gi, k, fd, pg[gi, k])
        for k in range(3):
            fp, fm = feats.copy(), feats.copy()
            fp[gi, k] += h
            fm[gi, k] -= h
            fd = (f(packed, fp) - f(packed, fm)) / (2 * h)
            assert abs(fd - g["colors"][gi, k]) <= 1e-6 * max(1.0, abs(fd))


def test_conic_rule_culls_like_snugbox():
    """Conic contract: opacity at or below the threshold, a <= 0, c <= 0 or a c - b^2 <= 1e-8 draw
    nothing (gsplat_kernels.metal:57-59)."""
    means = np.array([[4.0, 4.0]] * 4)
    conics = np.array([[0.5, 0.0, 0.5], [-0.5, 0.0, 0.5], [0.5, 0.5, 0.5], [0.5, 0.0, 0.5]])
    ops = np.array([1.0 / 255.0, 0.5, 0.5, 0.5])
    cols = np.ones((4, 3))
    img, w = so.render_conic(means, conics, cols, ops, np.arange(4.0), 8, 8)
    only_last, w_last = so.render_conic(means[3:], conics[3:], cols[3:], ops[3:], np.zeros(1), 8, 8)
    assert np.array_equal(img, only_last) and np.array_equal(w, w_last)


def test_splats2d_structs_match_header():
    # 4 ints + 6 pointers; 5 pointers
    assert ctypes.sizeof(_lib.Splats2D) == 16 + 6 * 8
    assert ctypes.sizeof(_lib.Splats2DGrads) == 5 * 8


def test_splats2d_argument_errors_are_host_side():
    L = _lib.load()
    s = _lib.Splats2D()
    s.n_views, s.n_gaussians, s.format = 1, 4, 5  # unknown format
    s.colors = s.packed = 16
    assert L.gsb_splats2d_order(ctypes.byref(s), 16, 16, 16, 1 << 20, None) == 7
    s.format = _lib.SPLATS2D_CONIC  # conic format without its arrays
    assert L.gsb_splats2d_order(ctypes.byref(s), 16, 16, 16, 1 << 20, None) == 7
    s.format = _lib.SPLATS2D_PACKED
    s.n_gaussians = 0
    assert L.gsb_splats2d_order(ctypes.byref(s), 16, 16, 16, 1 << 20, None) == 1
    s.n_gaussians = 4
    o = _lib.Options()
    o.tile_size, o.near_plane, o.flags = 16, 1e-4, _lib.RENDER_TILED_COMPAT
    assert L.gsb_splats2d_preprocess(ctypes.byref(s), 8, 8, ctypes.byref(o), 16, 16, 16, 16, 16, 1 << 20,
                                     None) == 7
    assert L.gsb_splats2d_order_workspace(ctypes.byref(s)) > 4 * 8


def test_python_contracts_validate_shapes_before_touching_a_device():
    from dynaworld_b200 import gsplat_bridge, packed_rasterizer

    cfg = gsplat_bridge.RasterConfig(height=8, width=8)
    with pytest.raises(ValueError, match="means2d"):
        gsplat_bridge.rasterize_projected_gaussians(torch.zeros(4, 3), torch.zeros(4, 3), torch.zeros(4, 3),
                                                    torch.zeros(4), torch.zeros(4), cfg)
    with pytest.raises(ValueError, match="opacities"):
        gsplat_bridge.rasterize_projected_gaussians(torch.zeros(4, 2), torch.zeros(4, 3), torch.zeros(4, 3),
                                                    torch.zeros(4, 1), torch.zeros(4), cfg)
    with pytest.raises(ValueError, match=r"\[G,7\]"):
        packed_rasterizer.rasterize(torch.zeros(4, 6), torch.zeros(4, 1), torch.zeros(4, 3), (8, 8),
                                    packed_rasterizer.RasterConfig())
    with pytest.raises(ValueError, match="antialias"):
        packed_rasterizer.RasterConfig(antialias=True).options()
    with pytest.raises(RuntimeError, match="CUDA"):  # no CPU fallback
        packed_rasterizer.rasterize(torch.zeros(4, 7), torch.zeros(4, 1), torch.zeros(4, 3), (8, 8),
                                    packed_rasterizer.RasterConfig())
