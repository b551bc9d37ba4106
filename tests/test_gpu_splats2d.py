"""CUDA 2-D entry (conic and packed contracts) against the reference's accuracy harness and the
float64 oracle.

Tolerances: the reference harness's own (splat_renderer_accuracy.py:62-70: image max 5e-4 / mean
5e-5, loss 5e-5, gradients max 2e-3 / mean 1e-4), and tighter checks of our own (image 2e-5 abs,
gradients 1e-3 of the largest magnitude) since the blend is float32 throughout.
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from dynaworld_b200 import gsplat_bridge, packed_rasterizer
from dynaworld_b200.splats2d import CONIC, PACKED, Splat2DOptions, render_splats2d
from oracle import splats2d_oracle as so

pytestmark = pytest.mark.gpu

ACC = load_golden("splats2d_accuracy")
CASES = list(range(int(ACC["n_cases"])))
TOL = dict(zip(["image_max", "image_mean", "loss", "pg_max", "pg_mean", "fg_max", "fg_mean"],
               ACC["tolerances"].tolist()))
DEV = "cuda:0"


def case(i):
    p = f"c{i}_"
    H, W, G, _set, _seed = (int(v) for v in ACC[p + "size"])
    return dict(H=H, W=W, G=G, packed=ACC[p + "packed"], depths=ACC[p + "depths"], features=ACC[p + "features"],
                target=ACC[p + "target"], background=ACC[p + "background"], image=ACC[p + "image"],
                loss=float(ACC[p + "loss"]), packed_grad=ACC[p + "packed_grad"], feature_grad=ACC[p + "feature_grad"])


def cuda(a, grad=False):
    t = torch.tensor(np.asarray(a), dtype=torch.float32, device=DEV)
    return t.requires_grad_(grad)


def packed_to_conic_f32(packed: np.ndarray):
    """The reference's packed -> conic conversion (raw_metal_mlx_bridge.py:106-121) in float32."""
    p = np.asarray(packed, dtype=np.float32)
    ux, uy, s0, s1 = p[:, 2], p[:, 3], p[:, 4], p[:, 5]
    i0, i1 = np.float32(1) / (s0 * s0), np.float32(1) / (s1 * s1)
    conics = np.stack([ux * ux * i0 + uy * uy * i1, ux * uy * (i0 - i1), uy * uy * i0 + ux * ux * i1], axis=-1)
    return p[:, 0:2].copy(), conics, p[:, 6].copy()


def harness_compare(image, loss, pg, fg, c):
    img_d = np.abs(image - c["image"])
    assert img_d.max() <= TOL["image_max"] and img_d.mean() <= TOL["image_mean"]
    assert img_d.max() <= 2e-5
    assert abs(loss - c["loss"]) <= TOL["loss"]
    for got, ref, mx, mean in ((pg, c["packed_grad"], "pg_max", "pg_mean"), (fg, c["feature_grad"], "fg_max",
                                                                            "fg_mean")):
        d = np.abs(got - ref)
        assert d.max() <= TOL[mx] and d.mean() <= TOL[mean]
        assert d.max() <= 1e-3 * np.abs(ref).max() + 1e-9


@pytest.mark.parametrize("i", CASES)
def test_packed_contract_matches_reference_harness(i):
    """What run_accuracy does with a renderer (splat_renderer_accuracy.py:586-600), through the
    taichi-style API: composite the background as taichi.py:309 does, mse loss, backward."""
    c = case(i)
    packed, feats = cuda(c["packed"], True), cuda(c["features"], True)
    cfg = packed_rasterizer.RasterConfig(tile_size=16, alpha_threshold=1.0 / 255.0, clamp_max_alpha=0.99,
                                         saturate_threshold=0.9999)
    r = packed_rasterizer.rasterize(packed, cuda(c["depths"]), feats, image_size=(c["W"], c["H"]), config=cfg)
    bg = cuda(c["background"])
    image = (r.image + (1.0 - r.image_weight).unsqueeze(-1).clamp(0.0, 1.0) * bg).permute(2, 0, 1)
    loss = (image - cuda(c["target"])).square().mean()
    loss.backward()
    harness_compare(image.detach().cpu().double().numpy(), float(loss.detach()), packed.grad.cpu().double().numpy(),
                    feats.grad.cpu().double().numpy(), c)


@pytest.mark.parametrize("i", CASES)
def test_conic_contract_matches_reference_harness(i):
    """The fast-mac bridge API on the same splats (packed -> conic as the reference converts it)."""
    c = case(i)
    m, q, o = packed_to_conic_f32(c["packed"])
    means, conics, ops, feats = cuda(m, True), cuda(q, True), cuda(o, True), cuda(c["features"], True)
    cfg = gsplat_bridge.RasterConfig(height=c["H"], width=c["W"], background=tuple(c["background"].tolist()))
    hwc = gsplat_bridge.rasterize_projected_gaussians(means, conics, feats, ops, cuda(c["depths"][:, 0]), cfg)
    image = hwc.permute(2, 0, 1)
    loss = (image - cuda(c["target"])).square().mean()
    loss.backward()
    assert np.abs(image.detach().cpu().double().numpy() - c["image"]).max() <= 2e-5
    assert abs(float(loss.detach()) - c["loss"]) <= TOL["loss"]
    # oracle gradients in the conic parameterisation (transmittance rule, float64)
    mean64, A, B, C = m.astype(np.float64), q[:, 0].astype(np.float64), 2.0 * q[:, 1], q[:, 2].astype(np.float64)
    img64, _w = so.blend_2d(mean64, A, B, C, o, c["features"], c["depths"], c["H"], c["W"],
                            background=c["background"], cull_conic=True)
    _l, d_img = so.mse_loss_and_grad(img64, c["target"].astype(np.float64))
    g = so.blend_2d_backward(mean64, A, B, C, o, c["features"], c["depths"], c["H"], c["W"], d_img,
                             background=c["background"], cull_conic=True)
    ref_conic = np.stack([g["A"], 2.0 * g["B"], g["C"]], axis=-1)
    for got, ref in ((means.grad, g["mean"]), (conics.grad, ref_conic), (ops.grad, g["opacity"]),
                     (feats.grad, g["colors"])):
        got = got.cpu().double().numpy()
        assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max() + 1e-9


def random_packed(rng, G, H, W, sigma=(0.8, 12.0), opacity=(0.05, 0.95)):
    packed = np.zeros((G, 7), dtype=np.float32)
    packed[:, 0] = rng.uniform(-0.1 * W, 1.1 * W, G)
    packed[:, 1] = rng.uniform(-0.1 * H, 1.1 * H, G)
    ang = rng.uniform(0, 2 * np.pi, G)
    packed[:, 2], packed[:, 3] = np.cos(ang), np.sin(ang)
    packed[:, 4:6] = np.exp(rng.uniform(np.log(sigma[0]), np.log(sigma[1]), (G, 2)))
    packed[:, 6] = rng.uniform(*opacity, G)
    feats = rng.uniform(0, 1, (G, 3)).astype(np.float32)
    depths = rng.uniform(0.1, 10.0, G).astype(np.float32)
    return packed, feats, depths


@pytest.mark.parametrize("tile", [8, 16])
def test_batched_packed_vs_oracle_with_weight_gradient(tile):
    """B=3 images of 1500 splats each, 131x97 (ragged tiles), loss on image and weight."""
    rng = np.random.default_rng(11)
    B, G, H, W = 3, 1500, 131, 97
    data = [random_packed(rng, G, H, W) for _ in range(B)]
    packed = cuda(np.stack([d[0] for d in data]), True)
    feats = cuda(np.stack([d[1] for d in data]), True)
    depths = cuda(np.stack([d[2] for d in data]))
    go = rng.normal(size=(B, 3, H, W)).astype(np.float32)
    gw = rng.normal(size=(B, H, W)).astype(np.float32)
    bg = (0.3, 0.6, 0.9)
    image, weight = render_splats2d(PACKED, H, W, Splat2DOptions(tile_size=tile, background=bg), colors=feats,
                                    depths=depths, packed=packed)
    ((image * cuda(go)).sum() + (weight * cuda(gw)).sum()).backward()
    for b in range(B):
        p, f, d = (x.astype(np.float64) for x in data[b])
        ref_img, ref_w = so.render_packed(p, d, f, H, W, background=bg)
        assert np.abs(image[b].detach().cpu().numpy() - ref_img).max() <= 2e-5
        assert np.abs(weight[b].detach().cpu().numpy() - ref_w).max() <= 2e-5
        mean, A, Bc, C, o = so.packed_to_conic(p)
        g = so.blend_2d_backward(mean, A, Bc, C, o, f, d, H, W, go[b], gw[b], background=bg)
        pg = so.packed_grads(p, g)
        got = packed.grad[b].cpu().double().numpy()
        # per column: positions, axes, sigmas and opacity have different scales
        for k in range(7):
            assert np.abs(got[:, k] - pg[:, k]).max() <= 2e-3 * np.abs(pg[:, k]).max() + 1e-7, k
        gf = feats.grad[b].cpu().double().numpy()
        assert np.abs(gf - g["colors"]).max() <= 1e-3 * np.abs(g["colors"]).max()


def test_batch_images_are_independent():
    rng = np.random.default_rng(5)
    data = [random_packed(rng, 300, 64, 80) for _ in range(2)]
    cfg = packed_rasterizer.RasterConfig()
    both = packed_rasterizer.rasterize_batch(cuda(np.stack([d[0] for d in data])),
                                             cuda(np.stack([d[2] for d in data])),
                                             cuda(np.stack([d[1] for d in data])), (80, 64), cfg)
    for b in range(2):
        one = packed_rasterizer.rasterize(cuda(data[b][0]), cuda(data[b][2]), cuda(data[b][1]), (80, 64), cfg)
        assert torch.equal(both.image[b], one.image) and torch.equal(both.image_weight[b], one.image_weight)


def test_tile_lists_agree_between_tile_sizes():
    rng = np.random.default_rng(9)
    p, f, d = random_packed(rng, 800, 100, 120)
    outs = []
    for tile in (8, 16):
        cfg = gsplat_bridge.RasterConfig(height=100, width=120, tile_size=tile)
        m, q, o = packed_to_conic_f32(p)
        outs.append(gsplat_bridge.rasterize_projected_gaussians(cuda(m), cuda(q), cuda(f), cuda(o), cuda(d), cfg))
    assert torch.allclose(outs[0], outs[1], atol=1e-6, rtol=0)


def test_edge_cases_conic():
    """Off-screen, culled (degenerate, non-positive, transparent) and clamped splats, a 1x1 and a
    ragged image, and an empty batch."""
    means = np.array([[-50.0, 3.0], [3.0, 3.0], [3.0, 3.0], [3.0, 3.0], [2.5, 2.0], [1.0, 1.0]], np.float32)
    conics = np.array([[0.5, 0, 0.5], [1e-5, 0, 1e-5 * 0.5], [-0.5, 0, 0.5], [0.5, 0, 0.5], [0.3, 0.1, 0.4],
                       [0.2, -0.05, 0.6]], np.float32)
    ops = np.array([0.9, 0.9, 0.9, 1.0 / 255.0, 3.0, 0.5], np.float32)  # [4] is clamped to 0.99
    cols = np.array([[1, 0, 0], [0, 1, 0], [0, 0, 1], [1, 1, 0], [0.2, 0.4, 0.6], [0.9, 0.1, 0.5]], np.float32)
    depths = np.arange(6, dtype=np.float32)[::-1].copy()
    for H, W in ((7, 5), (1, 1), (17, 33)):
        cm, cq, co, cc = cuda(means, True), cuda(conics, True), cuda(ops, True), cuda(cols, True)
        cfg = gsplat_bridge.RasterConfig(height=H, width=W, background=(0.1, 0.2, 0.3))
        out = gsplat_bridge.rasterize_projected_gaussians(cm, cq, cc, co, cuda(depths), cfg)
        go = np.random.default_rng(H).normal(size=(H, W, 3)).astype(np.float32)
        (out * cuda(go)).sum().backward()
        A, B, C = so.conic_to_abc(conics)
        kw = dict(background=(0.1, 0.2, 0.3), alpha_threshold=float(np.float32(1.0 / 255.0)), cull_conic=True)
        ref, _w = so.blend_2d(means, A, B, C, ops, cols, depths, H, W, **kw)
        assert np.abs(out.detach().cpu().numpy().transpose(2, 0, 1) - ref).max() <= 2e-5
        g = so.blend_2d_backward(means, A, B, C, ops, cols, depths, H, W, go.transpose(2, 0, 1), **kw)
        assert np.abs(cm.grad.cpu().numpy() - g["mean"]).max() <= 1e-3 * max(np.abs(g["mean"]).max(), 1e-3)
        assert np.abs(co.grad.cpu().numpy() - g["opacity"]).max() <= 1e-3 * max(np.abs(g["opacity"]).max(), 1e-3)
        assert float(cm.grad[1:4].abs().sum()) == 0.0  # culled splats get no gradient
    empty = gsplat_bridge.rasterize_projected_gaussians(
        cuda(np.zeros((2, 0, 2))), cuda(np.zeros((2, 0, 3))), cuda(np.zeros((2, 0, 3))), cuda(np.zeros((2, 0))),
        cuda(np.zeros((2, 0))), gsplat_bridge.RasterConfig(height=4, width=4, background=(0.5, 0.5, 0.5)))
    assert empty.shape == (2, 4, 4, 3) and torch.all(empty == 0.5)


def test_index_order_without_depths_equals_arange_depths():
    rng = np.random.default_rng(2)
    p, f, _d = random_packed(rng, 400, 48, 48)
    opt = Splat2DOptions()
    a, wa = render_splats2d(PACKED, 48, 48, opt, colors=cuda(f)[None], depths=None, packed=cuda(p)[None])
    b, wb = render_splats2d(PACKED, 48, 48, opt, colors=cuda(f)[None],
                            depths=torch.arange(400, dtype=torch.float32, device=DEV)[None], packed=cuda(p)[None])
    assert torch.equal(a, b) and torch.equal(wa, wb)


def test_conic_and_packed_formats_agree():
    rng = np.random.default_rng(4)
    p, f, d = random_packed(rng, 1000, 90, 110, opacity=(0.05, 0.5))
    m, q, o = packed_to_conic_f32(p)
    opt = Splat2DOptions(background=(1.0, 1.0, 1.0))
    a, _ = render_splats2d(PACKED, 90, 110, opt, colors=cuda(f)[None], depths=cuda(d)[None], packed=cuda(p)[None])
    b, _ = render_splats2d(CONIC, 90, 110, opt, colors=cuda(f)[None], depths=cuda(d)[None], means=cuda(m)[None],
                           conics=cuda(q)[None], opacities=cuda(o)[None])
    assert torch.allclose(a, b, atol=2e-5, rtol=0)
