"""NumPy float64 restatement of the reference's 2-D (already-projected) Gaussian rasterizers.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): what the tests compare the CUDA 2-D entry with, never a
compute path.  Citations are to files of nbardy/dynaworld.

Restated:
  * packed -> conic   src/benchmarks/raw_metal_mlx_bridge.py:106-121 (_packed_to_conics_mx);
                      the same quadratic form as src/benchmarks/splat_renderer_accuracy.py:
                      289-297 (tx = d.axis / s0, ty = d.perp / s1, q = tx^2 + ty^2)
  * blend, rule "saturation"    splat_renderer_accuracy.py:262-305 (torch_reference_rasterize):
                      active = alpha > threshold and W < saturate, w = alpha (1 - W),
                      image = accum + (1 - W) background
  * blend, rule "transmittance" third_party/fast-mac-gsplat-scaffold/csrc/metal/
                      gsplat_kernels.metal:160-204 (tile_forward): skip power > 0 and
                      alpha < threshold, w = T alpha, T *= 1 - alpha, stop once T < threshold,
                      image = accum + T background; culling of snugbox_count (:57-59)
  * gradients         the exact derivative of the blend (what torch autograd gives through
                      torch_reference_rasterize): reverse scan with the suffix colour
                      R_j = alpha_j c_j + (1 - alpha_j) R_{j+1}, zero through a clamped alpha.
                      The Metal scaffold's tile_backward (gsplat_kernels.metal:206-297) differs
                      from this derivative in two places -- its suffix update leaves out the
                      alpha_j factor and it ignores the 0.99 clamp -- and is not followed.

Pinned against the reference's own torch_reference_rasterize run in float64 with autograd
(tests/golden/make_golden_2d.py -> splats2d_accuracy.npz).
"""
from __future__ import annotations

import numpy as np

PACKED_FLOATS = 7


def packed_to_conic(packed: np.ndarray):
    """packed [..., 7] -> (mean [..., 2], A, B, C, opacity) with q = A dx^2 + B dx dy + C dy^2
    (B is twice the reference's conic_b)."""
    p = np.asarray(packed, dtype=np.float64)
    ax, ay, s0, s1 = p[..., 2], p[..., 3], p[..., 4], p[..., 5]
    u0, u1 = 1.0 / (s0 * s0), 1.0 / (s1 * s1)
    A = ax * ax * u0 + ay * ay * u1
    B = 2.0 * ax * ay * (u0 - u1)
    C = ay * ay * u0 + ax * ax * u1
    return p[..., 0:2], A, B, C, p[..., 6]


def conic_to_abc(conics: np.ndarray):
    """Reference conic (a, b, c), q = a dx^2 + 2 b dx dy + c dy^2 -> (A, B, C)."""
    q = np.asarray(conics, dtype=np.float64)
    return q[..., 0], 2.0 * q[..., 1], q[..., 2]


def blend_order(depths: np.ndarray | None, G: int) -> np.ndarray:
    if depths is None:
        return np.arange(G)
    return np.argsort(np.asarray(depths, dtype=np.float64).reshape(-1), kind="stable")


def _pixels(H: int, W: int):
    y, x = np.meshgrid(np.arange(H, dtype=np.float64), np.arange(W, dtype=np.float64), indexing="ij")
    return x + 0.5, y + 0.5


def blend_2d(mean, A, B, C, opacity, colors, depths, H: int, W: int, *, alpha_threshold: float = 1.0 / 255.0,
             alpha_clamp: float = 0.99, t_threshold: float = 1e-4, background=(0.0, 0.0, 0.0),
             rule: str = "transmittance", cull_conic: bool = False, keep_trace: bool = False):
    """One image.  Returns image [3,H,W], weight sum [H,W] and (keep_trace) the per-entry
    trace the backward needs."""
    mean = np.asarray(mean, dtype=np.float64)
    colors = np.asarray(colors, dtype=np.float64)
    A, B, C, opacity = (np.asarray(v, dtype=np.float64) for v in (A, B, C, opacity))
    G = mean.shape[0]
    px, py = _pixels(H, W)
    bg = np.asarray(background, dtype=np.float64)
    accum = np.zeros((3, H, W))
    T = np.ones((H, W))
    Wsum = np.zeros((H, W))
    done = np.zeros((H, W), dtype=bool)
    trace = []
    for g in blend_order(depths, G):
        if cull_conic:
            hb = 0.5 * B[g]
            if not (opacity[g] > alpha_threshold and A[g] > 0 and C[g] > 0 and A[g] * C[g] - hb * hb > 1e-8):
                continue
        dx, dy = px - mean[g, 0], py - mean[g, 1]
        q = A[g] * dx * dx + B[g] * dx * dy + C[g] * dy * dy
        raw = opacity[g] * np.exp(-0.5 * q)
        alpha = np.minimum(raw, alpha_clamp)
        if rule == "saturation":
            active = (alpha > alpha_threshold) & (Wsum < 1.0 - t_threshold)
            w = np.where(active, alpha * (1.0 - Wsum), 0.0)
            Tprev = 1.0 - Wsum
            Wsum = Wsum + w
            T = 1.0 - Wsum
        else:
            active = (~done) & (q >= 0.0) & (alpha >= alpha_threshold)
            w = np.where(active, T * alpha, 0.0)
            Tprev = T
            Wsum = Wsum + w
            T = np.where(active, T * (1.0 - alpha), T)
            done = done | (active & (T < t_threshold))
        accum += w[None] * colors[g][:, None, None]
        if keep_trace and active.any():  # entries that touch no pixel have no gradient
            rows = np.flatnonzero(active.any(axis=1))
            r0, r1 = rows[0], rows[-1] + 1  # keep the band of rows the entry touches
            trace.append((g, r0, active[r0:r1], alpha[r0:r1], Tprev[r0:r1], (raw <= alpha_clamp)[r0:r1]))
    if rule == "saturation":
        image = accum + (1.0 - Wsum)[None] * bg[:, None, None]
    else:
        image = accum + T[None] * bg[:, None, None]
    return (image, Wsum, trace) if keep_trace else (image, Wsum)


def blend_2d_backward(mean, A, B, C, opacity, colors, depths, H: int, W: int, d_image, d_weight=None, **kw):
    """Gradients of sum(d_image * image) + sum(d_weight * weight) of blend_2d w.r.t. mean [G,2],
    (A, B, C) [G] each, opacity [G] and colors [G,3]."""
    colors = np.asarray(colors, dtype=np.float64)
    opacity = np.asarray(opacity, dtype=np.float64)
    A, B, C = (np.asarray(v, dtype=np.float64) for v in (A, B, C))
    image, Wsum, trace = blend_2d(mean, A, B, C, opacity, colors, depths, H, W, keep_trace=True, **kw)
    go = np.asarray(d_image, dtype=np.float64)
    gw = np.zeros((H, W)) if d_weight is None else np.asarray(d_weight, dtype=np.float64)
    bg = np.asarray(kw.get("background", (0.0, 0.0, 0.0)), dtype=np.float64)
    G = len(colors)
    g_mean = np.zeros((G, 2))
    gA, gB, gC, g_op = np.zeros(G), np.zeros(G), np.zeros(G), np.zeros(G)
    g_col = np.zeros((G, 3))
    # L = sum_{k<j} T_k alpha_k D_k + T_j R_j with D_k = go . c_k + gw (each weight enters the
    # image and the weight sum) and R_j = alpha_j D_j + (1 - alpha_j) R_{j+1}, R_{n+1} = go . bg;
    # so dL/d alpha_j = T_j (D_j - R_{j+1}).
    gR = np.einsum("chw,c->hw", go, bg)
    px, py = _pixels(H, W)
    mean = np.asarray(mean, dtype=np.float64)
    for g, r0, active, alpha, Tprev, unclamped in reversed(trace):
        r1 = r0 + active.shape[0]
        gob, gRb = go[:, r0:r1], gR[r0:r1]
        dx, dy = px[r0:r1] - mean[g, 0], py[r0:r1] - mean[g, 1]
        q = A[g] * dx * dx + B[g] * dx * dy + C[g] * dy * dy
        alpha = np.where(active, alpha, 0.0)
        dot_gc = np.einsum("chw,c->hw", gob, colors[g]) + gw[r0:r1]
        g_alpha = np.where(active, Tprev * (dot_gc - gRb), 0.0)
        g_col[g] += np.einsum("chw,hw->c", gob, np.where(active, Tprev * alpha, 0.0))
        gR[r0:r1] = np.where(active, alpha * dot_gc + (1.0 - alpha) * gRb, gRb)
        e = np.exp(-0.5 * q)
        g_raw = np.where(active & unclamped, g_alpha, 0.0)
        g_op[g] += np.sum(g_raw * e)
        g_q = g_raw * opacity[g] * e * -0.5
        gA[g] += np.sum(g_q * dx * dx)
        gB[g] += np.sum(g_q * dx * dy)
        gC[g] += np.sum(g_q * dy * dy)
        g_mean[g, 0] += np.sum(g_q * -(2.0 * A[g] * dx + B[g] * dy))
        g_mean[g, 1] += np.sum(g_q * -(B[g] * dx + 2.0 * C[g] * dy))
    return dict(mean=g_mean, A=gA, B=gB, C=gC, opacity=g_op, colors=g_col)


def packed_grads(packed: np.ndarray, g: dict) -> np.ndarray:
    """Chain rule from blend_2d_backward's (mean, A, B, C, opacity) to the packed rows [G,7]."""
    p = np.asarray(packed, dtype=np.float64)
    ax, ay, s0, s1 = p[:, 2], p[:, 3], p[:, 4], p[:, 5]
    u0, u1 = 1.0 / (s0 * s0), 1.0 / (s1 * s1)
    gA, gB, gC = g["A"], g["B"], g["C"]
    out = np.zeros_like(p)
    out[:, 0:2] = g["mean"]
    out[:, 2] = gA * 2 * ax * u0 + gB * 2 * ay * (u0 - u1) + gC * 2 * ax * u1
    out[:, 3] = gA * 2 * ay * u1 + gB * 2 * ax * (u0 - u1) + gC * 2 * ay * u0
    gu0 = gA * ax * ax + gB * 2 * ax * ay + gC * ay * ay
    gu1 = gA * ay * ay - gB * 2 * ax * ay + gC * ax * ax
    out[:, 4] = gu0 * -2.0 * u0 / s0
    out[:, 5] = gu1 * -2.0 * u1 / s1
    out[:, 6] = g["opacity"]
    return out


def render_packed(packed, depths, features, H: int, W: int, background=(0.0, 0.0, 0.0), **kw):
    """image [3,H,W], weight [H,W] of packed splats (the accuracy harness's contract)."""
    mean, A, B, C, o = packed_to_conic(packed)
    return blend_2d(mean, A, B, C, o, features, depths, H, W, background=background, **kw)


def render_conic(means2d, conics, colors, opacities, depths, H: int, W: int, background=(0.0, 0.0, 0.0), **kw):
    """image [3,H,W], weight [H,W] of the fast-mac bridge's contract (conic culling on)."""
    A, B, C = conic_to_abc(conics)
    kw.setdefault("cull_conic", True)
    return blend_2d(means2d, A, B, C, opacities, colors, depths, H, W, background=background, **kw)


def mse_loss_and_grad(image: np.ndarray, target: np.ndarray):
    """The accuracy harness's loss, mean((image - target)^2) (splat_renderer_accuracy.py:446-447)."""
    d = image - target
    return float(np.mean(d * d)), 2.0 * d / d.size
