"""Torch restatement of the reference's differentiable splat render + loss.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Every function here is a
plain-torch restatement, differentiable through torch autograd, usable in
float32 (to mirror the reference's own arithmetic) or float64 (as a tighter
oracle).  Citations are to files of nbardy/dynaworld.

Reference semantics restated:
  * projection  src/train/renderers/common.py:149-231 (project_gaussians_2d_batch)
  * lenses      src/train/renderers/projection.py:75-214 (camera_model projection:
                radial-tangential and OpenCV fisheye distortion, closed-form Jacobians)
  * dense blend src/train/renderers/dense.py:170-236  (render_pytorch_3dgs_batch)
  * loss        src/train/losses.py:13-85             (ssim_per_image,
                reconstruction_loss_per_image)
Extensions with no reference code (parity pinned only against this file):
  activation of raw parameters, real spherical harmonics of degree 0..3,
  per-view time offset (means + t * velocity), alpha (sum of blend weights)
  and depth (sum of weight * camera z) outputs, Gaussian-window SSIM.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

MIN_RENDER_DEPTH = 1e-4  # common.py:3

# Real spherical-harmonic normalisation constants, derived from
# Y_lm = sqrt((2l+1)/(4 pi) * (l-|m|)!/(l+|m|)!) P_l^|m| with the usual
# sqrt(2) factor for m != 0 (3DGS sign convention).
SH_C0 = 0.5 / math.sqrt(math.pi)
SH_C1 = math.sqrt(3.0 / (4.0 * math.pi))
SH_C2 = (
    0.5 * math.sqrt(15.0 / math.pi),
    -0.5 * math.sqrt(15.0 / math.pi),
    0.25 * math.sqrt(5.0 / math.pi),
    -0.5 * math.sqrt(15.0 / math.pi),
    0.25 * math.sqrt(15.0 / math.pi),
)
SH_C3 = (
    -0.25 * math.sqrt(35.0 / (2.0 * math.pi)),
    0.5 * math.sqrt(105.0 / math.pi),
    -0.25 * math.sqrt(21.0 / (2.0 * math.pi)),
    0.25 * math.sqrt(7.0 / math.pi),
    -0.25 * math.sqrt(21.0 / (2.0 * math.pi)),
    0.25 * math.sqrt(105.0 / math.pi),
    -0.25 * math.sqrt(35.0 / (2.0 * math.pi)),
)


def sh_basis(dirs: torch.Tensor, degree: int) -> torch.Tensor:
    """Real SH basis values [..., (degree+1)^2] for unit directions [..., 3]."""
    x, y, z = dirs.unbind(-1)
    out = [torch.full_like(x, SH_C0)]
    if degree >= 1:
        out += [-SH_C1 * y, SH_C1 * z, -SH_C1 * x]
    if degree >= 2:
        xx, yy, zz, xy, yz, xz = x * x, y * y, z * z, x * y, y * z, x * z
        out += [
            SH_C2[0] * xy,
            SH_C2[1] * yz,
            SH_C2[2] * (2.0 * zz - xx - yy),
            SH_C2[3] * xz,
            SH_C2[4] * (xx - yy),
        ]
    if degree >= 3:
        out += [
            SH_C3[0] * y * (3.0 * xx - yy),
            SH_C3[1] * xy * z,
            SH_C3[2] * y * (4.0 * zz - xx - yy),
            SH_C3[3] * z * (2.0 * zz - 3.0 * xx - 3.0 * yy),
            SH_C3[4] * x * (4.0 * zz - xx - yy),
            SH_C3[5] * z * (xx - yy),
            SH_C3[6] * x * (xx - 3.0 * yy),
        ]
    return torch.stack(out, dim=-1)


@dataclass
class RawGaussians:
    """Raw (pre-activation) Gaussian parameters of S sets of G Gaussians.

    means [S,G,3], log_scales [S,G,3], quats [S,G,4] (any norm),
    opacity_logits [S,G,1], sh [S,G,(deg+1)^2,3], velocity [S,G,3] or None.
    View b uses set b // views_per_set.
    """

    means: torch.Tensor
    log_scales: torch.Tensor
    quats: torch.Tensor
    opacity_logits: torch.Tensor
    sh: torch.Tensor
    velocity: torch.Tensor | None = None

    @property
    def sh_degree(self) -> int:
        return int(round(math.sqrt(self.sh.shape[-2]))) - 1


def time_offset_means(means: torch.Tensor, velocity: torch.Tensor | None, t: torch.Tensor) -> torch.Tensor:
    """means + t * velocity, rounded as two float ops (no fused multiply-add)."""
    if velocity is None:
        return means
    return means + t.to(means.dtype).view(-1, 1, 1) * velocity


def activate(
    raw: RawGaussians,
    times: torch.Tensor | None,
    camera_to_world: torch.Tensor,
    views_per_set: int,
    sh_clamp_min: float | None = 0.0,
):
    """Raw parameters -> per-view activated tensors [B,G,*] (extension).

    scales = exp(log_scales); quats = q/|q|; opacity = sigmoid(logit);
    rgb = SH(dir) + 0.5 (clamped below at ``sh_clamp_min`` if given) with
    dir = normalise(mean_t - camera centre); mean_t = mean + t * velocity.
    The reference receives these already activated from its model heads
    (src/train/gs_models/blocks.py:172-186).
    """
    B = camera_to_world.shape[0]
    set_index = torch.arange(B) // views_per_set
    means = raw.means[set_index]
    vel = raw.velocity[set_index] if raw.velocity is not None else None
    if times is None:
        times = torch.zeros(B, dtype=means.dtype)
    means_t = time_offset_means(means, vel, times)
    scales = torch.exp(raw.log_scales[set_index])
    q = raw.quats[set_index]
    quats = q / torch.linalg.norm(q, dim=-1, keepdim=True)
    opac = torch.sigmoid(raw.opacity_logits[set_index])
    centre = camera_to_world[:, :3, 3].to(means.dtype)
    d = means_t - centre[:, None, :]
    dirs = d / torch.linalg.norm(d, dim=-1, keepdim=True)
    basis = sh_basis(dirs, raw.sh_degree)  # [B,G,K]
    rgb = torch.einsum("bgk,bgkc->bgc", basis, raw.sh[set_index]) + 0.5
    if sh_clamp_min is not None:
        rgb = torch.clamp(rgb, min=sh_clamp_min)
    return means_t, scales, quats, opac, rgb


def activate_head(xyz_raw, scale_raw, rot_raw, opacity_raw, rgb_raw, xy_extent, z_min, z_max, scale_init):
    """GaussianParameterHeads.forward's output activation (src/train/gs_models/blocks.py:172-186)
    restated: xyz = (tanh(x, y) * xy_extent, sigmoid(z) * (z_max - z_min) + z_min), scales =
    exp * scale_init, quats = F.normalize, opacity = sigmoid, rgb = sigmoid."""
    xyz = torch.cat([torch.tanh(xyz_raw[..., :2]) * xy_extent,
                     torch.sigmoid(xyz_raw[..., 2:]) * (z_max - z_min) + z_min], dim=-1)
    scales = torch.exp(scale_raw) * scale_init
    quats = F.normalize(rot_raw, p=2, dim=-1)
    return xyz, scales, quats, torch.sigmoid(opacity_raw), torch.sigmoid(rgb_raw)


def quat_to_rotation(q: torch.Tensor) -> torch.Tensor:
    """Unnormalised-safe rotation formula of common.py:169-179 (q = r,i,j,k)."""
    qr, qi, qj, qk = q.unbind(-1)
    rows = [
        torch.stack([1.0 - 2 * (qj * qj + qk * qk), 2 * (qi * qj - qr * qk), 2 * (qi * qk + qr * qj)], -1),
        torch.stack([2 * (qi * qj + qr * qk), 1.0 - 2 * (qi * qi + qk * qk), 2 * (qj * qk - qr * qi)], -1),
        torch.stack([2 * (qi * qk - qr * qj), 2 * (qj * qk + qr * qi), 1.0 - 2 * (qi * qi + qj * qj)], -1),
    ]
    return torch.stack(rows, dim=-2)


def fma_f32(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    """float32 fused multiply-add: round32(a*b + c) with one rounding.

    a*b of two float32 values is exact in float64; the sum is formed in
    80-bit extended precision (numpy longdouble) before the single rounding.
    """
    import numpy as np

    an, bn, cn = (x.detach().cpu().float().numpy().astype(np.longdouble) for x in (a, b, c))
    return torch.from_numpy((an * bn + cn).astype(np.float32))


def camera_depth_fp32(means: torch.Tensor, camera_to_world: torch.Tensor) -> torch.Tensor:
    """Camera-space z in float32 as the CUDA preprocess computes it.

    z = fma(d2, R22, fma(d1, R12, d0*R02)), d = fl32(mean - t).  This is the
    depth-sort key.  The reference computes the same quantity as a float32
    matmul (common.py:39-51, 191); on x86 CPUs with FMA, torch's matmul
    rounds it exactly this way, so the sort keys agree bit for bit.
    """
    m = means.float()
    c2w = camera_to_world.float()
    d = m - c2w[:, None, :3, 3]
    r = c2w[:, :3, 2]
    shape = d.shape[:-1]
    r0, r1, r2 = (r[:, None, k].expand(shape) for k in range(3))
    p0 = d[..., 0] * r0
    return fma_f32(d[..., 2], r2, fma_f32(d[..., 1], r1, p0)).reshape(shape)


def lens_distort(x: torch.Tensor, y: torch.Tensor, lens: str, c: torch.Tensor):
    """Distorted normalised coordinates and the closed-form lens Jacobian [...,2,2] of
    projection.py:93-116 (radial_tangential, c = k1, k2, p1, p2, k3) and :119-161
    (opencv_fisheye, c = k1, k2, k3, k4)."""
    if lens == "radial_tangential":
        k1, k2, p1, p2, k3 = (c[i] for i in range(5))
        r2 = x * x + y * y
        r4 = r2 * r2
        r6 = r4 * r2
        radial = 1.0 + k1 * r2 + k2 * r4 + k3 * r6
        xd = x * radial + 2.0 * p1 * x * y + p2 * (r2 + 2.0 * x * x)
        yd = y * radial + p1 * (r2 + 2.0 * y * y) + 2.0 * p2 * x * y
        rd = k1 + 2.0 * k2 * r2 + 3.0 * k3 * r4
        rdx, rdy = 2.0 * x * rd, 2.0 * y * rd
        l00 = radial + x * rdx + 2.0 * p1 * y + 6.0 * p2 * x
        l01 = x * rdy + 2.0 * p1 * x + 2.0 * p2 * y
        l10 = y * rdx + 2.0 * p1 * x + 2.0 * p2 * y
        l11 = radial + y * rdy + 6.0 * p1 * y + 2.0 * p2 * x
    elif lens == "opencv_fisheye":
        k1, k2, k3, k4 = (c[i] for i in range(4))
        eps = 1.0e-8
        r2 = x * x + y * y
        radius = torch.sqrt(torch.clamp(r2, min=eps * eps))
        theta = torch.atan(radius)
        t2 = theta * theta
        t4 = t2 * t2
        t6 = t4 * t2
        t8 = t4 * t4
        theta_d = theta * (1.0 + k1 * t2 + k2 * t4 + k3 * t6 + k4 * t8)
        valid = r2 > eps * eps
        scale = torch.where(valid, theta_d / radius, torch.ones_like(radius))
        xd, yd = scale * x, scale * y
        dtd = 1.0 + 3.0 * k1 * t2 + 5.0 * k2 * t4 + 7.0 * k3 * t6 + 9.0 * k4 * t8
        dtdr = 1.0 / (1.0 + radius * radius)
        dsdr = torch.where(valid, (dtd * dtdr * radius - theta_d) / (radius * radius), torch.zeros_like(radius))
        inv_r = torch.where(valid, 1.0 / radius, torch.zeros_like(radius))
        dsdx, dsdy = dsdr * x * inv_r, dsdr * y * inv_r
        l00, l01, l10, l11 = scale + x * dsdx, x * dsdy, y * dsdx, scale + y * dsdy
    else:
        raise ValueError(f"Unknown lens_model: {lens}")
    lj = torch.stack([torch.stack([l00, l01], -1), torch.stack([l10, l11], -1)], -2)
    return xd, yd, lj


def project_batch(
    means: torch.Tensor,
    scales: torch.Tensor,
    quats: torch.Tensor,
    opacities: torch.Tensor,
    rgbs: torch.Tensor,
    fx: torch.Tensor,
    fy: torch.Tensor,
    cx: torch.Tensor,
    cy: torch.Tensor,
    camera_to_world: torch.Tensor,
    near_plane: float = MIN_RENDER_DEPTH,
    sort_key: torch.Tensor | None = None,
    lens_models: list[str] | None = None,
    distortion: torch.Tensor | None = None,
):
    """Restates project_gaussians_2d_batch (common.py:149-231); views whose ``lens_models`` entry
    is not "pinhole" take the pixel position and Jacobian of project_gaussians_2d_camera
    (projection.py:75-90, 164-214, 253-263) with ``distortion[b]`` (zero-padded to 5).

    Returns, in per-view depth order: means2d [B,G,2], inv_cov [B,G,2,2],
    cov2d [B,G,2,2], opacity [B,G,1] (zeroed behind the near plane), rgb
    [B,G,3], camera z [B,G] and the sort permutation [B,G] (stable argsort of
    ``sort_key``, default the camera z).
    """
    dtype = means.dtype
    B = means.shape[0]
    fx, fy, cx, cy = (v.to(dtype).reshape(B, 1) for v in (fx, fy, cx, cy))
    rot = quat_to_rotation(quats)
    basis = rot * scales.unsqueeze(-2)  # R @ diag(s)
    cov3 = basis @ basis.transpose(-1, -2)
    c2w = camera_to_world.to(dtype)
    rcw = c2w[:, :3, :3]
    t = c2w[:, :3, 3]
    m_cam = torch.einsum("bgj,bjk->bgk", means - t[:, None, :], rcw)
    cov_cam = rcw.transpose(1, 2).unsqueeze(1) @ cov3 @ rcw.unsqueeze(1)

    key = m_cam[..., 2] if sort_key is None else sort_key
    order = torch.argsort(key, dim=1, stable=True)  # common.py:191

    def gather(v):
        idx = order
        for _ in v.shape[2:]:
            idx = idx.unsqueeze(-1)
        return torch.gather(v, 1, idx.expand_as(v))

    m_cam, cov_cam, opacities, rgbs = gather(m_cam), gather(cov_cam), gather(opacities), gather(rgbs)
    x, y, z = m_cam.unbind(-1)
    front = z > near_plane  # common.py:197-203
    z_safe = torch.where(front, torch.clamp(z, min=near_plane), torch.ones_like(z))
    xp = torch.where(front, x, torch.zeros_like(x))
    yp = torch.where(front, y, torch.zeros_like(y))
    opacities = opacities * front.to(dtype).unsqueeze(-1)

    zero = torch.zeros_like(z_safe)
    jac = torch.stack(
        [
            torch.stack([fx / z_safe, zero, -(fx * xp) / (z_safe * z_safe)], -1),
            torch.stack([zero, fy / z_safe, -(fy * yp) / (z_safe * z_safe)], -1),
        ],
        dim=-2,
    )
    means2d = torch.stack([(fx * xp) / z_safe + cx, (fy * yp) / z_safe + cy], -1)
    if lens_models is not None and any(m != "pinhole" for m in lens_models):
        jac_rows, m2_rows = [], []
        for b, lens in enumerate(lens_models):
            if lens == "pinhole":
                jac_rows.append(jac[b])
                m2_rows.append(means2d[b])
                continue
            zs = z_safe[b]
            nj = torch.stack([torch.stack([1.0 / zs, torch.zeros_like(zs), -xp[b] / (zs ** 2)], -1),
                              torch.stack([torch.zeros_like(zs), 1.0 / zs, -yp[b] / (zs ** 2)], -1)], -2)
            nj = nj * front[b].to(dtype).view(-1, 1, 1)
            xd, yd, lj = lens_distort(xp[b] / zs, yp[b] / zs, lens, distortion[b].to(dtype))
            kj = torch.zeros(2, 2, dtype=dtype)
            kj[0, 0], kj[1, 1] = fx[b, 0], fy[b, 0]
            jac_rows.append(kj @ lj @ nj)
            m2_rows.append(torch.stack([fx[b, 0] * xd + cx[b, 0], fy[b, 0] * yd + cy[b, 0]], -1))
        jac, means2d = torch.stack(jac_rows), torch.stack(m2_rows)
    cov2 = jac @ cov_cam @ jac.transpose(-1, -2)
    cov2 = cov2 + 0.3 * torch.eye(2, dtype=dtype)  # EWA low-pass, common.py:216-218
    det = torch.clamp(cov2[..., 0, 0] * cov2[..., 1, 1] - cov2[..., 0, 1] * cov2[..., 1, 0], min=1e-6)
    inv = torch.stack(
        [
            torch.stack([cov2[..., 1, 1] / det, -cov2[..., 0, 1] / det], -1),
            torch.stack([-cov2[..., 1, 0] / det, cov2[..., 0, 0] / det], -1),
        ],
        dim=-2,
    )
    return means2d, inv, cov2, opacities, rgbs, z, order


def transmittance_factors(alpha: torch.Tensor, eps: float) -> torch.Tensor:
    """1 - alpha + eps with the reference's float32 roundings.

    dense.py:225 forms (1 - alpha) + 1e-6 in float32, so an alpha of zero
    gives 1 + 2^-20, not 1 + 1e-6; at G = 4096 the difference is 2e-4 in T.
    The factor is formed in float32 and returned in alpha's dtype.
    """
    a32 = alpha.float()
    return ((1.0 - a32) + eps).to(alpha.dtype)


def blend_dense(
    means2d: torch.Tensor,
    inv_cov: torch.Tensor,
    opacities: torch.Tensor,
    rgbs: torch.Tensor,
    depth: torch.Tensor | None,
    H: int,
    W: int,
    *,
    pixel_center: float = 0.0,
    eps: float = 1e-6,
    alpha_clamp: float = 0.99,
    background=(1.0, 1.0, 1.0),
    x0: int = 0,
    y0: int = 0,
    flip_wsum: torch.Tensor | None = None,
    flip_image: torch.Tensor | None = None,
    return_pre: bool = False,
):
    """All-pairs blend of dense.py:208-233 for a window [y0,y0+H) x [x0,x0+W).

    ``flip_wsum`` [B,H,W] / ``flip_image`` [B,3,H,W] (bool, optional): pixels where the clamp of
    the weight sum (dense.py:232) / of the image (:233) takes the other side of its kink, for
    values within rounding of 0 or 1 (see flip_clamp); the default is torch.clamp's.
    ``return_pre``: also return the image before its clamp [B,3,H,W].

    Returns image [B,3,H,W] (clamped to [0,1]), alpha = sum of weights
    [B,H,W] (before the clamp dense.py:232 applies), depth = sum of
    weight * z [B,H,W] (or None).  Pixels are independent given the
    projected Gaussians, so a window of a larger image is exact.
    """
    dtype = means2d.dtype
    B, G = means2d.shape[:2]
    gy, gx = torch.meshgrid(
        torch.arange(y0, y0 + H, dtype=dtype) + pixel_center,
        torch.arange(x0, x0 + W, dtype=dtype) + pixel_center,
        indexing="ij",
    )
    dx = gx.view(1, 1, H, W) - means2d[..., 0].view(B, G, 1, 1)
    dy = gy.view(1, 1, H, W) - means2d[..., 1].view(B, G, 1, 1)
    a = inv_cov[..., 0, 0].view(B, G, 1, 1)
    b = (inv_cov[..., 0, 1] + inv_cov[..., 1, 0]).view(B, G, 1, 1)
    c = inv_cov[..., 1, 1].view(B, G, 1, 1)
    power = -0.5 * (a * dx.square() + b * dx * dy + c * dy.square())
    power = torch.minimum(power, torch.zeros((), dtype=dtype))
    alpha = torch.clamp(opacities.reshape(B, G, 1, 1) * torch.exp(power), 0.0, alpha_clamp)
    factors = transmittance_factors(alpha[:, :-1], eps)
    T = torch.cat([alpha.new_ones((B, 1, H, W)), torch.cumprod(factors, dim=1)], dim=1)
    w = T * alpha
    color = (w.unsqueeze(-1) * rgbs[:, :, None, None, :]).sum(dim=1)  # [B,H,W,3]
    wsum = w.sum(dim=1)
    bg = torch.as_tensor(background, dtype=dtype)
    ws_c = wsum.clamp(0, 1)
    if flip_wsum is not None:  # the other side of the clamp's kink at these pixels
        ws_c = torch.where(flip_wsum, flip_clamp(wsum, ws_c), ws_c)
    out = color + (1.0 - ws_c).unsqueeze(-1) * bg
    out_c = out.clamp(0.0, 1.0)
    if flip_image is not None:
        out_c = torch.where(flip_image.permute(0, 2, 3, 1), flip_clamp(out, out_c), out_c)
    pre = out.permute(0, 3, 1, 2)
    out = out_c.permute(0, 3, 1, 2)
    d = None
    if depth is not None:
        d = (w * depth[:, :, None, None]).sum(dim=1)
    if return_pre:
        return out, wsum, d, pre
    return out, wsum, d


def flip_clamp(x: torch.Tensor, clamped: torch.Tensor) -> torch.Tensor:
    """The clamp of ``x`` to [0, 1] from the other side of its kink: where torch.clamp passes the
    gradient (0 <= x <= 1) the value is kept and the gradient blocked; where it blocks it, x itself
    (within rounding of the bound at the pixels this is used for) passes it."""
    inside = (x >= 0) & (x <= 1)
    return torch.where(inside, clamped.detach(), x)


def render_dense(
    means, scales, quats, opacities, rgbs, H, W, fx, fy, cx, cy, camera_to_world,
    *, near_plane=MIN_RENDER_DEPTH, pixel_center=0.0, eps=1e-6, alpha_clamp=0.99,
    background=(1.0, 1.0, 1.0), sort_key=None, x0=0, y0=0, lens_models=None, distortion=None,
    flip_wsum=None, flip_image=None, return_pre=False,
):
    """Projection + dense blend: render_pytorch_3dgs_batch restated (dense.py:170-236)."""
    m2, inv, _cov, op, rgb, z, _order = project_batch(
        means, scales, quats, opacities, rgbs, fx, fy, cx, cy, camera_to_world,
        near_plane=near_plane, sort_key=sort_key, lens_models=lens_models, distortion=distortion,
    )
    return blend_dense(
        m2, inv, op, rgb, z, H, W, pixel_center=pixel_center, eps=eps,
        alpha_clamp=alpha_clamp, background=background, x0=x0, y0=y0,
        flip_wsum=flip_wsum, flip_image=flip_image, return_pre=return_pre,
    )


# ----------------------------------------------------------------------------------------------
# Loss: losses.py:9-85
# ----------------------------------------------------------------------------------------------


def gaussian_window_1d(size: int, sigma: float, dtype=torch.float32) -> torch.Tensor:
    x = torch.arange(size, dtype=torch.float64) - (size // 2)
    g = torch.exp(-(x * x) / (2.0 * sigma * sigma))
    return (g / g.sum()).to(dtype)


def local_mean(images: torch.Tensor, window_size: int, window: str = "box", sigma: float = 1.5) -> torch.Tensor:
    """Reflect-padded window mean (losses.py:13-18); ``window='gaussian'`` is the extension."""
    if window_size <= 1:
        return images
    pad = window_size // 2
    padded = F.pad(images, (pad, pad, pad, pad), mode="reflect")
    if window == "box":
        return F.avg_pool2d(padded, kernel_size=window_size, stride=1)
    g = gaussian_window_1d(window_size, sigma, images.dtype)
    C = images.shape[1]
    kx = g.view(1, 1, 1, -1).expand(C, 1, 1, window_size)
    ky = g.view(1, 1, -1, 1).expand(C, 1, window_size, 1)
    return F.conv2d(F.conv2d(padded, kx, groups=C), ky, groups=C)


def ssim_per_image(pred, target, *, window_size=11, c1=1e-4, c2=9e-4, window="box", sigma=1.5):
    """losses.py:21-44 (map mean per image, clamped to [-1, 1])."""
    mu_x = local_mean(pred, window_size, window, sigma)
    mu_y = local_mean(target, window_size, window, sigma)
    mu_x_sq, mu_y_sq, mu_xy = mu_x.square(), mu_y.square(), mu_x * mu_y
    sxx = local_mean(pred.square(), window_size, window, sigma) - mu_x_sq
    syy = local_mean(target.square(), window_size, window, sigma) - mu_y_sq
    sxy = local_mean(pred * target, window_size, window, sigma) - mu_xy
    num = (2.0 * mu_xy + c1) * (2.0 * sxy + c2)
    den = (mu_x_sq + mu_y_sq + c1) * (sxx + syy + c2)
    smap = num / den.clamp_min(1.0e-12)
    return smap.flatten(1).mean(dim=1).clamp(-1.0, 1.0)


LOSS_DEFAULTS = {  # src/train/dynamicTokenGS.py:115-123
    "type": "standard_gs",
    "l1_weight": 0.8,
    "dssim_weight": 0.2,
    "mse_weight": 0.2,
    "ssim_window_size": 11,
    "ssim_c1": 1e-4,
    "ssim_c2": 9e-4,
}


def reconstruction_loss_per_image(pred, target, loss_cfg=None):
    """losses.py:58-85; extra keys ``ssim_window`` ('box'|'gaussian'),
    ``ssim_sigma`` and ``dssim_half`` (True: (1-SSIM)/2 as the reference)."""
    cfg = dict(LOSS_DEFAULTS)
    cfg.update(loss_cfg or {})
    kind = cfg["type"]
    delta = pred - target
    l1 = delta.abs().flatten(1).mean(dim=1)
    if kind == "l1":
        return l1
    mse = delta.square().flatten(1).mean(dim=1)
    if kind == "mse":
        return mse
    if kind == "l1_mse":
        return float(cfg["l1_weight"]) * l1 + float(cfg["mse_weight"]) * mse
    if kind == "standard_gs":
        ssim = ssim_per_image(
            pred, target,
            window_size=int(cfg["ssim_window_size"]), c1=float(cfg["ssim_c1"]), c2=float(cfg["ssim_c2"]),
            window=str(cfg.get("ssim_window", "box")), sigma=float(cfg.get("ssim_sigma", 1.5)),
        )
        dssim = (1.0 - ssim) * (0.5 if cfg.get("dssim_half", True) else 1.0)
        return float(cfg["l1_weight"]) * l1 + float(cfg["dssim_weight"]) * dssim
    raise ValueError(f"Unknown reconstruction loss type: {kind!r}")
