"""Public render functions.

* ``render_b200_3dgs_batch`` / ``render_b200_3dgs``: drop-ins for the reference's backend entry
  points (``render_pytorch_3dgs_batch``, src/train/renderers/dense.py:170-236, and
  ``render_fast_mac_3dgs[_batch]``, src/train/renderers/fast_mac.py:216-309): activated per-frame
  Gaussians [K,G,C], one camera per frame, image [K,3,H,W] (or [3,H,W]).
* ``render_b200``: raw parameters (means, log-scales, quaternions, opacity logits, SH, optional
  velocity with per-view times) shared by groups of views; returns image, alpha and depth.
* ``render_b200_head``: the decoder head's raw outputs (GaussianParameterHeads, src/train/
  gs_models/blocks.py:172-186) with the head's activation fused into the projection.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .config import B200RendererConfig
from .render import MIN_RENDER_DEPTH, SceneSpec, ViewSpec, lens_tensors, render_scene


def _per_view(value, K: int, device) -> torch.Tensor:
    if torch.is_tensor(value):  # keeps the autograd graph: learned intrinsics get gradients
        v = value.to(device=device, dtype=torch.float32)
        return v.expand(K) if v.ndim == 0 else v.reshape(K)
    return torch.full((K,), float(value), device=device, dtype=torch.float32)


def _intrinsics(fx, fy, cx, cy, K, device) -> torch.Tensor:
    return torch.stack([_per_view(v, K, device) for v in (fx, fy, cx, cy)], dim=-1).contiguous()


def _lens_of(projection_mode: str, cameras, K: int, device):
    """Lens models of the views.  ``legacy_pinhole`` projects every view as a pinhole
    (common.py); ``camera_model`` takes each CameraSpec's lens_model and distortion
    (projection.py:227-330: pinhole views keep the common.py projection)."""
    if projection_mode == "legacy_pinhole":
        return None
    if projection_mode != "camera_model":
        raise ValueError(f"Unknown projection_mode: {projection_mode}")
    cams = list(cameras) if isinstance(cameras, (list, tuple)) else ([cameras] if cameras is not None else [])
    if not cams:
        raise ValueError("camera_model projection requires CameraSpec values.")
    if len(cams) != K:
        raise ValueError(f"Expected {K} cameras, got {len(cams)}.")
    models = [getattr(c, "lens_model", "pinhole") for c in cams]
    for m in models:
        if m not in _lib.LENS_CODES:
            raise ValueError(f"Unknown lens_model: {m}")
    return lens_tensors(models, [getattr(c, "distortion", None) for c in cams], K, device)


def render_b200_3dgs_batch(
    means3d: torch.Tensor,
    scales: torch.Tensor,
    quats: torch.Tensor,
    opacities: torch.Tensor,
    rgbs: torch.Tensor,
    height: int,
    width: int,
    fx,
    fy,
    cx,
    cy,
    *,
    cameras=None,
    projection_mode: str = "legacy_pinhole",
    camera_to_world: torch.Tensor | None = None,
    near_plane: float = MIN_RENDER_DEPTH,
    config: B200RendererConfig | None = None,
) -> torch.Tensor:
    """[K,G,3] means, [K,G,3] scales, [K,G,4] quaternions, [K,G,1] opacities, [K,G,3] rgbs and
    per-frame intrinsics / camera_to_world [K,4,4] -> image [K,3,H,W] in [0,1]."""
    config = config or B200RendererConfig()
    K, G = int(means3d.shape[0]), int(means3d.shape[1])
    dev = means3d.device
    lens = _lens_of(projection_mode, cameras, K, dev)
    intr = _intrinsics(fx, fy, cx, cy, K, dev)
    if camera_to_world is None:
        c2w = torch.eye(4, device=dev, dtype=torch.float32).expand(K, 4, 4).contiguous()
    else:
        c2w = camera_to_world.to(device=dev, dtype=torch.float32)
        c2w = (c2w.unsqueeze(0).expand(K, 4, 4) if c2w.ndim == 2 else c2w).contiguous()
    sspec = SceneSpec(n_sets=K, n_gaussians=G, raw=False, sh_degree=0, velocity=False, sh_clamp=False)
    vspec = ViewSpec(n_views=K, views_per_set=1, height=int(height), width=int(width))
    image, _alpha, _depth = render_scene(
        sspec, vspec, config, near_plane, means=means3d, scales=scales, quats=quats,
        opacities=opacities.reshape(K, G), colors=rgbs, velocity=None, intrinsics=intr, camera_to_world=c2w,
        times=None, lens=lens,
    )
    return image


def render_b200_3dgs(
    means3d: torch.Tensor,
    scales: torch.Tensor,
    quats: torch.Tensor,
    opacities: torch.Tensor,
    rgbs: torch.Tensor,
    height: int,
    width: int,
    fx,
    fy,
    cx,
    cy,
    *,
    camera=None,
    projection_mode: str = "legacy_pinhole",
    camera_to_world: torch.Tensor | None = None,
    near_plane: float = MIN_RENDER_DEPTH,
    config: B200RendererConfig | None = None,
) -> torch.Tensor:
    """Single frame: [G,*] Gaussians -> image [3,H,W] (render_pytorch_3dgs, dense.py:105-167)."""
    c2w = None if camera_to_world is None else camera_to_world.reshape(1, 4, 4)
    return render_b200_3dgs_batch(
        means3d.unsqueeze(0), scales.unsqueeze(0), quats.unsqueeze(0), opacities.reshape(1, -1, 1),
        rgbs.unsqueeze(0), height, width, fx, fy, cx, cy, cameras=[camera] if camera is not None else None,
        projection_mode=projection_mode, camera_to_world=c2w, near_plane=near_plane, config=config,
    )[0]


def render_b200(
    means: torch.Tensor,
    log_scales: torch.Tensor,
    quats: torch.Tensor,
    opacity_logits: torch.Tensor,
    sh: torch.Tensor,
    *,
    intrinsics: torch.Tensor,
    camera_to_world: torch.Tensor,
    height: int,
    width: int,
    velocity: torch.Tensor | None = None,
    times: torch.Tensor | None = None,
    views_per_set: int | None = None,
    near_plane: float = MIN_RENDER_DEPTH,
    config: B200RendererConfig | None = None,
    lens_models=None,
    distortion=None,
):
    """Raw-parameter render.

    means/log_scales [S,G,3] (or [G,3]), quats [S,G,4] (normalised here), opacity_logits [S,G,1]
    or [S,G], sh [S,G,(d+1)^2,3] (rgb = SH(view dir) + 0.5), velocity [S,G,3] with times [B]
    (means_t = means + t * velocity).  View b uses set b // views_per_set (default: all views
    share set 0 when S == 1, else B // S views per set).  intrinsics [B,4] = fx, fy, cx, cy;
    camera_to_world [B,4,4].  ``lens_models`` (per view: "pinhole", "radial_tangential",
    "opencv_fisheye", or their GSB_LENS_* codes) with ``distortion`` (per view [k1, k2, p1, p2, k3]
    or [k1, k2, k3, k4]) project as project_gaussians_2d_camera does.  Returns image [B,3,H,W],
    alpha [B,H,W] (sum of blend weights) and depth [B,H,W] (sum of weight * camera z; None unless
    ``config.depth``).
    """
    config = config or B200RendererConfig()
    if means.ndim == 2:
        means, log_scales, quats = means.unsqueeze(0), log_scales.unsqueeze(0), quats.unsqueeze(0)
        opacity_logits, sh = opacity_logits.unsqueeze(0), sh.unsqueeze(0)
        velocity = None if velocity is None else velocity.unsqueeze(0)
    S, G = int(means.shape[0]), int(means.shape[1])
    B = int(camera_to_world.shape[0])
    k = int(sh.shape[-2])
    degree = {1: 0, 4: 1, 9: 2, 16: 3}.get(k)
    if degree is None:
        raise ValueError(f"sh must have 1, 4, 9 or 16 coefficients per channel, got {k}")
    if views_per_set is None:
        views_per_set = B if S == 1 else B // S
    if views_per_set <= 0 or (B - 1) // views_per_set >= S:
        raise ValueError(f"{B} views with views_per_set={views_per_set} need more than {S} sets")
    if velocity is not None and times is None:
        raise ValueError("velocity needs per-view times")
    sspec = SceneSpec(n_sets=S, n_gaussians=G, raw=True, sh_degree=degree, velocity=velocity is not None,
                      sh_clamp=config.sh_clamp)
    vspec = ViewSpec(n_views=B, views_per_set=views_per_set, height=int(height), width=int(width))
    image, alpha, depth = render_scene(
        sspec, vspec, config, near_plane, means=means, scales=log_scales, quats=quats,
        opacities=opacity_logits.reshape(S, G), colors=sh, velocity=velocity,
        intrinsics=intrinsics.reshape(B, 4), camera_to_world=camera_to_world, times=times,
        lens=lens_tensors(lens_models, distortion, B, means.device),
    )
    return image, alpha, (depth if config.depth else None)


@dataclass(frozen=True)
class HeadActivation:
    """Constants of the decoder head's output activation (GaussianParameterHeads, src/train/
    gs_models/blocks.py:110-186): xy bound, z range and the scale multiplier."""

    xy_extent: float = 1.5
    z_min: float = 0.5
    z_max: float = 2.5
    scale_init: float = 0.05

    @classmethod
    def from_heads(cls, heads) -> "HeadActivation":
        """Reads a GaussianParameterHeads-like module's xy_extent, z_min, z_extent, scale_init."""
        return cls(float(heads.xy_extent), float(heads.z_min), float(heads.z_min) + float(heads.z_extent),
                   float(heads.scale_init))

    def constants(self) -> tuple[float, float, float, float]:
        return (self.xy_extent, self.z_min, self.z_max - self.z_min, self.scale_init)


def render_b200_head(
    xyz_raw: torch.Tensor,
    scale_raw: torch.Tensor,
    rot_raw: torch.Tensor,
    opacity_raw: torch.Tensor,
    rgb_raw: torch.Tensor,
    *,
    head: HeadActivation,
    intrinsics: torch.Tensor,
    camera_to_world: torch.Tensor,
    height: int,
    width: int,
    velocity: torch.Tensor | None = None,
    times: torch.Tensor | None = None,
    views_per_set: int | None = None,
    near_plane: float = MIN_RENDER_DEPTH,
    config: B200RendererConfig | None = None,
    lens_models=None,
    distortion=None,
):
    """Render straight from the decoder head's raw outputs [S,G,*] (the five head MLPs' reshaped
    outputs of GaussianParameterHeads.forward, blocks.py:172-186), with the head's activation fused
    into the projection, so the activated [S,G,*] tensors are never written:

        xyz = (tanh(x) xy_extent, tanh(y) xy_extent, sigmoid(z) (z_max - z_min) + z_min)
        scales = exp(scale_raw) scale_init, quats = normalize(rot_raw), opacity = sigmoid,
        rgb = sigmoid(rgb_raw)

    Gradients flow to the five raw tensors (and ``velocity``).  Sets, views, lenses and outputs as
    render_b200."""
    config = config or B200RendererConfig()
    if xyz_raw.ndim == 2:
        xyz_raw, scale_raw, rot_raw = xyz_raw.unsqueeze(0), scale_raw.unsqueeze(0), rot_raw.unsqueeze(0)
        opacity_raw, rgb_raw = opacity_raw.unsqueeze(0), rgb_raw.unsqueeze(0)
        velocity = None if velocity is None else velocity.unsqueeze(0)
    S, G = int(xyz_raw.shape[0]), int(xyz_raw.shape[1])
    B = int(camera_to_world.shape[0])
    if rgb_raw.shape[-1] != 3 or rgb_raw.numel() != S * G * 3:
        raise ValueError(f"rgb_raw must be [S,G,3], got {tuple(rgb_raw.shape)}")
    if views_per_set is None:
        views_per_set = B if S == 1 else B // S
    if views_per_set <= 0 or (B - 1) // views_per_set >= S:
        raise ValueError(f"{B} views with views_per_set={views_per_set} need more than {S} sets")
    if velocity is not None and times is None:
        raise ValueError("velocity needs per-view times")
    sspec = SceneSpec(n_sets=S, n_gaussians=G, raw=False, sh_degree=0, velocity=velocity is not None,
                      sh_clamp=False, head=head.constants())
    vspec = ViewSpec(n_views=B, views_per_set=views_per_set, height=int(height), width=int(width))
    image, alpha, depth = render_scene(
        sspec, vspec, config, near_plane, means=xyz_raw, scales=scale_raw, quats=rot_raw,
        opacities=opacity_raw.reshape(S, G), colors=rgb_raw.reshape(S, G, 3), velocity=velocity,
        intrinsics=intrinsics.reshape(B, 4), camera_to_world=camera_to_world, times=times,
        lens=lens_tensors(lens_models, distortion, B, xyz_raw.device),
    )
    return image, alpha, (depth if config.depth else None)
