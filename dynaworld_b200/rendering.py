"""Trainer-facing render dispatch with the ``"b200"`` renderer mode.

Same call shapes as the reference's src/train/rendering.py (render_gaussian_frame :106-212,
render_gaussian_frames :230-351, pick_renderer_mode :50-61, camera_for_viewport :25-47,
_resolve_camera_projection_mode :88-103).  ``frame`` / ``sequence`` are any objects with the
reference's GaussianFrame / GaussianSequence fields (xyz, scales, quats, opacities, rgbs) and
cameras any objects with CameraSpec's fields (fx, fy, cx, cy, camera_to_world, lens_model).
The reference's own modes (dense, tiled, taichi, fast_mac) stay in the reference; this module
only renders ``"b200"``.
"""
from __future__ import annotations

import torch

from .config import B200RendererConfig
from .renderer import render_b200_3dgs, render_b200_3dgs_batch

CAMERA_PROJECTION_MODES = {"auto", "legacy_pinhole", "camera_model"}
REFERENCE_MODES = ("dense", "tiled", "taichi", "fast_mac")


def pick_renderer_mode(renderer: str, gaussian_count: int, height: int, width: int, auto_dense_limit: int) -> str:
    """``"b200"`` (and ``"auto"``, which resolves to it here) are this library's; the reference's
    modes are refused with a pointer to the reference module (rendering.py:50-61 raises the same
    way for unknown modes)."""
    if renderer in ("auto", "b200"):
        return "b200"
    if renderer in REFERENCE_MODES:
        raise ValueError(f"renderer mode {renderer!r} is served by the reference's rendering module, not b200")
    raise ValueError(f"Unknown renderer mode: {renderer}")


def _normalize_camera_projection_mode(camera_projection: str | None) -> str:
    mode = "auto" if camera_projection is None else str(camera_projection).lower()
    if mode == "legacy":
        mode = "legacy_pinhole"
    if mode not in CAMERA_PROJECTION_MODES:
        raise ValueError(
            f"Unknown render.camera_projection={camera_projection!r}. Expected auto, legacy_pinhole, or camera_model."
        )
    return mode


def resolve_camera_projection_mode(cameras, camera_projection: str | None) -> str:
    mode = _normalize_camera_projection_mode(camera_projection)
    cams = list(cameras) if isinstance(cameras, (list, tuple)) else [cameras]
    lens = sorted({getattr(c, "lens_model", "pinhole") for c in cams})
    has_non_pinhole = lens != ["pinhole"]
    if mode == "legacy_pinhole" and has_non_pinhole:
        raise ValueError(
            "render.camera_projection='legacy_pinhole' cannot render non-pinhole CameraSpec values "
            f"(lens models: {lens}). Use render.camera_projection='camera_model' or 'auto'."
        )
    if mode == "auto":
        return "camera_model" if has_non_pinhole else "legacy_pinhole"
    return mode


def camera_for_viewport(camera, source_height: int, source_width: int, target_height: int, target_width: int):
    """Same pose, intrinsics rescaled to the target viewport (rendering.py:25-47)."""
    if source_height < 1 or source_width < 1:
        raise ValueError(f"source viewport must be positive, got {source_width}x{source_height}.")
    if target_height < 1 or target_width < 1:
        raise ValueError(f"target viewport must be positive, got {target_width}x{target_height}.")
    sx = float(target_width) / float(source_width)
    sy = float(target_height) / float(source_height)
    import dataclasses

    fields = dict(fx=camera.fx * sx, fy=camera.fy * sy, cx=camera.cx * sx, cy=camera.cy * sy)
    if dataclasses.is_dataclass(camera):
        return dataclasses.replace(camera, **fields)
    out = type(camera).__new__(type(camera))
    out.__dict__.update(camera.__dict__)
    out.__dict__.update(fields)
    return out


def _config(b200_options, tile_size, alpha_threshold) -> B200RendererConfig:
    return B200RendererConfig.from_mapping(b200_options, fallback_tile_size=tile_size,
                                           fallback_alpha_threshold=alpha_threshold)


def render_gaussian_frame(frame, camera, height: int, width: int, mode: str, dense_grid=None, tile_size: int = 8,
                          bound_scale: float = 3.0, alpha_threshold: float = 1.0 / 255.0, near_plane: float = 1.0e-4,
                          taichi_options: dict | None = None, fast_mac_options: dict | None = None,
                          camera_projection: str | None = "auto", return_aux: bool = False,
                          b200_options: dict | None = None) -> torch.Tensor:
    projection_mode = resolve_camera_projection_mode(camera, camera_projection)
    if mode != "b200":
        pick_renderer_mode(mode, 0, height, width, 0)
    if return_aux:
        raise ValueError("return_aux is only supported by the dense renderer.")
    options = dict(b200_options or {})
    options.setdefault("bound_scale", bound_scale)
    return render_b200_3dgs(
        frame.xyz, frame.scales, frame.quats, frame.opacities, frame.rgbs, height, width,
        camera.fx, camera.fy, camera.cx, camera.cy, camera=camera, projection_mode=projection_mode,
        camera_to_world=camera.camera_to_world, near_plane=near_plane,
        config=_config(options, tile_size, alpha_threshold),
    )


def render_gaussian_frames(sequence, cameras, height: int, width: int, mode: str, dense_grid=None,
                           tile_size: int = 8, bound_scale: float = 3.0, alpha_threshold: float = 1.0 / 255.0,
                           near_plane: float = 1.0e-4, taichi_options: dict | None = None,
                           fast_mac_options: dict | None = None, camera_projection: str | None = "auto",
                           return_aux: bool = False, b200_options: dict | None = None) -> torch.Tensor:
    frame_count = int(sequence.xyz.shape[0])
    if frame_count != len(cameras):
        raise ValueError(f"Expected {frame_count} cameras, got {len(cameras)}.")
    projection_mode = resolve_camera_projection_mode(cameras, camera_projection)
    if mode != "b200":
        pick_renderer_mode(mode, 0, height, width, 0)
    if return_aux:
        raise ValueError("return_aux is only supported by the dense renderer.")
    device = sequence.xyz.device

    def vec(name):
        vals = [getattr(c, name) for c in cameras]
        return torch.stack([torch.as_tensor(v, dtype=torch.float32, device=device).reshape(()) for v in vals])

    c2w = torch.stack([c.camera_to_world.to(device=device, dtype=torch.float32) for c in cameras], dim=0)
    options = dict(b200_options or {})
    options.setdefault("bound_scale", bound_scale)
    return render_b200_3dgs_batch(
        sequence.xyz, sequence.scales, sequence.quats, sequence.opacities, sequence.rgbs, height, width,
        vec("fx"), vec("fy"), vec("cx"), vec("cy"), cameras=cameras, projection_mode=projection_mode,
        camera_to_world=c2w, near_plane=near_plane, config=_config(options, tile_size, alpha_threshold),
    )
