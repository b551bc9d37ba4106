"""The video trainer's reconstruction backward as one multi-view launch.

The reference's implicit-camera video trainer renders a clip in temporal micro-batches and
back-propagates each (src/train/train_video_token_implicit_dynamic.py:881-925): every chunk
renders its frames (render_clip_sequence, :382-403), computes reconstruction_loss_per_image and
calls backward(retain_graph=True), so the decoder's graph is walked once per chunk -- frame_count
times with the "framewise" strategy -- because the dense renderer's [B, G, H, W] intermediates do
not fit for a whole clip.  The B200 renderer keeps only per-pixel state, so ``recon_backward``
renders every frame of the clip in one launch of each stage, computes the fused loss of all of
them and walks the decoder's graph once.  The chunk losses sum to the clip loss, so the loss and
the gradients are the same (up to float summation order) with one backward pass instead of one
per chunk.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .losses import reconstruction_loss_per_image
from .rendering import camera_for_viewport, render_gaussian_frames


def temporal_recon_chunk_size(strategy: str, frame_count: int, microbatch_size: int) -> int:
    """Frames per chunk of the reference trainer (:881-886): "batched" renders the clip at once,
    "framewise" one frame at a time, anything else ``microbatch_size`` frames."""
    if strategy == "batched":
        return frame_count
    if strategy == "framewise":
        return 1
    return min(microbatch_size, frame_count)


def resize_images(images: torch.Tensor, image_size: int) -> torch.Tensor:
    """[..., C, H, W] -> [..., C, S, S], bilinear without corner alignment (rendering.py:16-22);
    returned unchanged at the size already."""
    if tuple(images.shape[-2:]) == (image_size, image_size):
        return images
    lead = images.shape[:-3]
    flat = images.reshape(-1, *images.shape[-3:])
    out = F.interpolate(flat, size=(image_size, image_size), mode="bilinear", align_corners=False)
    return out.reshape(*lead, *out.shape[-3:])


def viewport_cameras(cameras, input_size: int, render_size: int) -> tuple:
    """Cameras of the input frames rescaled to the render size, camera_for_viewport per camera
    (train_video_token_implicit_dynamic.py:348-363)."""
    return tuple(camera_for_viewport(c, input_size, input_size, render_size, render_size) for c in cameras)


def recon_backward(clip_frames: torch.Tensor, decoded, regularizer_loss, keep_preview: bool, *,
                   render_size: int, loss_cfg: dict | None = None, input_size: int | None = None,
                   render_cfg: dict | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Drop-in for the trainer's ``recon_backward`` (:887-925) with the renderer in "b200" mode.

    ``clip_frames`` [1, K, 3, H, W] targets, ``decoded`` a GaussianSequence-like object (xyz,
    scales, quats, opacities, rgbs [K, G, *] and K cameras), ``regularizer_loss`` a scalar added
    to the backward (or 0).  ``render_cfg`` holds the trainer's render options (tile_size,
    bound_scale, alpha_threshold, near_plane, camera_projection, and "b200" backend options);
    ``input_size`` the size the cameras' intrinsics refer to (None: ``render_size``).

    Returns (reconstruction loss, detached: sum over frames / K; the first frame's render,
    detached, when ``keep_preview``).  Gradients are accumulated into the decoder's parameters by
    one backward pass."""
    if decoded.cameras is None:
        raise ValueError("Implicit-camera video decode must include cameras.")
    cfg = dict(render_cfg or {})
    frame_count = len(decoded.cameras)
    cameras = viewport_cameras(decoded.cameras, input_size or render_size, render_size)
    renders = render_gaussian_frames(
        decoded, cameras, render_size, render_size, "b200", tile_size=cfg.get("tile_size", 8),
        bound_scale=cfg.get("bound_scale", 3.0), alpha_threshold=cfg.get("alpha_threshold", 1.0 / 255.0),
        near_plane=cfg.get("near_plane", 1.0e-4), camera_projection=cfg.get("camera_projection", "auto"),
        b200_options=cfg.get("b200"),
    )
    target = resize_images(clip_frames[0], render_size)
    recon = reconstruction_loss_per_image(renders, target, loss_cfg).sum() / frame_count
    (recon + regularizer_loss).backward()
    return recon.detach(), (renders[0].detach() if keep_preview else None)
