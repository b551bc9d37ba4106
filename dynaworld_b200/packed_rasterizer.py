"""Drop-in for the packed-splat rasterizer the reference calls through taichi-splatting, on B200.

Mirrors the calls of src/train/renderers/taichi.py:301-308 and :364-371
(``rasterize`` / ``rasterize_batch(packed, depths, features, image_size=(W, H), config=...,
use_depth16=...)`` returning ``.image`` [H,W,C] and ``.image_weight`` [H,W]) and the
``RasterConfig`` fields of taichi.py:94-104.  taichi-splatting is an un-vendored submodule
(third_party/taichi-splatting); the semantics follow the reference's float64 restatement of it,
``torch_reference_rasterize`` (src/benchmarks/splat_renderer_accuracy.py:262-305):

* packed rows [mean x, y, axis x, y, sigma0, sigma1, opacity]; pixel p = (x + 0.5, y + 0.5);
  q = ((p - mean).axis / sigma0)^2 + ((p - mean).perp / sigma1)^2, perp = (-axis y, axis x);
* Gaussians in ascending depth order; alpha = min(clamp_max_alpha, opacity exp(-q/2)), skipped
  unless above alpha_threshold; w = alpha (1 - W) while W = sum of earlier w is below
  saturate_threshold (1 - W is the transmittance T; the pixel stops after the entry that takes
  T below 1 - saturate_threshold);
* image = sum w features (no background), image_weight = W.  The caller composites the
  background (taichi.py:309,372, splat_renderer_accuracy.py:341).

The Taichi kernel-selection fields (``kernel_variant``, ``sort_backend``, ``backward_variant``,
``metal_block_dim``, ``metal_compatible``) and ``use_depth16`` pick among Taichi implementations
of the same blend; they are accepted and have no effect here.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from .splats2d import PACKED, PACKED_FLOATS, Splat2DOptions, render_splats2d


@dataclass(frozen=True)
class RasterConfig:
    tile_size: int = 16
    alpha_threshold: float = 1.0 / 255.0
    clamp_max_alpha: float = 0.99
    saturate_threshold: float = 0.9999
    metal_compatible: bool = False
    kernel_variant: str = "cuda_simt"
    sort_backend: str = "auto"
    backward_variant: str = "pixel_reference"
    metal_block_dim: int = 0
    use_alpha_blending: bool = True
    antialias: bool = False

    def options(self) -> Splat2DOptions:
        if not self.use_alpha_blending:
            raise ValueError("only alpha blending is implemented (use_alpha_blending=True).")
        if self.antialias:
            raise ValueError("the antialiased Gaussian PDF is not implemented (antialias=False).")
        return Splat2DOptions(tile_size=int(self.tile_size), alpha_threshold=float(self.alpha_threshold),
                              transmittance_threshold=float(1.0 - self.saturate_threshold),
                              alpha_clamp=float(self.clamp_max_alpha), background=(0.0, 0.0, 0.0),
                              clamp_image=False)


@dataclass
class Rasterization:
    image: Tensor         # [H,W,C] or [B,H,W,C]: sum of weights x features (no background)
    image_weight: Tensor  # [H,W] or [B,H,W]: sum of weights


def _unpack_size(image_size) -> tuple[int, int]:
    width, height = (int(v) for v in image_size)
    return height, width


def rasterize_batch(gaussians: Tensor, depths: Tensor, features: Tensor, image_size, config: RasterConfig,
                    use_depth16: bool = False) -> Rasterization:
    """gaussians [B,G,7], depths [B,G] or [B,G,1], features [B,G,3], image_size (width, height)."""
    del use_depth16
    if gaussians.ndim != 3 or gaussians.shape[-1] != PACKED_FLOATS:
        raise ValueError("gaussians must have shape [B,G,7]")
    if features.ndim != 3 or features.shape[:2] != gaussians.shape[:2]:
        raise ValueError("features must have shape [B,G,C]")
    if features.shape[-1] != 3:
        raise ValueError(f"features must have 3 channels, got {features.shape[-1]}")
    height, width = _unpack_size(image_size)
    image, weight = render_splats2d(PACKED, height, width, config.options(), colors=features,
                                    depths=depths.reshape(gaussians.shape[0], gaussians.shape[1]),
                                    packed=gaussians)
    return Rasterization(image=image.permute(0, 2, 3, 1), image_weight=weight)


def rasterize(gaussians: Tensor, depths: Tensor, features: Tensor, image_size, config: RasterConfig,
              use_depth16: bool = False) -> Rasterization:
    """gaussians [G,7], depths [G] or [G,1], features [G,3], image_size (width, height)."""
    if gaussians.ndim != 2 or gaussians.shape[-1] != PACKED_FLOATS:
        raise ValueError("gaussians must have shape [G,7]")
    r = rasterize_batch(gaussians[None], depths.reshape(1, -1), features[None], image_size, config, use_depth16)
    return Rasterization(image=r.image[0], image_weight=r.image_weight[0])


__all__ = ["RasterConfig", "Rasterization", "rasterize", "rasterize_batch"]
