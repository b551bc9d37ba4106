"""Drop-in for the fast-mac bridge's projected-Gaussian rasterizer, on B200.

Mirrors ``torch_gsplat_bridge`` (third_party/fast-mac-gsplat-scaffold/torch_gsplat_bridge/
rasterize.py:15-141) and the fields its v5 successor takes from src/train/renderers/fast_mac.py:
62-76 (``_make_v5_config``): same names, argument shapes, output layout (image HWC, or BHWC for a
batch) and validation errors.  The v5 package itself is an un-vendored submodule
(third_party/fast-mac-gsplat); the blend follows the vendored Metal kernels
(csrc/metal/gsplat_kernels.metal:40-297), which define the same contract:

* tiles from the Gaussian's q <= tau ellipse, tau = -2 ln(alpha_threshold / opacity);
* per pixel p = (x + 0.5, y + 0.5), Gaussians in ascending ``depths`` order (ties by index):
  alpha = min(0.99, o exp(-q/2)), skipped below ``alpha_threshold``; w = T alpha; T *= 1 - alpha;
  the pixel stops once T < ``transmittance_threshold``;
* out = sum w c + T background, not clamped (the caller clamps, fast_mac.py:261,309).

The v5-only fields (``max_fast_pairs``, ``enable_overflow_fallback``, ``batch_strategy`` and the
launch limits) tune the Metal scheduler; they are accepted and have no effect here: this
rasterizer has no per-tile pair cap to overflow, and a batch is one launch.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple

import torch
from torch import Tensor

from .splats2d import CONIC, Splat2DOptions, render_splats2d


@dataclass(frozen=True)
class RasterConfig:
    height: int
    width: int
    tile_size: int = 16
    chunk_size: int = 32
    alpha_threshold: float = 1.0 / 255.0
    transmittance_threshold: float = 1e-4
    background: Tuple[float, float, float] = (0.0, 0.0, 0.0)
    max_fast_pairs: int = 2048
    enable_overflow_fallback: bool = True
    batch_strategy: str = "flatten"
    batch_launch_limit_tiles: int = 262144
    batch_launch_limit_gaussians: int = 262144

    def options(self) -> Splat2DOptions:
        if len(self.background) != 3:
            raise ValueError(f"background must contain three values, got {self.background!r}.")
        return Splat2DOptions(tile_size=int(self.tile_size), alpha_threshold=float(self.alpha_threshold),
                              transmittance_threshold=float(self.transmittance_threshold), alpha_clamp=0.99,
                              background=tuple(float(v) for v in self.background), clamp_image=False)


def _check(name: str, t: Tensor, ndim: int, last: int | None, shape_text: str) -> None:
    if t.ndim != ndim or (last is not None and t.shape[-1] != last):
        raise ValueError(f"{name} must have shape {shape_text}")


def rasterize_projected_gaussians(
    means2d: Tensor,
    conics: Tensor,
    colors: Tensor,
    opacities: Tensor,
    depths: Tensor,
    config: RasterConfig,
) -> Tensor:
    """means2d [G,2], conics [G,3] (a, b, c: q = a dx^2 + 2 b dx dy + c dy^2), colors [G,3],
    opacities [G], depths [G] -> image [H,W,3]; or the same with a leading batch dimension
    [B,G,...] -> [B,H,W,3].  Differentiable in means2d, conics, colors and opacities."""
    batched = means2d.ndim == 3
    if batched:
        _check("means2d", means2d, 3, 2, "[B,G,2]")
        _check("conics", conics, 3, 3, "[B,G,3]")
        _check("colors", colors, 3, 3, "[B,G,3]")
        _check("opacities", opacities, 2, None, "[B,G]")
        _check("depths", depths, 2, None, "[B,G]")
        m, q, c, o, d = means2d, conics, colors, opacities, depths
    else:
        _check("means2d", means2d, 2, 2, "[G,2]")
        _check("conics", conics, 2, 3, "[G,3]")
        _check("colors", colors, 2, 3, "[G,3]")
        _check("opacities", opacities, 1, None, "[G]")
        _check("depths", depths, 1, None, "[G]")
        m, q, c, o, d = means2d[None], conics[None], colors[None], opacities[None], depths[None]
    image, _alpha = render_splats2d(CONIC, config.height, config.width, config.options(), colors=c, depths=d,
                                    means=m, conics=q, opacities=o)
    image = image.permute(0, 2, 3, 1)
    return image if batched else image[0]


class ProjectedGaussianRasterizer(torch.nn.Module):
    def __init__(self, config: RasterConfig):
        super().__init__()
        self.config = config

    def forward(self, means2d: Tensor, conics: Tensor, colors: Tensor, opacities: Tensor, depths: Tensor) -> Tensor:
        return rasterize_projected_gaussians(means2d, conics, colors, opacities, depths, self.config)


__all__ = ["RasterConfig", "rasterize_projected_gaussians", "ProjectedGaussianRasterizer"]
