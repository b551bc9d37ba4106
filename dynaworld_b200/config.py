"""Renderer options, read from a trainer's ``render.b200`` mapping.

Same construction contract as the reference's backend configs
(src/train/renderers/fast_mac.py:17-52, taichi.py:18-50):
``B200RendererConfig.from_mapping(values, *, fallback_tile_size, fallback_alpha_threshold)``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

from . import _lib

# alpha at or below 2^-25 leaves fl32(1 - alpha) == 1, so skipping such pairs reproduces the
# reference's transmittance factors bit for bit.
EXACT_ALPHA_CUTOFF = 2.0 ** -25

MODES = ("exact", "tiled_compat")


@dataclass(frozen=True)
class B200RendererConfig:
    """Options of the B200 renderer.

    mode="exact" reproduces the reference's dense renderer (src/train/renderers/dense.py):
    every Gaussian of the view contributes its (1 + eps) transmittance factor, pairs with alpha
    below ``alpha_cutoff`` count as alpha = 0, and a pixel stops once its transmittance drops
    below ``transmittance_threshold``.  mode="tiled_compat" reproduces the reference's tiled
    renderer (src/train/renderers/tiled.py): its tile bounds (``bound_scale``,
    ``tiled_alpha_threshold``) and its tile-local (1 + eps) products.
    """

    tile_size: int = 16
    mode: str = "exact"
    alpha_cutoff: float = EXACT_ALPHA_CUTOFF
    transmittance_threshold: float = 1e-7
    alpha_clamp: float = 0.99
    eps: float = 1e-6
    pixel_center: float = 0.0
    background: tuple[float, float, float] = (1.0, 1.0, 1.0)
    bound_scale: float = 3.0
    tiled_alpha_threshold: float = 1.0 / 255.0
    ellipse_culling: bool = True
    sh_clamp: bool = True
    depth: bool = False
    check_status: bool = False  # wait for binning's status word at once (else: at the next sync point)
    check_finite: bool = True  # raise FloatingPointError on non-finite projected Gaussians
    backward_segments: int = 0  # 1, 2, 4: pieces of each tile list in the reverse blend; 0: automatic

    def __post_init__(self):
        if self.mode not in MODES:
            raise ValueError(f"b200.mode must be one of {MODES}, got {self.mode!r}.")
        if self.tile_size not in (8, 16):
            raise ValueError(f"b200.tile_size must be 8 or 16, got {self.tile_size}.")
        if self.backward_segments not in (0, 1, 2, 4):
            raise ValueError(f"b200.backward_segments must be 0, 1, 2 or 4, got {self.backward_segments}.")
        if len(self.background) != 3:
            raise ValueError(f"b200.background must contain three values, got {self.background!r}.")

    @classmethod
    def from_mapping(
        cls,
        values: dict[str, Any] | None,
        *,
        fallback_tile_size: int,
        fallback_alpha_threshold: float,
    ) -> "B200RendererConfig":
        """Reads ``render.b200``.  The fallbacks are the trainer's generic ``tile_size`` and
        ``alpha_threshold``; they define the tile lists of tiled_compat mode (as they do for the
        reference's tiled renderer, src/train/rendering.py:191-211).  Exact mode uses 16x16 tiles
        unless ``tile_size`` is given, because its output does not depend on the tile size."""
        values = dict(values or {})
        mode = str(values.get("mode", cls.mode))
        default_tile = fallback_tile_size if mode == "tiled_compat" else cls.tile_size
        background = values.get("background", cls.background)
        if len(background) != 3:
            raise ValueError(f"b200.background must contain three values, got {background!r}.")
        return cls(
            tile_size=int(values.get("tile_size", default_tile)),
            mode=mode,
            alpha_cutoff=float(values.get("alpha_cutoff", cls.alpha_cutoff)),
            transmittance_threshold=float(values.get("transmittance_threshold", cls.transmittance_threshold)),
            alpha_clamp=float(values.get("alpha_clamp", cls.alpha_clamp)),
            eps=float(values.get("eps", cls.eps)),
            pixel_center=float(values.get("pixel_center", cls.pixel_center)),
            background=tuple(float(v) for v in background),
            bound_scale=float(values.get("bound_scale", cls.bound_scale)),
            tiled_alpha_threshold=float(values.get("alpha_threshold", fallback_alpha_threshold)),
            ellipse_culling=bool(values.get("ellipse_culling", cls.ellipse_culling)),
            sh_clamp=bool(values.get("sh_clamp", cls.sh_clamp)),
            depth=bool(values.get("depth", cls.depth)),
            check_status=bool(values.get("check_status", cls.check_status)),
            check_finite=bool(values.get("check_finite", cls.check_finite)),
            backward_segments=int(values.get("backward_segments", cls.backward_segments)),
        )

    def options(self, near_plane: float) -> "_lib.Options":
        o = _lib.Options()
        o.tile_size = self.tile_size
        flags = 0
        if self.mode == "tiled_compat":
            flags |= _lib.RENDER_TILED_COMPAT
        if self.depth:
            flags |= _lib.RENDER_DEPTH
        if not self.ellipse_culling:
            flags |= _lib.RENDER_NO_ELLIPSE
        o.flags = flags
        o.near_plane = float(near_plane)
        o.alpha_clamp = self.alpha_clamp
        o.alpha_cutoff = self.alpha_cutoff
        o.transmittance_threshold = self.transmittance_threshold
        o.eps = self.eps
        o.pixel_center = self.pixel_center
        for k in range(3):
            o.background[k] = self.background[k]
        o.bound_scale = self.bound_scale
        o.tiled_alpha_threshold = self.tiled_alpha_threshold
        o.backward_segments = self.backward_segments
        return o


LOSS_TYPES = {"standard_gs": 0, "l1": 1, "mse": 2, "l1_mse": 3}


@dataclass(frozen=True)
class LossConfig:
    """losses.py options (src/train/dynamicTokenGS.py:115-123 defaults) plus the SSIM window
    ('box' as the reference, or 'gaussian' with ``ssim_sigma``) and the D-SSIM 1/2 factor."""

    type: str = "standard_gs"
    l1_weight: float = 0.8
    dssim_weight: float = 0.2
    mse_weight: float = 0.2
    ssim_window_size: int = 11
    ssim_c1: float = 1e-4
    ssim_c2: float = 9e-4
    ssim_window: str = "box"
    ssim_sigma: float = 1.5
    dssim_half: bool = True
    extra: dict = field(default_factory=dict, compare=False)

    @classmethod
    def from_mapping(cls, values: dict[str, Any] | None) -> "LossConfig":
        values = dict(values or {})
        kind = str(values.get("type", cls.type)).lower()
        if kind not in LOSS_TYPES:
            raise ValueError(f"Unknown reconstruction loss type: {kind!r}")
        window = str(values.get("ssim_window", cls.ssim_window))
        if window not in ("box", "gaussian"):
            raise ValueError(f"ssim_window must be 'box' or 'gaussian', got {window!r}")
        return cls(
            type=kind,
            l1_weight=float(values.get("l1_weight", cls.l1_weight)),
            dssim_weight=float(values.get("dssim_weight", cls.dssim_weight)),
            mse_weight=float(values.get("mse_weight", cls.mse_weight)),
            ssim_window_size=int(values.get("ssim_window_size", cls.ssim_window_size)),
            ssim_c1=float(values.get("ssim_c1", cls.ssim_c1)),
            ssim_c2=float(values.get("ssim_c2", cls.ssim_c2)),
            ssim_window=window,
            ssim_sigma=float(values.get("ssim_sigma", cls.ssim_sigma)),
            dssim_half=bool(values.get("dssim_half", cls.dssim_half)),
        )

    def options(self) -> "_lib.LossOptions":
        o = _lib.LossOptions()
        o.type = LOSS_TYPES[self.type]
        o.window_size = self.ssim_window_size
        o.window = 1 if self.ssim_window == "gaussian" else 0
        o.dssim_half = 1 if self.dssim_half else 0
        o.l1_weight = self.l1_weight
        o.dssim_weight = self.dssim_weight
        o.mse_weight = self.mse_weight
        o.c1 = self.ssim_c1
        o.c2 = self.ssim_c2
        o.sigma = self.ssim_sigma
        return o
