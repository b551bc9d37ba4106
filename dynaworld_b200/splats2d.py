"""Already-projected 2-D Gaussians over the C ABI, and their torch.autograd wrapper.

Shared core of the two 2-D contracts the reference renders through:

* conic -- ``rasterize_projected_gaussians(means2d, conics, colors, opacities, depths, config)`` of
  the fast-mac bridge (third_party/fast-mac-gsplat-scaffold/torch_gsplat_bridge/rasterize.py:93-126;
  kernels csrc/metal/gsplat_kernels.metal:40-297), used by src/train/renderers/fast_mac.py:253,301;
  :mod:`dynaworld_b200.gsplat_bridge` mirrors it.
* packed -- ``rasterize(packed, depths, features, image_size, config)`` of taichi-splatting as
  src/train/renderers/taichi.py:301-308 calls it, with the float64 restatement of
  src/benchmarks/splat_renderer_accuracy.py:262-305; :mod:`dynaworld_b200.packed_rasterizer`
  mirrors it.

Stages: gsb_splats2d_order -> gsb_splats2d_preprocess -> (one host read of the pair count) ->
gsb_bin -> gsb_raster_fwd; backward gsb_raster_bwd -> gsb_splats2d_preprocess_bwd.  The bin and
raster kernels are the ones the 3-D path uses.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .render import FrameState, _defer_status, _stage, _stream, _ws, check_pending, checkpoint_buffer, read_words

CONIC = _lib.SPLATS2D_CONIC
PACKED = _lib.SPLATS2D_PACKED
PACKED_FLOATS = 7


@dataclass(frozen=True)
class Splat2DOptions:
    """Blend semantics of the reference's 2-D kernels (gsplat_kernels.metal:160-204):
    pixel centres at +0.5, alpha = min(alpha_clamp, o exp(-q/2)), pairs with alpha below
    ``alpha_threshold`` skipped, a pixel stops after the entry that takes T below
    ``transmittance_threshold``, no (1 + eps) factor, image not clamped."""

    tile_size: int = 16
    alpha_threshold: float = 1.0 / 255.0
    transmittance_threshold: float = 1.0e-4
    alpha_clamp: float = 0.99
    background: tuple[float, float, float] = (0.0, 0.0, 0.0)
    clamp_image: bool = False

    def options(self) -> _lib.Options:
        if self.tile_size not in (8, 16):
            raise ValueError(f"tile_size must be 8 or 16, got {self.tile_size}")
        if not self.alpha_threshold > 0.0:
            raise ValueError("alpha_threshold must be positive")
        o = _lib.Options()
        o.tile_size = int(self.tile_size)
        o.flags = 0 if self.clamp_image else _lib.RENDER_NO_CLAMP
        o.near_plane = 1e-4  # unused by the 2-D stages
        o.alpha_clamp = float(self.alpha_clamp)
        o.alpha_cutoff = float(self.alpha_threshold)
        o.transmittance_threshold = float(self.transmittance_threshold)
        o.eps = 0.0
        o.pixel_center = 0.5
        for k in range(3):
            o.background[k] = float(self.background[k])
        o.bound_scale = 3.0
        o.tiled_alpha_threshold = float(self.alpha_threshold)
        return o


def _splats_struct(fmt: int, B: int, G: int, t: dict) -> _lib.Splats2D:
    s = _lib.Splats2D()
    s.n_views, s.n_gaussians, s.format = B, G, fmt
    s.means = _lib.ptr(t.get("means"))
    s.conics = _lib.ptr(t.get("conics"))
    s.opacities = _lib.ptr(t.get("opacities"))
    s.packed = _lib.ptr(t.get("packed"))
    s.colors = t["colors"].data_ptr()
    s.depths = _lib.ptr(t.get("depths"))
    return s


def _frame(B: int, H: int, W: int) -> _lib.Views:
    v = _lib.Views()
    v.n_views, v.views_per_set, v.height, v.width = B, 1, H, W
    return v


def forward_stages_2d(fmt: int, B: int, G: int, H: int, W: int, opt: Splat2DOptions, t: dict):
    """image [B,3,H,W], alpha (sum of weights) [B,H,W] and the state the backward reads."""
    L = _lib.lib()
    dev = t["colors"].device
    st = _stream(dev)
    sp = _splats_struct(fmt, B, G, t)
    frame = _frame(B, H, W)
    opts = opt.options()
    sorted_ids = torch.empty(B * G, dtype=torch.int32, device=dev)
    rank_of = torch.empty(B * G, dtype=torch.int32, device=dev)
    ws1 = _ws(L.gsb_splats2d_order_workspace(sp), dev)
    with _stage("order_2d"):
        _lib.check("gsb_splats2d_order", L.gsb_splats2d_order(sp, sorted_ids.data_ptr(), rank_of.data_ptr(),
                                                              ws1.data_ptr(), ws1.numel(), st))
    records = torch.empty(B * G * _lib.RECORD_FLOATS, dtype=torch.float32, device=dev)
    rects = torch.empty(B * G * 4, dtype=torch.int32, device=dev)
    offsets = torch.empty(B * G + 1, dtype=torch.int32, device=dev)
    ws2 = _ws(L.gsb_splats2d_preprocess_workspace(sp), dev)
    with _stage("preprocess_2d"):
        _lib.check("gsb_splats2d_preprocess",
                   L.gsb_splats2d_preprocess(sp, H, W, opts, rank_of.data_ptr(), records.data_ptr(), rects.data_ptr(),
                                             offsets.data_ptr(), ws2.data_ptr(), ws2.numel(), st))
    head = read_words([offsets[-1:], ws1.view(torch.int32)[:1], ws2.view(torch.int32)[:1]])
    n_tiles = -(-H // opt.tile_size) * -(-W // opt.tile_size)
    ranges = torch.empty(B * n_tiles * 2, dtype=torch.int32, device=dev)
    order = torch.empty(B * n_tiles, dtype=torch.int32, device=dev)
    image = torch.empty(B, 3, H, W, dtype=torch.float32, device=dev)
    alpha = torch.empty(B, H, W, dtype=torch.float32, device=dev)
    pixel_t = torch.empty(B, H, W, dtype=torch.float32, device=dev)
    pixel_state = torch.empty(B, H, W, dtype=torch.int32, device=dev)
    ckpt = checkpoint_buffer(frame, opts, dev)
    head = head.wait()
    check_pending(dev)
    n_pairs = head[0] & 0xFFFFFFFF
    for name, code in (("gsb_splats2d_order", head[1]), ("gsb_splats2d_preprocess", head[2])):
        _lib.check(name, code)
    keys = torch.empty(max(n_pairs, 1), dtype=torch.int64, device=dev)
    ws3 = _ws(L.gsb_bin_workspace(frame, opts, G, n_pairs), dev)
    with _stage("bin"):
        _lib.check("gsb_bin", L.gsb_bin(frame, opts, G, records.data_ptr(), rects.data_ptr(), offsets.data_ptr(),
                                        n_pairs, keys.data_ptr(), ranges.data_ptr(), order.data_ptr(),
                                        ws3.data_ptr(), ws3.numel(), st))
    with _stage("raster_fwd"):
        _lib.check("gsb_raster_fwd", L.gsb_raster_fwd(frame, opts, G, records.data_ptr(), keys.data_ptr(),
                                                      ranges.data_ptr(), order.data_ptr(), image.data_ptr(),
                                                      alpha.data_ptr(), None, pixel_t.data_ptr(),
                                                      pixel_state.data_ptr(), _lib.ptr(ckpt), st))
    _defer_status(dev, "gsb_bin", ws3.view(torch.int32)[:1])
    state = FrameState(rank_of, records, keys, ranges, order, pixel_t, pixel_state, n_pairs, ckpt)
    return image, alpha, state


def backward_stages_2d(fmt: int, B: int, G: int, H: int, W: int, opt: Splat2DOptions, t: dict, state: FrameState,
                       d_image: torch.Tensor, d_alpha: torch.Tensor | None) -> dict:
    L = _lib.lib()
    dev = t["colors"].device
    st = _stream(dev)
    sp = _splats_struct(fmt, B, G, t)
    frame = _frame(B, H, W)
    opts = opt.options()
    grad2d = torch.empty(B * G * _lib.GRAD2D_FLOATS, dtype=torch.float32, device=dev)
    with _stage("raster_bwd"):
        _lib.check("gsb_raster_bwd", L.gsb_raster_bwd(frame, opts, G, state.records.data_ptr(),
                                                      state.keys.data_ptr(), state.ranges.data_ptr(),
                                                      state.order.data_ptr(), state.pixel_t.data_ptr(),
                                                      state.pixel_state.data_ptr(), _lib.ptr(state.ckpt),
                                                      d_image.data_ptr(),
                                                      _lib.ptr(d_alpha), None, None, grad2d.data_ptr(), st))
    names = ("packed", "colors") if fmt == PACKED else ("means", "conics", "opacities", "colors")
    out = {k: torch.empty_like(t[k]) for k in names}
    g = _lib.Splats2DGrads()
    for k in names:
        setattr(g, k, out[k].data_ptr())
    with _stage("preprocess_2d_bwd"):
        _lib.check("gsb_splats2d_preprocess_bwd",
                   L.gsb_splats2d_preprocess_bwd(sp, state.rank_of.data_ptr(), grad2d.data_ptr(), g, st))
    return out


def _f32(x: torch.Tensor | None) -> torch.Tensor | None:
    return None if x is None else x.detach().to(torch.float32).contiguous()


class _Splats2DFunction(torch.autograd.Function):
    """(image [B,3,H,W], alpha [B,H,W]); gradients to (means, conics, opacities) or packed, and
    colors.  Depths only order the blend and get no gradient (gsplat_kernels.metal returns zeros)."""

    @staticmethod
    def forward(ctx, fmt, dims, opt, means, conics, opacities, packed, colors, depths):
        B, G, H, W = dims
        t = {"means": _f32(means), "conics": _f32(conics), "opacities": _f32(opacities), "packed": _f32(packed),
             "colors": _f32(colors), "depths": _f32(depths)}
        image, alpha, state = forward_stages_2d(fmt, B, G, H, W, opt, t)
        ctx.fmt, ctx.dims, ctx.opt, ctx.t, ctx.state = fmt, dims, opt, t, state
        ctx.meta = [None if x is None else (x.shape, x.dtype) for x in (means, conics, opacities, packed, colors)]
        return image, alpha

    @staticmethod
    def backward(ctx, d_image, d_alpha):
        B, G, H, W = ctx.dims
        dev = ctx.t["colors"].device
        if d_image is None:
            d_image = torch.zeros(B, 3, H, W, dtype=torch.float32, device=dev)
        d_image = d_image.to(torch.float32).contiguous()
        d_alpha = None if d_alpha is None else d_alpha.to(torch.float32).contiguous()
        grads = backward_stages_2d(ctx.fmt, B, G, H, W, ctx.opt, ctx.t, ctx.state, d_image, d_alpha)
        out = []
        for name, meta in zip(("means", "conics", "opacities", "packed", "colors"), ctx.meta):
            if meta is None or name not in grads:
                out.append(None)
            else:
                out.append(grads[name].reshape(meta[0]).to(meta[1]))
        ctx.state = None
        return (None, None, None, *out, None)


def render_splats2d(fmt: int, height: int, width: int, opt: Splat2DOptions, *, colors: torch.Tensor,
                    depths: torch.Tensor | None = None, means: torch.Tensor | None = None,
                    conics: torch.Tensor | None = None, opacities: torch.Tensor | None = None,
                    packed: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Batched entry: tensors carry a leading batch dimension [B, G, ...] (depths [B, G] or
    [B, G, 1]).  Returns image [B,3,H,W] and the summed weights [B,H,W]."""
    if not colors.is_cuda:
        raise RuntimeError("the b200 rasterizer runs on CUDA devices only (got a tensor on %s)" % colors.device)
    if colors.ndim != 3 or colors.shape[-1] != 3:
        raise ValueError("colors must have shape [B,G,3] (three channels)")
    B, G = int(colors.shape[0]), int(colors.shape[1])
    if fmt == PACKED:
        if packed is None or tuple(packed.shape) != (B, G, PACKED_FLOATS):
            raise ValueError(f"packed must have shape [B,G,7] = [{B},{G},7]")
    elif fmt == CONIC:
        if means is None or tuple(means.shape) != (B, G, 2):
            raise ValueError(f"means2d must have shape [{B},{G},2]")
        if conics is None or tuple(conics.shape) != (B, G, 3):
            raise ValueError(f"conics must have shape [{B},{G},3]")
        if opacities is None or opacities.numel() != B * G:
            raise ValueError(f"opacities must have {B * G} elements")
    else:
        raise ValueError(f"unknown 2-D format {fmt}")
    if depths is not None and depths.numel() != B * G:
        raise ValueError(f"depths must have {B * G} elements")
    if B == 0 or G == 0:
        dev = colors.device
        bg = torch.tensor(opt.background, dtype=torch.float32, device=dev).view(1, 3, 1, 1)
        image = bg.expand(B, 3, height, width).clone()
        return image, torch.zeros(B, height, width, dtype=torch.float32, device=dev)
    return _Splats2DFunction.apply(fmt, (B, G, int(height), int(width)), opt, means, conics, opacities, packed,
                                   colors, depths)
