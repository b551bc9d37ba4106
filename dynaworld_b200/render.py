"""Render pipeline over the C ABI, and its torch.autograd wrapper.

Forward: depth order -> projection/bounds/pair offsets -> (one host read of the pair count) ->
pair keys + radix sort + tile ranges -> blend.  Backward: reverse blend -> chain rule to the scene
parameters.  Every stage is a libgsb200 kernel; torch only allocates memory and supplies the
stream.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass

import torch

from . import _lib
from .config import B200RendererConfig

MIN_RENDER_DEPTH = 1e-4  # src/train/renderers/common.py:3

# Optional stage timing: when set to a list, every C-ABI stage call appends
# (stage name, start event, end event), both recorded on the launching stream; STAGE_FILTER (a set
# of stage names, or None for all) limits which stages are bracketed.
STAGE_EVENTS: list | None = None
STAGE_FILTER: set | None = None
# NVTX ranges "gsb:<stage>" around every C-ABI stage call (diagnostics.nvtx).
NVTX = False
# When a list, every forward appends the lists it built (diagnostics.collect / FrameLists).
STATS_FRAMES: list | None = None


class _stage:
    """Brackets one C-ABI call with CUDA events when STAGE_EVENTS is enabled, and with an NVTX
    range when NVTX is."""

    def __init__(self, name: str):
        self.name = name
        self.ev = None
        self.nvtx = False

    def __enter__(self):
        if NVTX:
            torch.cuda.nvtx.range_push("gsb:" + self.name)
            self.nvtx = True
        if STAGE_EVENTS is not None and (STAGE_FILTER is None or self.name in STAGE_FILTER):
            self.ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self.ev[0].record()
        return self

    def __exit__(self, *exc):
        if self.ev is not None:
            self.ev[1].record()
            STAGE_EVENTS.append((self.name, *self.ev))
        if self.nvtx:
            torch.cuda.nvtx.range_pop()
        return False


@dataclass
class SceneSpec:
    """Non-tensor description of a scene (Gaussian parameter sets)."""

    n_sets: int
    n_gaussians: int
    raw: bool
    sh_degree: int
    velocity: bool
    sh_clamp: bool
    bank_basis: int = 0  # dynamic bank: temporal basis functions M (0: no bank)
    bank_first: int = 0  # dynamic bank: Gaussians before this index are static
    # decoder-head activation (xy_extent, z_min, z_extent, scale_init) of the head's raw outputs, or None
    head: tuple[float, float, float, float] | None = None


@dataclass
class ViewSpec:
    n_views: int
    views_per_set: int
    height: int
    width: int


@dataclass
class FrameState:
    """What the backward needs from the forward (all device tensors)."""

    rank_of: torch.Tensor
    records: torch.Tensor
    keys: torch.Tensor
    ranges: torch.Tensor
    order: torch.Tensor
    pixel_t: torch.Tensor
    pixel_state: torch.Tensor
    n_pairs: int
    ckpt: torch.Tensor | None = None  # backward segment checkpoints (None: one segment)


def checkpoint_buffer(views: _lib.Views, opts: _lib.Options, device) -> torch.Tensor | None:
    n = int(_lib.lib().gsb_raster_checkpoint_floats(views, opts))
    return torch.empty(n, dtype=torch.float32, device=device) if n else None


def _stream(device) -> int:
    """Raw handle of the device's current stream (the handle torch.cuda.current_stream(device)
    wraps, without building the Stream object: this runs several times per step on the host)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(index)


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


_PINNED = threading.local()


class _Words:
    """Device int32 words on their way to a pinned host buffer (see read_words)."""

    def __init__(self, buf: torch.Tensor, n: int, event: torch.cuda.Event):
        self.buf, self.n, self.event = buf, n, event

    def wait(self) -> list[int]:
        self.event.synchronize()
        return self.buf[: self.n].tolist()


def read_words(words: list[torch.Tensor], own_buffer: bool = False) -> _Words:
    """Queues device->host copies of single int32 words (all on one device) behind that device's
    current stream and returns at once; .wait() blocks until they have landed.  One pinned buffer
    per host thread (each wait completes before that thread queues its next read), or with
    ``own_buffer`` a pinned buffer of the read's own (for reads that are waited for later, possibly
    by another thread)."""
    if own_buffer:
        buf = torch.empty(max(4, len(words)), dtype=torch.int32, pin_memory=True)
    else:
        buf = getattr(_PINNED, "buf", None)
        if buf is None or buf.numel() < len(words):
            buf = torch.empty(max(8, len(words)), dtype=torch.int32, pin_memory=True)
            _PINNED.buf = buf
    dev = words[0].device
    with torch.cuda.device(dev):
        for i, w in enumerate(words):
            buf[i : i + 1].copy_(w, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(dev))
    return _Words(buf, len(words), ev)


# Status words of stages whose result the host does not wait for (binning's sort and emission):
# read into pinned memory behind the kernels and checked at the device's next synchronisation
# point, i.e. when the backward of that frame has been queued or when the next forward waits for
# its pair count, whichever comes first.  No extra host-device synchronisation.
_PENDING: dict[int, list[tuple[str, _Words]]] = {}

# Data-parallel gradient reducer (distributed.GradientAllReduce) the backward hands its parameter
# gradients to, or None.
_GRAD_REDUCER = None


def set_gradient_reducer(reducer) -> None:
    """Installs (or, with None, removes) the reducer the render backward sums its parameter
    gradients over ranks with (distributed.GradientAllReduce): the sum then happens inside the
    backward, overlapped with the chain-rule kernel, and the returned gradients are already
    summed.  Scenes with per-clip Gaussian sets or a dynamic bank are not reduced."""
    global _GRAD_REDUCER
    _GRAD_REDUCER = reducer
_PENDING_LOCK = threading.Lock()


def _defer_status(dev: torch.device, name: str, word: torch.Tensor) -> None:
    words = read_words([word], own_buffer=True)
    with _PENDING_LOCK:
        _PENDING.setdefault(dev.index, []).append((name, words))


def check_pending(dev: torch.device) -> None:
    """Waits for the deferred status words of ``dev`` and raises on the first error among them."""
    with _PENDING_LOCK:
        pending = _PENDING.pop(dev.index, [])
    for name, words in pending:
        code = words.wait()[0]
        if code != _lib.GSB_OK:
            raise _lib.GsbError(f"{name} (reported at the next synchronisation point)", code)


def _f32(t: torch.Tensor | None) -> torch.Tensor | None:
    if t is None:
        return None
    return t.detach().to(dtype=torch.float32).contiguous()


def scene_struct(spec: SceneSpec, means, scales, quats, opacities, colors, velocity, bank=None) -> _lib.Scene:
    """``bank``: (bank_mu, bank_rot, bank_alpha) device tensors when spec.bank_basis > 0."""
    s = _lib.Scene()
    s.n_sets = spec.n_sets
    s.n_gaussians = spec.n_gaussians
    s.sh_degree = spec.sh_degree
    flags = 0
    if spec.head is not None:
        flags |= _lib.SCENE_HEAD
        s.head_xy_extent, s.head_z_min, s.head_z_extent, s.head_scale_init = (float(v) for v in spec.head)
    elif spec.raw:
        flags |= _lib.SCENE_RAW
        if spec.sh_clamp:
            flags |= _lib.SCENE_SH_CLAMP
    if spec.velocity:
        flags |= _lib.SCENE_VELOCITY
    if spec.bank_basis:
        flags |= _lib.SCENE_BANK
        s.bank_mu, s.bank_rot, s.bank_alpha = (t.data_ptr() for t in bank)
        s.bank_first, s.bank_basis = spec.bank_first, spec.bank_basis
    s.flags = flags
    s.means, s.scales, s.quats = means.data_ptr(), scales.data_ptr(), quats.data_ptr()
    s.opacities, s.colors = opacities.data_ptr(), colors.data_ptr()
    s.velocity = velocity.data_ptr() if velocity is not None else None
    return s


def _scene_of(sspec: SceneSpec, t: dict) -> _lib.Scene:
    bank = (t["bank_mu"], t["bank_rot"], t["bank_alpha"]) if sspec.bank_basis else None
    return scene_struct(sspec, t["means"], t["scales"], t["quats"], t["opacities"], t["colors"], t.get("velocity"),
                        bank)


def views_struct(spec: ViewSpec, intrinsics, camera_to_world, times, lens_models=None, distortion=None,
                 basis=None) -> _lib.Views:
    v = _lib.Views()
    v.n_views, v.views_per_set, v.height, v.width = spec.n_views, spec.views_per_set, spec.height, spec.width
    v.intrinsics = intrinsics.data_ptr()
    v.camera_to_world = camera_to_world.data_ptr()
    v.times = times.data_ptr() if times is not None else None
    v.lens_models = lens_models.data_ptr() if lens_models is not None else None
    v.distortion = distortion.data_ptr() if lens_models is not None else None
    v.basis = basis.data_ptr() if basis is not None else None
    return v


def _views_of(vspec: ViewSpec, tensors: dict) -> _lib.Views:
    return views_struct(vspec, tensors["intrinsics"], tensors["camera_to_world"], tensors.get("times"),
                        tensors.get("lens_models"), tensors.get("distortion"), tensors.get("basis"))


# Pair-key capacity per frame shape (device, views, Gaussians, image, tile size, mode), from the
# frames rendered before: binning and the blend are queued with it before the exact count reaches
# the host, so the GPU does not wait on the host there.  A count above it (first frames, growth)
# re-runs the two stages with the count.
_PAIR_CAPACITY: dict = {}


def _next_capacity(n_pairs: int, cap: int | None) -> int:
    if cap is not None and n_pairs <= cap and 2 * n_pairs >= cap:
        return cap
    return -(-(n_pairs + n_pairs // 4 + 4096) // 65536) * 65536


def forward_stages(sspec: SceneSpec, vspec: ViewSpec, cfg: B200RendererConfig, near_plane: float,
                   tensors: dict) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None, FrameState]:
    L = _lib.lib()
    dev = tensors["means"].device
    st = _stream(dev)
    B, G, H, W = vspec.n_views, sspec.n_gaussians, vspec.height, vspec.width
    scene = _scene_of(sspec, tensors)
    views = _views_of(vspec, tensors)
    opts = cfg.options(near_plane)

    sorted_ids = torch.empty(B * G, dtype=torch.int32, device=dev)
    rank_of = torch.empty(B * G, dtype=torch.int32, device=dev)
    ws1 = _ws(L.gsb_depth_order_workspace(scene, views), dev)
    with _stage("depth_order"):
        _lib.check("gsb_depth_order", L.gsb_depth_order(scene, views, sorted_ids.data_ptr(), rank_of.data_ptr(),
                                                        ws1.data_ptr(), ws1.numel(), st))
    records = torch.empty(B * G * _lib.RECORD_FLOATS, dtype=torch.float32, device=dev)
    rects = torch.empty(B * G * 4, dtype=torch.int32, device=dev)
    offsets = torch.empty(B * G + 1, dtype=torch.int32, device=dev)
    ws2 = _ws(L.gsb_preprocess_workspace(views, G), dev)
    with _stage("preprocess_fwd"):
        _lib.check("gsb_preprocess_fwd", L.gsb_preprocess_fwd(scene, views, opts, rank_of.data_ptr(),
                                                              records.data_ptr(), rects.data_ptr(),
                                                              offsets.data_ptr(), None, ws2.data_ptr(), ws2.numel(),
                                                              st))
    # The one host synchronisation of the forward: the pair count plus the device status words,
    # copied into pinned memory behind the kernels.  Binning reads the count on the device, so with
    # a capacity known from earlier frames of this shape it and the blend are queued first.
    ws2w = ws2.view(torch.int32)
    head = read_words([offsets[-1:], ws1.view(torch.int32)[:1], ws2w[0:1], ws2w[1:2], ws2w[2:3]])
    n_tiles = -(-H // cfg.tile_size) * -(-W // cfg.tile_size)
    ranges = torch.empty(B * n_tiles * 2, dtype=torch.int32, device=dev)
    order = torch.empty(B * n_tiles, dtype=torch.int32, device=dev)
    image = torch.empty(B, 3, H, W, dtype=torch.float32, device=dev)
    alpha = torch.empty(B, H, W, dtype=torch.float32, device=dev)
    depth = torch.empty(B, H, W, dtype=torch.float32, device=dev) if cfg.depth else None
    pixel_t = torch.empty(B, H, W, dtype=torch.float32, device=dev)
    pixel_state = torch.empty(B, H, W, dtype=torch.int32, device=dev)
    ckpt = checkpoint_buffer(views, opts, dev)

    def bin_and_blend(capacity: int):
        keys = torch.empty(max(capacity, 1), dtype=torch.int64, device=dev)
        ws3 = _ws(L.gsb_bin_workspace(views, opts, G, capacity), dev)
        with _stage("bin"):
            _lib.check("gsb_bin", L.gsb_bin(views, opts, G, records.data_ptr(), rects.data_ptr(),
                                            offsets.data_ptr(), capacity, keys.data_ptr(), ranges.data_ptr(),
                                            order.data_ptr(), ws3.data_ptr(), ws3.numel(), st))
        with _stage("raster_fwd"):
            _lib.check("gsb_raster_fwd", L.gsb_raster_fwd(views, opts, G, records.data_ptr(), keys.data_ptr(),
                                                          ranges.data_ptr(), order.data_ptr(), image.data_ptr(),
                                                          alpha.data_ptr(), _lib.ptr(depth), pixel_t.data_ptr(),
                                                          pixel_state.data_ptr(), _lib.ptr(ckpt), st))
        return keys, ws3

    shape = (dev.index, B, G, H, W, cfg.tile_size, cfg.mode)
    cap = _PAIR_CAPACITY.get(shape)
    if cap is not None:
        keys, ws3 = bin_and_blend(cap)
    head = head.wait()
    check_pending(dev)  # earlier frames' deferred status words have landed by now
    n_pairs = head[0] & 0xFFFFFFFF
    _lib.check("gsb_depth_order", head[1])
    if head[2] == _lib.GSB_ERR_NONFINITE:
        if cfg.check_finite:
            first = head[3]
            raise FloatingPointError(
                f"Non-finite render input: {head[4]} projected Gaussians are not finite (first: view "
                f"{first // G}, Gaussian {first % G}).")
    else:
        _lib.check("gsb_preprocess_fwd", head[2])
    if cap is None or n_pairs > cap:  # no guess yet, or too small: again with the count
        keys, ws3 = bin_and_blend(n_pairs)
    _PAIR_CAPACITY[shape] = _next_capacity(n_pairs, cap)
    if cfg.check_status:
        _lib.check("gsb_bin", int(ws3.view(torch.int32)[0].item()))
    else:
        _defer_status(dev, "gsb_bin", ws3.view(torch.int32)[:1])
    state = FrameState(rank_of, records, keys, ranges, order, pixel_t, pixel_state, n_pairs, ckpt)
    if STATS_FRAMES is not None:
        from .diagnostics import FrameLists

        STATS_FRAMES.append(FrameLists(B, G, n_tiles, cfg.tile_size, cfg.mode, offsets, ranges))
    return image, alpha, depth, state


def backward_stages(sspec: SceneSpec, vspec: ViewSpec, cfg: B200RendererConfig, near_plane: float, tensors: dict,
                    state: FrameState, d_image: torch.Tensor, d_alpha: torch.Tensor | None,
                    d_depth: torch.Tensor | None, view_scale: torch.Tensor | None = None,
                    camera: bool = False) -> dict:
    """Gradients of the scene tensors; with ``camera`` also "cam_intrinsics" [B,4],
    "cam_camera_to_world" [B,4,4] and, with lenses, "cam_distortion" [B,5]."""
    L = _lib.lib()
    dev = tensors["means"].device
    st = _stream(dev)
    B, G = vspec.n_views, sspec.n_gaussians
    scene = _scene_of(sspec, tensors)
    views = _views_of(vspec, tensors)
    opts = cfg.options(near_plane)
    grad2d = torch.empty(B * G * _lib.GRAD2D_FLOATS, dtype=torch.float32, device=dev)
    with _stage("raster_bwd"):
        _lib.check("gsb_raster_bwd", L.gsb_raster_bwd(views, opts, G, state.records.data_ptr(),
                                                      state.keys.data_ptr(), state.ranges.data_ptr(),
                                                      state.order.data_ptr(),
                                                      state.pixel_t.data_ptr(), state.pixel_state.data_ptr(),
                                                      _lib.ptr(state.ckpt),
                                                      d_image.data_ptr(), _lib.ptr(d_alpha), _lib.ptr(d_depth),
                                                      _lib.ptr(view_scale), grad2d.data_ptr(), st))
    # every parameter gradient is a view of one flat buffer: a data-parallel sum over ranks is then
    # one in-place collective (distributed.allreduce_gradients), with no gather or scatter copies
    names = ["means", "scales", "quats", "opacities", "colors"] + (["velocity"] if sspec.velocity else [])
    flat = torch.empty(sum(tensors[k].numel() for k in names), dtype=torch.float32, device=dev)
    out, off = {}, 0
    for k in names:
        n = tensors[k].numel()
        out[k] = flat[off:off + n].view(tensors[k].shape)
        off += n
    g = _lib.SceneGrads()
    g.means, g.scales, g.quats = out["means"].data_ptr(), out["scales"].data_ptr(), out["quats"].data_ptr()
    g.opacities, g.colors = out["opacities"].data_ptr(), out["colors"].data_ptr()
    g.velocity = out["velocity"].data_ptr() if "velocity" in out else None
    if sspec.bank_basis:
        for k in ("bank_mu", "bank_rot", "bank_alpha"):
            out[k] = torch.empty_like(tensors[k])
        g.bank_mu, g.bank_rot, g.bank_alpha = (out[k].data_ptr() for k in ("bank_mu", "bank_rot", "bank_alpha"))
    reducer = _GRAD_REDUCER
    if reducer is not None and sspec.n_sets == 1 and not sspec.bank_basis and reducer.active():
        # chain rule in ranges of Gaussians; each range's rows are summed over the ranks (on the
        # collective's stream) while the next range is computed
        G1 = sspec.n_gaussians
        with _stage("preprocess_bwd"):
            for c in range(reducer.buckets):
                g0, g1 = c * G1 // reducer.buckets, (c + 1) * G1 // reducer.buckets
                _lib.check("gsb_preprocess_bwd_range",
                           L.gsb_preprocess_bwd_range(scene, views, opts, state.rank_of.data_ptr(), grad2d.data_ptr(),
                                                      g, g0, g1 - g0, st))
                reducer.reduce([out[k].view(G1, -1)[g0:g1] for k in names])
            reducer.finish()
    else:
        with _stage("preprocess_bwd"):
            _lib.check("gsb_preprocess_bwd", L.gsb_preprocess_bwd(scene, views, opts, state.rank_of.data_ptr(),
                                                                  grad2d.data_ptr(), g, st))
    check_pending(dev)  # the forward's binning status, while the GPU runs the kernels just queued
    if camera:
        out["cam_intrinsics"] = torch.empty(B, 4, dtype=torch.float32, device=dev)
        out["cam_camera_to_world"] = torch.empty(B, 4, 4, dtype=torch.float32, device=dev)
        cg = _lib.CameraGrads()
        cg.intrinsics, cg.camera_to_world = out["cam_intrinsics"].data_ptr(), out["cam_camera_to_world"].data_ptr()
        if tensors.get("lens_models") is not None:
            out["cam_distortion"] = torch.empty(B, _lib.DISTORTION_FLOATS, dtype=torch.float32, device=dev)
            cg.distortion = out["cam_distortion"].data_ptr()
        with _stage("camera_bwd"):
            _lib.check("gsb_camera_bwd", L.gsb_camera_bwd(scene, views, opts, state.rank_of.data_ptr(),
                                                          grad2d.data_ptr(), cg, st))
    return out


_PARAM_NAMES = ("means", "scales", "quats", "opacities", "colors", "velocity")
_BANK_NAMES = ("bank_mu", "bank_rot", "bank_alpha")


_CAMERA_NAMES = ("cam_intrinsics", "cam_camera_to_world", None, "cam_distortion")  # times get none


class _RenderFunction(torch.autograd.Function):
    """(image [B,3,H,W], alpha [B,H,W], depth [B,H,W]) of the scene; gradients flow to the six
    scene tensors, the dynamic bank's coefficients and, when they require them, to the
    intrinsics, camera_to_world and lens distortion (not to the per-view times or the basis)."""

    @staticmethod
    def forward(ctx, sspec, vspec, cfg, near_plane, lens_models, means, scales, quats, opacities, colors, velocity,
                intrinsics, camera_to_world, times, distortion, bank_mu, bank_rot, bank_alpha, basis):
        tensors = {
            "means": _f32(means), "scales": _f32(scales), "quats": _f32(quats), "opacities": _f32(opacities),
            "colors": _f32(colors), "velocity": _f32(velocity), "intrinsics": _f32(intrinsics),
            "camera_to_world": _f32(camera_to_world), "times": _f32(times), "bank_mu": _f32(bank_mu),
            "bank_rot": _f32(bank_rot), "bank_alpha": _f32(bank_alpha), "basis": _f32(basis),
        }
        if lens_models is not None:
            tensors["lens_models"], tensors["distortion"] = lens_models, _f32(distortion)
        image, alpha, depth, state = forward_stages(sspec, vspec, cfg, near_plane, tensors)
        ctx.sspec, ctx.vspec, ctx.cfg, ctx.near_plane = sspec, vspec, cfg, near_plane
        ctx.tensors = tensors
        ctx.state = state
        ctx.shapes = [None if t is None else (t.shape, t.dtype) for t in (means, scales, quats, opacities, colors,
                                                                          velocity)]
        ctx.camera_shapes = [None if t is None else (t.shape, t.dtype) for t in (intrinsics, camera_to_world, times,
                                                                                 distortion)]
        ctx.bank_shapes = [None if t is None else (t.shape, t.dtype) for t in (bank_mu, bank_rot, bank_alpha)]
        if depth is None:
            depth = image.new_zeros(0)
            ctx.mark_non_differentiable(depth)
        return image, alpha, depth

    @staticmethod
    def backward(ctx, d_image, d_alpha, d_depth):
        vspec = ctx.vspec
        B, H, W = vspec.n_views, vspec.height, vspec.width
        t = ctx.tensors
        if d_image is None:
            d_image = torch.zeros(B, 3, H, W, dtype=torch.float32, device=t["means"].device)
        d_image = d_image.to(torch.float32).contiguous()
        d_alpha = None if d_alpha is None else d_alpha.to(torch.float32).contiguous()
        d_depth = None if (d_depth is None or d_depth.numel() == 0) else d_depth.to(torch.float32).contiguous()
        need = ctx.needs_input_grad
        camera = bool(need[11] or need[12] or need[14])
        grads = backward_stages(ctx.sspec, vspec, ctx.cfg, ctx.near_plane, t, ctx.state, d_image, d_alpha, d_depth,
                                camera=camera)
        out = []
        for name, shp in zip(_PARAM_NAMES + _CAMERA_NAMES + _BANK_NAMES,
                             ctx.shapes + ctx.camera_shapes + ctx.bank_shapes):
            if shp is None or name not in grads:
                out.append(None)
            else:
                out.append(grads[name].reshape(shp[0]).to(shp[1]))
        ctx.state = None
        # sspec, vspec, cfg, near_plane, lens_models | 6 scene tensors | intrinsics, c2w, times, distortion
        # | bank_mu, bank_rot, bank_alpha, basis
        return (None, None, None, None, None, *out[:6], out[6], out[7], None, out[9], *out[10:13], None)


def _check_times_no_grad(times):
    if isinstance(times, torch.Tensor) and times.requires_grad:
        raise NotImplementedError(
            "the b200 renderer does not differentiate the per-view times; detach them (the reference's "
            "renderers take the time-offset means, not times)."
        )


def lens_tensors(lens_models, distortion, n_views: int, device):
    """(int32 [B] GSB_LENS_* codes, float32 [B,5] coefficients) on ``device``, or None when every
    view is pinhole.  ``lens_models`` holds names ("pinhole", "radial_tangential",
    "opencv_fisheye") or codes; ``distortion`` per-view coefficient lists (None: zeros)."""
    if lens_models is None:
        return None
    if torch.is_tensor(lens_models):
        codes = [int(c) for c in lens_models.reshape(-1).tolist()]
    else:
        for m in lens_models:
            if isinstance(m, str) and m not in _lib.LENS_CODES:
                raise ValueError(f"Unknown lens_model: {m}")  # projection.py:203-204
        codes = [_lib.LENS_CODES[m] if isinstance(m, str) else int(m) for m in lens_models]
    if len(codes) != n_views:
        raise ValueError(f"expected {n_views} lens models, got {len(codes)}")
    if any(c not in _lib.LENS_CODES.values() for c in codes):
        raise ValueError(f"unknown lens model code in {codes}")
    if all(c == _lib.LENS_PINHOLE for c in codes):
        return None
    nd = _lib.DISTORTION_FLOATS
    padded = torch.is_tensor(distortion) and distortion.ndim == 2 and distortion.shape[-1] == nd
    rows = [None] * n_views
    if distortion is not None:
        rows = list(distortion.unbind(0)) if torch.is_tensor(distortion) else list(distortion)
        if len(rows) != n_views:
            raise ValueError(f"expected {n_views} distortion rows, got {len(rows)}")
    names = {v: k for k, v in _lib.LENS_CODES.items()}
    out = []
    for code, row in zip(codes, rows):
        if row is None or code == _lib.LENS_PINHOLE:  # pinhole views ignore distortion
            out.append(torch.zeros(nd, dtype=torch.float32, device=device))
            continue
        # tensors keep their autograd graph: the coefficients can be learned through the render
        r = (row if torch.is_tensor(row) else torch.as_tensor(row)).to(device=device, dtype=torch.float32).reshape(-1)
        limit = nd if padded else _lib.LENS_COEFFS[names[code]]
        if r.numel() > limit:  # projection.py:38-50 (_distortion_tensor)
            raise ValueError(f"{names[code]} expects at most {limit} distortion coefficients, got {r.numel()}.")
        out.append(torch.nn.functional.pad(r, (0, nd - r.numel())))
    return (torch.tensor(codes, dtype=torch.int32, device=device).contiguous(), torch.stack(out).contiguous())


def render_scene(sspec: SceneSpec, vspec: ViewSpec, cfg: B200RendererConfig, near_plane: float, *, means, scales,
                 quats, opacities, colors, velocity, intrinsics, camera_to_world, times, lens=None, bank=None,
                 basis=None):
    """Autograd entry used by every public render function.  ``lens``: the pair lens_tensors()
    returns, or None for pinhole views only.  Intrinsics, camera_to_world and the distortion may
    require gradients (cameras learned through the render call).  ``bank``: (bank_mu, bank_rot,
    bank_alpha) with ``basis`` [B, M] when sspec.bank_basis > 0."""
    if not means.is_cuda:
        raise RuntimeError("the b200 renderer runs on CUDA devices only (got a tensor on %s)" % means.device)
    _check_times_no_grad(times)
    lens_models, distortion = lens if lens is not None else (None, None)
    bank_mu, bank_rot, bank_alpha = bank if bank is not None else (None, None, None)
    if sspec.bank_basis and (bank is None or basis is None):
        raise ValueError("a scene with a dynamic bank needs the bank tensors and the per-view basis")
    return _RenderFunction.apply(sspec, vspec, cfg, float(near_plane), lens_models, means, scales, quats, opacities,
                                 colors, velocity, intrinsics, camera_to_world, times, distortion, bank_mu, bank_rot,
                                 bank_alpha, basis)
