"""ctypes binding of libgsb200.so (the C ABI of include/gsb200.h).

The library is the only compute path: if it cannot be loaded, every render or loss call raises
``RuntimeError``; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libgsb200.so"
_lib = None
_load_error: str | None = None

GSB_OK = 0
GSB_ERR_NONFINITE = 4
GSB_ERR_TIMEOUT = 5
STATUS_NAMES = {
    0: "GSB_OK", 1: "GSB_ERR_SHAPE", 2: "GSB_ERR_WORKSPACE", 3: "GSB_ERR_KEY_OVERFLOW",
    4: "GSB_ERR_NONFINITE", 5: "GSB_ERR_TIMEOUT", 6: "GSB_ERR_CUDA", 7: "GSB_ERR_ARG", 8: "GSB_ERR_CAPACITY",
}

SCENE_RAW = 0x1
SCENE_VELOCITY = 0x2
SCENE_SH_CLAMP = 0x4
SCENE_BANK = 0x8
SCENE_HEAD = 0x10
BANK_MAX_BASIS = 16
RENDER_TILED_COMPAT = 0x1
RENDER_DEPTH = 0x2
RENDER_NO_ELLIPSE = 0x4
RENDER_NO_CLAMP = 0x8
LENS_PINHOLE = 0
LENS_RADIAL_TANGENTIAL = 1
LENS_OPENCV_FISHEYE = 2
LENS_CODES = {"pinhole": LENS_PINHOLE, "radial_tangential": LENS_RADIAL_TANGENTIAL,
              "opencv_fisheye": LENS_OPENCV_FISHEYE}
LENS_COEFFS = {"pinhole": 0, "radial_tangential": 5, "opencv_fisheye": 4}
DISTORTION_FLOATS = 5
SPLATS2D_CONIC = 0
SPLATS2D_PACKED = 1
RECORD_FLOATS = 16
GRAD2D_FLOATS = 10

vp = C.c_void_p


class Scene(C.Structure):
    _fields_ = [
        ("n_sets", C.c_int32), ("n_gaussians", C.c_int32), ("sh_degree", C.c_int32), ("flags", C.c_uint32),
        ("means", vp), ("scales", vp), ("quats", vp), ("opacities", vp), ("colors", vp), ("velocity", vp),
        ("bank_mu", vp), ("bank_rot", vp), ("bank_alpha", vp), ("bank_first", C.c_int32), ("bank_basis", C.c_int32),
        ("head_xy_extent", C.c_float), ("head_z_min", C.c_float), ("head_z_extent", C.c_float),
        ("head_scale_init", C.c_float),
    ]


class Views(C.Structure):
    _fields_ = [
        ("n_views", C.c_int32), ("views_per_set", C.c_int32), ("height", C.c_int32), ("width", C.c_int32),
        ("intrinsics", vp), ("camera_to_world", vp), ("times", vp), ("lens_models", vp), ("distortion", vp),
        ("basis", vp),
    ]


class Options(C.Structure):
    _fields_ = [
        ("tile_size", C.c_int32), ("flags", C.c_uint32), ("near_plane", C.c_float), ("alpha_clamp", C.c_float),
        ("alpha_cutoff", C.c_float), ("transmittance_threshold", C.c_float), ("eps", C.c_float),
        ("pixel_center", C.c_float), ("background", C.c_float * 3), ("bound_scale", C.c_float),
        ("tiled_alpha_threshold", C.c_float), ("backward_segments", C.c_int32),
    ]


class SceneGrads(C.Structure):
    _fields_ = [("means", vp), ("scales", vp), ("quats", vp), ("opacities", vp), ("colors", vp), ("velocity", vp),
                ("bank_mu", vp), ("bank_rot", vp), ("bank_alpha", vp)]


class CameraGrads(C.Structure):
    _fields_ = [("intrinsics", vp), ("camera_to_world", vp), ("distortion", vp)]


class LossOptions(C.Structure):
    _fields_ = [
        ("type", C.c_int32), ("window_size", C.c_int32), ("window", C.c_int32), ("dssim_half", C.c_int32),
        ("l1_weight", C.c_float), ("dssim_weight", C.c_float), ("mse_weight", C.c_float),
        ("c1", C.c_float), ("c2", C.c_float), ("sigma", C.c_float),
    ]


class Splats2D(C.Structure):
    _fields_ = [
        ("n_views", C.c_int32), ("n_gaussians", C.c_int32), ("format", C.c_int32), ("reserved", C.c_int32),
        ("means", vp), ("conics", vp), ("opacities", vp), ("packed", vp), ("colors", vp), ("depths", vp),
    ]


class Splats2DGrads(C.Structure):
    _fields_ = [("means", vp), ("conics", vp), ("opacities", vp), ("packed", vp), ("colors", vp)]


P = C.POINTER
# name -> (restype, argtypes)
SIGNATURES = {
    "gsb_version": (C.c_char_p, []),
    "gsb_kernel_launches": (C.c_uint64, []),
    "gsb_status_string": (C.c_char_p, [C.c_int]),
    "gsb_read_status": (C.c_int, [vp, P(C.c_int), vp]),
    "gsb_depth_order_workspace": (C.c_size_t, [P(Scene), P(Views)]),
    "gsb_depth_order": (C.c_int, [P(Scene), P(Views), vp, vp, vp, C.c_size_t, vp]),
    "gsb_preprocess_workspace": (C.c_size_t, [P(Views), C.c_int32]),
    "gsb_preprocess_fwd": (C.c_int, [P(Scene), P(Views), P(Options), vp, vp, vp, vp, vp, vp, C.c_size_t, vp]),
    "gsb_bin_workspace": (C.c_size_t, [P(Views), P(Options), C.c_int32, C.c_uint32]),
    "gsb_bin": (C.c_int, [P(Views), P(Options), C.c_int32, vp, vp, vp, C.c_uint32, vp, vp, vp, vp, C.c_size_t,
                          vp]),
    "gsb_raster_checkpoint_floats": (C.c_size_t, [P(Views), P(Options)]),
    "gsb_raster_fwd": (C.c_int, [P(Views), P(Options), C.c_int32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "gsb_loss_workspace": (C.c_size_t, [C.c_int32]),
    "gsb_loss_fwd_bwd": (C.c_int, [P(LossOptions), C.c_int32, C.c_int32, C.c_int32, C.c_int32, vp, vp, vp, vp, vp,
                                   C.c_size_t, vp]),
    "gsb_loss_fwd_bwd_noalloc": (C.c_int, [P(LossOptions), C.c_int32, C.c_int32, C.c_int32, C.c_int32, vp, vp, vp,
                                           vp, vp]),
    "gsb_scale_planes": (C.c_int, [vp, vp, vp, C.c_int32, C.c_int64, vp]),
    "gsb_raster_bwd": (C.c_int, [P(Views), P(Options), C.c_int32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                 vp]),
    "gsb_preprocess_bwd": (C.c_int, [P(Scene), P(Views), P(Options), vp, vp, P(SceneGrads), vp]),
    "gsb_preprocess_bwd_range": (C.c_int, [P(Scene), P(Views), P(Options), vp, vp, P(SceneGrads), C.c_int64,
                                           C.c_int64, vp]),
    "gsb_camera_bwd": (C.c_int, [P(Scene), P(Views), P(Options), vp, vp, P(CameraGrads), vp]),
    "gsb_splats2d_order_workspace": (C.c_size_t, [P(Splats2D)]),
    "gsb_splats2d_order": (C.c_int, [P(Splats2D), vp, vp, vp, C.c_size_t, vp]),
    "gsb_splats2d_preprocess_workspace": (C.c_size_t, [P(Splats2D)]),
    "gsb_splats2d_preprocess": (C.c_int, [P(Splats2D), C.c_int32, C.c_int32, P(Options), vp, vp, vp, vp, vp,
                                          C.c_size_t, vp]),
    "gsb_splats2d_preprocess_bwd": (C.c_int, [P(Splats2D), vp, vp, P(Splats2DGrads), vp]),
    "gsb_radix_sort_workspace": (C.c_size_t, [C.c_uint32, C.c_int, C.c_int]),
    "gsb_radix_sort": (C.c_int, [vp, vp, vp, vp, C.c_uint32, C.c_int, C.c_int, C.c_int, vp, C.c_size_t, vp]),
    "gsb_debug_sort_lookback_timeout": (C.c_int, [vp, vp, C.c_uint32, C.c_uint32, vp, C.c_size_t, vp]),
}


def library_path() -> Path:
    return Path(os.environ.get("GSB200_LIB", str(_LIB_PATH)))


def load(path: str | Path | None = None):
    """Loads the shared library (once) and declares every entry point's signature."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    p = Path(path) if path else library_path()
    if not p.exists():
        _load_error = f"{p} not found: build it with `python -m dynaworld_b200.build`"
        raise RuntimeError(f"libgsb200 is not built: {_load_error}")
    try:
        lib = C.CDLL(str(p))
    except OSError as exc:  # pragma: no cover - depends on the box
        _load_error = str(exc)
        raise RuntimeError(f"libgsb200 failed to load: {exc}") from exc
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def lib():
    return _lib if _lib is not None else load()


class GsbError(RuntimeError):
    def __init__(self, fn: str, status: int):
        self.status = status
        name = STATUS_NAMES.get(status, str(status))
        detail = lib().gsb_status_string(status).decode()
        super().__init__(f"{fn} failed: {name} ({detail})")


def check(fn: str, status: int) -> None:
    if status != GSB_OK:
        raise GsbError(fn, status)


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    if t is None:
        return None
    return t.data_ptr()
