"""libgsb200.so loads and exports every entry point include/gsb200.h declares (no GPU needed)."""
import ctypes
import re

import pytest

from conftest import ROOT
from dynaworld_b200 import _lib, build

HEADER = ROOT / "include" / "gsb200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"GSB_API\s+[\w\s\*]+?\b(gsb_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "gsb_raster_fwd" in names and "gsb_preprocess_bwd" in names and len(names) >= 15


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_the_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_version_and_status_strings(lib):
    assert b"sm_100a" in lib.gsb_version()
    for code in range(9):
        assert lib.gsb_status_string(code) != b"unknown status"
    assert lib.gsb_status_string(99) == b"unknown status"


def test_struct_sizes_match_header():
    # 4 ints + 9 pointers + 2 ints; 4 ints + 6 pointers; 2 ints + 11 floats (incl. background[3])
    # + 1 int; 9 pointers
    assert ctypes.sizeof(_lib.Scene) == 16 + 9 * 8 + 8 + 4 * 4
    assert ctypes.sizeof(_lib.Views) == 16 + 6 * 8
    assert ctypes.sizeof(_lib.SceneGrads) == 9 * 8
    assert ctypes.sizeof(_lib.Options) == 8 + 11 * 4 + 4
    assert ctypes.sizeof(_lib.LossOptions) == 16 + 6 * 4


def test_argument_errors_return_codes_without_touching_a_gpu(lib):
    """Invalid arguments are rejected on the host with a status, before any CUDA call."""
    v = _lib.Views()
    assert lib.gsb_depth_order(None, None, None, None, None, 0, None) == 7  # GSB_ERR_ARG
    # the raster stages need no cameras: an empty frame is a shape error, a missing option block an
    # argument error
    assert lib.gsb_raster_fwd(ctypes.byref(v), None, 1, None, None, None, None, None, None, None, None, None,
                              None, None) == 1
    v.n_views = v.height = v.width = 1
    assert lib.gsb_raster_fwd(ctypes.byref(v), None, 1, None, None, None, None, None, None, None, None, None,
                              None, None) == 7
    o = _lib.Options()
    o.tile_size = 12
    v.intrinsics = v.camera_to_world = 16
    v.n_views = v.height = v.width = v.views_per_set = 1
    assert lib.gsb_raster_fwd(ctypes.byref(v), ctypes.byref(o), 1, 16, 16, 16, None, 16, 16, 16, 16, 16,
                              None, None) == 7
    # backward segments: 3 is not a valid count; 2 segments need the checkpoint buffer
    o.tile_size, o.near_plane, o.backward_segments = 16, 1e-4, 3
    assert lib.gsb_raster_checkpoint_floats(ctypes.byref(v), ctypes.byref(o)) == 0
    assert lib.gsb_raster_fwd(ctypes.byref(v), ctypes.byref(o), 1, 16, 16, 16, None, 16, 16, 16, 16, 16,
                              None, None) == 7
    o.backward_segments = 2
    assert lib.gsb_raster_checkpoint_floats(ctypes.byref(v), ctypes.byref(o)) == 6
    assert lib.gsb_raster_fwd(ctypes.byref(v), ctypes.byref(o), 1, 16, 16, 16, None, 16, 16, 16, 16, 16,
                              None, None) == 7
    o.backward_segments = 1
    assert lib.gsb_raster_checkpoint_floats(ctypes.byref(v), ctypes.byref(o)) == 0
    # the backward adds to grad2d in pairs of floats: a buffer off an 8-byte boundary is refused
    assert lib.gsb_raster_bwd(ctypes.byref(v), ctypes.byref(o), 1, 16, 16, 16, None, 16, 16, None, 16, None, None,
                              None, 20, None) == 7
    lo = _lib.LossOptions()
    lo.type = 0
    lo.window_size = 4  # even window
    assert lib.gsb_loss_fwd_bwd(ctypes.byref(lo), 1, 3, 16, 16, 16, 16, 16, None, 16, 4096, None) == 7


def test_bank_scene_checks_are_host_only(lib):
    """A dynamic bank needs the activated scene without velocity, its three coefficient arrays, a
    per-view basis, 1..16 basis functions and 0 <= bank_first <= G; anything else is rejected
    before a kernel runs."""
    s, v = _lib.Scene(), _lib.Views()
    s.n_sets, s.n_gaussians = 1, 10
    s.means = s.scales = s.quats = s.opacities = s.colors = 16
    v.n_views = v.views_per_set = v.height = v.width = 1
    v.intrinsics = v.camera_to_world = 16

    def depth_order():
        return lib.gsb_depth_order(ctypes.byref(s), ctypes.byref(v), 16, 16, 16, 1 << 30, None)

    s.flags = _lib.SCENE_BANK
    assert depth_order() == 7  # no coefficient arrays
    s.bank_mu = s.bank_rot = s.bank_alpha = 16
    s.bank_basis = 8
    assert depth_order() == 7  # no basis
    v.basis = 16
    s.flags = _lib.SCENE_BANK | _lib.SCENE_RAW
    assert depth_order() == 7
    s.flags = _lib.SCENE_BANK | _lib.SCENE_VELOCITY
    s.velocity = 16
    assert depth_order() == 7
    s.flags = _lib.SCENE_BANK
    for m in (0, 17):
        s.bank_basis = m
        assert depth_order() == 7
    s.bank_basis, s.bank_first = 8, 11
    assert depth_order() == 1  # GSB_ERR_SHAPE


def test_workspace_queries_are_host_only(lib):
    s, v = _lib.Scene(), _lib.Views()
    s.n_gaussians = 1000
    v.n_views = 4
    assert lib.gsb_depth_order_workspace(ctypes.byref(s), ctypes.byref(v)) > 4 * 1000 * 16
    assert lib.gsb_preprocess_workspace(ctypes.byref(v), 1000) >= 4 * 1000 * 4
    assert lib.gsb_bin_workspace(ctypes.byref(v), None, 1000, 5000) >= 5000 * 16
    assert lib.gsb_radix_sort_workspace(10000, 8, 1) > 10000 * 12
    assert lib.gsb_loss_workspace(8) >= 256 + 8 * 24
