"""Host-side logic: configs, dispatch, argument checks, synthetic workloads (CPU only)."""
import pytest
import torch

from dynaworld_b200 import rendering, synthetic
from dynaworld_b200.config import EXACT_ALPHA_CUTOFF, B200RendererConfig, LossConfig
from dynaworld_b200.losses import reconstruction_loss_per_image
from dynaworld_b200.renderer import render_b200, render_b200_3dgs_batch


def test_from_mapping_contract():
    cfg = B200RendererConfig.from_mapping(None, fallback_tile_size=8, fallback_alpha_threshold=1 / 255)
    assert cfg.tile_size == 16 and cfg.mode == "exact" and cfg.alpha_cutoff == EXACT_ALPHA_CUTOFF
    assert cfg.tiled_alpha_threshold == pytest.approx(1 / 255)
    compat = B200RendererConfig.from_mapping({"mode": "tiled_compat"}, fallback_tile_size=8,
                                             fallback_alpha_threshold=0.01)
    assert compat.tile_size == 8 and compat.tiled_alpha_threshold == 0.01
    with pytest.raises(ValueError):
        B200RendererConfig.from_mapping({"background": [1, 1]}, fallback_tile_size=8, fallback_alpha_threshold=0.1)
    with pytest.raises(ValueError):
        B200RendererConfig(mode="fast")
    with pytest.raises(ValueError):
        B200RendererConfig(tile_size=32)


def test_exact_cutoff_is_the_float32_identity_boundary():
    a = torch.tensor([EXACT_ALPHA_CUTOFF], dtype=torch.float32)
    assert (1.0 - a).item() == 1.0
    b = torch.tensor([EXACT_ALPHA_CUTOFF], dtype=torch.float32).nextafter(torch.tensor(1.0))
    assert (1.0 - b).item() < 1.0


def test_options_struct():
    o = B200RendererConfig(mode="tiled_compat", depth=True).options(0.05)
    assert o.flags & 1 and o.flags & 2 and o.near_plane == pytest.approx(0.05)


def test_loss_config():
    c = LossConfig.from_mapping({"type": "L1"})
    assert c.type == "l1" and c.options().type == 1
    with pytest.raises(ValueError):
        LossConfig.from_mapping({"type": "huber"})
    with pytest.raises(ValueError):
        LossConfig.from_mapping({"ssim_window": "tri"})


def test_pick_renderer_mode():
    assert rendering.pick_renderer_mode("b200", 1, 1, 1, 0) == "b200"
    assert rendering.pick_renderer_mode("auto", 1, 1, 1, 0) == "b200"
    with pytest.raises(ValueError):
        rendering.pick_renderer_mode("dense", 1, 1, 1, 0)
    with pytest.raises(ValueError):
        rendering.pick_renderer_mode("nope", 1, 1, 1, 0)


class _Cam:
    def __init__(self, lens="pinhole"):
        self.fx, self.fy, self.cx, self.cy = 10.0, 10.0, 4.0, 4.0
        self.camera_to_world = torch.eye(4)
        self.lens_model = lens


def test_projection_mode_resolution():
    assert rendering.resolve_camera_projection_mode([_Cam()], "auto") == "legacy_pinhole"
    assert rendering.resolve_camera_projection_mode([_Cam("opencv_fisheye")], "auto") == "camera_model"
    with pytest.raises(ValueError):
        rendering.resolve_camera_projection_mode([_Cam("opencv_fisheye")], "legacy_pinhole")
    with pytest.raises(ValueError):
        rendering.resolve_camera_projection_mode([_Cam()], "orthographic")


def test_camera_for_viewport():
    c = rendering.camera_for_viewport(_Cam(), 8, 8, 16, 32)
    assert (c.fx, c.fy, c.cx, c.cy) == (40.0, 20.0, 16.0, 8.0)
    with pytest.raises(ValueError):
        rendering.camera_for_viewport(_Cam(), 0, 8, 16, 16)


def test_cpu_tensors_fail_loudly():
    """No CPU fallback: the product path refuses CPU tensors."""
    wl = synthetic.static64(scale=0.01)
    K, G = 1, wl.n_gaussians
    with pytest.raises(RuntimeError, match="CUDA"):
        render_b200_3dgs_batch(torch.zeros(K, G, 3), torch.ones(K, G, 3), torch.ones(K, G, 4), torch.ones(K, G, 1),
                               torch.ones(K, G, 3), 8, 8, 8.0, 8.0, 4.0, 4.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        render_b200(wl.means, wl.log_scales, wl.quats, wl.opacity_logits, wl.sh,
                    intrinsics=torch.tensor([[64.0, 64, 32, 32]]), camera_to_world=torch.eye(4)[None],
                    height=64, width=64)
    with pytest.raises(RuntimeError, match="CUDA"):
        reconstruction_loss_per_image(torch.zeros(1, 3, 16, 16), torch.zeros(1, 3, 16, 16))


def test_lens_tables_and_their_argument_errors():
    """Lens models become per-view codes and zero-padded coefficient rows; the reference's
    argument errors (projection.py:38-50, :287-288) are raised on the host."""
    from dynaworld_b200 import _lib
    from dynaworld_b200.render import lens_tensors

    assert lens_tensors(["pinhole", "pinhole"], None, 2, "cpu") is None
    codes, coeffs = lens_tensors(["radial_tangential", "pinhole", "opencv_fisheye"],
                                 [[0.1, -0.02], [9.0, 9.0, 9.0, 9.0, 9.0, 9.0], (0.01, 0.0, 0.002, -0.001)], 3, "cpu")
    assert codes.tolist() == [_lib.LENS_RADIAL_TANGENTIAL, _lib.LENS_PINHOLE, _lib.LENS_OPENCV_FISHEYE]
    assert coeffs.shape == (3, 5)
    assert coeffs[0].tolist() == pytest.approx([0.1, -0.02, 0, 0, 0])
    assert coeffs[1].tolist() == [0, 0, 0, 0, 0]  # pinhole views ignore distortion
    assert coeffs[2].tolist() == pytest.approx([0.01, 0.0, 0.002, -0.001, 0])
    with pytest.raises(ValueError, match="at most 4"):
        lens_tensors(["opencv_fisheye"], [[0.1] * 5], 1, "cpu")
    with pytest.raises(ValueError, match="at most 5"):
        lens_tensors(["radial_tangential"], [[0.1] * 6], 1, "cpu")
    with pytest.raises(ValueError, match="Unknown lens_model"):
        lens_tensors(["orthographic"], None, 1, "cpu")
    args = (torch.zeros(2, 2, 3), torch.ones(2, 2, 3), torch.ones(2, 2, 4), torch.ones(2, 2, 1), torch.ones(2, 2, 3),
            8, 8, 8.0, 8.0, 4.0, 4.0)
    with pytest.raises(ValueError, match="Expected 2 cameras, got 1"):
        render_b200_3dgs_batch(*args, cameras=[_Cam("radial_tangential")], projection_mode="camera_model")
    with pytest.raises(ValueError, match="requires CameraSpec"):
        render_b200_3dgs_batch(*args, cameras=None, projection_mode="camera_model")
    with pytest.raises(RuntimeError, match="CUDA"):  # lens views run on the GPU kernels only
        render_b200_3dgs_batch(*args, cameras=[_Cam("radial_tangential"), _Cam("opencv_fisheye")],
                               projection_mode="camera_model")


@pytest.mark.parametrize("name", sorted(synthetic.WORKLOADS))
def test_synthetic_workloads_small(name):
    wl = synthetic.WORKLOADS[name](scale=0.002, image_scale=0.05)
    assert wl.means.shape[-1] == 3 and wl.target.shape[0] == wl.n_views
    assert wl.camera_to_world.shape == (wl.n_views, 4, 4)
    assert (wl.n_views - 1) // wl.views_per_set < wl.n_sets
    assert torch.isfinite(wl.means).all()


def test_synthetic_shapes_full_size_metadata():
    wl = synthetic.dynamic128()
    assert wl.n_views == 16 and wl.n_gaussians == 32768 and wl.height == 128 and wl.sh_degree == 1
    assert wl.times[-1].item() == pytest.approx(1.0)
    cont = synthetic.dynamic128(frames=2, frame_offset=14, total_frames=16)
    torch.testing.assert_close(cont.camera_to_world, wl.camera_to_world[14:16])
    torch.testing.assert_close(cont.target, wl.target[14:16])
    torch.testing.assert_close(cont.times, wl.times[14:16])


def test_pair_capacity_guess():
    """The binning capacity guessed from earlier frames: 1.25x the count plus slack, in 64 Ki steps,
    kept while the count stays between half the capacity and the capacity."""
    from dynaworld_b200.render import _next_capacity

    first = _next_capacity(1_000_000, None)
    assert first % 65536 == 0 and first >= 1_250_000
    assert _next_capacity(1_100_000, first) == first          # still fits: keep
    assert _next_capacity(first + 1, first) > first + 1        # overflow: grow past the count
    assert _next_capacity(first // 3, first) < first           # far below: shrink
    assert _next_capacity(0, None) == 65536


def test_training_host_helpers():
    from types import SimpleNamespace

    from dynaworld_b200.training import resize_images, temporal_recon_chunk_size, viewport_cameras

    assert [temporal_recon_chunk_size(s, 8, 3) for s in ("batched", "framewise", "microbatch")] == [8, 1, 3]
    x = torch.rand(2, 4, 3, 16, 16)
    assert resize_images(x, 16) is x
    y = resize_images(x, 8)
    assert y.shape == (2, 4, 3, 8, 8)
    torch.testing.assert_close(y[0, 0], torch.nn.functional.interpolate(x[0, :1], size=(8, 8), mode="bilinear",
                                                                        align_corners=False)[0])
    cam = SimpleNamespace(fx=100.0, fy=80.0, cx=32.0, cy=30.0, camera_to_world=torch.eye(4))
    (c,) = viewport_cameras((cam,), 64, 32)
    assert (c.fx, c.fy, c.cx, c.cy) == (50.0, 40.0, 16.0, 15.0) and c.camera_to_world is cam.camera_to_world


def test_bank_basis_and_argument_checks_on_cpu():
    from dynaworld_b200.bank import DynamicGaussianBank, render_dynamic_bank, temporal_basis

    phi = temporal_basis(torch.tensor([0.0, 0.25]), 5, 8.0)
    assert phi.shape == (2, 5)
    torch.testing.assert_close(phi[:, 4], torch.tensor([-1.0, -0.5]))  # odd count: 2t - 1
    bank = DynamicGaussianBank(*(torch.zeros(3, c) for c in (3, 3, 4, 1, 3)), torch.zeros(3, 2, 3),
                               torch.zeros(3, 2, 3), torch.zeros(3, 2, 1))
    with pytest.raises(RuntimeError, match="CUDA"):
        render_dynamic_bank(bank, torch.zeros(2), 8, 8, 10.0, 10.0, 4.0, 4.0)
