"""recon_backward (one multi-view launch, one backward pass) against the reference trainer's
micro-batched loop (train_video_token_implicit_dynamic.py:887-925: render a chunk, loss, backward
with retain_graph, chunk after chunk) run with the same renderer."""
import math
from types import SimpleNamespace

import pytest
import torch

from conftest import grad_close
from dynaworld_b200 import synthetic as syn
from dynaworld_b200.losses import reconstruction_loss_per_image
from dynaworld_b200.rendering import render_gaussian_frames
from dynaworld_b200.training import recon_backward, resize_images, temporal_recon_chunk_size, viewport_cameras
from gpu_helpers import DEV

pytestmark = pytest.mark.gpu


class TinyDecoder(torch.nn.Module):
    """Shared parameters decoded into K frames (means move with time): a graph every chunk's
    backward walks again in the reference loop."""

    def __init__(self, wl):
        super().__init__()
        self.xyz = torch.nn.Parameter(wl.means[0].clone())
        self.vel = torch.nn.Parameter(wl.velocity[0].clone())
        self.log_scales = torch.nn.Parameter(wl.log_scales[0].clone())
        self.quats = torch.nn.Parameter(wl.quats[0].clone())
        self.logits = torch.nn.Parameter(wl.opacity_logits[0].clone())
        self.rgb = torch.nn.Parameter(wl.sh[0, :, 0].clone())

    def forward(self, times, cameras):
        K = times.shape[0]
        exp = lambda t: t[None].expand(K, *t.shape)  # noqa: E731
        return SimpleNamespace(
            xyz=self.xyz[None] + times[:, None, None] * self.vel[None],
            scales=exp(torch.exp(self.log_scales)), quats=exp(torch.nn.functional.normalize(self.quats, dim=-1)),
            opacities=exp(torch.sigmoid(self.logits)), rgbs=exp(torch.sigmoid(self.rgb)), cameras=cameras)


def setup(frames=6):
    wl = syn.dynamic128(scale=0.05, image_scale=0.5, frames=frames)
    cams = tuple(SimpleNamespace(fx=float(wl.fx[k]) * 2, fy=float(wl.fy[k]) * 2, cx=float(wl.cx[k]) * 2,
                                 cy=float(wl.cy[k]) * 2, camera_to_world=wl.camera_to_world[k].to(DEV),
                                 lens_model="pinhole", distortion=None) for k in range(frames))
    dec = TinyDecoder(wl).to(DEV)
    clip = wl.target[None].to(DEV)  # [1, K, 3, S, S] at the render size
    return wl, cams, dec, clip


def reference_loop(dec, times, cams, clip, render_size, chunk, reg):
    """The trainer's recon_backward structure with the b200 renderer in every chunk."""
    decoded = dec(times, cams)
    K = len(cams)
    target = resize_images(clip[0], render_size)
    total, preview = 0.0, None
    for s in range(0, K, chunk):
        e = min(s + chunk, K)
        seq = SimpleNamespace(xyz=decoded.xyz[s:e], scales=decoded.scales[s:e], quats=decoded.quats[s:e],
                              opacities=decoded.opacities[s:e], rgbs=decoded.rgbs[s:e])
        renders = render_gaussian_frames(seq, viewport_cameras(cams[s:e], 2 * render_size, render_size),
                                         render_size, render_size, "b200")
        if preview is None:
            preview = renders[0].detach()
        loss = reconstruction_loss_per_image(renders, target[s:e]).sum() / K
        total = total + loss.detach()
        (loss + (reg(dec) if e == K else 0.0)).backward(retain_graph=e != K)
    return total, preview


@pytest.mark.parametrize("chunk", [1, 4])
def test_one_launch_matches_the_chunked_loop(chunk):
    wl, cams, dec, clip = setup()
    S = wl.height
    times = wl.times.to(DEV)
    reg = lambda d: 1e-3 * d.vel.square().sum()  # noqa: E731
    ref_loss, ref_preview = reference_loop(dec, times, cams, clip, S, chunk, reg)
    ref_grads = {k: p.grad.clone() for k, p in dec.named_parameters()}
    dec.zero_grad(set_to_none=True)
    loss, preview = recon_backward(clip, dec(times, cams), reg(dec), True, render_size=S, input_size=2 * S)
    torch.testing.assert_close(loss, ref_loss, rtol=1e-5, atol=1e-7)
    assert torch.equal(preview, ref_preview)
    for k, p in dec.named_parameters():
        ok, e, s = grad_close(p.grad, ref_grads[k], 1e-4)
        assert ok, f"chunk={chunk} {k}: {e:.3e} vs {s:.3e}"


def test_chunk_sizes_and_errors():
    assert temporal_recon_chunk_size("batched", 8, 2) == 8
    assert temporal_recon_chunk_size("framewise", 8, 2) == 1
    assert temporal_recon_chunk_size("microbatch", 8, 3) == 3
    assert temporal_recon_chunk_size("microbatch", 2, 3) == 2
    wl, cams, dec, clip = setup(2)
    with pytest.raises(ValueError, match="cameras"):
        recon_backward(clip, SimpleNamespace(cameras=None), 0.0, False, render_size=wl.height)
    assert math.isfinite(float(recon_backward(clip, dec(wl.times.to(DEV), cams), 0.0, False,
                                              render_size=wl.height, input_size=2 * wl.height)[0]))
