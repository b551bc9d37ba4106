"""Seeded synthetic workloads for the render + loss path.

Five scenes, each a set of raw Gaussian parameters, cameras, frame times and
uniform [0, 1] targets.  The reference measures on no dataset for this path,
so these generators are the whole workload.  All draws come from one CPU
``torch.Generator`` per scene (per clip for ``clips``), in a fixed order.

  static64   one 64x64 pinhole view (f=64, c=32, identity pose), G=4096,
             SH degree 0.
  dynamic128 16 frames at 128x128 (f=128, c=64) on an arc of radius 0.3
             about the origin, yaw 2 degrees per frame, G=32768 with
             velocities, t = k/15, SH degree 1.
  multiview384 8 views at 384x384 (f=384, c=192) evenly on a 30 degree arc
             of radius 4 looking at the origin, G=200000 around z=+4 with 5%
             anisotropic outliers, SH degree 3.
  large1080  32 views at 1920x1080 (f=1500, c=(960,540)) on a 4x8 grid of
             translations over [-0.5,0.5]^2, identity rotation, G=1000000,
             SH degree 3.
  clips256   64 clips x 8 frames at 256x256 (f=256, c=128), 65536 Gaussians
             per clip with velocities, t = k/7, identity rotation with
             N(0, 0.05^2) translations, SH degree 1, per-clip gradients.

``scale`` shrinks G (and ``image_scale`` the image) for test-sized variants;
the full-size workloads use scale = image_scale = 1.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class Workload:
    name: str
    means: torch.Tensor          # [S,G,3]
    log_scales: torch.Tensor     # [S,G,3]
    quats: torch.Tensor          # [S,G,4] raw (unnormalised)
    opacity_logits: torch.Tensor # [S,G,1]
    sh: torch.Tensor             # [S,G,(d+1)^2,3]
    velocity: torch.Tensor | None  # [S,G,3]
    fx: torch.Tensor             # [B]
    fy: torch.Tensor
    cx: torch.Tensor
    cy: torch.Tensor
    camera_to_world: torch.Tensor  # [B,4,4]
    times: torch.Tensor          # [B]
    views_per_set: int
    height: int
    width: int
    target: torch.Tensor         # [B,3,H,W]

    @property
    def n_views(self) -> int:
        return int(self.camera_to_world.shape[0])

    @property
    def n_gaussians(self) -> int:
        return int(self.means.shape[1])

    @property
    def n_sets(self) -> int:
        return int(self.means.shape[0])

    @property
    def sh_degree(self) -> int:
        return int(round(math.sqrt(self.sh.shape[-2]))) - 1

    def pixels(self) -> int:
        return self.n_views * self.height * self.width

    def views(self, start: int, stop: int) -> "Workload":
        """Views [start, stop) with the parameter sets they use (whole sets only
        when sets are per-clip)."""
        vps = self.views_per_set
        if vps >= self.n_views:
            sets = slice(0, self.n_sets)
        else:
            if start % vps or stop % vps:
                raise ValueError("per-set workloads split on set boundaries only")
            sets = slice(start // vps, stop // vps)
        return Workload(
            name=self.name,
            means=self.means[sets], log_scales=self.log_scales[sets], quats=self.quats[sets],
            opacity_logits=self.opacity_logits[sets], sh=self.sh[sets],
            velocity=None if self.velocity is None else self.velocity[sets],
            fx=self.fx[start:stop], fy=self.fy[start:stop], cx=self.cx[start:stop], cy=self.cy[start:stop],
            camera_to_world=self.camera_to_world[start:stop], times=self.times[start:stop],
            views_per_set=min(vps, stop - start), height=self.height, width=self.width,
            target=self.target[start:stop],
        )


def look_at_camera_to_world(position: torch.Tensor, target=None, up=None) -> torch.Tensor:
    """Camera-to-world [4,4] whose columns are (right, up, forward), +z forward.

    Same convention as the reference's build_look_at_camera_to_world
    (src/train/camera.py:105-120).
    """
    position = position.to(torch.float32)
    target = torch.zeros(3) if target is None else target
    up = torch.tensor([0.0, 1.0, 0.0]) if up is None else up

    def unit(v):
        return v / torch.linalg.norm(v).clamp_min(1e-6)

    forward = unit(target - position)
    right = unit(torch.cross(up, forward, dim=0))
    cam_up = unit(torch.cross(forward, right, dim=0))
    m = torch.eye(4)
    m[:3, :3] = torch.stack([right, cam_up, forward], dim=1)
    m[:3, 3] = position
    return m


def orbit_camera_to_world(radius: float, azimuth: float, elevation: float = 0.0) -> torch.Tensor:
    """Pose of the reference's make_orbit_camera (src/train/camera.py:123-150)."""
    r = torch.tensor(radius, dtype=torch.float32)
    az = torch.tensor(azimuth, dtype=torch.float32)
    el = torch.tensor(elevation, dtype=torch.float32)
    pos = torch.stack([r * torch.cos(el) * torch.sin(az), r * torch.sin(el), -r * torch.cos(el) * torch.cos(az)])
    return look_at_camera_to_world(pos)


def _uniform(g, shape, lo, hi):
    return torch.rand(shape, generator=g) * (hi - lo) + lo


def _normal(g, shape, mean, std):
    return torch.randn(shape, generator=g) * std + mean


def _sh(g, G, degree, dc_std, rest_std):
    k = (degree + 1) ** 2
    sh = torch.zeros(G, k, 3)
    sh[:, 0, :] = _normal(g, (G, 3), 0.0, dc_std)
    if k > 1:
        sh[:, 1:, :] = _normal(g, (G, k - 1, 3), 0.0, rest_std)
    return sh


def _intrinsics(B, f, cxy):
    return (torch.full((B,), float(f)), torch.full((B,), float(f)),
            torch.full((B,), float(cxy[0])), torch.full((B,), float(cxy[1])))


def static64(scale: float = 1.0, image_scale: float = 1.0, seed: int = 0) -> Workload:
    g = torch.Generator().manual_seed(seed)
    G = max(1, int(4096 * scale))
    S = max(8, int(round(64 * image_scale)))
    means = torch.stack([_uniform(g, (G,), -1, 1), _uniform(g, (G,), -1, 1), _uniform(g, (G,), 2, 4)], -1)
    log_scales = _normal(g, (G, 3), -3.0, 0.5)
    quats = torch.randn(G, 4, generator=g)
    logits = _normal(g, (G, 1), 0.0, 1.0)
    sh = _sh(g, G, 0, 0.3, 0.0)
    target = torch.rand(1, 3, S, S, generator=g)
    fx, fy, cx, cy = _intrinsics(1, 64 * S / 64, (32 * S / 64, 32 * S / 64))
    return Workload("static64", means[None], log_scales[None], quats[None], logits[None], sh[None], None,
                    fx, fy, cx, cy, torch.eye(4)[None], torch.zeros(1), 1, S, S, target)


def dynamic128(scale: float = 1.0, image_scale: float = 1.0, frames: int = 16, seed: int = 1,
               frame_offset: int = 0, total_frames: int | None = None) -> Workload:
    """16 frames by default; ``frame_offset``/``total_frames`` continue the same
    arc for weak-scaling runs (frame k of ``total_frames``: yaw 2k degrees,
    t = k/(total_frames-1))."""
    g = torch.Generator().manual_seed(seed)
    G = max(1, int(32768 * scale))
    S = max(8, int(round(128 * image_scale)))
    total = frames if total_frames is None else total_frames
    means = torch.stack([_uniform(g, (G,), -1.5, 1.5), _uniform(g, (G,), -1.5, 1.5), _uniform(g, (G,), 2, 5)], -1)
    velocity = _normal(g, (G, 3), 0.0, 0.05)
    log_scales = _normal(g, (G, 3), -3.5, 0.6)
    quats = torch.randn(G, 4, generator=g)
    logits = _normal(g, (G, 1), 0.0, 1.0)
    sh = _sh(g, G, 1, 0.3, 0.1)
    ks = list(range(frame_offset, frame_offset + frames))
    target = torch.stack([torch.rand(3, S, S, generator=torch.Generator().manual_seed(seed * 7919 + k)) for k in ks])
    c2w = torch.stack([orbit_camera_to_world(0.3, math.radians(2.0 * k)) for k in ks])
    times = torch.tensor([k / max(total - 1, 1) for k in ks], dtype=torch.float32)
    fx, fy, cx, cy = _intrinsics(frames, 128 * S / 128, (64 * S / 128, 64 * S / 128))
    return Workload("dynamic128", means[None], log_scales[None], quats[None], logits[None], sh[None],
                    velocity[None], fx, fy, cx, cy, c2w, times, frames, S, S, target)


def multiview384(scale: float = 1.0, image_scale: float = 1.0, views: int = 8, seed: int = 2) -> Workload:
    g = torch.Generator().manual_seed(seed)
    G = max(1, int(200_000 * scale))
    S = max(8, int(round(384 * image_scale)))
    means = torch.randn(G, 3, generator=g) * 0.8 + torch.tensor([0.0, 0.0, 4.0])
    log_scales = _normal(g, (G, 3), -4.0, 0.7)
    outlier = torch.rand(G, generator=g) < 0.05
    axis = torch.randint(0, 3, (G,), generator=g)
    bump = torch.zeros(G, 3)
    bump[torch.arange(G), axis] = 2.0
    log_scales = log_scales + bump * outlier[:, None].float()
    quats = torch.randn(G, 4, generator=g)
    logits = _normal(g, (G, 1), 0.0, 1.5)
    sh = _sh(g, G, 3, 0.3, 0.05)
    target = torch.rand(views, 3, S, S, generator=g)
    az = [(-15.0 + 30.0 * i / max(views - 1, 1)) for i in range(views)]
    c2w = torch.stack([orbit_camera_to_world(4.0, math.radians(a)) for a in az])
    fx, fy, cx, cy = _intrinsics(views, 384 * S / 384, (192 * S / 384, 192 * S / 384))
    return Workload("multiview384", means[None], log_scales[None], quats[None], logits[None], sh[None], None,
                    fx, fy, cx, cy, c2w, torch.zeros(views), views, S, S, target)


def large1080(scale: float = 1.0, image_scale: float = 1.0, views: int = 32, seed: int = 3) -> Workload:
    g = torch.Generator().manual_seed(seed)
    G = max(1, int(1_000_000 * scale))
    Wd = max(8, int(round(1920 * image_scale)))
    Ht = max(8, int(round(1080 * image_scale)))
    means = torch.stack([_uniform(g, (G,), -3, 3), _uniform(g, (G,), -3, 3), _uniform(g, (G,), 2, 10)], -1)
    log_scales = torch.clamp(_normal(g, (G, 3), -4.5, 0.8), max=-1.0)
    quats = torch.randn(G, 4, generator=g)
    logits = _normal(g, (G, 1), 0.0, 2.0)
    sh = _sh(g, G, 3, 0.3, 0.05)
    target = torch.rand(views, 3, Ht, Wd, generator=g)
    c2w = torch.eye(4).repeat(views, 1, 1)
    for i in range(views):
        gx, gy = i % 8, i // 8
        c2w[i, 0, 3] = -0.5 + gx / 7.0
        c2w[i, 1, 3] = -0.5 + gy / 3.0
    f = 1500 * image_scale
    fx, fy, cx, cy = _intrinsics(views, f, (960 * Wd / 1920, 540 * Ht / 1080))
    return Workload("large1080", means[None], log_scales[None], quats[None], logits[None], sh[None], None,
                    fx, fy, cx, cy, c2w, torch.zeros(views), views, Ht, Wd, target)


def clips256(scale: float = 1.0, image_scale: float = 1.0, clips: int = 64, frames: int = 8,
             seed: int = 4, clip_offset: int = 0) -> Workload:
    G = max(1, int(65536 * scale))
    S = max(8, int(round(256 * image_scale)))
    parts = []
    c2ws, targets = [], []
    for clip in range(clip_offset, clip_offset + clips):
        g = torch.Generator().manual_seed(seed + clip)
        means = torch.stack([_uniform(g, (G,), -1, 1), _uniform(g, (G,), -1, 1), _uniform(g, (G,), 2, 4)], -1)
        vel = _normal(g, (G, 3), 0.0, 0.03)
        log_scales = _normal(g, (G, 3), -3.2, 0.6)
        quats = torch.randn(G, 4, generator=g)
        logits = _normal(g, (G, 1), 0.0, 1.0)
        sh = _sh(g, G, 1, 0.3, 0.1)
        parts.append((means, log_scales, quats, logits, sh, vel))
        for _k in range(frames):
            m = torch.eye(4)
            m[:3, 3] = _normal(g, (3,), 0.0, 0.05)
            c2ws.append(m)
        targets.append(torch.rand(frames, 3, S, S, generator=g))
    stack = [torch.stack([p[i] for p in parts]) for i in range(6)]
    B = clips * frames
    times = torch.tensor([k / max(frames - 1, 1) for _ in range(clips) for k in range(frames)], dtype=torch.float32)
    fx, fy, cx, cy = _intrinsics(B, 256 * S / 256, (128 * S / 256, 128 * S / 256))
    return Workload("clips256", stack[0], stack[1], stack[2], stack[3], stack[4], stack[5],
                    fx, fy, cx, cy, torch.stack(c2ws), times, frames, S, S, torch.cat(targets))


WORKLOADS = {
    "static64": static64,
    "dynamic128": dynamic128,
    "multiview384": multiview384,
    "large1080": large1080,
    "clips256": clips256,
}
