"""Benchmark of the fused render + L1/SSIM loss step (forward and backward) on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

One step = depth order -> projection/binning -> blend -> fused L1+SSIM loss and gradient ->
reverse blend -> chain rule to the Gaussian parameters (+ one NCCL all-reduce of the gradients
when N > 1).  Default workload: "large1080" (32 views of 1920x1080, 1,000,000 Gaussians, SH degree
3, cameras on a 4x8 grid of translations, gradients summed over views), the largest of the five
seeded workloads that fits one GPU.  With N GPUs the views are sharded over the ranks (4 per GPU at
8) against one replicated Gaussian set: the total work is fixed (strong scaling).  Per-clip
workloads (clips256) shard whole clips and need no all-reduce.

Prints one JSON line (rank 0).  Metric: Mpix/s (rendered pixels per second, all ranks).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "Mpix/s fwd+bwd render+SSIM at 1/2/4/8 B200; % HBM roofline; vs ref CPU"
UNIT = "Mpix/s"
PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024

# Algorithmic bytes of one raster launch:
#   backward: per (tile, Gaussian) pair an 8 B key + a 48 B projected record read and a 40 B
#   gradient record read-modify-written (80 B); per pixel 4 B transmittance + 4 B state + 12 B
#   image gradient read.   forward: per pair key + record (56 B); per pixel 24 B written.
BWD_BYTES_PER_PAIR, BWD_BYTES_PER_PIXEL = 136, 20
FWD_BYTES_PER_PAIR, FWD_BYTES_PER_PIXEL = 56, 24


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="large1080")
    ap.add_argument("--scale", type=float, default=1.0, help="Gaussian-count scale (1 = full workload)")
    ap.add_argument("--image-scale", type=float, default=1.0)
    ap.add_argument("--views", type=int, default=0,
                    help="render only the first N views of the workload (a slice for profiling; 0 = all)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--stages", action="store_true", help="print per-stage times to stderr")
    ap.add_argument("--tile", type=int, default=None, help="tile size (8 or 16; default: the renderer's)")
    ap.add_argument("--segments", type=int, default=0, help="backward list segments (1, 2, 4; default: automatic)")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------
# workloads


def make_workload(name: str, rank: int, world: int, scale: float, image_scale: float, views: int = 0):
    """(the whole workload, this rank's shard of its views).  Views are sharded over the ranks;
    per-clip Gaussian sets keep a clip's frames on one rank."""
    from dynaworld_b200 import synthetic as syn
    from dynaworld_b200.distributed import shard_views

    full = syn.WORKLOADS[name](scale=scale, image_scale=image_scale)
    if views:
        full = full.views(0, min(views, full.n_views))
    shared = full.views_per_set >= full.n_views
    sh = shard_views(full.n_views, world, rank, full.views_per_set, shared_set=shared)
    return full, full.views(sh.start, sh.stop)


def workload_config(name, full, shard, world):
    return {
        "workload": f"{name}: {full.n_views} views/frames at {full.height}x{full.width}, {full.n_gaussians} "
                    f"Gaussians per set ({full.n_sets} set{'s' if full.n_sets > 1 else ''}), SH degree {full.sh_degree}"
                    + (", velocities" if full.velocity is not None else ""),
        "views": full.n_views,
        "views_per_gpu": shard.n_views,
        "gaussians": full.n_gaussians,
        "height": full.height,
        "width": full.width,
        "sh_degree": full.sh_degree,
        "loss": "standard_gs: 0.8*L1 + 0.2*(1-SSIM)/2, 11x11 box window (reference losses.py)",
        "renderer": "exact (dense.py semantics), tile 16, alpha cutoff 2^-25",
        "parallelism": (f"dp{world} over views, Gaussians replicated, NCCL all-reduce of the Gaussian gradients"
                        if full.views_per_set >= full.n_views else f"dp{world} over clips, per-clip gradients")
        if world > 1 else "single GPU",
        "l2": "flushed between timed steps (256 MiB write outside the timed events); inputs larger than L2",
    }


# ---------------------------------------------------------------------------------------------
# the step


class Step:
    """One render + loss forward/backward of a workload resident on the device."""

    def __init__(self, wl, device, world, tile=None, segments=0, shared_set=True):
        from dynaworld_b200.config import B200RendererConfig
        from dynaworld_b200.distributed import GradientAllReduce
        from dynaworld_b200.render import set_gradient_reducer

        self.wl = wl
        self.dev = device
        self.world = world
        # one Gaussian set shared by every rank: the backward sums its gradients over the ranks
        # (bucketed NCCL all-reduce overlapped with the chain rule); per-clip sets need no exchange
        set_gradient_reducer(GradientAllReduce() if (world > 1 and shared_set) else None)
        self.cfg = B200RendererConfig(tile_size=tile or 16, backward_segments=segments)
        self.params = {k: getattr(wl, k).to(device).contiguous().requires_grad_(True)
                       for k in ("means", "log_scales", "quats", "opacity_logits", "sh")}
        if wl.velocity is not None:
            self.params["velocity"] = wl.velocity.to(device).contiguous().requires_grad_(True)
        self.intr = torch.stack([wl.fx, wl.fy, wl.cx, wl.cy], -1).to(device).contiguous()
        self.c2w = wl.camera_to_world.to(device).contiguous()
        self.times = wl.times.to(device).contiguous()
        self.target = wl.target.to(device).contiguous()

    def run(self, params=None, intr=None, c2w=None, times=None, target=None):
        from dynaworld_b200.losses import reconstruction_loss_per_image
        from dynaworld_b200.renderer import render_b200

        p = params or self.params
        for v in p.values():
            v.grad = None
        image, _alpha, _ = render_b200(
            p["means"], p["log_scales"], p["quats"], p["opacity_logits"], p["sh"],
            intrinsics=self.intr if intr is None else intr, camera_to_world=self.c2w if c2w is None else c2w,
            height=self.wl.height, width=self.wl.width, velocity=p.get("velocity"),
            times=self.times if times is None else times, views_per_set=self.wl.views_per_set, config=self.cfg,
        )
        loss = reconstruction_loss_per_image(image, self.target if target is None else target)
        loss.sum().backward()
        return loss


# ---------------------------------------------------------------------------------------------
# clocks


class ClockSampler:
    """nvidia-smi samples of the local GPU while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
# CPU ports of the reference's renderers (the oracle's restatements of dense.py + losses.py and of
# tiled.py), timed on this host's cores on bounded samples of the workload


# Window side of the dense samples: pixels x Gaussians of about 30-70 M pair evaluations, so one
# fwd+bwd sample takes seconds.  The dense renderer blends every Gaussian at every pixel, so its
# cost is the same at every pixel and Mpix/s on a window is Mpix/s on the frame.
CPU_WINDOW = {"static64": 64, "dynamic128": 32, "multiview384": 16, "large1080": 8, "clips256": 32}
TILED_SAMPLE_TILES = 32
TILED_TILE = 8  # tiled.py's default tile size


def _view_leaves(wl, frame):
    s = 0 if wl.views_per_set >= wl.n_views else frame // wl.views_per_set
    leaves = {k: getattr(wl, k)[s][None].clone().requires_grad_(True)
              for k in ("means", "log_scales", "quats", "opacity_logits", "sh")}
    vel = wl.velocity[s][None].clone().requires_grad_(True) if wl.velocity is not None else None
    return leaves, vel


def cpu_sample_time(wl, window: int, frame: int = 0):
    """Seconds for one fwd+bwd of the reference algorithm (dense render of every Gaussian at every
    pixel + standard_gs loss) on the centre window x window of one frame, on this host's cores."""
    from oracle import splat_oracle as so

    x0 = (wl.width - window) // 2
    y0 = (wl.height - window) // 2
    sl = slice(frame, frame + 1)
    leaves, vel = _view_leaves(wl, frame)
    t0 = time.perf_counter()
    raw = so.RawGaussians(leaves["means"], leaves["log_scales"], leaves["quats"], leaves["opacity_logits"],
                          leaves["sh"], vel)
    m, s, q, o, rgb = so.activate(raw, wl.times[sl], wl.camera_to_world[sl], 1)
    key = so.camera_depth_fp32(m.detach(), wl.camera_to_world[sl])
    img, _, _ = so.render_dense(m, s, q, o, rgb, window, window, wl.fx[sl], wl.fy[sl], wl.cx[sl], wl.cy[sl],
                                wl.camera_to_world[sl], sort_key=key, x0=x0, y0=y0)
    tgt = wl.target[sl][:, :, y0:y0 + window, x0:x0 + window]
    so.reconstruction_loss_per_image(img, tgt).sum().backward()
    return time.perf_counter() - t0


def cpu_window(name: str, wl) -> int:
    return min(CPU_WINDOW.get(name, 16), wl.height, wl.width)


def cpu_baseline(name, wl, reps: int = 2):
    """Dense line: the centre window of frame 0, one warm-up on an 8x8 window (the SSIM window's
    reflect padding needs at least 6 pixels a side), median of ``reps``."""
    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    window = cpu_window(name, wl)
    cpu_sample_time(wl, min(8, window))
    t = statistics.median(cpu_sample_time(wl, window) for _ in range(reps))
    return {
        "value": (window * window) / t / 1e6,
        "unit": UNIT,
        "cores": cores,
        "kind": "port",
        "sample": f"dense.py + losses.py restated (oracle/splat_oracle.py): {window}x{window} centre window of frame 0 "
                  f"({wl.n_gaussians} Gaussians, all blended at every pixel as dense.py does), fwd+bwd with the "
                  f"standard_gs loss, median of {reps}; the same window as the --impl reference arm. Mpix/s "
                  f"extrapolated from the window (dense cost is the same at every pixel)",
    }


def cpu_tiled_baseline(wl, tiles: int = TILED_SAMPLE_TILES, tile: int = TILED_TILE, seed: int = 0):
    """Tiled line (tiled.py's faster CPU renderer, restated per tile in oracle/tiled_oracle.py):
    frame 0's activation, projection and tile bounds over every Gaussian (forward and backward),
    plus the blend and loss of ``tiles`` random tiles (forward and backward), extrapolated to the
    frame's tiles."""
    from oracle import splat_oracle as so
    from oracle import tiled_oracle as to

    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    sl = slice(0, 1)
    leaves, vel = _view_leaves(wl, 0)
    t0 = time.perf_counter()
    raw = so.RawGaussians(leaves["means"], leaves["log_scales"], leaves["quats"], leaves["opacity_logits"],
                          leaves["sh"], vel)
    m, s, q, o, rgb = so.activate(raw, wl.times[sl], wl.camera_to_world[sl], 1)
    proj = to.project_view(m[0], s[0], q[0], o[0], rgb[0], wl.fx[0], wl.fy[0], wl.cx[0], wl.cy[0],
                           wl.camera_to_world[0])
    m2, inv, cov, op, rgbp = proj
    bounds = to.gaussian_bounds(m2.detach(), cov.detach(), op.detach(), wl.height, wl.width)
    g = torch.Generator().manual_seed(seed)
    torch.autograd.backward([m2, inv, op, rgbp], [torch.randn(v.shape, generator=g) for v in (m2, inv, op, rgbp)])
    t_frame_fixed = time.perf_counter() - t0

    tiles_x, tiles_y = -(-wl.width // tile), -(-wl.height // tile)
    n_tiles = tiles_x * tiles_y
    # stratified sample: the image's border tiles hold the off-screen Gaussians that tiled.py
    # clamps onto the edge (long lists), the interior ones the rest; each stratum's time is
    # extrapolated to its own tile count
    ids = torch.arange(n_tiles)
    tx, ty = ids % tiles_x, ids // tiles_x
    border = (tx == 0) | (ty == 0) | (tx == tiles_x - 1) | (ty == tiles_y - 1)
    strata = [ids[border], ids[~border]]
    picks = [st[torch.randperm(st.numel(), generator=g)[: tiles // 2]].tolist() for st in strata]
    lf = [v.detach().clone().requires_grad_(True) for v in (m2, inv, op, rgbp)]
    t_tiles = 0.0
    for stratum, pick in zip(strata, picks):
        if pick:
            t_tiles += _tiled_sample_time(to, so, wl, bounds, lf, pick, tile, tiles_x) * stratum.numel() / len(pick)
    t_frame = t_frame_fixed + t_tiles
    return {
        "value": wl.height * wl.width / t_frame / 1e6,
        "unit": UNIT,
        "cores": cores,
        "kind": "port",
        "sample": f"tiled.py restated per tile (oracle/tiled_oracle.py, tile {tile}): frame 0's activation, projection "
                  f"and bounds over all {wl.n_gaussians} Gaussians fwd+bwd ({t_frame_fixed:.2f} s) plus the blend and "
                  f"standard_gs loss fwd+bwd of {sum(len(p) for p in picks)} tiles sampled from the border and the "
                  f"interior tiles of the frame's {n_tiles}, extrapolated per stratum ({t_tiles:.2f} s for the "
                  f"frame). The reference's tiled.py pads every tile to the longest list ([tiles, longest, "
                  f"{tile}, {tile}] tensors) and is slower than this restatement; at 1920x1080 with 1M Gaussians "
                  f"it does not fit in memory",
    }


def _tiled_sample_time(to, so, wl, bounds, lf, pick, tile, tiles_x):
    """Seconds for the tiled blend + loss fwd+bwd of the tiles ``pick`` of frame 0."""
    t0 = time.perf_counter()
    lists = to.tile_lists(*bounds, tile, tiles_x, only=pick)
    outs, tgts = [], []
    for tid in pick:
        ox, oy = (tid % tiles_x) * tile, (tid // tiles_x) * tile
        if tid in lists:
            outs.append(to.blend_tile(*lf, lists[tid], ox, oy, tile).clamp(0.0, 1.0).permute(2, 0, 1))
        else:
            outs.append(torch.ones(3, tile, tile))
        tgt = torch.ones(3, tile, tile)
        h, w = min(tile, wl.height - oy), min(tile, wl.width - ox)
        tgt[:, :h, :w] = wl.target[0, :, oy:oy + h, ox:ox + w]
        tgts.append(tgt)
    loss = so.reconstruction_loss_per_image(torch.stack(outs), torch.stack(tgts)).sum()
    if loss.requires_grad:
        loss.backward()
    return time.perf_counter() - t0


def reference_arm(args, rank, world):
    """--impl reference: the reference's CPU algorithm (the oracle's port of dense.py + losses.py),
    one centre window of one frame per step (frames cycled), the window cpu_baseline also uses."""
    if rank != 0:
        return 0
    full, _ = make_workload(args.workload, 0, 1, args.scale, args.image_scale, args.views)
    wl = full
    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    window = cpu_window(args.workload, wl)
    steps = max(1, args.steps)
    for k in range(args.warmup):
        cpu_sample_time(wl, window, frame=k % wl.n_views)
    total = 0.0
    for k in range(steps):
        total += cpu_sample_time(wl, window, frame=k % wl.n_views)
    value = steps * window * window / total / 1e6
    sample = (f"dense.py + losses.py restated (oracle/splat_oracle.py): {window}x{window} centre window of one frame "
              f"per step ({wl.n_gaussians} Gaussians, dense all-pairs blend + standard_gs loss, fwd+bwd), frames "
              f"cycled; Mpix/s extrapolated from the window (dense cost is the same at every pixel)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.workload, full, make_workload(args.workload, 0, world, args.scale,
                                                                     args.image_scale, args.views)[1], world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------
# main GPU arm


def _profile_rows(kernel: str, workload: str):
    """Rows `| `metric` | value unit |` of the committed ncu summary profiles/<kernel>_<workload>.md
    as {metric: (value, unit)}, and its path; (None, None) when there is none."""
    path = ROOT / "profiles" / f"{kernel}_{workload}.md"
    if not path.exists():
        return None, None
    rows = {}
    for line in path.read_text().splitlines():
        cells = line.split("|")
        if len(cells) >= 3 and cells[1].strip().startswith("`"):
            parts = cells[2].split()
            try:
                rows[cells[1].strip().strip("`")] = (float(parts[0]), parts[1] if len(parts) > 1 else "")
            except (ValueError, IndexError):
                pass
    return rows, str(path.relative_to(ROOT))


def ncu_traffic(kernel: str, workload: str, n_pairs: int):
    """DRAM bytes (read + write) of one launch of `kernel` from the committed ncu summary,
    per launch of this run: a summary of a smaller slice of the workload (its `pairs` row) is
    scaled by the pair count, which the traffic follows.  (None, None) when there is no summary."""
    rows, src = _profile_rows(kernel, workload)
    if rows is None or "dram__bytes_read.sum" not in rows or "dram__bytes_write.sum" not in rows:
        return None, src
    scale = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    total = sum(rows[m][0] * scale.get(rows[m][1], 1.0) for m in ("dram__bytes_read.sum", "dram__bytes_write.sum"))
    if "pairs" in rows and rows["pairs"][0] > 0:
        total *= n_pairs / rows["pairs"][0]
    return total, src


# FP32 operations one B200 SM can retire per cycle (128 lanes, an FMA counted as two).
FP32_FLOP_PER_SM_CYCLE = 256
B200_SMS = 148


def ncu_issue(kernel: str, workload: str):
    """The compute-side bound of `kernel` from the same committed ncu summary: issue-slot use,
    FP32 operations per cycle as a fraction of the SMs' peak, warp instructions per (tile,
    Gaussian) pair.  None without a summary."""
    rows, src = _profile_rows(kernel, workload)
    if rows is None:
        return None
    out = {}
    for metric, key in (("smsp__issue_active.avg.pct_of_peak_sustained_active", "issue_active_pct"),
                        ("sm__throughput.avg.pct_of_peak_sustained_elapsed", "sm_throughput_pct"),
                        ("smsp__inst_executed.sum", "warp_instructions"),
                        ("sm__pipe_fma_cycles_active.avg.pct_of_peak_sustained_active", "fma_pipe_pct")):
        if metric in rows:
            out[key] = rows[metric][0]
    if "fp32_flop_per_cycle" in rows:
        out["fp32_flop_per_cycle"] = rows["fp32_flop_per_cycle"][0]
        out["fp32_frac"] = rows["fp32_flop_per_cycle"][0] / (FP32_FLOP_PER_SM_CYCLE * B200_SMS)
    if "pairs" in rows and "warp_instructions" in out:
        out["warp_instructions_per_pair"] = out["warp_instructions"] / rows["pairs"][0]
    if "issue_active_pct" not in out:
        return None
    out["source"] = src
    return out


def hbm_peak():
    try:
        p = json.loads(PEAKS.read_text())
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def main():
    args = parse_args()
    rank, local_rank, world = (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
                               int(os.environ.get("WORLD_SIZE", 1)))
    if args.impl == "reference":
        return reference_arm(args, rank, world)

    from dynaworld_b200 import _lib, build
    from dynaworld_b200 import render as R

    build.build()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    L = _lib.load()
    full, wl = make_workload(args.workload, rank, world, args.scale, args.image_scale, args.views)
    step = Step(wl, dev, world, args.tile, args.segments, shared_set=full.views_per_set >= full.n_views)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step.run()
    barrier()

    # ---- timed region: inputs resident in HBM; events bracket only the two raster stages ----
    R.STAGE_EVENTS, R.STAGE_FILTER = [], {"raster_fwd", "raster_bwd"}
    sampler = ClockSampler(local_rank if "CUDA_VISIBLE_DEVICES" not in os.environ else local_rank)
    sampler.start()
    launches0 = L.gsb_kernel_launches()
    evs = []
    barrier()
    for _ in range(args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step.run()
        b.record()
        evs.append((a, b))
    barrier()
    launches = L.gsb_kernel_launches() - launches0
    clocks = sampler.stop()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    local_total = sum(step_ms)
    raster_ms: dict[str, list[float]] = {}
    for name, a, b in R.STAGE_EVENTS:
        raster_ms.setdefault(name, []).append(a.elapsed_time(b))
    # every other stage from a separate run of the same steps (events around every stage call)
    R.STAGE_EVENTS, R.STAGE_FILTER = [], None
    for _ in range(min(args.steps, 50)):
        flush.zero_()
        step.run()
    torch.cuda.synchronize()
    stage_ms: dict[str, list[float]] = {}
    for name, a, b in R.STAGE_EVENTS:
        stage_ms.setdefault(name, []).append(a.elapsed_time(b))
    stage_ms.update(raster_ms)  # the raster stages as timed inside the timed region
    R.STAGE_EVENTS = None
    n_pairs = int(getattr(step, "last_pairs", 0))

    t = torch.tensor([local_total], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    pixels_per_step = full.n_views * full.height * full.width  # every rank's views
    value = pixels_per_step * args.steps / (total_ms / 1e3) / 1e6

    # pair count of the workload (for the roofline), from one more forward
    from dynaworld_b200.render import SceneSpec, ViewSpec, forward_stages

    sspec = SceneSpec(wl.n_sets, wl.n_gaussians, True, wl.sh_degree, wl.velocity is not None, True)
    vspec = ViewSpec(wl.n_views, wl.views_per_set, wl.height, wl.width)
    tens = {"means": step.params["means"].detach(), "scales": step.params["log_scales"].detach(),
            "quats": step.params["quats"].detach(),
            "opacities": step.params["opacity_logits"].detach().reshape(wl.n_sets, wl.n_gaussians),
            "colors": step.params["sh"].detach(),
            "velocity": step.params["velocity"].detach() if "velocity" in step.params else None,
            "intrinsics": step.intr, "camera_to_world": step.c2w, "times": step.times}
    _, _, _, fstate = forward_stages(sspec, vspec, step.cfg, 1e-4, tens)
    n_pairs = fstate.n_pairs
    del fstate

    # ---- end to end: host buffers in, loss out, through the public API ----
    e2e = None
    if not args.no_e2e:
        host = {k: v.detach().cpu().pin_memory() for k, v in step.params.items()}
        h_intr, h_c2w = step.intr.cpu().pin_memory(), step.c2w.cpu().pin_memory()
        h_times, h_target = step.times.cpu().pin_memory(), step.target.cpu().pin_memory()
        h2d = sum(v.numel() * v.element_size() for v in host.values()) + sum(
            v.numel() * v.element_size() for v in (h_intr, h_c2w, h_times, h_target))
        d2h = wl.n_views * 4

        # A training loop's input pipeline: step k+1's inputs are copied on a side stream while
        # step k computes, and each step's loss goes to pinned host memory behind its kernels
        # (read on the host after the last step).  Step k's timed events bracket its compute, the
        # copy of step k+1 (issued after step k's start and waited for before its end) and the
        # loss read-back, so every byte of H2D and D2H traffic lies inside a timed step.
        copy_stream = torch.cuda.Stream(dev)
        main = torch.cuda.current_stream(dev)
        host_in = (h_intr, h_c2w, h_times, h_target)
        losses_host = torch.empty(max(args.steps, args.warmup, 2), wl.n_views, dtype=torch.float32).pin_memory()

        def fetch():
            with torch.cuda.stream(copy_stream):
                p = {k: v.to(dev, non_blocking=True) for k, v in host.items()}
                rest = tuple(v.to(dev, non_blocking=True) for v in host_in)
                done = torch.cuda.Event()
                done.record(copy_stream)
            for t in (*p.values(), *rest):
                t.record_stream(main)
            return p, rest, done

        def e2e_steps(n, events=None):
            pending = None
            for k in range(n):
                if events is not None:
                    flush.zero_()
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                if pending is None:
                    pending = fetch()
                p, rest, done = pending
                main.wait_event(done)
                loss = step.run({k2: v.requires_grad_(True) for k2, v in p.items()}, *rest)
                losses_host[k].copy_(loss.detach(), non_blocking=True)
                pending = fetch() if k + 1 < n else None
                if pending is not None:
                    main.wait_event(pending[2])
                if events is not None:
                    b.record()
                    events.append((a, b))
            torch.cuda.synchronize()
            return losses_host[:n].clone()

        e2e_steps(max(2, args.warmup))
        barrier()
        e_evs = []
        e2e_losses = e2e_steps(args.steps, e_evs)
        if not torch.isfinite(e2e_losses).all():
            raise RuntimeError("non-finite loss in the end-to-end run")
        barrier()
        et = torch.tensor([sum(a.elapsed_time(b) for a, b in e_evs)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": pixels_per_step * args.steps / (float(et.item()) / 1e3) / 1e6, "unit": UNIT,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)}

    # ---- roofline of the dominant kernel ----
    means = {k: sum(v) / len(v) for k, v in stage_ms.items()}
    dominant = max(("raster_bwd", "raster_fwd"), key=lambda k: means.get(k, 0.0))
    px = wl.n_views * wl.height * wl.width
    if dominant == "raster_bwd":
        alg_bytes = BWD_BYTES_PER_PAIR * n_pairs + BWD_BYTES_PER_PIXEL * px
    else:
        alg_bytes = FWD_BYTES_PER_PAIR * n_pairs + FWD_BYTES_PER_PIXEL * px
    peak, peak_kind = hbm_peak()
    dur_s = means[dominant] / 1e3
    achieved = alg_bytes / dur_s / 1e9
    traffic, traffic_src = (ncu_traffic(dominant, args.workload, n_pairs) if (args.tile is None and args.segments == 0
                                                                             and not args.views) else (None, None))
    roofline = {"bound": "hbm", "kernel": f"{dominant} (gsb_{dominant})", "achieved": achieved, "peak": peak,
                "unit": "GB/s", "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_src,
                "peak_source": peak_kind, "bytes_per_launch": int(alg_bytes), "pairs": int(n_pairs),
                "pixels": int(px), "launch_ms": means[dominant],
                "issue": (ncu_issue(dominant, args.workload) if (args.tile is None and args.segments == 0
                                                                 and not args.views) else None),
                "note": "the raster is issue-bound (records re-read from L2, DRAM traffic below the algorithmic "
                        "bytes): 'issue' gives the same kernel's ncu issue-slot use, FP32 operations as a "
                        "fraction of the SMs' FP32 peak and warp instructions per pair (profiles/)"}
    stage_share = {k: round(v / sum(means.values()), 4) for k, v in means.items()} if means else {}

    if rank == 0:
        cpu = cpu_tiled = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(args.workload, wl)
            cpu_tiled = cpu_tiled_baseline(wl)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args.workload, full, wl, world),
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "cpu_baseline_tiled": cpu_tiled,
            "clocks": clocks,
            "gpu_launches": int(launches), "stage_ms": {k: round(v, 4) for k, v in means.items()},
            "stage_share": stage_share,
        }
        print(json.dumps(line), flush=True)
        if args.stages:
            print(json.dumps(means, indent=1), file=sys.stderr)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
