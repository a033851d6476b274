#!/usr/bin/env python
"""Benchmark: data-parallel 3DGS training step on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU, NCCL)

A step is one view per GPU: render forward, L1 + D-SSIM loss, render backward,
all-reduce (pmean) of the flat gradient buffer, densification statistics and
the masked multi-group Adam update -- trainer.py:55-123 on the native
kernels. Prints ONE JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "jax-gs_b200"), ROOT]

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "train views/s (fwd+bwd)"
UNIT = "views/s"
WORKLOAD = ("BASELINE config 2: data-parallel train step, one view per GPU; 100k active Gaussians in "
            "a 200k static capacity, SH degree 3, 504x378, 20 cameras on a 30 deg arc at r=4; "
            "0.8 L1 + 0.2 D-SSIM, masked multi-group Adam, pmean over GPUs")
HBM_FALLBACK = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["train", "render", "train-large", "densify", "2dgs"], default="train",
                    help="train: config 2 train step (default); render: config 3 render-only Mpix/s; "
                         "train-large: the same train step on the config 3 scene (1M Gaussians, SH3, 1920x1080); "
                         "densify: config 4 (4M capacity, 3M active, 1600x1064) with densify_and_prune every "
                         "100 steps amortised; 2dgs: config 5 surfel train step (500k surfels, 1264x832)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--render-streams", type=int, default=4,
                    help="render workload: streams (each with its own workspace) the 8 views are spread over")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-fused", action="store_true",
                    help="N>1: NCCL all-reduces + replicated Adam instead of the fused peer-memory update")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch the step's kernels one by one instead of replaying a CUDA graph")
    ap.add_argument("--profile", type=int, default=0,
                    help="run warm-up + this many train steps and exit (for ncu captures)")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled by NVML every
    ~2 ms from a background thread during the timed region (nvidia-smi's
    200 ms minimum interval is longer than the region itself)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device: torch.device):
        self.device = device
        self.samples = []
        self.smax = None
        self.err = None
        self._stop = threading.Event()
        self.thread = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(self.device)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception as e:  # no NVML: report it instead of guessing
            self.err = f"nvml unavailable: {e}"
            return

        def loop():
            while not self._stop.is_set():
                try:
                    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((float(sm), int(rs)))
                except Exception as e:
                    self.err = str(e)
                    return
                time.sleep(0.002)

        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()

    def stop(self):
        self._stop.set()
        if self.thread:
            self.thread.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.smax, "reasons": [], "samples": 0,
                    "note": self.err or "no samples"}
        reasons = set()
        for _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm for sm, _ in self.samples), "sm_max_mhz": self.smax,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml"}


def alg_bytes(kernel, st):
    """Algorithmic bytes of one launch: the bytes the kernel must move per
    unit (pair, pixel, Gaussian, element) times the units of one launch."""
    N, Na, K, M, P, Nv = st["N"], st["Na"], st["K"], st["M"], st["P"], st["Nv"]
    table = {
        "preprocess_fwd": N * 1 + Na * (44 + 12 * K) + Na * 48,
        "raster_fwd": M * 40 + P * 20,
        "raster_bwd": M * 40 + P * 20 + Nv * 72,
        "preprocess_bwd": Na * (44 + 12 * K + 36 + 48) + Na * (40 + 12 * K),
        "adam": N * (11 + 3 * K) * 4 * 7 + N,
        "sort_tile": M * 16,
        "sort_depth": Nv * 16,
        "emit_pairs": M * 8 + Nv * 12,
        # 2DGS (config 5): Mc = composited pairs (first 512 per tile); a
        # Splat2 record is 64 B, a pixel has 9 output maps + pix_T
        "raster2d_fwd": st.get("Mc", 0) * 68 + P * 40,
        "raster2d_bwd": st.get("Mc", 0) * 68 + P * 72 + Nv * 64,
        "preprocess2d_fwd": N * (52 + 13) + Nv * 64,
        "preprocess2d_bwd": N * (52 + 64 + 40 + 12 * K),
        "adam_flat": N * (10 + 3 * K) * 4 * 7,
        "ssim_fwd": P * 3 * 4 * (2 + 3),
        "ssim_bwd": P * 3 * 4 * (3 + 2 + 2),
        "l1_loss": P * 3 * 4 * 3,
    }
    return table.get(kernel)


def read_loss_lagged(loss, i, loss_h, loss_ev):
    """End-to-end loop's loss read: step i's loss is copied to pinned host
    memory as soon as it is enqueued, and read (after its copy completes)
    once step i + 1 has been enqueued, so the host keeps one step in flight.
    loss=None reads the last step's value (i = number of steps)."""
    if loss is not None:
        loss_h[i % 2].copy_(loss.reshape(()), non_blocking=True)
        loss_ev[i % 2].record()
    if i > 0:
        loss_ev[(i - 1) % 2].synchronize()
        v = float(loss_h[(i - 1) % 2])
        if not math.isfinite(v):
            raise RuntimeError(f"non-finite loss at end-to-end step {i - 1}")


def build_state(scene, device):
    from gs_b200.core.gaussians import Gaussians
    from gs_b200.training.trainer import AdamConfig, init_density_state
    na = int(scene.active.sum())
    t = lambda a: torch.as_tensor(a[:na], device=device)  # noqa: E731
    g = Gaussians(means=t(scene.means), scales=t(scene.scales), quaternions=t(scene.quats),
                  opacities=t(scene.opacities), sh_coeffs=t(scene.sh))
    m = scene.means[:na]
    extent = float(np.max(np.linalg.norm(m - m.mean(0), axis=1)))
    opt = AdamConfig.from_extent(extent, 30000)
    return init_density_state(g, opt, scene.n), opt


def view_stats(state, scene, device, capacity=None):
    """M (pairs per view, averaged over the cameras), visible Gaussians N_v."""
    from gs_b200.core.camera import Camera
    from gs_b200.renderer.projection import project_gaussians
    from gs_b200.renderer.rasterizer import get_tile_interactions
    Ms, Nvs = [], []
    for w2c in scene.w2cs[:4]:
        cam = Camera(scene.W, scene.H, scene.fx, scene.fy, scene.cx, scene.cy,
                     torch.as_tensor(w2c, device=device), None)
        m2, _, radii, valid, z = project_gaussians(state.gaussians, cam, mask=state.active_mask)
        _, gids, n = get_tile_interactions(m2, radii, valid, z, scene.H, scene.W, capacity=capacity)
        n = int(n)
        Ms.append(n)
        Nvs.append(int(torch.unique(gids[:n]).numel()))
    return float(np.mean(Ms)), float(np.mean(Nvs))


def cpu_baseline_sample(scene, seed):
    """One oracle train step of view 0 on the host cores (torch CPU)."""
    from oracle import ref_restated as R
    torch.set_num_threads(os.cpu_count() or 1)
    params = {"means": torch.tensor(scene.means), "scales": torch.tensor(scene.scales),
              "quaternions": torch.tensor(scene.quats), "opacities": torch.tensor(scene.opacities),
              "sh_coeffs": torch.tensor(scene.sh)}
    zeros = {k: torch.zeros_like(v) for k, v in params.items()}
    from gs_b200 import synthetic
    tgt = torch.tensor(synthetic.target_image(seed, scene.H, scene.W))
    lrs = dict(zip(R.GROUPS, [1e-4, 0.005, 0.001, 0.05, 0.0025]))
    t0 = time.perf_counter()
    R.train_step(params, zeros, dict(zeros), 1, lrs, torch.tensor(scene.active), tgt,
                 torch.tensor(scene.w2cs[0]), scene.camera_static(), sh_degree=scene.sh_degree,
                 compact_sort=False)
    return time.perf_counter() - t0


LARGE_SAMPLE_TILES = 960  # about 1/8 of the tiles of a 1080p view (the central band)


def large_cpu_sample(scene, seed, cfg_id):
    """Oracle train step (torch-CPU autograd, L1 + D-SSIM, Adam) of view 0
    with only the central band of about LARGE_SAMPLE_TILES tiles composited
    (projection, SH, sort, loss and Adam on everything); views/s scaled by the
    tile share. densify_and_prune (every 100 steps) is not in the sample."""
    from oracle import ref_restated as R
    torch.set_num_threads(os.cpu_count() or 1)
    from gs_b200 import synthetic
    params = {"means": torch.tensor(scene.means), "scales": torch.tensor(scene.scales),
              "quaternions": torch.tensor(scene.quats), "opacities": torch.tensor(scene.opacities),
              "sh_coeffs": torch.tensor(scene.sh)}
    zeros = {k: torch.zeros_like(v) for k, v in params.items()}
    tgt = torch.tensor(synthetic.target_image(seed, scene.H, scene.W))
    lrs = dict(zip(R.GROUPS, [1e-4, 0.005, 0.001, 0.05, 0.0025]))
    tx, ty = (scene.W + 15) // 16, (scene.H + 15) // 16
    rows = max(1, LARGE_SAMPLE_TILES // tx)
    r0 = (ty - rows) // 2
    subset = list(range(r0 * tx, (r0 + rows) * tx))
    t0 = time.perf_counter()
    R.train_step(params, zeros, dict(zeros), 1, lrs, torch.tensor(scene.active), tgt, torch.tensor(scene.w2cs[0]),
                 scene.camera_static(), sh_degree=scene.sh_degree, compact_sort=True, tile_subset=subset)
    dt = time.perf_counter() - t0
    share = len(subset) / (tx * ty)
    return {"value": share / dt, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"1 oracle train step of config {cfg_id} view 0 with the central {len(subset)} of "
                      f"{tx * ty} tiles composited (projection, SH, sort, loss, Adam on all Gaussians; "
                      f"densify_and_prune not sampled); {dt:.1f} s, scaled by the tile share"}


WORKLOAD_LARGE = ("north-star train step: the config 3 scene (1M Gaussians, all active, SH degree 3) at "
                  "1920x1080, one of 64 sphere views per GPU per step, targets uniform [0,1]; 0.8 L1 + 0.2 "
                  "D-SSIM, masked multi-group Adam, pmean over GPUs")
DENSIFY_EVERY = 100
WORKLOAD_DENSIFY = ("BASELINE config 4: 4M capacity, 3M active (8 Gaussian blobs, sigma 1.5, in a 20^3 box), "
                    "SH degree 3, 1600x1064, 200 orbit cameras at r=15, one view per GPU per step; "
                    "densify_and_prune (grad threshold 2e-4) every 100 steps, its time amortised")
RENDER_METRIC = "render Mpix/s"
RENDER_WORKLOAD = ("BASELINE config 3: render-only, 1M Gaussians (uniform in a 10^3 box), SH degree 3, "
                   "1920x1080, fx=fy=1200, 64 views on a sphere of radius 12, 8 views per GPU per step")
RENDER_SAMPLE_TILES = 1020  # 1/8 of the 8160 tiles of a 1920x1080 view (the central band)


def render_cpu_sample(scene, view=0):
    """Oracle render of one config-3 view restricted to the central 1/8 of
    its tiles (projection, SH and the full sort still run for all 1M
    Gaussians); returns (pixels composited, seconds)."""
    from oracle import ref_restated as R
    torch.set_num_threads(os.cpu_count() or 1)
    tx = (scene.W + 15) // 16
    ty = (scene.H + 15) // 16
    rows = RENDER_SAMPLE_TILES // tx
    r0 = (ty - rows) // 2
    subset = list(range(r0 * tx, (r0 + rows) * tx))
    t = lambda a: torch.tensor(a)  # noqa: E731
    t0 = time.perf_counter()
    with torch.no_grad():
        R.render(t(scene.means), t(scene.scales), t(scene.quats), t(scene.opacities), t(scene.sh),
                 t(scene.w2cs[view]), scene.W, scene.H, scene.fx, scene.fy, scene.cx, scene.cy,
                 sh_degree=scene.sh_degree, tile_subset=subset)
    return len(subset) * 256, time.perf_counter() - t0


def run_reference(args, world, rank):
    """Reference arm: the reference's algorithm on the host CPU (the torch-CPU
    restatement in oracle/, since JAX is not installable here), rank 0 only."""
    if rank != 0:
        return
    if args.workload == "render":
        from gs_b200 import synthetic
        scene = synthetic.config3(args.seed)
        cores = os.cpu_count() or 1
        pix, secs = 0, 0.0
        render_cpu_sample(scene, 0)  # warm-up
        steps = 0
        while steps < max(1, min(args.steps, 3)):
            p, t = render_cpu_sample(scene, steps % len(scene.w2cs))
            pix += p
            secs += t
            steps += 1
        v = pix / secs / 1e6
        sample = (f"{steps} view(s) of config 3, central {RENDER_SAMPLE_TILES} of 8160 tiles composited "
                  f"(projection, SH, sort of all 1M Gaussians), torch-CPU restatement, {cores} threads; "
                  "JAX reference not installable")
        print(json.dumps({
            "impl": "reference", "metric": RENDER_METRIC, "value": v, "unit": "Mpix/s", "n_gpus": world,
            "steps": steps, "warmup": 1, "ms_per_step": 1000.0 * secs / steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": RENDER_WORKLOAD, "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "Mpix/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "Mpix/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    if args.workload == "2dgs":
        from gs_b200 import synthetic
        sc = synthetic.config5(args.seed)
        twod_cpu_sample(sc, args.seed)  # warm-up
        res = [twod_cpu_sample(sc, args.seed) for _ in range(max(1, min(args.steps, 2)))]
        v = len(res) / sum(1.0 / r["value"] for r in res)
        cpu = dict(res[0], value=v, sample=f"{len(res)} x " + res[0]["sample"] + "; JAX reference not installable")
        print(json.dumps({
            "impl": "reference", "metric": "2DGS train views/s (fwd+bwd)", "value": v, "unit": "views/s",
            "n_gpus": world, "steps": len(res), "warmup": 1, "ms_per_step": 1000.0 / v, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD_2DGS, "parallelism": "cpu"}, "cpu_baseline": cpu,
            "e2e": {"value": v, "unit": "views/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    if args.workload in ("train-large", "densify"):
        from gs_b200 import synthetic
        dens = args.workload == "densify"
        cfg_id = 4 if dens else 3
        scene = (synthetic.config4 if dens else synthetic.config3)(args.seed)
        res = [large_cpu_sample(scene, args.seed, cfg_id) for _ in range(max(1, min(args.steps, 2)))]
        v = len(res) / sum(1.0 / r["value"] for r in res)
        cpu = dict(res[0], value=v, sample=f"{len(res)} x " + res[0]["sample"] + "; JAX reference not installable")
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world,
            "steps": len(res), "warmup": 0, "ms_per_step": 1000.0 / v, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD_DENSIFY if dens else WORKLOAD_LARGE, "parallelism": "cpu"},
            "cpu_baseline": cpu,
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    from gs_b200 import synthetic
    scene = synthetic.config2(args.seed)
    cores = os.cpu_count() or 1
    t_first = cpu_baseline_sample(scene, args.seed)  # warm-up (1 step is enough for the CPU path)
    steps = max(1, min(args.steps, int(150.0 / max(t_first, 1e-3))))
    times = [cpu_baseline_sample(scene, args.seed) for _ in range(steps)]
    total = sum(times)
    v = steps / total
    sample = (f"{steps} oracle train step(s) of config 2 view 0 (literal N*256-slot sort, torch-CPU "
              f"autograd, L1+D-SSIM, Adam), {cores} threads; JAX reference not installable")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": 1, "ms_per_step": 1000.0 * total / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse()
    world, rank, local = dist_env()
    if args.impl == "reference":
        # rank 0 alone runs the host-CPU reference and prints; the other ranks
        # exit at once (no process group: nothing to exchange, and a barrier
        # would time out while rank 0 spends minutes on the CPU)
        run_reference(args, world, rank)
        return
    group = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        group = dist.group.WORLD

    if args.workload in ("render", "2dgs"):
        (run_render if args.workload == "render" else run_2dgs)(args, world, rank, local, group)
        if group is not None:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return

    from gs_b200 import _lib, synthetic
    from gs_b200.training.trainer import CapturedStep, train_step_internal
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dens = args.workload == "densify"
    large = args.workload in ("train-large", "densify")
    cfg_id = 4 if dens else 3 if large else 2
    scene = {2: synthetic.config2, 3: synthetic.config3, 4: synthetic.config4}[cfg_id](args.seed)
    workload = WORKLOAD_DENSIFY if dens else WORKLOAD_LARGE if large else WORKLOAD
    state, opt = build_state(scene, dev)
    n_cams = len(scene.w2cs)
    n_tgt = 8 if large else n_cams  # 1080p targets: 8 distinct images, cycled
    # pair capacity: 16 per Gaussian at 1080p (about 12 are used; checked below)
    cap = 16 * scene.n if large else None
    targets_h = [torch.tensor(synthetic.target_image(args.seed + i, scene.H, scene.W)).pin_memory()
                 for i in range(n_tgt)]
    w2cs_h = [torch.tensor(w).pin_memory() for w in scene.w2cs]
    targets_d = [t.to(dev) for t in targets_h]
    w2cs_d = [w.to(dev) for w in w2cs_h]
    cam = scene.camera_static()
    deg = scene.sh_degree

    captured = None
    if not args.no_graph:
        # the whole step (NCCL all-reduces included when N > 1) as one CUDA
        # graph; its construction trains one step
        v0 = rank % n_cams
        captured = CapturedStep(state, targets_d[v0 % n_tgt], w2cs_d[v0], cam, opt, sh_degree=deg, group=group,
                                fused=not args.no_fused, capacity=cap)

    def step(i, host=False):
        v = (i * world + rank) % n_cams
        tgt = targets_h[v % n_tgt] if host else targets_d[v % n_tgt]
        w2c = w2cs_h[v] if host else w2cs_d[v]
        if captured is not None:
            return captured(tgt, w2c)
        return train_step_internal(state, tgt, w2c, cam, opt, sh_degree=deg, group=group,
                                   fused=not args.no_fused, capacity=cap)

    def barrier():
        if group is not None:
            import torch.distributed as dist
            dist.barrier(group=group)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    if args.profile:
        for i in range(args.profile):
            step(args.warmup + i)
        torch.cuda.synchronize()
        if rank == 0:
            print(f"profile: {args.profile} train steps done", flush=True)
        return

    # ---- device-timed region (inputs resident in HBM; L2 flushed between steps)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    K = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    clocks = ClockSampler(dev)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    for i in range(K):
        flush.zero_()
        ev[i][0].record()
        step(args.warmup + i)
        ev[i][1].record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = sum(a.elapsed_time(b) for a, b in ev)
    tmax = torch.tensor([ms], dtype=torch.float64, device=dev)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX, group=group)
    ms_total = float(tmax)
    value = world * K / (ms_total / 1000.0)

    # ---- end to end through the public API: pinned host inputs, loss read back
    barrier()
    torch.cuda.synchronize()
    loss_h = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(2)]
    loss_ev = [torch.cuda.Event() for _ in range(2)]
    t0 = time.perf_counter()
    for i in range(K):
        _, loss, _ = step(args.warmup + K + i, host=True)
        read_loss_lagged(loss, i, loss_h, loss_ev)
    read_loss_lagged(None, K, loss_h, loss_ev)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(te, op=dist.ReduceOp.MAX, group=group)
    e2e_value = world * K / float(te)
    h2d = scene.H * scene.W * 3 * 4 + 16 * 4
    d2h = 4

    dens_cfg = {}
    if dens:
        # densify_and_prune (density.py:98-211) every DENSIFY_EVERY steps, on the
        # statistics the steps above accumulated; device time of each call
        from gs_b200.training.density import densify_and_prune
        extent = float(np.max(np.linalg.norm(scene.means[scene.active] - scene.means[scene.active].mean(0),
                                             axis=1)))
        dms = []
        info = None
        for j in range(2):
            barrier()
            a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            densify_and_prune(state, rng_key=args.seed + j, grad_threshold=0.0002, extent=extent)
            b_.record()
            torch.cuda.synchronize()
            dms.append(a.elapsed_time(b_))
            info = [int(x) for x in state.densify_info.cpu()]
            for i in range(5):  # a few steps in between, so the second call has statistics
                step(args.warmup + 2 * K + i)
            torch.cuda.synchronize()
        dm = torch.tensor([max(dms)], dtype=torch.float64, device=dev)
        if group is not None:
            import torch.distributed as dist
            dist.all_reduce(dm, op=dist.ReduceOp.MAX, group=group)
        d_ms = float(dm)
        step_ms, e2e_step_ms = ms_total / K, 1000.0 * float(te) / K
        value = world * DENSIFY_EVERY / ((DENSIFY_EVERY * step_ms + d_ms) / 1000.0)
        e2e_value = world * DENSIFY_EVERY / ((DENSIFY_EVERY * e2e_step_ms + d_ms) / 1000.0)
        dens_cfg = {"densify_every": DENSIFY_EVERY, "densify_ms": d_ms, "train_step_ms": step_ms,
                    "densify_last": dict(zip(("pruned", "clones", "splits", "applied"), info)),
                    "extent": extent}

    # ---- per-kernel device time (CUDA events around every library launch)
    _lib.lib().gs_timing_enable(64 * K)
    torch.cuda.synchronize()
    for i in range(K):
        v = ((args.warmup + 3 * K + i) * world + rank) % n_cams
        train_step_internal(state, targets_d[v % n_tgt], w2cs_d[v], cam, opt, sh_degree=deg, group=group,
                            fused=not args.no_fused, capacity=cap)
    torch.cuda.synchronize()
    kt = _lib.kernel_times()
    if cap is not None:
        assert int(state.buffers(scene.W, scene.H, cap)["extras"][8]) == 0, "pair capacity overflow"
    _lib.lib().gs_timing_disable()
    launches = sum(c for _, c in kt.values())
    kernels = {k: round(v[0] / K, 4) for k, v in sorted(kt.items(), key=lambda x: -x[1][0])}

    out = None
    if rank == 0:
        M, Nv = view_stats(state, scene, dev, cap)
        st = {"N": scene.n, "Na": int(scene.active.sum()), "K": 16, "M": M, "P": scene.W * scene.H,
              "Nv": Nv}
        hbm, src = peaks()
        dom = max(kt.items(), key=lambda x: x[1][0])[0]
        per_launch_ms = kt[dom][0] / kt[dom][1]
        b = alg_bytes(dom, st)
        achieved = (b / (per_launch_ms / 1000.0)) / 1e9 if b else None
        traffic = read_traffic(dom + ("_config%d" % cfg_id if large else ""))
        roof = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": (achieved / hbm) if achieved else None, "traffic": traffic,
                "peak_source": f"{src} hbm_gbs (MEASURED_PEAKS.json)" if src == "measured" else "fallback",
                "alg_bytes_per_launch": b, "ms_per_launch": per_launch_ms}
        roof.update(limiter(dom + ("_config%d" % cfg_id if large else ""), roof["frac"]))
        cpu = None
        if world == 1 and not args.no_cpu_baseline and not large:
            t_cpu = cpu_baseline_sample(scene, args.seed)
            cpu = {"value": 1.0 / t_cpu, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                   "sample": "1 oracle train step of config 2 view 0 (literal N*256-slot sort, torch-CPU "
                             "autograd, L1+D-SSIM, Adam)"}
        elif world == 1 and not args.no_cpu_baseline:
            cpu = large_cpu_sample(scene, args.seed, cfg_id)
        out = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_total / K, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE config %d distributions)" % cfg_id,
            "config": {"workload": workload, "gaussians_capacity": scene.n,
                       "gaussians_active": int(scene.active.sum()), "image": [scene.W, scene.H],
                       "views_per_gpu_per_step": 1, "pairs_per_view": M, "visible_per_view": Nv,
                       "l2": "flushed between timed steps (256 MiB write, outside the step events)",
                       "parallelism": f"dp{world}",
                       "step_launch": "cuda graph replay" if captured is not None else "eager",
                       "dp_update": ("n/a" if world == 1 else "nccl all-reduce" if args.no_fused
                                     else "fused peer-memory kernel"), **dens_cfg},
            "clocks": clk,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches, "roofline": roof, "cpu_baseline": cpu,
            "kernels_ms_per_step": kernels,
        }
        print(json.dumps(out), flush=True)
    # a graph holding NCCL calls must be released before the process group
    del captured, step
    torch.cuda.synchronize()
    for v in state._buffers.values():
        if hasattr(v, "close"):
            v.close()
    if group is not None:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def run_render(args, world, rank, local, group):
    """Config 3: each GPU renders 8 of the 64 views per step (replicas, no
    exchange). value = pixels of all ranks' views / max-over-ranks time."""
    from gs_b200 import _lib, synthetic
    from gs_b200.core.camera import Camera
    from gs_b200.core.gaussians import Gaussians
    from gs_b200.renderer.renderer import render
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    scene = synthetic.config3(args.seed)
    n, W, H, k = scene.n, scene.W, scene.H, 16
    V = 8
    tt = lambda a: torch.as_tensor(a, device=dev).contiguous()  # noqa: E731
    means, scales, quats, opac, sh = (tt(scene.means), tt(scene.scales), tt(scene.quats),
                                      tt(scene.opacities), tt(scene.sh))
    w2cs_h = [torch.tensor(w).pin_memory() for w in scene.w2cs]
    w2cs_d = torch.stack([w.to(dev) for w in w2cs_h])
    cap = 16 * n  # pairs per view; overflow is checked below
    P = _lib.ptr
    lib = _lib.lib()
    # the step's views run on S streams with a workspace each, so that one
    # view's sort overlaps another's compositing on the GPU
    S = max(1, min(args.render_streams, V))
    wss = [torch.empty(lib.gs_workspace_bytes(n, W, H, cap), dtype=torch.uint8, device=dev) for _ in range(S)]
    images = torch.empty((V, H, W, 3), dtype=torch.float32, device=dev)
    radii = [torch.empty(n, dtype=torch.float32, device=dev) for _ in range(S)]
    valid = [torch.empty(n, dtype=torch.uint8, device=dev) for _ in range(S)]
    extras = torch.zeros((V, 16), dtype=torch.int32, device=dev)
    views_d = torch.zeros(V, 4, 4, dtype=torch.float32, device=dev)
    side = [torch.cuda.Stream(dev) for _ in range(S - 1)]

    def forward_views():
        main = torch.cuda.current_stream(dev)
        for s2 in side:
            s2.wait_stream(main)
        for i in range(V):
            j = i % S
            st = main.cuda_stream if j == 0 else side[j - 1].cuda_stream
            ws = wss[j]
            _lib.call("gs_render_image", P(means), P(scales), P(quats), P(opac), P(sh), n, k, None,
                      P(views_d[i]), W, H, scene.fx, scene.fy, scene.cx, scene.cy, None, scene.sh_degree,
                      cap, P(ws), ws.numel(), P(images[i]), P(radii[j]), P(valid[j]), P(extras[i]), st)
        for s2 in side:
            main.wait_stream(s2)

    def set_views(step):
        base = (step * world + rank) * V
        views_d.copy_(w2cs_d[[(base + i) % len(scene.w2cs) for i in range(V)]])

    for i in range(max(args.warmup, 3)):
        set_views(i)
        forward_views()
    torch.cuda.synchronize()
    assert int(extras[:, 8].max()) == 0, "pair capacity overflow"
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        forward_views()
    K = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    clocks = ClockSampler(dev)
    clocks.start()
    if group is not None:
        import torch.distributed as dist
        dist.barrier(group=group)
    torch.cuda.synchronize()
    for i in range(K):
        set_views(i)
        flush.zero_()
        ev[i][0].record()
        graph.replay()
        ev[i][1].record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = sum(a.elapsed_time(b) for a, b in ev)
    tm = torch.tensor([ms], dtype=torch.float64, device=dev)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(tm, op=dist.ReduceOp.MAX, group=group)
    pix = W * H * V * world * K
    value = pix / (float(tm) / 1000.0) / 1e6
    assert int(extras[:, 8].max()) == 0, "pair capacity overflow"
    M = float(extras[:, 0].float().mean())
    # end to end through the public render(): W2C from pinned host memory,
    # image copied back to pinned host memory, every view; the views are
    # issued round-robin on the same S streams (render() takes its scratch
    # from the stream-aware allocator, so concurrent calls do not share it),
    # so one view's copies overlap other views' kernels
    g = Gaussians(means=means, scales=scales, quaternions=quats, opacities=opac, sh_coeffs=sh)
    e2e_streams = [torch.cuda.current_stream(dev)] + side
    host_imgs = [torch.empty((H, W, 3), dtype=torch.float32).pin_memory() for _ in range(S)]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.no_grad():
        for i in range(K):
            base = (i * world + rank) * V
            for j in range(V):
                with torch.cuda.stream(e2e_streams[j % S]):
                    w = w2cs_h[(base + j) % len(scene.w2cs)]
                    cam = Camera(W, H, scene.fx, scene.fy, scene.cx, scene.cy, w.to(dev, non_blocking=True),
                                 None)
                    img, _ = render(g, cam, sh_degree=scene.sh_degree, capacity=cap)
                    host_imgs[j % S].copy_(img, non_blocking=True)
        torch.cuda.synchronize()
    te = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(te, op=dist.ReduceOp.MAX, group=group)
    e2e = pix / float(te) / 1e6
    # per-kernel device time of the same work (eager, timing hook)
    lib.gs_timing_enable(64 * K * V)
    for i in range(K):
        set_views(i)
        forward_views()
    torch.cuda.synchronize()
    kt = _lib.kernel_times()
    lib.gs_timing_disable()
    launches = sum(c for _, c in kt.values())
    del graph
    if rank != 0:
        return
    hbm, src = peaks()
    dom = max(kt.items(), key=lambda x: x[1][0])[0]
    per_ms = kt[dom][0] / kt[dom][1]
    st = {"N": n, "Na": n, "K": 16, "M": M, "P": W * H, "Nv": n}
    b = alg_bytes(dom, st)
    achieved = (b / (per_ms / 1000.0)) / 1e9 if b else None
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        pix_c, secs = render_cpu_sample(scene, 0)
        cpu = {"value": pix_c / secs / 1e6, "unit": "Mpix/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"1 view of config 3, central {RENDER_SAMPLE_TILES} of 8160 tiles composited "
                         "(projection, SH, sort of all 1M Gaussians), torch-CPU restatement"}
    print(json.dumps({
        "metric": RENDER_METRIC, "value": value, "unit": "Mpix/s", "n_gpus": world, "steps": K,
        "warmup": max(args.warmup, 3), "ms_per_step": float(tm) / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE config 3)",
        "config": {"workload": RENDER_WORKLOAD, "gaussians": n, "image": [W, H], "views_per_gpu_per_step": V,
                   "pairs_per_view": M, "capacity_per_view": cap,
                   "l2": "flushed between timed steps (256 MiB write, outside the step events)",
                   "parallelism": f"replicas x{world}", "step_launch": "cuda graph replay",
                   "streams_per_gpu": S},
        "clocks": clk,
        "e2e": {"value": e2e, "unit": "Mpix/s", "h2d_bytes_per_step": 64 * V,
                "d2h_bytes_per_step": W * H * 3 * 4 * V},
        "gpu_launches": launches,
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": (achieved / hbm) if achieved else None, "traffic": read_traffic(dom + "_config3"),
                     "peak_source": f"{src} hbm_gbs (MEASURED_PEAKS.json)", "alg_bytes_per_launch": b,
                     "ms_per_launch": per_ms,
                     **limiter(dom + "_config3", (achieved / hbm) if achieved else None)},
        "cpu_baseline": cpu,
        "kernels_ms_per_step": {k2: round(v2[0] / K, 4) for k2, v2 in sorted(kt.items(), key=lambda x: -x[1][0])},
    }), flush=True)


TWOD_SAMPLE_TILES = 632  # 8 of the 52 tile rows of a 1264x832 view (the central band)


def twod_cpu_sample(sc, seed):
    """Oracle 2DGS train loss fwd+bwd of config 5 view 0 with only the
    central TWOD_SAMPLE_TILES tiles composited (projection, sort, losses and
    their backward run on the full view); views/s scaled by the tile share."""
    from oracle import ref_restated_2d as R2
    torch.set_num_threads(os.cpu_count() or 1)
    from gs_b200 import synthetic
    p = {k: torch.tensor(sc[k]).requires_grad_(True)
         for k in ("means", "scales", "quaternions", "opacities", "sh_coeffs")}
    tgt = torch.tensor(synthetic.target_image(seed, sc["H"], sc["W"]))
    tx, ty = (sc["W"] + 15) // 16, (sc["H"] + 15) // 16
    rows = TWOD_SAMPLE_TILES // tx
    r0 = (ty - rows) // 2
    subset = list(range(r0 * tx, (r0 + rows) * tx))
    t0 = time.perf_counter()
    loss, _ = R2.train_loss_2d(p, tgt, torch.tensor(sc["w2cs"][0]), sc["W"], sc["H"], sc["fx"], sc["fy"],
                               sc["cx"], sc["cy"], tile_subset=subset)
    loss.backward()
    dt = time.perf_counter() - t0
    share = len(subset) / (tx * ty)
    return {"value": share / dt, "unit": "views/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"oracle 2DGS train loss fwd+bwd (torch-CPU autograd) of config 5 view 0 with the central "
                      f"{len(subset)} of {tx * ty} tiles composited; {dt:.1f} s, scaled by the tile share"}


WORKLOAD_2DGS = ("BASELINE config 5: 2DGS train step (render fwd with RGB, depth, depth^2, normal and 1 - T maps; "
                 "0.8 L1 + 0.2 D-SSIM + 1e-4 distortion + 1e-4 normal consistency; bwd; Adam 1e-3), 500k surfels "
                 "uniform in a 6^3 box, log-scales N(-3.5, 0.5), SH degree 3 (DC used), 1264x832, one of 20 sphere "
                 "views per GPU per step")


def run_2dgs(args, world, rank, local, group):
    """Config 5: 2DGS fwd+bwd train steps, one view per GPU, gradients
    averaged over the GPUs (NCCL) when N > 1."""
    from gs_b200 import _lib, synthetic
    from gs_b200.twod.core.gaussians_2d import Gaussians2D
    from gs_b200.twod.training.trainer import CapturedStep2D, State2D, train_step
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    sc = synthetic.config5(args.seed)
    n = sc["means"].shape[0]
    t = {k: torch.as_tensor(sc[k], device=dev) for k in ("means", "scales", "quaternions", "opacities", "sh_coeffs")}
    st = State2D(Gaussians2D(t["means"], t["scales"], t["quaternions"], t["opacities"], t["sh_coeffs"]))
    cam = (sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"])
    n_cams = len(sc["w2cs"])
    targets_h = [torch.tensor(synthetic.target_image(args.seed + i, sc["H"], sc["W"])).pin_memory() for i in range(4)]
    targets_d = [x.to(dev) for x in targets_h]
    w2cs_h = [torch.tensor(w).pin_memory() for w in sc["w2cs"]]
    w2cs_d = [w.to(dev) for w in w2cs_h]
    cap = 16 * n

    captured = None
    if not args.no_graph:
        v0 = rank % n_cams
        captured = CapturedStep2D(st, targets_d[v0 % 4], w2cs_d[v0], cam, group=group, capacity=cap)

    def step(i, host=False):
        v = (i * world + rank) % n_cams
        tg = targets_h[v % 4] if host else targets_d[v % 4]
        w = w2cs_h[v] if host else w2cs_d[v]
        if captured is not None:
            return captured(tg, w)
        return train_step(st, tg, w, cam, group=group, capacity=cap)

    def barrier():
        if group is not None:
            import torch.distributed as dist
            dist.barrier(group=group)

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    K = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    clocks = ClockSampler(dev)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    for i in range(K):
        flush.zero_()
        ev[i][0].record()
        step(args.warmup + i)
        ev[i][1].record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    tm = torch.tensor([sum(a.elapsed_time(b) for a, b in ev)], dtype=torch.float64, device=dev)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(tm, op=dist.ReduceOp.MAX, group=group)
    value = world * K / (float(tm) / 1000.0)
    barrier()
    torch.cuda.synchronize()
    loss_h = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(2)]
    loss_ev = [torch.cuda.Event() for _ in range(2)]
    t0 = time.perf_counter()
    for i in range(K):
        _, loss, _ = step(args.warmup + K + i, host=True)
        read_loss_lagged(loss, i, loss_h, loss_ev)
    read_loss_lagged(None, K, loss_h, loss_ev)
    torch.cuda.synchronize()
    te = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(te, op=dist.ReduceOp.MAX, group=group)
    e2e = world * K / float(te)
    b = st.buffers(sc["W"], sc["H"], cap)
    _lib.lib().gs_timing_enable(64 * K)
    for i in range(K):  # eager launches: the timing hook sees each kernel
        v = ((args.warmup + 2 * K + i) * world + rank) % n_cams
        train_step(st, targets_d[v % 4], w2cs_d[v], cam, group=group, capacity=cap)
    torch.cuda.synchronize()
    kt = _lib.kernel_times()
    _lib.lib().gs_timing_disable()
    ex = b["extras"].cpu()
    assert int(ex[8]) == 0, "pair capacity overflow"
    # composited pairs: all pairs minus those past the first 512 of a tile
    Mc = float(int(ex[0]) - int(ex[4]))
    Nv = float(((b["valid"] != 0) & (b["radii"] > 0)).sum())
    if rank != 0:
        return
    hbm, src = peaks()
    dom = max(kt.items(), key=lambda x: x[1][0])[0]
    M = float(ex[0])
    P = sc["W"] * sc["H"]
    stats = {"N": n, "Na": n, "K": sc["sh_coeffs"].shape[1], "M": M, "P": P, "Nv": Nv, "Mc": Mc}
    ab = alg_bytes(dom, stats)
    ms_dom = kt[dom][0] / kt[dom][1]
    achieved = ab / (ms_dom * 1e6) if ab else None
    traffic = read_traffic(dom + "_config5")
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = twod_cpu_sample(sc, args.seed)
    print(json.dumps({
        "metric": "2DGS train views/s (fwd+bwd)", "value": value, "unit": "views/s", "n_gpus": world, "steps": K,
        "warmup": max(args.warmup, 3), "ms_per_step": float(tm) / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE config 5 distributions)",
        "config": {"workload": WORKLOAD_2DGS, "surfels": n, "image": [sc["W"], sc["H"]], "pairs_per_view": M,
                   "composited_pairs_per_view": Mc, "visible_upper_bound": Nv,
                   "l2": "flushed between timed steps (256 MiB write, outside the step events)",
                   "parallelism": f"dp{world}",
                   "step_launch": "eager" if captured is None else "cuda graph replay"},
        "clocks": clk,
        "e2e": {"value": e2e, "unit": "views/s", "h2d_bytes_per_step": sc["H"] * sc["W"] * 12 + 64,
                "d2h_bytes_per_step": 4},
        "gpu_launches": sum(c for _, c in kt.values()),
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm if achieved else None, "traffic": traffic,
                     "peak_source": f"{src} hbm_gbs (MEASURED_PEAKS.json)", "alg_bytes_per_launch": ab,
                     "ms_per_launch": ms_dom, **limiter(dom + "_config5", achieved / hbm if achieved else None)},
        "cpu_baseline": cpu,
        "kernels_ms_per_step": {k2: round(v2[0] / K, 4) for k2, v2 in sorted(kt.items(), key=lambda x: -x[1][0])},
    }), flush=True)


def _profile_figure(name, kernel):
    """The number on the line 'kernel value' of profiles/<name>, or None."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        with open(path) as f:
            for ln in f:
                p = ln.split()
                if len(p) >= 2 and p[0] == kernel:
                    return float(p[1])
    except OSError:
        pass
    return None


def read_traffic(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary
    (profiles/dram_traffic.txt, lines 'kernel bytes'), or None."""
    return _profile_figure("dram_traffic.txt", kernel)


def limiter(kernel, frac):
    """What bounds `kernel` when it is far below the HBM roofline: the
    compositors spend their time on per-(splat, pixel) arithmetic on the CUDA
    cores, so their bound is instruction issue, given as smsp__issue_active
    from the committed ncu capture (profiles/issue_active.txt)."""
    ia = _profile_figure("issue_active.txt", kernel)
    if ia is None or (frac is not None and frac > 0.5):
        return {}
    return {"limiter": "instruction issue", "issue_active": ia,
            "issue_source": "ncu smsp__issue_active, profiles/issue_active.txt"}


if __name__ == "__main__":
    main()
