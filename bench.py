#!/usr/bin/env python
"""Benchmark: data-parallel 3DGS training step on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]
  torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU, NCCL)

Default workload: a step is one view per GPU -- render forward, L1 + D-SSIM
loss, render backward, the gradient average over the GPUs (pmean), the
densification statistics and the masked multi-group Adam update
(trainer.py:55-123 on the native kernels). At N = 1 the line also carries,
under "north_star", the config 3 render throughput and the 1M-Gaussian
1080p train step time, each device-timed with its own clock record.
Other workloads: config1 (single-view fwd+bwd), render
(config 3), train-large (the north-star 1080p step), densify (config 4),
2dgs (config 5). Prints ONE JSON line on rank 0.

The reference arm (--impl reference) times the reference's algorithm on the
host cores (the CPU restatement under oracle/, since JAX is not installable
here) on the same workload, with the same `config` keys and W warm-up
samples.
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
HBM_FALLBACK = 6650.0
L2_NOTE = "flushed between timed steps (256 MiB write, outside the step events)"
DENSIFY_EVERY = 100
RENDER_VIEWS = 8  # config 3: views per GPU per step
REFERENCE_BUDGET_S = 120.0  # timed CPU samples of the reference arm stop after this much time

WORKLOADS = {
    "train": ("BASELINE config 2: data-parallel train step, one view per GPU; 100k active Gaussians in "
              "a 200k static capacity, SH degree 3, 504x378, 20 cameras on a 30 deg arc at r=4; "
              "0.8 L1 + 0.2 D-SSIM, masked multi-group Adam, pmean over GPUs"),
    "config1": ("BASELINE config 1: single-view fwd+bwd, 10,000 Gaussians (x,y uniform in [-1,1], z in [2,6]), "
                "SH degree 0, 504x378, fx=fy=400, L1 loss against a uniform [0,1] target; image plus every "
                "per-Gaussian gradient"),
    "render": ("BASELINE config 3: render-only, 1M Gaussians (uniform in a 10^3 box), SH degree 3, "
               "1920x1080, fx=fy=1200, 64 views on a sphere of radius 12, 8 views per GPU per step"),
    "train-large": ("north-star train step: the config 3 scene (1M Gaussians, all active, SH degree 3) at "
                    "1920x1080, one of 64 sphere views per GPU per step, targets uniform [0,1]; 0.8 L1 + 0.2 "
                    "D-SSIM, masked multi-group Adam, pmean over GPUs"),
    "densify": ("BASELINE config 4: 4M capacity, 3M active (8 Gaussian blobs, sigma 1.5, in a 20^3 box), "
                "SH degree 3, 1600x1064, 200 orbit cameras at r=15, one view per GPU per step; "
                "densify_and_prune (grad threshold 2e-4) every 100 steps on rank 0's state, copied to every "
                "rank, its time amortised"),
    "2dgs": ("BASELINE config 5: 2DGS train step (render fwd with RGB, depth, depth^2, normal and 1 - T maps; "
             "0.8 L1 + 0.2 D-SSIM + 1e-4 distortion + 1e-4 normal consistency; bwd; Adam 1e-3), 500k surfels "
             "uniform in a 6^3 box, log-scales N(-3.5, 0.5), SH degree 3 (DC used), 1264x832, one of 20 sphere "
             "views per GPU per step"),
}
METRICS = {"train": (METRIC, UNIT), "config1": ("fwd+bwd views/s", UNIT), "render": ("render Mpix/s", "Mpix/s"),
           "train-large": (METRIC, UNIT), "densify": (METRIC, UNIT),
           "2dgs": ("2DGS train views/s (fwd+bwd)", UNIT)}


def static_config(workload: str, world: int) -> dict:
    """The `config` object of a workload: its fixed description, printed
    identically by both arms (measured figures go under "details")."""
    shapes = {"train": dict(gaussians_capacity=200_000, gaussians_active=100_000, image=[504, 378],
                            views_per_gpu_per_step=1),
              "config1": dict(gaussians_capacity=10_000, gaussians_active=10_000, image=[504, 378],
                              views_per_gpu_per_step=1),
              "render": dict(gaussians_capacity=1_000_000, gaussians_active=1_000_000, image=[1920, 1080],
                             views_per_gpu_per_step=RENDER_VIEWS),
              "train-large": dict(gaussians_capacity=1_000_000, gaussians_active=1_000_000, image=[1920, 1080],
                                  views_per_gpu_per_step=1),
              "densify": dict(gaussians_capacity=4_000_000, gaussians_active=3_000_000, image=[1600, 1064],
                              views_per_gpu_per_step=1, densify_every=DENSIFY_EVERY),
              "2dgs": dict(gaussians_capacity=500_000, gaussians_active=500_000, image=[1264, 832],
                           views_per_gpu_per_step=1)}[workload]
    par = f"replicas x{world}" if workload in ("render", "config1") else f"dp{world}"
    return {"workload": WORKLOADS[workload], **shapes, "l2": L2_NOTE, "parallelism": par}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=list(WORKLOADS), default="train",
                    help="train: config 2 train step (default); config1: config 1 single-view fwd+bwd; "
                         "render: config 3 render-only Mpix/s; train-large: the same train step on the config 3 "
                         "scene (1M Gaussians, SH3, 1920x1080); densify: config 4 (4M capacity, 3M active, "
                         "1600x1064) with densify_and_prune every 100 steps amortised; 2dgs: config 5 surfel "
                         "train step (500k surfels, 1264x832)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-north-star", action="store_true",
                    help="default workload: skip the config 3 render and 1080p train-step figures")
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


def _oracle_params(scene):
    return {"means": torch.tensor(scene.means), "scales": torch.tensor(scene.scales),
            "quaternions": torch.tensor(scene.quats), "opacities": torch.tensor(scene.opacities),
            "sh_coeffs": torch.tensor(scene.sh)}


def sample_config2(scene, seed):
    """One oracle train step of config 2 view 0 on the host cores (torch CPU,
    literal N*256-slot sort). Returns (views, seconds, description)."""
    from gs_b200 import synthetic
    from oracle import ref_restated as R
    torch.set_num_threads(os.cpu_count() or 1)
    params = _oracle_params(scene)
    zeros = {k: torch.zeros_like(v) for k, v in params.items()}
    tgt = torch.tensor(synthetic.target_image(seed, scene.H, scene.W))
    lrs = dict(zip(R.GROUPS, [1e-4, 0.005, 0.001, 0.05, 0.0025]))
    t0 = time.perf_counter()
    R.train_step(params, zeros, dict(zeros), 1, lrs, torch.tensor(scene.active), tgt,
                 torch.tensor(scene.w2cs[0]), scene.camera_static(), sh_degree=scene.sh_degree,
                 compact_sort=False)
    return 1.0, time.perf_counter() - t0, ("oracle train step of config 2 view 0 (literal N*256-slot sort, "
                                          "torch-CPU autograd, L1+D-SSIM, Adam)")


def sample_config1(scene, seed):
    """Oracle render fwd + L1 loss + backward of config 1 (every per-Gaussian
    gradient) on the host cores. Returns (views, seconds, description)."""
    from gs_b200 import synthetic
    from oracle import ref_restated as R
    torch.set_num_threads(os.cpu_count() or 1)
    p = {k: v.requires_grad_(True) for k, v in _oracle_params(scene).items()}
    tgt = torch.tensor(synthetic.target_image(seed, scene.H, scene.W))
    t0 = time.perf_counter()
    img, _ = R.render(p["means"], p["scales"], p["quaternions"], p["opacities"], p["sh_coeffs"],
                      torch.tensor(scene.w2cs[0]), scene.W, scene.H, scene.fx, scene.fy, scene.cx, scene.cy,
                      mask=torch.tensor(scene.active), sh_degree=scene.sh_degree, compact_sort=False)
    R.l1_loss(img, tgt).backward()
    return 1.0, time.perf_counter() - t0, ("oracle render + L1 loss + backward of config 1 (literal N*256-slot "
                                          "sort, torch-CPU autograd)")


LARGE_SAMPLE_TILES = 960  # about 1/8 of the tiles of a 1080p view (the central band)


def _central_tiles(W, H, n_tiles):
    tx, ty = (W + 15) // 16, (H + 15) // 16
    rows = max(1, n_tiles // tx)
    r0 = (ty - rows) // 2
    return list(range(r0 * tx, (r0 + rows) * tx)), tx * ty


def sample_large(scene, seed, cfg_id):
    """Oracle train step (torch-CPU autograd, L1 + D-SSIM, Adam) of view 0
    with only the central band of about LARGE_SAMPLE_TILES tiles composited
    (projection, SH, sort, loss and Adam on everything). Returns (views
    scaled by the tile share, seconds, description). densify_and_prune
    (every 100 steps) is not in the sample."""
    from gs_b200 import synthetic
    from oracle import ref_restated as R
    torch.set_num_threads(os.cpu_count() or 1)
    params = _oracle_params(scene)
    zeros = {k: torch.zeros_like(v) for k, v in params.items()}
    tgt = torch.tensor(synthetic.target_image(seed, scene.H, scene.W))
    lrs = dict(zip(R.GROUPS, [1e-4, 0.005, 0.001, 0.05, 0.0025]))
    subset, total = _central_tiles(scene.W, scene.H, LARGE_SAMPLE_TILES)
    t0 = time.perf_counter()
    R.train_step(params, zeros, dict(zeros), 1, lrs, torch.tensor(scene.active), tgt, torch.tensor(scene.w2cs[0]),
                 scene.camera_static(), sh_degree=scene.sh_degree, compact_sort=True, tile_subset=subset)
    dt = time.perf_counter() - t0
    return len(subset) / total, dt, (f"oracle train step of config {cfg_id} view 0 with the central {len(subset)} "
                                     f"of {total} tiles composited (projection, SH, sort, loss, Adam on all "
                                     "Gaussians; densify_and_prune not sampled), scaled by the tile share")


RENDER_SAMPLE_TILES = 1020  # 1/8 of the 8160 tiles of a 1920x1080 view (the central band)


def sample_render(scene, view=0):
    """Oracle render of one config-3 view restricted to the central 1/8 of
    its tiles (projection, SH and the full sort still run for all 1M
    Gaussians). Returns (Mpix composited, seconds, description)."""
    from oracle import ref_restated as R
    torch.set_num_threads(os.cpu_count() or 1)
    subset, total = _central_tiles(scene.W, scene.H, RENDER_SAMPLE_TILES)
    t = lambda a: torch.tensor(a)  # noqa: E731
    t0 = time.perf_counter()
    with torch.no_grad():
        R.render(t(scene.means), t(scene.scales), t(scene.quats), t(scene.opacities), t(scene.sh),
                 t(scene.w2cs[view]), scene.W, scene.H, scene.fx, scene.fy, scene.cx, scene.cy,
                 sh_degree=scene.sh_degree, tile_subset=subset)
    return len(subset) * 256 / 1e6, time.perf_counter() - t0, (
        f"oracle render of a config 3 view, central {len(subset)} of {total} tiles composited (projection, SH, "
        "sort of all 1M Gaussians)")


TWOD_SAMPLE_TILES = 632  # 8 of the 52 tile rows of a 1264x832 view (the central band)


def sample_2dgs(sc, seed):
    """Oracle 2DGS train loss fwd+bwd of config 5 view 0 with only the
    central TWOD_SAMPLE_TILES tiles composited (projection, sort, losses and
    their backward run on the full view). Returns (views scaled by the tile
    share, seconds, description)."""
    from gs_b200 import synthetic
    from oracle import ref_restated_2d as R2
    torch.set_num_threads(os.cpu_count() or 1)
    p = {k: torch.tensor(sc[k]).requires_grad_(True)
         for k in ("means", "scales", "quaternions", "opacities", "sh_coeffs")}
    tgt = torch.tensor(synthetic.target_image(seed, sc["H"], sc["W"]))
    subset, total = _central_tiles(sc["W"], sc["H"], TWOD_SAMPLE_TILES)
    t0 = time.perf_counter()
    loss, _ = R2.train_loss_2d(p, tgt, torch.tensor(sc["w2cs"][0]), sc["W"], sc["H"], sc["fx"], sc["fy"],
                               sc["cx"], sc["cy"], tile_subset=subset)
    loss.backward()
    return len(subset) / total, time.perf_counter() - t0, (
        f"oracle 2DGS train loss fwd+bwd (torch-CPU autograd) of config 5 view 0 with the central {len(subset)} "
        f"of {total} tiles composited, scaled by the tile share")


def cpu_sampler(workload, seed):
    """(sample function, description prefix) of the reference's algorithm on
    the host cores for `workload`; the function returns (units, seconds,
    description) for one bounded sample."""
    from gs_b200 import synthetic
    if workload == "config1":
        scene = synthetic.config1(seed)
        return lambda i: sample_config1(scene, seed)
    if workload == "render":
        scene = synthetic.config3(seed)
        return lambda i: sample_render(scene, i % len(scene.w2cs))
    if workload == "2dgs":
        sc = synthetic.config5(seed)
        return lambda i: sample_2dgs(sc, seed)
    if workload in ("train-large", "densify"):
        dens = workload == "densify"
        scene = (synthetic.config4 if dens else synthetic.config3)(seed)
        return lambda i: sample_large(scene, seed, 4 if dens else 3)
    scene = synthetic.config2(seed)
    return lambda i: sample_config2(scene, seed)


def cpu_baseline(workload, seed):
    """The GPU arm's cpu_baseline object: one bounded sample of the
    reference's algorithm on the host cores (rank 0, N = 1)."""
    u, s, desc = cpu_sampler(workload, seed)(0)
    return {"value": u / s, "unit": METRICS[workload][1], "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"1 x {desc}; {s:.1f} s"}


def run_reference(args, world, rank):
    """Reference arm: the reference's algorithm on the host CPU (the torch-CPU
    restatement in oracle/, since JAX is not installable here), rank 0 only:
    W warm-up samples, then up to K timed samples (stopping once
    REFERENCE_BUDGET_S of them have run)."""
    if rank != 0:
        return
    sample = cpu_sampler(args.workload, args.seed)
    for i in range(args.warmup):
        sample(i)
    units = secs = 0.0
    steps, desc = 0, ""
    while steps < max(1, args.steps) and (steps == 0 or secs < REFERENCE_BUDGET_S):
        u, s, desc = sample(args.warmup + steps)
        units, secs, steps = units + u, secs + s, steps + 1
    v = units / secs
    metric, unit = METRICS[args.workload]
    cores = torch.get_num_threads()
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": v, "unit": unit, "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * secs / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; the GPU arm's inputs)",
        "config": static_config(args.workload, world),
        "cpu_baseline": {"value": v, "unit": unit, "cores": cores, "kind": "port",
                         "sample": f"{steps} x {desc}, torch-CPU restatement, {cores} threads; "
                                   "JAX reference not installable"},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def timed_region(run_step, K, dev, group=None, first=0):
    """K steps run_step(first + i), each bracketed by CUDA events on the
    current stream with an L2 flush (256 MiB write) before it, outside the
    events; barrier + synchronize on both sides; SM clocks sampled
    throughout. Returns (total ms, max over ranks; clock record)."""
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    clocks = ClockSampler(dev)
    clocks.start()
    if group is not None:
        import torch.distributed as dist
        dist.barrier(group=group)
    torch.cuda.synchronize()
    for i in range(K):
        flush.zero_()
        ev[i][0].record()
        run_step(first + i)
        ev[i][1].record()
    torch.cuda.synchronize()
    if group is not None:
        import torch.distributed as dist
        dist.barrier(group=group)
    clk = clocks.stop()
    tm = torch.tensor([sum(a.elapsed_time(b) for a, b in ev)], dtype=torch.float64, device=dev)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(tm, op=dist.ReduceOp.MAX, group=group)
    return float(tm), clk


def max_over_ranks(x, dev, group):
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t)


def roofline(kt, st, kernel_suffix=""):
    """The roofline object of the kernel with the largest device time:
    achieved = its algorithmic bytes (alg_bytes) / mean launch time, against
    the measured HBM copy rate; traffic from the committed ncu summary."""
    hbm, src = peaks()
    dom = max(kt.items(), key=lambda x: x[1][0])[0]
    per_ms = kt[dom][0] / kt[dom][1]
    b = alg_bytes(dom, st)
    achieved = (b / (per_ms / 1000.0)) / 1e9 if b else None
    frac = (achieved / hbm) if achieved else None
    roof = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": frac,
            "traffic": read_traffic(dom + kernel_suffix),
            "peak_source": f"{src} hbm_gbs (MEASURED_PEAKS.json)" if src == "measured" else "fallback",
            "alg_bytes_per_launch": b, "ms_per_launch": per_ms}
    roof.update(limiter(dom + kernel_suffix, frac))
    roof.update(l2_figures(dom + kernel_suffix))
    return roof


def kernel_table(kt, K):
    return {k: round(v[0] / K, 4) for k, v in sorted(kt.items(), key=lambda x: -x[1][0])}


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
        # NCCL's communicator set-up is logged (ranks, devices, transports), so
        # that a reader of the run's output sees every rank join
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        group = dist.group.WORLD
    run = {"render": run_render, "2dgs": run_2dgs, "config1": run_config1}.get(args.workload, run_train)
    run(args, world, rank, local, group)
    if group is not None:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


class TrainRun:
    """A training workload on one rank: the state, its cameras and targets
    (device and pinned host copies), and the step (a CUDA graph replay of
    the whole step unless no_graph)."""

    def __init__(self, scene, dev, seed, world, rank, group, fused=True, no_graph=False, large=False):
        from gs_b200 import synthetic
        from gs_b200.training.trainer import CapturedStep
        self.scene, self.dev, self.world, self.rank, self.group, self.fused = scene, dev, world, rank, group, fused
        self.state, self.opt = build_state(scene, dev)
        self.n_cams = len(scene.w2cs)
        self.n_tgt = 8 if large else self.n_cams  # 1080p targets: 8 distinct images, cycled
        # pair capacity: 16 per Gaussian at 1080p (about 12 are used; checked after the run)
        self.cap = 16 * scene.n if large else None
        self.targets_h = [torch.tensor(synthetic.target_image(seed + i, scene.H, scene.W)).pin_memory()
                          for i in range(self.n_tgt)]
        self.w2cs_h = [torch.tensor(w).pin_memory() for w in scene.w2cs]
        self.targets_d = [t.to(dev) for t in self.targets_h]
        self.w2cs_d = [w.to(dev) for w in self.w2cs_h]
        self.cam = scene.camera_static()
        self.captured = None
        if not no_graph:
            # the whole step (NCCL all-reduces included when N > 1) as one
            # CUDA graph; its construction trains one step
            v0 = rank % self.n_cams
            self.captured = CapturedStep(self.state, self.targets_d[v0 % self.n_tgt], self.w2cs_d[v0], self.cam,
                                         self.opt, sh_degree=scene.sh_degree, group=group, fused=fused,
                                         capacity=self.cap)

    def view(self, i):
        return (i * self.world + self.rank) % self.n_cams

    def step(self, i, host=False):
        from gs_b200.training.trainer import train_step_internal
        v = self.view(i)
        tgt = (self.targets_h if host else self.targets_d)[v % self.n_tgt]
        w2c = (self.w2cs_h if host else self.w2cs_d)[v]
        if self.captured is not None:
            return self.captured(tgt, w2c)
        return train_step_internal(self.state, tgt, w2c, self.cam, self.opt, sh_degree=self.scene.sh_degree,
                                   group=self.group, fused=self.fused, capacity=self.cap)

    def eager_step(self, i):
        from gs_b200.training.trainer import train_step_internal
        v = self.view(i)
        return train_step_internal(self.state, self.targets_d[v % self.n_tgt], self.w2cs_d[v], self.cam, self.opt,
                                   sh_degree=self.scene.sh_degree, group=self.group, fused=self.fused,
                                   capacity=self.cap)

    def close(self):
        # a graph holding NCCL calls must be released before the process group
        self.captured = None
        torch.cuda.synchronize()
        for v in self.state._buffers.values():
            if hasattr(v, "close"):
                v.close()


def run_train(args, world, rank, local, group):
    """Configs 2 (default), 4 (densify) and the north-star 1080p step
    (train-large): device-timed steps, the same steps end to end through the
    public API, per-kernel times, roofline and CPU baseline."""
    from gs_b200 import _lib, synthetic
    from gs_b200.training.trainer import check_step
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dens = args.workload == "densify"
    large = args.workload in ("train-large", "densify")
    cfg_id = 4 if dens else 3 if large else 2
    scene = {2: synthetic.config2, 3: synthetic.config3, 4: synthetic.config4}[cfg_id](args.seed)
    tr = TrainRun(scene, dev, args.seed, world, rank, group, fused=not args.no_fused, no_graph=args.no_graph,
                  large=large)
    W0 = max(args.warmup, 3)
    for i in range(W0):
        tr.step(i)
    torch.cuda.synchronize()
    if args.profile:
        for i in range(args.profile):
            tr.step(W0 + i)
        torch.cuda.synchronize()
        if rank == 0:
            print(f"profile: {args.profile} train steps done", flush=True)
        tr.close()
        return
    K = args.steps
    # ---- device-timed region (inputs resident in HBM; L2 flushed between steps)
    last = {}

    def timed_step(i):
        last["m"] = tr.step(i)[2]

    ms_total, clk = timed_region(timed_step, K, dev, group, first=W0)
    check_step(last["m"])  # no bounded device wait gave up in the timed steps
    value = world * K / (ms_total / 1000.0)

    # ---- end to end through the public API: pinned host inputs, loss read back
    if group is not None:
        import torch.distributed as dist
        dist.barrier(group=group)
    torch.cuda.synchronize()
    loss_h = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(2)]
    loss_ev = [torch.cuda.Event() for _ in range(2)]
    t0 = time.perf_counter()
    for i in range(K):
        _, loss, _ = tr.step(W0 + K + i, host=True)
        read_loss_lagged(loss, i, loss_h, loss_ev)
    read_loss_lagged(None, K, loss_h, loss_ev)
    torch.cuda.synchronize()
    te = max_over_ranks(time.perf_counter() - t0, dev, group)
    e2e_value = world * K / te
    h2d = scene.H * scene.W * 3 * 4 + 16 * 4
    d2h = 4

    details = {"step_launch": "cuda graph replay" if tr.captured is not None else "eager",
               "dp_update": ("n/a" if world == 1 else "nccl all-reduce" if args.no_fused
                             else "fused peer-memory kernel")}
    if dens:
        details.update(densify_amortised(args, tr, scene, dev, group, world, K))
        step_ms, e2e_step_ms, d_ms = ms_total / K, 1000.0 * te / K, details["densify_ms"]
        value = world * DENSIFY_EVERY / ((DENSIFY_EVERY * step_ms + d_ms) / 1000.0)
        e2e_value = world * DENSIFY_EVERY / ((DENSIFY_EVERY * e2e_step_ms + d_ms) / 1000.0)

    # ---- per-kernel device time (CUDA events around every library launch)
    _lib.lib().gs_timing_enable(64 * K)
    torch.cuda.synchronize()
    for i in range(K):
        tr.eager_step(W0 + 3 * K + i)
    torch.cuda.synchronize()
    kt = _lib.kernel_times()
    if tr.cap is not None:
        assert int(tr.state.buffers(scene.W, scene.H, tr.cap)["extras"][8]) == 0, "pair capacity overflow"
    _lib.lib().gs_timing_disable()
    launches = sum(c for _, c in kt.values())

    north = None
    if rank == 0 and world == 1 and args.workload == "train" and not args.no_north_star:
        north = north_star_figures(args, dev)
    out = None
    if rank == 0:
        M, Nv = view_stats(tr.state, scene, dev, tr.cap)
        st = {"N": scene.n, "Na": int(scene.active.sum()), "K": 16, "M": M, "P": scene.W * scene.H, "Nv": Nv}
        details.update(pairs_per_view=M, visible_per_view=Nv)
        roof = roofline(kt, st, "_config%d" % cfg_id if large else "")
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(args.workload, args.seed)
        out = {
            "metric": METRICS[args.workload][0], "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": W0, "ms_per_step": ms_total / K, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE config %d distributions)" % cfg_id,
            "config": static_config(args.workload, world), "details": details,
            "clocks": clk,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches, "roofline": roof, "cpu_baseline": cpu,
            "device_timeouts": int(float(last["m"]["device_timeouts"])),
            "kernels_ms_per_step": kernel_table(kt, K),
        }
        if north is not None:
            out["north_star"] = north
        print(json.dumps(out), flush=True)
    tr.close()


def densify_amortised(args, tr, scene, dev, group, world, K):
    """densify_and_prune (density.py:98-211) on the statistics the steps above
    accumulated, device time of each call (two calls, a few steps apart);
    with N > 1 the data-parallel version (rank 0's state, copied to every
    rank, train_parallel.py:269-283)."""
    from gs_b200.training.density import densify_and_prune, densify_and_prune_parallel
    extent = float(np.max(np.linalg.norm(scene.means[scene.active] - scene.means[scene.active].mean(0), axis=1)))
    dms = []
    info = None
    for j in range(2):
        if group is not None:
            import torch.distributed as dist
            dist.barrier(group=group)
        torch.cuda.synchronize()
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        if group is None:
            densify_and_prune(tr.state, rng_key=args.seed + j, grad_threshold=0.0002, extent=extent)
        else:
            densify_and_prune_parallel(tr.state, group, rng_key=args.seed + j, grad_threshold=0.0002,
                                       extent=extent, fused=not args.no_fused)
        b_.record()
        torch.cuda.synchronize()
        dms.append(a.elapsed_time(b_))
        info = [int(x) for x in tr.state.densify_info.cpu()]
        for i in range(5):  # a few steps in between, so the second call has statistics
            tr.step(args.warmup + 2 * K + i)
        torch.cuda.synchronize()
    d_ms = max_over_ranks(max(dms), dev, group)
    return {"densify_every": DENSIFY_EVERY, "densify_ms": d_ms,
            "densify_on": "rank 0, copied to every rank" if world > 1 else "the one rank",
            "densify_last": dict(zip(("pruned", "clones", "splits", "applied"), info)), "extent": extent}


def north_star_figures(args, dev):
    """The north star's other headline numbers, device-timed on this GPU
    after the main line's run: config 3 render throughput (8 views per step
    over the render streams, CUDA graph replay) and the 1M-Gaussian SH3
    1920x1080 train step (target < 5 ms), each with its own clock record.
    No CPU sample here (the render and train-large workloads carry one)."""
    from gs_b200 import synthetic
    from gs_b200.training.trainer import check_step
    K = max(3, min(args.steps, 10))
    scene = synthetic.config3(args.seed)
    out = {"steps": K, "warmup": max(args.warmup, 3), "l2": L2_NOTE,
           "cpu_baseline": "not sampled in this line (bench.py --workload render / train-large carry theirs)"}
    rs = RenderSetup(scene, dev, max(1, min(args.render_streams, RENDER_VIEWS)), 1, 0)
    for i in range(max(args.warmup, 3)):
        rs.set_views(i)
        rs.forward_views()
    torch.cuda.synchronize()
    rs.capture()

    def render_step(i):
        rs.set_views(i)
        rs.graph.replay()

    ms, clk = timed_region(render_step, K, dev)
    rs.check()
    out["render_config3"] = {"value": scene.W * scene.H * RENDER_VIEWS * K / (ms / 1000.0) / 1e6,
                             "unit": "Mpix/s", "ms_per_step": ms / K, "views_per_step": RENDER_VIEWS,
                             "workload": WORKLOADS["render"], "clocks": clk}
    rs.close()
    del rs
    tr = TrainRun(scene, dev, args.seed, 1, 0, None, large=True)
    for i in range(max(args.warmup, 3)):
        tr.step(i)
    torch.cuda.synchronize()
    last = {}

    def train_step_(i):
        last["m"] = tr.step(i)[2]

    ms, clk = timed_region(train_step_, K, dev, first=max(args.warmup, 3))
    check_step(last["m"])
    assert int(tr.state.buffers(scene.W, scene.H, tr.cap)["extras"][8]) == 0, "pair capacity overflow"
    out["train_1080p"] = {"ms_per_step": ms / K, "target_ms": 5.0, "value": K / (ms / 1000.0), "unit": UNIT,
                          "workload": WORKLOADS["train-large"], "clocks": clk}
    tr.close()
    return out


class RenderSetup:
    """Config 3 render step on one GPU: RENDER_VIEWS views per step issued
    round-robin on S streams, each with its own workspace, so that one
    view's pair sort overlaps another view's compositing."""

    def __init__(self, scene, dev, S, world, rank):
        from gs_b200 import _lib
        self.scene, self.dev, self.S, self.world, self.rank = scene, dev, S, world, rank
        n, W, H = scene.n, scene.W, scene.H
        tt = lambda a: torch.as_tensor(a, device=dev).contiguous()  # noqa: E731
        self.means, self.scales, self.quats, self.opac, self.sh = (tt(scene.means), tt(scene.scales),
                                                                   tt(scene.quats), tt(scene.opacities),
                                                                   tt(scene.sh))
        self.w2cs_h = [torch.tensor(w).pin_memory() for w in scene.w2cs]
        self.w2cs_d = torch.stack([w.to(dev) for w in self.w2cs_h])
        self.cap = 16 * n  # pairs per view; overflow is checked
        lib = _lib.lib()
        self.wss = [torch.empty(lib.gs_workspace_bytes(n, W, H, self.cap), dtype=torch.uint8, device=dev)
                    for _ in range(S)]
        self.images = torch.empty((RENDER_VIEWS, H, W, 3), dtype=torch.float32, device=dev)
        self.radii = [torch.empty(n, dtype=torch.float32, device=dev) for _ in range(S)]
        self.valid = [torch.empty(n, dtype=torch.uint8, device=dev) for _ in range(S)]
        self.extras = torch.zeros((RENDER_VIEWS, 16), dtype=torch.int32, device=dev)
        self.views_d = torch.zeros(RENDER_VIEWS, 4, 4, dtype=torch.float32, device=dev)
        self.side = [torch.cuda.Stream(dev) for _ in range(S - 1)]
        self.graph = None

    def forward_views(self):
        from gs_b200 import _lib
        P, sc = _lib.ptr, self.scene
        main = torch.cuda.current_stream(self.dev)
        for s2 in self.side:
            s2.wait_stream(main)
        for i in range(RENDER_VIEWS):
            j = i % self.S
            st = main.cuda_stream if j == 0 else self.side[j - 1].cuda_stream
            ws = self.wss[j]
            _lib.call("gs_render_image", P(self.means), P(self.scales), P(self.quats), P(self.opac), P(self.sh),
                      sc.n, 16, None, P(self.views_d[i]), sc.W, sc.H, sc.fx, sc.fy, sc.cx, sc.cy, None,
                      sc.sh_degree, self.cap, P(ws), ws.numel(), P(self.images[i]), P(self.radii[j]),
                      P(self.valid[j]), P(self.extras[i]), st)
        for s2 in self.side:
            main.wait_stream(s2)

    def set_views(self, step):
        base = (step * self.world + self.rank) * RENDER_VIEWS
        n = len(self.scene.w2cs)
        self.views_d.copy_(self.w2cs_d[[(base + i) % n for i in range(RENDER_VIEWS)]])

    def capture(self):
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.forward_views()

    def check(self):
        ex = self.extras.cpu()
        assert int(ex[:, 8].max()) == 0, "pair capacity overflow"
        assert int(ex[:, 10].max()) == 0, "a bounded device wait gave up"

    def close(self):
        self.graph = None
        torch.cuda.synchronize()


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
    W, H, V = scene.W, scene.H, RENDER_VIEWS
    S = max(1, min(args.render_streams, V))
    rs = RenderSetup(scene, dev, S, world, rank)
    W0 = max(args.warmup, 3)
    for i in range(W0):
        rs.set_views(i)
        rs.forward_views()
    torch.cuda.synchronize()
    rs.check()
    rs.capture()
    K = args.steps

    def step(i):
        rs.set_views(i)
        rs.graph.replay()

    ms, clk = timed_region(step, K, dev, group)
    pix = W * H * V * world * K
    value = pix / (ms / 1000.0) / 1e6
    rs.check()
    M = float(rs.extras[:, 0].float().mean())
    # end to end through the public render(): W2C from pinned host memory,
    # image copied back to pinned host memory, every view; the views are
    # issued round-robin on the same S streams (render() takes its scratch
    # from the stream-aware allocator, so concurrent calls do not share it),
    # so one view's copies overlap other views' kernels
    g = Gaussians(means=rs.means, scales=rs.scales, quaternions=rs.quats, opacities=rs.opac, sh_coeffs=rs.sh)
    e2e_streams = [torch.cuda.current_stream(dev)] + rs.side
    host_imgs = [torch.empty((H, W, 3), dtype=torch.float32).pin_memory() for _ in range(S)]

    def api_views(i):
        base = (i * world + rank) * V
        for j in range(V):
            with torch.cuda.stream(e2e_streams[j % S]):
                w = rs.w2cs_h[(base + j) % len(scene.w2cs)]
                cam = Camera(W, H, scene.fx, scene.fy, scene.cx, scene.cy, w.to(dev, non_blocking=True), None)
                img, _ = render(g, cam, sh_degree=scene.sh_degree, capacity=rs.cap)
                host_imgs[j % S].copy_(img, non_blocking=True)

    with torch.no_grad():
        api_views(0)  # the API path's own warm-up (allocator)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(K):
            api_views(i)
        torch.cuda.synchronize()
    e2e = pix / max_over_ranks(time.perf_counter() - t0, dev, group) / 1e6
    # per-kernel device time of the same work (eager, timing hook)
    lib = _lib.lib()
    lib.gs_timing_enable(64 * K * V)
    for i in range(K):
        rs.set_views(i)
        rs.forward_views()
    torch.cuda.synchronize()
    kt = _lib.kernel_times()
    lib.gs_timing_disable()
    rs.close()
    if rank != 0:
        return
    st = {"N": scene.n, "Na": scene.n, "K": 16, "M": M, "P": W * H, "Nv": scene.n}
    cpu = cpu_baseline("render", args.seed) if world == 1 and not args.no_cpu_baseline else None
    print(json.dumps({
        "metric": METRICS["render"][0], "value": value, "unit": "Mpix/s", "n_gpus": world, "steps": K,
        "warmup": W0, "ms_per_step": ms / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE config 3)",
        "config": static_config("render", world),
        "details": {"pairs_per_view": M, "capacity_per_view": rs.cap, "step_launch": "cuda graph replay",
                    "streams_per_gpu": S},
        "clocks": clk,
        "e2e": {"value": e2e, "unit": "Mpix/s", "h2d_bytes_per_step": 64 * V,
                "d2h_bytes_per_step": W * H * 3 * 4 * V},
        "gpu_launches": sum(c for _, c in kt.values()),
        "roofline": roofline(kt, st, "_config3"),
        "cpu_baseline": cpu,
        "kernels_ms_per_step": kernel_table(kt, K),
    }), flush=True)


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

    W0 = max(args.warmup, 3)
    for i in range(W0):
        step(i)
    torch.cuda.synchronize()
    K = args.steps
    ms, clk = timed_region(step, K, dev, group, first=W0)
    value = world * K / (ms / 1000.0)
    if group is not None:
        import torch.distributed as dist
        dist.barrier(group=group)
    torch.cuda.synchronize()
    loss_h = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(2)]
    loss_ev = [torch.cuda.Event() for _ in range(2)]
    t0 = time.perf_counter()
    for i in range(K):
        _, loss, _ = step(W0 + K + i, host=True)
        read_loss_lagged(loss, i, loss_h, loss_ev)
    read_loss_lagged(None, K, loss_h, loss_ev)
    torch.cuda.synchronize()
    e2e = world * K / max_over_ranks(time.perf_counter() - t0, dev, group)
    b = st.buffers(sc["W"], sc["H"], cap)
    _lib.lib().gs_timing_enable(64 * K)
    for i in range(K):  # eager launches: the timing hook sees each kernel
        v = ((W0 + 2 * K + i) * world + rank) % n_cams
        train_step(st, targets_d[v % 4], w2cs_d[v], cam, group=group, capacity=cap)
    torch.cuda.synchronize()
    kt = _lib.kernel_times()
    _lib.lib().gs_timing_disable()
    ex = b["extras"].cpu()
    assert int(ex[8]) == 0, "pair capacity overflow"
    assert int(ex[10]) == 0, "a bounded device wait gave up"
    # composited pairs: all pairs minus those past the first 512 of a tile
    Mc = float(int(ex[0]) - int(ex[4]))
    Nv = float(((b["valid"] != 0) & (b["radii"] > 0)).sum())
    del captured
    if rank != 0:
        return
    M = float(ex[0])
    stats = {"N": n, "Na": n, "K": sc["sh_coeffs"].shape[1], "M": M, "P": sc["W"] * sc["H"], "Nv": Nv, "Mc": Mc}
    cpu = cpu_baseline("2dgs", args.seed) if world == 1 and not args.no_cpu_baseline else None
    print(json.dumps({
        "metric": METRICS["2dgs"][0], "value": value, "unit": "views/s", "n_gpus": world, "steps": K,
        "warmup": W0, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE config 5 distributions)",
        "config": static_config("2dgs", world),
        "details": {"pairs_per_view": M, "composited_pairs_per_view": Mc, "visible_upper_bound": Nv,
                    "step_launch": "eager" if args.no_graph else "cuda graph replay"},
        "clocks": clk,
        "e2e": {"value": e2e, "unit": "views/s", "h2d_bytes_per_step": sc["H"] * sc["W"] * 12 + 64,
                "d2h_bytes_per_step": 4},
        "gpu_launches": sum(c for _, c in kt.values()),
        "roofline": roofline(kt, stats, "_config5"),
        "cpu_baseline": cpu,
        "kernels_ms_per_step": kernel_table(kt, K),
    }), flush=True)


def run_config1(args, world, rank, local, group):
    """Config 1: single-view forward + L1 loss + backward (the image and every
    per-Gaussian gradient), no optimizer. Device-timed: gs_render_forward,
    gs_l1_loss, gs_render_backward replayed as one CUDA graph. End to end:
    render() + l1_loss + backward through the torch mirror, the target copied
    from pinned host memory and the loss read back every step. N > 1: each
    GPU runs its own replica (no exchange)."""
    from gs_b200 import _lib, synthetic
    from gs_b200.core.camera import Camera
    from gs_b200.core.gaussians import Gaussians
    from gs_b200.renderer.rasterizer import workspace
    from gs_b200.renderer.renderer import render
    from gs_b200.training.losses import l1_loss
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    scene = synthetic.config1(args.seed)
    n, W, H, k = scene.n, scene.W, scene.H, scene.sh.shape[1]
    tt = lambda a: torch.as_tensor(a, device=dev).contiguous()  # noqa: E731
    means, scales, quats, opac, sh = (tt(scene.means), tt(scene.scales), tt(scene.quats), tt(scene.opacities),
                                      tt(scene.sh))
    w2c = tt(scene.w2cs[0])
    target_h = torch.tensor(synthetic.target_image(args.seed, H, W)).pin_memory()
    target = target_h.to(dev)
    cap = int(_lib.lib().gs_default_capacity(n))
    ws = workspace(n, W, H, cap, dev)
    image = torch.empty((H, W, 3), dtype=torch.float32, device=dev)
    gimg = torch.empty_like(image)
    radii = torch.empty(n, dtype=torch.float32, device=dev)
    valid = torch.empty(n, dtype=torch.uint8, device=dev)
    ex = torch.zeros(16, dtype=torch.int32, device=dev)
    loss = torch.zeros((), dtype=torch.float32, device=dev)
    lws = torch.empty(_lib.L1_WORKSPACE_BYTES, dtype=torch.uint8, device=dev)
    grads = [torch.empty_like(x) for x in (means, scales, quats, opac, sh)]
    P = _lib.ptr

    def kernels():
        st = _lib.stream(dev)
        cam = (W, H, scene.fx, scene.fy, scene.cx, scene.cy)
        _lib.call("gs_render_forward", P(means), P(scales), P(quats), P(opac), P(sh), n, k, None, P(w2c),
                  *cam, None, scene.sh_degree, cap, P(ws), ws.numel(), P(image), P(radii), P(valid), P(ex), st)
        _lib.call("gs_l1_loss", P(image), P(target), image.numel(), 1.0, P(loss), P(gimg), P(lws), lws.numel(), st)
        _lib.call("gs_render_backward", P(means), P(scales), P(quats), P(opac), P(sh), n, k, None, P(w2c),
                  *cam, None, scene.sh_degree, cap, P(ws), ws.numel(), P(gimg), *[P(g) for g in grads], None, None,
                  st)

    W0 = max(args.warmup, 3)
    for _ in range(W0):
        kernels()
    torch.cuda.synchronize()
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            kernels()
    K = args.steps
    ms, clk = timed_region(lambda i: graph.replay() if graph is not None else kernels(), K, dev, group)
    assert int(ex[10]) == 0 and int(ex[8]) == 0, "invalid render (device timeout or capacity overflow)"
    value = world * K / (ms / 1000.0)
    # end to end through the public API
    params = [x.clone().requires_grad_(True) for x in (means, scales, quats, opac, sh)]
    g = Gaussians(*params)
    camera = Camera(W, H, scene.fx, scene.fy, scene.cx, scene.cy, w2c, None)
    tgt_d = torch.empty_like(target)
    loss_h = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(2)]
    loss_ev = [torch.cuda.Event() for _ in range(2)]

    def api_step():
        for p in params:
            p.grad = None
        tgt_d.copy_(target_h, non_blocking=True)
        img, _ = render(g, camera, sh_degree=scene.sh_degree)
        lv = l1_loss(img, tgt_d)
        lv.backward()
        return lv.detach()

    for _ in range(W0):  # the API path's own warm-up (allocator, autograd)
        api_step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(K):
        read_loss_lagged(api_step(), i, loss_h, loss_ev)
    read_loss_lagged(None, K, loss_h, loss_ev)
    torch.cuda.synchronize()
    e2e = world * K / max_over_ranks(time.perf_counter() - t0, dev, group)
    lib = _lib.lib()
    lib.gs_timing_enable(64 * K)
    for _ in range(K):
        kernels()
    torch.cuda.synchronize()
    kt = _lib.kernel_times()
    lib.gs_timing_disable()
    launch = "cuda graph replay" if graph is not None else "eager"
    del graph
    if rank != 0:
        return

    class _View:
        gaussians = Gaussians(means, scales, quats, opac, sh)
        active_mask = torch.ones(n, dtype=torch.bool, device=dev)

    M, Nv = view_stats(_View, scene, dev)
    st = {"N": n, "Na": n, "K": k, "M": M, "P": W * H, "Nv": Nv}
    cpu = cpu_baseline("config1", args.seed) if world == 1 and not args.no_cpu_baseline else None
    print(json.dumps({
        "metric": METRICS["config1"][0], "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W0,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; BASELINE config 1 distributions)",
        "config": static_config("config1", world),
        "details": {"pairs_per_view": M, "visible_per_view": Nv,
                    "step_launch": launch},
        "clocks": clk,
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": H * W * 3 * 4, "d2h_bytes_per_step": 4},
        "gpu_launches": sum(c for _, c in kt.values()),
        "roofline": roofline(kt, st, "_config1"),
        "cpu_baseline": cpu,
        "kernels_ms_per_step": kernel_table(kt, K),
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


def l2_figures(kernel):
    """L2 traffic of `kernel` from the committed one-kernel ncu captures
    (profiles/l2_traffic.txt, lines 'kernel lts_bytes_per_launch
    l2_throughput_pct shared_pipe_pct'), or {}."""
    path = os.path.join(ROOT, "profiles", "l2_traffic.txt")
    try:
        with open(path) as f:
            for ln in f:
                p = ln.split()
                if len(p) >= 4 and p[0] == kernel:
                    return {"l2_bytes_per_launch": float(p[1]), "l2_throughput_pct": float(p[2]),
                            "shared_pipe_pct": float(p[3]), "l2_source": "ncu, profiles/l2_traffic.txt"}
    except OSError:
        pass
    return {}


if __name__ == "__main__":
    main()
