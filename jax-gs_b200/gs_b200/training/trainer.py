"""Training step on the native kernels: mirror of jax_gs/training/trainer.py
and the static-capacity DensityState of jax_gs/training/density.py:9-61.

One step (trainer.py:55-123 / :125-169) is a fixed sequence of libgsb200
calls on buffers owned by the state:

  gs_render_forward -> gs_l1_dssim_loss (0.8 L1 + 0.2 D-SSIM and the image
  gradient) -> gs_render_backward -> [all-reduce of the flat
  gradient buffer, data parallel only] -> gs_grad2d_magnitude ->
  [all-reduces of grad_2d / radii / visibility] -> gs_adam_step ->
  gs_accumulate_density_stats.

Parameters, Adam moments and gradients live in flat fp32 buffers laid out as
[means (N,3) | scales (N,3) | quaternions (N,4) | opacities (N,1) |
sh_coeffs (N,K,3)] so one NCCL all-reduce averages every gradient leaf (the
pmean of trainer.py:69) and one kernel applies Adam to all groups. The
state is updated in place and returned.
"""
from __future__ import annotations

import ctypes
import dataclasses
from typing import Dict, Optional, Tuple

import torch

from gs_b200 import _lib
from gs_b200._staging import InputStager
from gs_b200.core.gaussians import Gaussians
from gs_b200.renderer.rasterizer import workspace

# Scalars appended to the gradient buffer so that they share its all-reduce:
# [l1, d_ssim, ssim_mean, 8 renderer health counters, the render's device
# timeouts, pad]. The NCCL path copies the counters in (_tail_counters); the
# fused peer-memory update reads them from every rank's GsExtras instead.
TAIL = 16
_METRIC_KEYS = ("n_interactions", "mean_interactions_per_tile", "max_interactions_per_tile",
                "overflow_tiles", "overflow_interactions", "truncated_tiles",
                "truncated_interactions", "radius_cap_violations", "device_timeouts")


@dataclasses.dataclass
class AdamConfig:
    """optax.multi_transform of per-group optax.adam (train.py:129-156)."""
    means_lr_init: float = 0.00016 * 3.0
    means_lr_end: float = 0.0000016 * 3.0
    transition_steps: int = 30000
    scales_lr: float = 0.005
    quaternions_lr: float = 0.001
    opacities_lr: float = 0.05
    sh_lr: float = 0.0025
    b1: float = 0.9
    b2: float = 0.999
    eps: float = 1e-8

    @classmethod
    def from_extent(cls, extent: float, num_iterations: int = 30000) -> "AdamConfig":
        return cls(means_lr_init=0.00016 * extent * 3.0, means_lr_end=0.0000016 * extent * 3.0,
                   transition_steps=num_iterations)

    def lrs(self, count: int):
        """Learning rates of the update whose optax count before increment is
        `count` (optax.exponential_decay for the means)."""
        rate = self.means_lr_end / self.means_lr_init
        m = self.means_lr_init * rate ** (count / self.transition_steps)
        return [m, self.scales_lr, self.quaternions_lr, self.opacities_lr, self.sh_lr]

    def schedule(self) -> "_lib.GsAdamSchedule":
        """The same schedule for the device-evaluated Adam step."""
        sc = _lib.GsAdamSchedule()
        lr = [self.means_lr_init, self.scales_lr, self.quaternions_lr, self.opacities_lr, self.sh_lr]
        for g in range(5):
            sc.lr_init[g] = lr[g]
            sc.decay_rate[g] = 1.0
            sc.transition_steps[g] = 1.0
        sc.decay_rate[0] = self.means_lr_end / self.means_lr_init
        sc.transition_steps[0] = float(self.transition_steps)
        sc.b1, sc.b2, sc.eps = self.b1, self.b2, self.eps
        return sc


DP_STRIPE = 32  # GS_DP_STRIPE (include/gsb200.h)
# From this many ranks on, a rank's gradient rows that are exact zeros (its
# view did not touch the Gaussian) are not read over NVLink: the touched flags
# are published to the owners at the first rendezvous (gs_dp_publish_barrier).
DP_SKIP_MIN_RANKS = 4


def dp_owner(n: int, world: int, device=None) -> torch.Tensor:
    """(n,) int64: the rank that owns each Gaussian's update under the fused
    data-parallel step (gs_dp_update): stripes of DP_STRIPE consecutive
    Gaussians dealt round-robin over the ranks."""
    return (torch.arange(n, device=device) // DP_STRIPE) % world


def _segments(n: int, k: int):
    widths = [3, 3, 4, 1, 3 * k]
    out, off = [], 0
    for w in widths:
        out.append((off, off + w * n))
        off += w * n
    return out, off


class DensityState:
    """Static-capacity training state (density.py:9-17) in flat buffers."""

    def __init__(self, n: int, sh_k: int, device):
        self.n, self.sh_k, self.device = int(n), int(sh_k), torch.device(device)
        self.segments, self.size = _segments(self.n, self.sh_k)
        f = dict(dtype=torch.float32, device=self.device)
        self.params = torch.zeros(self.size, **f)
        self.mu = torch.zeros(self.size, **f)
        self.nu = torch.zeros(self.size, **f)
        self.grads = torch.zeros(self.size + TAIL, **f)
        self.active_mask = torch.zeros(self.n, dtype=torch.bool, device=self.device)
        self.num_active = 0
        self.grad_accum = torch.zeros(self.n, **f)
        self.denom = torch.zeros(self.n, dtype=torch.int32, device=self.device)
        self.max_radii = torch.zeros(self.n, **f)
        self.count = 0  # optax step count (host mirror)
        # device [optax count, ticket] read and advanced by gs_adam_step_scheduled
        self.adam_state = torch.zeros(2, dtype=torch.int32, device=self.device)
        self._buffers: Dict = {}

    def _view(self, buf: torch.Tensor, i: int, shape):
        a, b = self.segments[i]
        return buf[a:b].view(*shape)

    def _fields(self, buf):
        n, k = self.n, self.sh_k
        return Gaussians(means=self._view(buf, 0, (n, 3)), scales=self._view(buf, 1, (n, 3)),
                         quaternions=self._view(buf, 2, (n, 4)),
                         opacities=self._view(buf, 3, (n, 1)),
                         sh_coeffs=self._view(buf, 4, (n, k, 3)))

    @property
    def gaussians(self) -> Gaussians:
        return self._fields(self.params)

    @property
    def grad_fields(self) -> Gaussians:
        return self._fields(self.grads)

    @property
    def tail(self) -> torch.Tensor:
        return self.grads[self.size:]

    def buffers(self, W: int, H: int, capacity: int):
        key = (W, H, capacity)
        b = self._buffers.get(key)
        if b is None:
            d = self.device
            b = {
                "ws": workspace(self.n, W, H, capacity, d),
                "image": torch.empty((H, W, 3), dtype=torch.float32, device=d),
                "grad_image": torch.empty((H, W, 3), dtype=torch.float32, device=d),
                "target": torch.empty((H, W, 3), dtype=torch.float32, device=d),
                "w2c": torch.empty((4, 4), dtype=torch.float32, device=d),
                "radii": torch.empty(self.n, dtype=torch.float32, device=d),
                "valid": torch.empty(self.n, dtype=torch.uint8, device=d),
                # per Gaussian: 0 where this view's gradient row is exact zeros
                # (gs_render_backward), so peers skip reading it
                "touched": torch.empty(self.n, dtype=torch.uint8, device=d),
                "extras": torch.empty(16, dtype=torch.int32, device=d),
                "g2d": torch.empty(self.n, dtype=torch.float32, device=d),
                "loss_ws": torch.empty(max(256, _lib.lib().gs_l1_dssim_workspace_bytes(H, W, 3)),
                                       dtype=torch.uint8, device=d),
                "lrs": (torch.zeros(5, dtype=torch.float32)),
            }
            self._buffers[key] = b
        return b


def init_density_state(gaussians: Gaussians, optimizer: AdamConfig, max_gaussians: int) -> DensityState:
    """Pad to the static capacity (density.py:19-61): padded quaternions are
    identity, everything else zero; active_mask marks the first n_init."""
    del optimizer
    n0 = int(gaussians.means.shape[0])
    k = int(gaussians.sh_coeffs.shape[1])
    st = DensityState(max_gaussians, k, gaussians.means.device)
    g = st.gaussians
    g.means[:n0] = gaussians.means
    g.scales[:n0] = gaussians.scales
    g.quaternions[:n0] = gaussians.quaternions
    g.quaternions[n0:, 0] = 1.0
    g.opacities[:n0] = gaussians.opacities
    g.sh_coeffs[:n0] = gaussians.sh_coeffs
    st.active_mask[:n0] = True
    st.num_active = n0
    return st


def _dev_tensor(x, like: torch.Tensor) -> torch.Tensor:
    """Copy x (host or device) into the preallocated device tensor `like`."""
    like.copy_(torch.as_tensor(x, dtype=torch.float32), non_blocking=True)
    return like


def _step(state: DensityState, target_image, w2c, camera_static, optimizer: AdamConfig,
          sh_degree: int, group, capacity: Optional[int], lambda_ssim: float = 0.2,
          fused: bool = True):
    W, H, fx, fy, cx, cy = camera_static
    W, H = int(W), int(H)
    fx, fy, cx, cy = float(fx), float(fy), float(cx), float(cy)
    dev = state.device
    n, k = state.n, state.sh_k
    cap = int(_lib.lib().gs_default_capacity(n)) if capacity is None else int(capacity)
    b = state.buffers(W, H, cap)
    st = _lib.stream(dev)
    p = state.gaussians
    gf = state.grad_fields
    target = target_image
    if not (isinstance(target, torch.Tensor) and target.is_cuda and target.dtype == torch.float32
            and target.is_contiguous()):
        target = _dev_tensor(target_image, b["target"])  # host -> device (pinned: async)
    w2c_d = w2c
    if group is not None and fused:
        # peers read this rank's camera from its static buffer
        if not (isinstance(w2c, torch.Tensor) and w2c.data_ptr() == b["w2c"].data_ptr()):
            _dev_tensor(w2c, b["w2c"])
        w2c_d = b["w2c"]
    elif not (isinstance(w2c, torch.Tensor) and w2c.is_cuda and w2c.dtype == torch.float32):
        w2c_d = _dev_tensor(w2c, b["w2c"])
    w2c_d = w2c_d.contiguous()
    mask = state.active_mask.view(torch.uint8)
    ws = b["ws"]
    P = _lib.ptr
    # render (trainer.py:21)
    _lib.call("gs_render_forward", P(p.means), P(p.scales), P(p.quaternions), P(p.opacities),
              P(p.sh_coeffs), n, k, P(mask), P(w2c_d), W, H, fx, fy, cx, cy, None, int(sh_degree),
              cap, P(ws), ws.numel(), P(b["image"]), P(b["radii"]), P(b["valid"]), P(b["extras"]), st)
    tail = state.tail
    # loss = 0.8 l1 + 0.2 d_ssim (trainer.py:18-26); gradient w.r.t. the image
    _lib.call("gs_l1_dssim_loss", P(b["image"]), P(target), H, W, 3, lambda_ssim, P(tail[0:1]),
              P(tail[1:2]), P(tail[2:3]), None, P(b["grad_image"]), P(b["loss_ws"]), b["loss_ws"].numel(),
              st)
    # value_and_grad (trainer.py:66/137)
    dp = _peer_set(state, b, group) if (group is not None and fused) else None
    touched = b["touched"] if (dp is not None and dp.skip_untouched) else None
    _lib.call("gs_render_backward", P(p.means), P(p.scales), P(p.quaternions), P(p.opacities),
              P(p.sh_coeffs), n, k, P(mask), P(w2c_d), W, H, fx, fy, cx, cy, None, int(sh_degree),
              cap, P(ws), ws.numel(), P(b["grad_image"]), P(gf.means), P(gf.scales),
              P(gf.quaternions), P(gf.opacities), P(gf.sh_coeffs), None, P(touched), st)
    valid = b["valid"]
    radii = b["radii"]
    radii_valid = valid
    if group is not None and fused:
        # gradient average + Adam + statistics over NVLink peer memory (the
        # update reads every rank's render counters from its extras)
        dp.barrier(touched)  # every rank's gradients (and touched flags) are final
        state.count += 1
        sched = optimizer.schedule()
        # a rendezvous that gave up (dp.status != 0) makes the update touch no
        # peer memory and change nothing; the step's metrics report it
        _lib.call("gs_dp_update", ctypes.byref(dp.peers), P(state.mu), P(state.nu), n, k, P(mask),
                  ctypes.byref(sched), P(state.adam_state), fx, fy, W, H, TAIL, P(dp.tail_out),
                  P(dp.status), st)
        dp.barrier()  # every rank's peer writes are done
        return b
    if group is None:
        # single device: grad_2d_mag (pre-update means) and the densification
        # statistics (trainer.py:143-159) in one kernel, then Adam
        _lib.call("gs_density_step_stats", P(gf.means), P(p.means), P(w2c_d), n, fx, fy, W, H, P(radii), P(valid),
                  P(mask), P(state.grad_accum), P(state.denom), P(state.max_radii), None, st)
        state.count += 1
        sched = optimizer.schedule()
        _lib.call("gs_adam_step_scheduled", P(state.params), P(state.grads), P(state.mu), P(state.nu), n,
                  k, P(mask), ctypes.byref(sched), P(state.adam_state), st)
        return b
    pmean_gradients(state.grads, tail, b["extras"], group)
    # grad_2d_mag from the averaged means gradient and pre-update means
    _lib.call("gs_grad2d_magnitude", P(gf.means), P(p.means), P(w2c_d), n, fx, fy, W, H, P(b["g2d"]), st)
    radii, radii_valid = pmean_grad2d_pmax_radii(b["g2d"], radii, valid, group)
    # Adam + masking + apply (trainer.py:73-77 / 139-141); the schedule is
    # evaluated on the device from state.adam_state so a graph can replay it
    state.count += 1
    sched = optimizer.schedule()
    _lib.call("gs_adam_step_scheduled", P(state.params), P(state.grads), P(state.mu), P(state.nu), n,
              k, P(mask), ctypes.byref(sched), P(state.adam_state), st)
    # densification statistics (trainer.py:100-113 / 152-159)
    # denom counts this rank's own visibility; max_radii uses the max over ranks
    _lib.call("gs_accumulate_density_stats", P(b["g2d"]), P(radii), P(valid), P(radii_valid), P(mask),
              n, P(state.grad_accum), P(state.denom), P(state.max_radii), st)
    return b


def pmean_gradients(grads: torch.Tensor, tail: torch.Tensor, extras: torch.Tensor, group) -> None:
    """trainer.py:69-71: average every gradient leaf, the loss and the
    metrics over the data-parallel group, in one all-reduce of the flat
    gradient buffer whose tail carries [l1, d_ssim, ssim, 8 health counters,
    device timeouts]."""
    _tail_counters(tail, extras)
    _all_reduce_mean(grads, group)


def _tail_counters(tail: torch.Tensor, extras: torch.Tensor) -> None:
    """tail[3:11] = the eight health counters of GsExtras as floats (the
    second one is a float field), tail[11] = its device_timeouts."""
    tail[3:11] = extras[0:8].to(torch.float32)
    tail[4] = extras[1:2].view(torch.float32)[0]
    tail[11] = extras[10].to(torch.float32)


def pmean_grad2d_pmax_radii(g2d: torch.Tensor, radii: torch.Tensor, valid: torch.Tensor, group):
    """trainer.py:97 and :108-111: average grad_2d_mag in place; return the
    max over ranks of the valid-masked radii and of the visibility (u8)."""
    import torch.distributed as dist
    _all_reduce_mean(g2d, group)
    rv = torch.stack([torch.where(valid.bool(), radii, torch.zeros((), device=radii.device)),
                      valid.to(torch.float32)])
    dist.all_reduce(rv, op=dist.ReduceOp.MAX, group=group)
    return rv[0].contiguous(), (rv[1] > 0).to(torch.uint8).contiguous()


def _all_reduce_mean(t: torch.Tensor, group) -> None:
    import torch.distributed as dist
    if dist.get_backend(group) == "nccl":
        dist.all_reduce(t, op=dist.ReduceOp.AVG, group=group)
    else:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
        t.div_(dist.get_world_size(group))


class PeerSet:
    """Every rank's training buffers mapped into this process (CUDA IPC), for
    gs_dp_update: parameters, gradients, the view's radii / valid mask / W2C
    and the densification statistics. Built once per state and image size."""

    FIELDS = ("params", "grads", "radii", "valid", "w2c", "grad_accum", "denom", "max_radii", "flags",
              "touched_in", "extras")

    def __init__(self, state: DensityState, b: Dict, group, skip_untouched: Optional[bool] = None):
        import torch.distributed as dist
        self.group = group
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        if world > _lib.GsPeerSet.MAX:
            raise ValueError(f"gs_dp_update supports at most {_lib.GsPeerSet.MAX} ranks")
        dev = state.device
        # rendezvous words (gs_dp_barrier): zeroed before any peer can see them
        self.flags = torch.zeros(_lib.GsPeerSet.MAX, dtype=torch.int32, device=dev)
        self.epoch = torch.zeros(2, dtype=torch.int32, device=dev)  # [epoch, ticket]
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        if skip_untouched is None:
            skip_untouched = world >= DP_SKIP_MIN_RANKS
        self.n = state.n
        local = {"params": state.params, "grads": state.grads, "radii": b["radii"], "valid": b["valid"],
                 "w2c": b["w2c"], "grad_accum": state.grad_accum, "denom": state.denom,
                 "max_radii": state.max_radii, "flags": self.flags, "extras": b["extras"]}
        if skip_untouched:
            # inbox of touched flags: row q = rank q's flags (for this rank's stripes)
            local["touched_in"] = torch.zeros(world * state.n, dtype=torch.uint8, device=dev)
        torch.cuda.synchronize(dev)
        info = {"uuid": str(torch.cuda.get_device_properties(dev).uuid)}
        for key, t in local.items():
            st = t.untyped_storage()
            shared = st._share_cuda_()
            handle, off = _raw_ipc_handle(bytes(shared[1])), int(shared[3])
            info[key] = (handle, off + t.storage_offset() * t.element_size())
        everyone = [None] * world
        dist.all_gather_object(everyone, info, group=group)
        # the peer-memory rendezvous spins on flags another rank writes: only
        # with one rank per GPU (else the one-element NCCL all-reduce)
        self.device_barrier = len({e["uuid"] for e in everyone}) == world
        # the flags travel with the peer-memory rendezvous only
        self.skip_untouched = bool(skip_untouched) and self.device_barrier
        self._bases = {}
        self.peers = _lib.GsPeerSet()
        self.peers.world, self.peers.rank = world, rank
        for r in range(world):
            for key in self.FIELDS:
                if key not in local or (key == "touched_in" and not self.skip_untouched):
                    continue  # NULL: every gradient row is read
                if r == rank:
                    ptr = local[key].data_ptr()
                else:
                    handle, off = everyone[r][key]
                    ptr = self._open(handle) + off
                getattr(self.peers, key)[r] = ptr
        self.local = local  # keep the exported tensors alive
        self.tail_out = torch.zeros(TAIL, dtype=torch.float32, device=state.device)
        self.flag = torch.zeros(1, dtype=torch.float32, device=state.device)

    def _open(self, handle: bytes) -> int:
        base = self._bases.get(handle)
        if base is None:
            out = ctypes.c_void_p()
            _lib.check("gs_ipc_open", _lib.lib().gs_ipc_open(handle, ctypes.byref(out)))
            base = self._bases[handle] = out.value
        return base

    def barrier(self, touched: Optional[torch.Tensor] = None):
        """Stream-ordered rendezvous: gs_dp_barrier over peer memory (a
        bounded wait; timeouts counted in self.status), or a one-element
        all-reduce on the stream when ranks share a GPU. With `touched` (this
        view's flags from gs_render_backward) and the skip on, the flags are
        first published to their owners (gs_dp_publish_barrier)."""
        if self.device_barrier:
            st = _lib.stream(self.flags.device)
            if touched is not None and self.skip_untouched:
                _lib.call("gs_dp_publish_barrier", ctypes.byref(self.peers), _lib.ptr(touched), self.n,
                          _lib.ptr(self.epoch), _lib.ptr(self.status), st)
                return
            _lib.call("gs_dp_barrier", ctypes.byref(self.peers), _lib.ptr(self.epoch), _lib.ptr(self.status), st)
            return
        import torch.distributed as dist
        dist.all_reduce(self.flag, group=self.group)

    def timeouts(self) -> int:
        """Rendezvous waits of this rank that expired (0 in a healthy run)."""
        return int(self.status.item())

    def close(self):
        for base in self._bases.values():
            _lib.lib().gs_ipc_close(base)
        self._bases = {}


def _raw_ipc_handle(h: bytes) -> bytes:
    """The 64-byte cudaIpcMemHandle_t inside torch's shareable handle, which
    torch writes as [format version][type 'c' = cudaMalloc segment][handle]."""
    if len(h) == 64:
        return h
    if len(h) == 66 and h[1:2] == b"c":
        return h[2:]
    raise RuntimeError("tensor memory cannot be shared through cudaIpc (expandable segments?); "
                       "use the NCCL path (fused=False)")


def _peer_set(state: DensityState, b: Dict, group) -> PeerSet:
    key = ("peers", b["ws"].data_ptr())
    dp = state._buffers.get(key)
    if dp is None:
        dp = state._buffers[key] = PeerSet(state, b, group)
    return dp


def train_step(state: DensityState, target_image, w2c, camera_static, optimizer: AdamConfig,
               fast_tpu_rasterizer: bool = False, sh_degree: int = 0,
               capacity: Optional[int] = None) -> Tuple[DensityState, torch.Tensor, Dict]:
    """Single-device step (trainer.py:125-169). Returns (state, loss, metrics);
    loss and metrics are device tensors (no synchronisation)."""
    del fast_tpu_rasterizer
    b = _step(state, target_image, w2c, camera_static, optimizer, sh_degree, None, capacity)
    return state, *_loss_metrics(state, b, None, True)


def train_step_internal(state: DensityState, target_image, w2c, camera_static,
                        optimizer: AdamConfig, fast_tpu_rasterizer: bool = False,
                        sh_degree: int = 0, group=None, capacity: Optional[int] = None,
                        fused: bool = True) -> Tuple[DensityState, torch.Tensor, Dict]:
    """Data-parallel step (trainer.py:55-123): each rank renders its own view;
    gradients, loss and metrics are averaged over `group` (torch.distributed,
    NCCL on GPUs), grad_2d is averaged again and radii / visibility are
    max-reduced before the statistics update."""
    del fast_tpu_rasterizer
    import torch.distributed as dist
    if group is None and dist.is_available() and dist.is_initialized():
        group = dist.group.WORLD
    if group is not None and dist.get_world_size(group) == 1:
        group = None
    b = _step(state, target_image, w2c, camera_static, optimizer, sh_degree, group, capacity,
              fused=fused)
    return state, *_loss_metrics(state, b, group, fused)


def _loss_metrics(state: DensityState, b: Dict, group, fused: bool):
    """(loss, metrics) of the step as views of one device vector filled by a
    single small kernel (gs_train_step_metrics): loss, l1, ssim, the
    health counters (this rank's, or averaged over the group) and
    device_timeouts (nonzero: the step's results are not valid;
    check_step raises)."""
    out = b.get("metrics_out")
    if out is None:
        out = b["metrics_out"] = torch.zeros(3 + len(_METRIC_KEYS), dtype=torch.float32, device=state.device)
    status = None
    if group is None:
        tail, ex = state.tail, b["extras"]
    elif fused:
        # tail_out: the tail averaged over the ranks by gs_dp_update (so a
        # render timeout on any rank shows); status: this rank's rendezvous
        # word (nonzero: the update was skipped)
        dp = _peer_set(state, b, group)
        tail, ex, status = dp.tail_out, None, dp.status
    else:
        tail, ex = state.tail, None
    _lib.call("gs_train_step_metrics", _lib.ptr(tail), _lib.ptr(ex), 0.2, _lib.ptr(status), _lib.ptr(out),
              _lib.stream(state.device))
    m = {"l1": out[1], "ssim": out[2]}
    for i, key in enumerate(_METRIC_KEYS):
        m[key] = out[3 + i]
    return out[0], m


def check_step(metrics: Dict[str, torch.Tensor]) -> None:
    """Raise GsError(GS_ERR_DEVICE_TIMEOUT) if a bounded device wait of the
    step gave up (the sort's look-back, or a data-parallel rendezvous, in
    which case the update touched no peer memory and changed nothing).
    Reads one device scalar (synchronises): call it where the loss is read
    back anyway."""
    if float(metrics["device_timeouts"]) != 0.0:
        _lib.check("train_step", _lib.GS_ERR_DEVICE_TIMEOUT)


class CapturedStep:
    """One training step captured in a CUDA graph and replayed.

    The step (train_step, or train_step_internal when `group` is given) is
    recorded once with static input buffers; __call__ copies the view's target
    image and W2C into them (host or device tensors) and replays the graph:
    one launch for the ~25 kernels and memsets of a step. The state is
    updated in place exactly as by the eager step (the Adam schedule lives on
    the device). One eager step runs first (priming the library's per-device
    launch configuration and the workspaces), so construction trains one step.
    """

    def __init__(self, state: DensityState, target_image, w2c, camera_static,
                 optimizer: AdamConfig, sh_degree: int = 0, group=None,
                 capacity: Optional[int] = None, fused: bool = True):
        self.state = state
        if group is not None:
            import torch.distributed as dist
            if dist.get_world_size(group) == 1:
                group = None
        W, H = int(camera_static[0]), int(camera_static[1])
        cap = int(_lib.lib().gs_default_capacity(state.n)) if capacity is None else int(capacity)
        b = state.buffers(W, H, cap)
        self.target, self.w2c = b["target"], b["w2c"]
        self.target.copy_(torch.as_tensor(target_image, dtype=torch.float32), non_blocking=True)
        self.w2c.copy_(torch.as_tensor(w2c, dtype=torch.float32), non_blocking=True)
        _step(state, self.target, self.w2c, camera_static, optimizer, sh_degree, group, capacity,
              fused=fused)
        torch.cuda.synchronize(state.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            _step(state, self.target, self.w2c, camera_static, optimizer, sh_degree, group, capacity,
                  fused=fused)
            self.loss, self.metrics = _loss_metrics(state, b, group, fused)
        self.state.count -= 1  # the capture did not run the step
        self._stager = InputStager(state.device)  # host inputs upload during the previous step

    def __call__(self, target_image, w2c):
        self._stager.upload([torch.as_tensor(target_image, dtype=torch.float32),
                             torch.as_tensor(w2c, dtype=torch.float32)], [self.target, self.w2c])
        self.graph.replay()
        self.state.count += 1
        return self.state, self.loss, self.metrics

