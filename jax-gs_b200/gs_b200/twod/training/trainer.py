"""Mirror of jax_2dgs/training/trainer.py: one 2DGS training step on the
native kernels.

loss = (1 - 0.2) L1 + 0.2 D-SSIM + 1e-4 distortion + 1e-4 normal consistency
(trainer.py:24-48), gradients by gs_render2d_backward, then optax.adam over
every parameter (gs_adam_step_flat; the reference passes an optax optimizer,
tests/test_benchmark_3dgs_vs_2dgs.py:58 uses adam(1e-3)). Data parallel: the
gradient buffer is averaged over `group` before the update (trainer.py:56-57).
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from gs_b200 import _lib
from gs_b200._staging import InputStager
from gs_b200.twod.core.gaussians_2d import Gaussians2D
from gs_b200.twod.renderer.renderer import workspace2d

LAMBDA_SSIM, LAMBDA_DIST, LAMBDA_NORMAL = 0.2, 1e-4, 1e-4
TAIL = 4  # l1, d_ssim, distortion, normal (ride the gradient average)


class State2D:
    """Parameters and Adam moments in flat float32 buffers
    [means | scales | quaternions | opacities | sh]."""

    def __init__(self, g: Gaussians2D, lr: float = 1e-3, b1: float = 0.9, b2: float = 0.999, eps: float = 1e-8):
        dev = g.means.device
        self.n, self.sh_k, self.device = int(g.means.shape[0]), int(g.sh_coeffs.shape[1]), dev
        self.widths = (3, 2, 4, 1, 3 * self.sh_k)
        self.size = self.n * sum(self.widths)
        f = dict(dtype=torch.float32, device=dev)
        self.params = torch.cat([t.reshape(-1).to(torch.float32) for t in
                                 (g.means, g.scales, g.quaternions, g.opacities, g.sh_coeffs)]).contiguous()
        self.mu = torch.zeros(self.size, **f)
        self.nu = torch.zeros(self.size, **f)
        self.grads = torch.zeros(self.size + TAIL, **f)
        self.lr, self.b1, self.b2, self.eps = lr, b1, b2, eps
        self.count = 0
        # optax count on the device [count, ticket], so a captured step replays
        self.adam_state = torch.zeros(2, dtype=torch.int32, device=dev)
        self._buffers: Dict = {}
        self.stager = InputStager(dev)  # host inputs upload during the previous step

    def _fields(self, buf) -> Gaussians2D:
        out, off = [], 0
        shapes = ((3,), (2,), (4,), (1,), (self.sh_k, 3))
        for w, shp in zip(self.widths, shapes):
            out.append(buf[off:off + self.n * w].view(self.n, *shp))
            off += self.n * w
        return Gaussians2D(*out)

    @property
    def gaussians(self) -> Gaussians2D:
        return self._fields(self.params)

    @property
    def grad_fields(self) -> Gaussians2D:
        return self._fields(self.grads)

    def buffers(self, W: int, H: int, capacity: int):
        key = (W, H, capacity)
        if key not in self._buffers:
            d = self.device
            f = dict(dtype=torch.float32, device=d)
            self._buffers[key] = {
                "ws": workspace2d(self.n, W, H, capacity, d),
                "image": torch.empty((H, W, 3), **f), "depth": torch.empty((H, W, 1), **f),
                "depth_sq": torch.empty((H, W, 1), **f), "normals": torch.empty((H, W, 3), **f),
                "accum": torch.empty((H, W, 1), **f), "g_image": torch.empty((H, W, 3), **f),
                "g_depth": torch.empty((H, W, 1), **f), "g_depth_sq": torch.empty((H, W, 1), **f),
                "g_normals": torch.empty((H, W, 3), **f),
                "target": torch.empty((H, W, 3), **f), "w2c": torch.empty((4, 4), **f),
                "radii": torch.empty(self.n, **f), "valid": torch.empty(self.n, dtype=torch.uint8, device=d),
                "extras": torch.empty(16, dtype=torch.int32, device=d),
                "loss_ws": torch.empty(max(256, _lib.lib().gs_l1_dssim_workspace_bytes(H, W, 3)),
                                       dtype=torch.uint8, device=d),
                "reg_ws": torch.empty(max(256, _lib.lib().gs_2dgs_regularizers_workspace_bytes()),
                                      dtype=torch.uint8, device=d),
            }
        return self._buffers[key]


def train_step(state: State2D, target_image: torch.Tensor, w2c: torch.Tensor, camera_static,
               group=None, capacity: Optional[int] = None) -> Tuple[State2D, torch.Tensor, Dict]:
    """trainer.py (jax_2dgs):8-62 (train_step_internal; the pmean when group is set)."""
    W, H, fx, fy, cx, cy = camera_static
    W, H = int(W), int(H)
    fx, fy, cx, cy = float(fx), float(fy), float(cx), float(cy)
    dev = state.device
    n, k = state.n, state.sh_k
    cap = int(_lib.lib().gs_default_capacity(n)) if capacity is None else int(capacity)
    b = state.buffers(W, H, cap)
    st = _lib.stream(dev)
    P = _lib.ptr
    g = state.gaussians
    gf = state.grad_fields
    tail = state.grads[state.size:]
    target, w2c_d = b["target"], b["w2c"]
    state.stager.upload([torch.as_tensor(target_image, dtype=torch.float32),
                         torch.as_tensor(w2c, dtype=torch.float32)], [target, w2c_d])
    _lib.call("gs_render2d_forward", P(g.means), P(g.scales), P(g.quaternions), P(g.opacities), P(g.sh_coeffs), n,
              k, P(w2c_d), W, H, fx, fy, cx, cy, None, cap, P(b["ws"]), b["ws"].numel(), P(b["image"]),
              P(b["depth"]), P(b["depth_sq"]), P(b["normals"]), P(b["accum"]), P(b["radii"]), P(b["valid"]),
              P(b["extras"]), st)
    _lib.call("gs_l1_dssim_loss", P(b["image"]), P(target), H, W, 3, LAMBDA_SSIM, P(tail[0:1]), P(tail[1:2]), None,
              None, P(b["g_image"]), P(b["loss_ws"]), b["loss_ws"].numel(), st)
    _lib.call("gs_2dgs_regularizers", P(b["depth"]), P(b["depth_sq"]), P(b["normals"]), P(b["accum"]), H, W,
              LAMBDA_DIST, LAMBDA_NORMAL, P(tail[2:3]), P(tail[3:4]), P(b["g_depth"]), P(b["g_depth_sq"]),
              P(b["g_normals"]), P(b["reg_ws"]), b["reg_ws"].numel(), st)
    _lib.call("gs_render2d_backward", P(g.means), P(g.scales), P(g.quaternions), P(g.opacities), P(g.sh_coeffs),
              n, k, P(w2c_d), W, H, fx, fy, cx, cy, cap, P(b["ws"]), b["ws"].numel(), P(b["image"]), P(b["depth"]),
              P(b["depth_sq"]), P(b["normals"]), P(b["accum"]), P(b["g_image"]), P(b["g_depth"]),
              P(b["g_depth_sq"]), P(b["g_normals"]), None, P(gf.means), P(gf.scales), P(gf.quaternions),
              P(gf.opacities), P(gf.sh_coeffs), st)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(state.grads, op=dist.ReduceOp.AVG, group=group)
    state.count += 1
    _lib.call("gs_adam_step_flat_device", P(state.params), P(state.grads), P(state.mu), P(state.nu), state.size,
              state.lr, state.b1, state.b2, state.eps, P(state.adam_state), st)
    loss = (1.0 - LAMBDA_SSIM) * tail[0] + LAMBDA_SSIM * tail[1] + LAMBDA_DIST * tail[2] + LAMBDA_NORMAL * tail[3]
    metrics = {"l1": tail[0], "ssim": 1.0 - tail[1] * 2.0, "dist_loss": tail[2], "normal_loss": tail[3]}
    return state, loss, metrics


def train_step_internal(state: State2D, target_image: torch.Tensor, w2c: torch.Tensor, camera_static,
                        optimizer=None, group=None) -> Tuple[State2D, torch.Tensor, Dict]:
    """trainer.py (jax_2dgs):10-66 under its own name. The optimizer argument
    is accepted for signature parity and not used: the Adam hyperparameters
    live in State2D (the reference passes optax.adam(1e-3), :70)."""
    del optimizer
    return train_step(state, target_image, w2c, camera_static, group=group)


class CapturedStep2D:
    """One 2DGS training step captured in a CUDA graph and replayed (the
    3DGS trainer's CapturedStep for jax_2dgs): one eager step primes the
    workspaces (so construction trains one step), then the step is recorded
    with the state's static target / W2C buffers; __call__ uploads the view
    (host inputs during the previous step) and replays."""

    def __init__(self, state: State2D, target_image, w2c, camera_static, group=None,
                 capacity: Optional[int] = None):
        self.state = state
        W, H = int(camera_static[0]), int(camera_static[1])
        cap = int(_lib.lib().gs_default_capacity(state.n)) if capacity is None else int(capacity)
        b = state.buffers(W, H, cap)
        self.target, self.w2c = b["target"], b["w2c"]
        train_step(state, target_image, w2c, camera_static, group=group, capacity=capacity)
        torch.cuda.synchronize(state.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            _, self.loss, self.metrics = train_step(state, self.target, self.w2c, camera_static, group=group,
                                                    capacity=capacity)
        state.count -= 1  # the capture did not run the step

    def __call__(self, target_image, w2c):
        self.state.stager.upload([torch.as_tensor(target_image, dtype=torch.float32),
                                  torch.as_tensor(w2c, dtype=torch.float32)], [self.target, self.w2c])
        self.graph.replay()
        self.state.count += 1
        return self.state, self.loss, self.metrics
