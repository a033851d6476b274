"""Mirror of jax_gs/training/density.py on the libgsb200 density kernels.

DensityState and init_density_state live in trainer.py (flat buffers);
densify_and_prune and reset_opacities update a state in place on the device
(gs_densify_and_prune, gs_reset_opacities) and return it, like the
reference's functional versions return a new state.

Data parallel (train_parallel.py:269-283): densify_and_prune_parallel runs
the density step on rank 0's state alone -- the reference's authoritative
state, unreplicate_tree takes device 0's copy -- with rank 0's own denom
(the ranks' denominators differ: each counts its own views), then copies the
result (parameters, both Adam moments, active mask, accumulators) from rank 0
to every rank, as replicate_tree does. Running the step on every replica
instead would diverge: avg_grad = grad_accum / denom differs per rank.
"""
from __future__ import annotations

from typing import Callable, Optional, Union

import torch

from gs_b200 import _lib
from gs_b200.training.trainer import DensityState, dp_owner, init_density_state  # noqa: F401  (re-export)


def _noise(state: DensityState, rng_key: Union[int, torch.Generator, None]) -> torch.Tensor:
    """Standard normal (N, 3) samples on the state's device: the reference's
    jax.random.normal(rng_key, (N, 3)) (density.py:188), from torch's
    generator (a seed or a torch.Generator)."""
    if isinstance(rng_key, torch.Generator):
        gen = rng_key
    else:
        gen = torch.Generator(device=state.device)
        gen.manual_seed(0 if rng_key is None else int(rng_key))
    return torch.randn((state.n, 3), generator=gen, device=state.device, dtype=torch.float32)


def densify_and_prune(state: DensityState, rng_key: Union[int, torch.Generator, None] = None,
                      densify_enabled: bool = True, grad_threshold: float = 0.0002,
                      min_opacity: float = 0.005, extent: float = 5.0, max_screen_size: int = 512,
                      noise: Optional[torch.Tensor] = None) -> DensityState:
    """density.py:98-211: prune, clone and split in the static capacity.

    `noise` (N, 3) overrides the samples drawn from `rng_key`. After the
    call, state.densify_info is a device int32 tensor [pruned, clones,
    splits, applied]."""
    dev = state.device
    if noise is None:
        noise = _noise(state, rng_key)
    noise = noise.to(device=dev, dtype=torch.float32).contiguous()
    if noise.shape != (state.n, 3):
        raise ValueError(f"noise must have shape ({state.n}, 3)")
    b = state._buffers.setdefault("density", {})
    if "ws" not in b:
        b["ws"] = torch.empty(max(256, _lib.lib().gs_density_workspace_bytes(state.n)), dtype=torch.uint8,
                              device=dev)
        b["info"] = torch.zeros(4, dtype=torch.int32, device=dev)
    P = _lib.ptr
    _lib.call("gs_densify_and_prune", P(state.params), P(state.mu), P(state.nu), state.n, state.sh_k,
              P(state.active_mask.view(torch.uint8)), P(state.grad_accum), P(state.denom), P(state.max_radii),
              P(noise), int(bool(densify_enabled)), float(grad_threshold), float(min_opacity), float(extent),
              float(max_screen_size), P(b["ws"]), b["ws"].numel(), P(b["info"]), _lib.stream(dev))
    state.densify_info = b["info"]
    return state


def reset_opacities(state: DensityState, reset_val: float = 0.01) -> DensityState:
    """density.py:76-96: active opacities to logit(reset_val)."""
    _lib.call("gs_reset_opacities", _lib.ptr(state.params), state.n, _lib.ptr(state.active_mask.view(torch.uint8)),
              float(reset_val), _lib.stream(state.device))
    return state


def gather_moments(state: DensityState, group) -> None:
    """Make every rank's Adam moments whole. Under the fused data-parallel
    update (gs_dp_update) rank r keeps mu / nu current only on the Gaussians
    it owns (dp_owner); every rank zeroes the entries it does not own and a
    sum over the ranks (exact: one nonzero term per entry) leaves every rank
    with the moments optax would hold on each pmap replica."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    foreign = dp_owner(state.n, world, state.device) != rank
    widths = [3, 3, 4, 1, 3 * state.sh_k]
    for (a, b), w in zip(state.segments, widths):
        for buf in (state.mu, state.nu):
            buf[a:b].view(state.n, w)[foreign] = 0.0
    for buf in (state.mu, state.nu):
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)


def update_from_rank0(state: DensityState, group, update: Callable[[DensityState], None],
                      fused: bool = True) -> DensityState:
    """Apply `update` to rank 0's state and copy the result to every rank
    (train_parallel.py:269-283: unreplicate_tree -> density_step /
    opacity_reset_step -> replicate_tree). With fused=True the moments are
    first gathered (gather_moments). Every rank takes the same collective
    steps; only rank 0 runs `update`. Copied from rank 0: params, mu, nu,
    active_mask, grad_accum, denom, max_radii and densify_info."""
    import torch.distributed as dist
    if fused:
        gather_moments(state, group)
    src = dist.get_global_rank(group, 0)
    if dist.get_rank(group) == 0:
        update(state)
    info = getattr(state, "densify_info", None)
    if info is None:
        info = state.densify_info = torch.zeros(4, dtype=torch.int32, device=state.device)
    for t in (state.params, state.mu, state.nu, state.active_mask.view(torch.uint8), state.grad_accum,
              state.denom, state.max_radii, info):
        dist.broadcast(t, src=src, group=group)
    return state


def densify_and_prune_parallel(state: DensityState, group=None, rng_key: Union[int, torch.Generator, None] = None,
                               densify_enabled: bool = True, grad_threshold: float = 0.0002,
                               min_opacity: float = 0.005, extent: float = 5.0, max_screen_size: int = 512,
                               reset_opacity: Optional[float] = None, fused: bool = True,
                               noise: Optional[torch.Tensor] = None) -> DensityState:
    """The density step of train_parallel.py:269-283 for a data-parallel
    state: densify_and_prune (and, when reset_opacity is given,
    reset_opacities to that value, train_parallel.py:276-280) on rank 0's
    state with rank 0's statistics, then the result copied to every rank.
    fused must match the train steps' setting (gs_dp_update keeps sliced Adam
    moments; the NCCL path keeps whole ones). rng_key / noise are used on
    rank 0 only. Returns the state, identical on every rank."""
    import torch.distributed as dist
    if group is None:
        group = dist.group.WORLD

    def update(st: DensityState) -> None:
        densify_and_prune(st, rng_key=rng_key, densify_enabled=densify_enabled, grad_threshold=grad_threshold,
                          min_opacity=min_opacity, extent=extent, max_screen_size=max_screen_size, noise=noise)
        if reset_opacity is not None:
            reset_opacities(st, reset_opacity)

    return update_from_rank0(state, group, update, fused=fused)
