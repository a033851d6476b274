"""Mirror of jax_gs/training/density.py on the libgsb200 density kernels.

DensityState and init_density_state live in trainer.py (flat buffers);
densify_and_prune and reset_opacities update a state in place on the device
(gs_densify_and_prune, gs_reset_opacities) and return it, like the
reference's functional versions return a new state.

Data parallel: every replica runs densify_and_prune with the same rng_key;
the kernels are deterministic, so the replicas stay identical without the
reference's broadcast from the authoritative state (train_parallel.py:269-283).
"""
from __future__ import annotations

from typing import Optional, Union

import torch

from gs_b200 import _lib
from gs_b200.training.trainer import DensityState, init_density_state  # noqa: F401  (re-export)


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
