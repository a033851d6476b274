"""ctypes binding of libgsb200.so (the C ABI declared in include/gsb200.h).

Every call passes plain device pointers, sizes and the current CUDA stream;
this module only converts torch tensors to pointers and turns non-zero status
codes into exceptions. There is no fallback: if the library cannot be loaded,
importing the renderer raises.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgsb200.so")

# Status codes (include/gsb200.h).
GS_OK = 0
GS_ERR_INVALID_ARGUMENT = 1
GS_ERR_CAPACITY = 2
GS_ERR_DEVICE_TIMEOUT = 3
GS_ERR_CUDA = 4
GS_ERR_WORKSPACE_TOO_SMALL = 5
GS_ERR_TOO_LARGE = 6

# Every symbol the header declares, with its ctypes signature.
_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_L = ctypes.c_int64
_S = ctypes.c_size_t
_D = ctypes.c_double

class GsAdamSchedule(ctypes.Structure):
    """struct GsAdamSchedule (include/gsb200.h)."""
    _fields_ = [("lr_init", ctypes.c_float * 5), ("decay_rate", ctypes.c_float * 5),
                ("transition_steps", ctypes.c_float * 5), ("b1", ctypes.c_double),
                ("b2", ctypes.c_double), ("eps", ctypes.c_double)]


class GsPeerSet(ctypes.Structure):
    """struct GsPeerSet (include/gsb200.h)."""
    MAX = 8
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32)] + [
        (name, ctypes.c_void_p * 8) for name in
        ("params", "grads", "radii", "valid", "w2c", "grad_accum", "denom", "max_radii", "flags", "touched_in",
         "extras")]


SIGNATURES = {
    "gs_status_string": (ctypes.c_char_p, [_I]),
    "gs_version": (_I, []),
    "gs_default_capacity": (_L, [_I]),
    "gs_workspace_bytes": (_S, [_I, _I, _I, _L]),
    "gs_project_gaussians": (_I, [_P, _P, _P, _I, _P, _P, _I, _I, _F, _F, _F, _F,
                                  _P, _P, _P, _P, _P, _P]),
    "gs_covariance_3d": (_I, [_P, _P, _I, _P, _P]),
    "gs_eval_sh": (_I, [_I, _P, _I, _I, _P, _P, _P]),
    "gs_get_tile_interactions": (_I, [_P, _P, _P, _P, _I, _I, _I, _L, _P, _S,
                                      _P, _P, _P, _P, _P]),
    "gs_render_tiles": (_I, [_P, _P, _P, _P, _I, _P, _P, _L, _I, _I, _P, _P, _S, _P, _P]),
    "gs_render_tiles_backward": (_I, [_P, _P, _P, _P, _I, _P, _P, _L, _I, _I, _P, _P,
                                      _P, _S, _P, _P, _P, _P, _P]),
    "gs_render_forward": (_I, [_P, _P, _P, _P, _P, _I, _I, _P, _P, _I, _I, _F, _F, _F, _F,
                               _P, _I, _L, _P, _S, _P, _P, _P, _P, _P]),
    "gs_render_image": (_I, [_P, _P, _P, _P, _P, _I, _I, _P, _P, _I, _I, _F, _F, _F, _F,
                             _P, _I, _L, _P, _S, _P, _P, _P, _P, _P]),
    "gs_render_backward": (_I, [_P, _P, _P, _P, _P, _I, _I, _P, _P, _I, _I, _F, _F, _F, _F,
                                _P, _I, _L, _P, _S, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "gs_render2d_forward": (_I, [_P, _P, _P, _P, _P, _I, _I, _P, _I, _I, _F, _F, _F, _F, _P, _L, _P, _S,
                                 _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "gs_render2d_workspace_bytes": (_S, [_I, _I, _I, _L]),
    "gs_render2d_backward": (_I, [_P, _P, _P, _P, _P, _I, _I, _P, _I, _I, _F, _F, _F, _F, _L, _P, _S,
                                  _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "gs_2dgs_regularizers": (_I, [_P, _P, _P, _P, _I, _I, _F, _F, _P, _P, _P, _P, _P, _P, _S, _P]),
    "gs_2dgs_regularizers_workspace_bytes": (_S, []),
    "gs_adam_step_flat": (_I, [_P, _P, _P, _P, _L, _F, _I, _D, _D, _D, _P]),
    "gs_adam_step_flat_device": (_I, [_P, _P, _P, _P, _L, _F, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                      _P, _P]),
    "gs_densify_and_prune": (_I, [_P, _P, _P, _I, _I, _P, _P, _P, _P, _P, _I, _F, _F, _F, _F, _P, _S, _P,
                                  _P]),
    "gs_density_workspace_bytes": (_S, [_I]),
    "gs_reset_opacities": (_I, [_P, _I, _P, _F, _P]),
    "gs_l1_dssim_loss": (_I, [_P, _P, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P, _S, _P]),
    "gs_l1_dssim_workspace_bytes": (_S, [_I, _I, _I]),
    "gs_l1_loss": (_I, [_P, _P, _L, _F, _P, _P, _P, _S, _P]),
    "gs_mse_loss": (_I, [_P, _P, _L, _F, _P, _P, _P, _S, _P]),
    "gs_dssim_loss": (_I, [_P, _P, _I, _I, _I, _F, _P, _P, _P, _P, _S, _P]),
    "gs_dssim_workspace_bytes": (_S, [_I, _I, _I]),
    "gs_dssim_loss_noalloc": (_I, [_P, _P, _I, _I, _I, _F, _P, _P, _P, _P]),
    "gs_adam_step": (_I, [_P, _P, _P, _P, _I, _I, _P, _P, _I, _D, _D, _D, _P]),
    "gs_adam_step_scheduled": (_I, [_P, _P, _P, _P, _I, _I, _P, ctypes.POINTER(GsAdamSchedule), _P,
                                    _P]),
    "gs_dp_update": (_I, [ctypes.POINTER(GsPeerSet), _P, _P, _I, _I, _P, ctypes.POINTER(GsAdamSchedule),
                          _P, _F, _F, _I, _I, _I, _P, _P, _P]),
    "gs_dp_barrier": (_I, [ctypes.POINTER(GsPeerSet), _P, _P, _P]),
    "gs_dp_publish_barrier": (_I, [ctypes.POINTER(GsPeerSet), _P, _I, _P, _P, _P]),
    "gs_train_step_metrics": (_I, [_P, _P, _F, _P, _P, _P]),
    "gs_check_extras": (_I, [_P, _P]),
    "gs_test_set_sort_wait": (_I, [_I, _I]),
    "gs_ipc_open": (_I, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "gs_ipc_close": (_I, [_P]),
    "gs_grad2d_magnitude": (_I, [_P, _P, _P, _I, _F, _F, _I, _I, _P, _P]),
    "gs_accumulate_density_stats": (_I, [_P, _P, _P, _P, _P, _I, _P, _P, _P, _P]),
    "gs_density_step_stats": (_I, [_P, _P, _P, _I, _F, _F, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "gs_timing_enable": (_I, [_I]),
    "gs_timing_disable": (_I, []),
    "gs_timing_reset": (_I, []),
    "gs_timing_collect": (_I, []),
    "gs_timing_get": (_I, [_I, ctypes.c_char_p, _I, ctypes.POINTER(ctypes.c_double),
                           ctypes.POINTER(ctypes.c_int)]),
}

# Bytes of scratch gs_l1_loss and gs_mse_loss need (a 64-byte scalar block +
# 296 partials, each region 256-byte aligned).
L1_WORKSPACE_BYTES = 2048


class GsError(RuntimeError):
    """A non-zero status returned by libgsb200."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise ImportError(
            f"libgsb200.so not found at {path}; build it with "
            "`python jax-gs_b200/build_lib.py` (or __graft_entry__.build())")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = load()
    return _lib


def check(fn: str, status: int) -> None:
    if status != GS_OK:
        msg = lib().gs_status_string(status).decode()
        raise GsError(fn, status, msg)


def call(fn: str, *args) -> None:
    check(fn, getattr(lib(), fn)(*args))


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    """Device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("libgsb200 needs CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("libgsb200 needs contiguous tensors")
    return t.data_ptr()


def kernel_times():
    """{kernel name: (total ms, launches)} recorded since gs_timing_enable /
    gs_timing_reset (synchronises on the recorded events)."""
    L = lib()
    n = L.gs_timing_collect()
    if n < 0:
        check("gs_timing_collect", -n)
    out = {}
    buf = ctypes.create_string_buffer(64)
    ms = ctypes.c_double()
    cnt = ctypes.c_int()
    for i in range(n):
        check("gs_timing_get", L.gs_timing_get(i, buf, 64, ctypes.byref(ms), ctypes.byref(cnt)))
        out[buf.value.decode()] = (ms.value, cnt.value)
    return out


def stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
