"""render() of jax_gs/renderer/renderer.py:15-107 on libgsb200.so through
XLA's typed FFI (gs_xla_ffi.cc), for jax-gs itself: same signature, same
return value (image (H,W,3), the extras dict of renderer.py:79-90), and
differentiable through a jax.custom_vjp whose forward and backward are one
ffi_call each. The FFI calls have static output shapes (the pair capacity is
an attribute), so render() composes with jit, lax.scan (train.py:101) and
pmap (train_parallel.py:26); vmap over views runs the calls one after the
other (vmap_method="sequential").

Build the handler library first: python jax-gs_b200/xla/build_ffi.py.
A jax-gs checkout uses it by making jax_gs.renderer.renderer.render this
function (the rest of jax_gs, train.py and train_parallel.py unchanged).
"""
from __future__ import annotations

import ctypes
import functools
import os

import jax
import jax.numpy as jnp
import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_GSLIB = os.path.join(os.path.dirname(_HERE), "gs_b200", "libgsb200.so")
_FFILIB = os.path.join(_HERE, "gs_xla_ffi.so")

TILE_SIZE, OFFSET_SIZE, BLOCK_SIZE = 16, 16, 512
_registered = None


def _libs():
    """Load both libraries once and register the three FFI targets."""
    global _registered
    if _registered is None:
        gs = ctypes.CDLL(_GSLIB, mode=ctypes.RTLD_GLOBAL)
        gs.gs_workspace_bytes.restype = ctypes.c_size_t
        gs.gs_workspace_bytes.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64]
        ffi_lib = ctypes.CDLL(_FFILIB)
        for name, sym in (("gs_render_fwd", "GsRenderFwd"), ("gs_render_bwd", "GsRenderBwd"),
                          ("gs_render_image", "GsRenderImage")):
            jax.ffi.register_ffi_target(name, jax.ffi.pycapsule(getattr(ffi_lib, sym)), platform="CUDA")
        _registered = gs
    return _registered


def _static(camera, sh_degree, n):
    cap = int(n) * OFFSET_SIZE * OFFSET_SIZE  # the reference's candidate count: never overflows
    ws = int(_libs().gs_workspace_bytes(int(n), int(camera.W), int(camera.H), cap)) + 256
    return (int(camera.W), int(camera.H), float(camera.fx), float(camera.fy), float(camera.cx),
            float(camera.cy), int(sh_degree), cap, ws)


def _attrs(static):
    W, H, fx, fy, cx, cy, deg, cap, _ = static
    return dict(W=np.int32(W), H=np.int32(H), fx=np.float32(fx), fy=np.float32(fy), cx=np.float32(cx),
                cy=np.float32(cy), sh_degree=np.int32(deg), capacity=np.int64(cap))


def _forward_types(static, n):
    W, H, ws = static[0], static[1], static[8]
    return (jax.ShapeDtypeStruct((H, W, 3), jnp.float32), jax.ShapeDtypeStruct((n,), jnp.float32),
            jax.ShapeDtypeStruct((n,), jnp.bool_), jax.ShapeDtypeStruct((16,), jnp.int32),
            jax.ShapeDtypeStruct((ws,), jnp.uint8))


def _call_forward(target, static, means, scales, quats, opac, sh, w2c, bg, mask):
    n = means.shape[0]
    return jax.ffi.ffi_call(target, _forward_types(static, n), vmap_method="sequential")(
        means, scales, quats, opac, sh, mask, w2c, bg, **_attrs(static))


@functools.partial(jax.custom_vjp, nondiff_argnums=(0,))
def _render_core(static, means, scales, quats, opac, sh, w2c, bg, mask):
    image, radii, valid, extras, _ = _call_forward("gs_render_image", static, means, scales, quats, opac, sh,
                                                   w2c, bg, mask)
    return image, radii, valid, extras


def _render_fwd(static, means, scales, quats, opac, sh, w2c, bg, mask):
    image, radii, valid, extras, ws = _call_forward("gs_render_fwd", static, means, scales, quats, opac, sh,
                                                    w2c, bg, mask)
    return (image, radii, valid, extras), (means, scales, quats, opac, sh, w2c, bg, mask, ws)


def _render_bwd(static, res, cot):
    means, scales, quats, opac, sh, w2c, bg, mask, ws = res
    g_image = cot[0]
    n = means.shape[0]
    types = (jax.ShapeDtypeStruct(means.shape, jnp.float32), jax.ShapeDtypeStruct(scales.shape, jnp.float32),
             jax.ShapeDtypeStruct(quats.shape, jnp.float32), jax.ShapeDtypeStruct(opac.shape, jnp.float32),
             jax.ShapeDtypeStruct(sh.shape, jnp.float32), jax.ShapeDtypeStruct((3,), jnp.float32),
             jax.ShapeDtypeStruct(ws.shape, jnp.uint8))
    del n
    gm, gs, gq, go, gsh, gbg, _ = jax.ffi.ffi_call("gs_render_bwd", types, vmap_method="sequential",
                                                   input_output_aliases={8: 6})(
        means, scales, quats, opac, sh, mask, w2c, bg, ws, g_image.astype(jnp.float32), **_attrs(static))
    return gm, gs, gq, go, gsh, None, gbg, None


_render_core.defvjp(_render_fwd, _render_bwd)


def render(gaussians, camera, background=None, fast_tpu_rasterizer: bool = False, mask=None, sh_degree: int = 0):
    """jax_gs.renderer.renderer.render on the native kernels (renderer.py:15-107).
    fast_tpu_rasterizer is accepted and has no effect: both reference
    rasterisers apply the same compositing rule."""
    del fast_tpu_rasterizer
    n = gaussians.means.shape[0]
    static = _static(camera, sh_degree, n)
    bg = jnp.zeros((3,), jnp.float32) if background is None else jnp.asarray(background, jnp.float32)
    m = jnp.ones((n,), jnp.bool_) if mask is None else jnp.asarray(mask, jnp.bool_)
    image, radii, valid, ex = _render_core(static, gaussians.means, gaussians.scales, gaussians.quaternions,
                                           gaussians.opacities, gaussians.sh_coeffs,
                                           jnp.asarray(camera.W2C, jnp.float32), bg, m)
    num_tiles = ((static[0] + TILE_SIZE - 1) // TILE_SIZE) * ((static[1] + TILE_SIZE - 1) // TILE_SIZE)
    extras = {
        "radii": radii,
        "valid_mask": valid,
        "n_interactions": ex[0],
        "mean_interactions_per_tile": ex[0] / jnp.maximum(num_tiles, 1),
        "max_interactions_per_tile": ex[2],
        "overflow_tiles": ex[3],
        "overflow_interactions": ex[4],
        "truncated_tiles": ex[5],
        "truncated_interactions": ex[6],
        "radius_cap_violations": ex[7],
    }
    return image, extras
