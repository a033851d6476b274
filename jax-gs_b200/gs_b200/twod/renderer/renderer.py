"""Mirror of jax_2dgs/renderer/renderer.py on gs_render2d_forward / _backward.

render(gaussians, camera, background=None) -> (image, extras) with extras
{"depth", "depth_sq", "normals", "accum_weight"}, differentiable w.r.t. the
Gaussians2D fields through torch.autograd (all five outputs carry gradients).
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from gs_b200 import _lib
from gs_b200.twod.core.gaussians_2d import Gaussians2D


def _f32(t, dev):
    return torch.as_tensor(t, dtype=torch.float32, device=dev).contiguous()


def workspace2d(n: int, W: int, H: int, capacity: int, dev) -> torch.Tensor:
    nbytes = _lib.lib().gs_render2d_workspace_bytes(n, W, H, capacity)
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)


class _Render2DFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, scales, quats, opacities, sh, w2c, bg, cam, capacity):
        W, H, fx, fy, cx, cy = cam
        dev = means.device
        n, k = int(means.shape[0]), int(sh.shape[1])
        ws = workspace2d(n, W, H, capacity, dev)
        f = dict(dtype=torch.float32, device=dev)
        image = torch.empty((H, W, 3), **f)
        depth = torch.empty((H, W, 1), **f)
        depth_sq = torch.empty((H, W, 1), **f)
        normals = torch.empty((H, W, 3), **f)
        accum = torch.empty((H, W, 1), **f)
        radii = torch.empty((n,), **f)
        valid = torch.empty((n,), dtype=torch.uint8, device=dev)
        ex = torch.empty((16,), dtype=torch.int32, device=dev)
        P = _lib.ptr
        _lib.call("gs_render2d_forward", P(means), P(scales), P(quats), P(opacities), P(sh), n, k, P(w2c), W, H,
                  fx, fy, cx, cy, P(bg), int(capacity), P(ws), ws.numel(), P(image), P(depth), P(depth_sq),
                  P(normals), P(accum), P(radii), P(valid), P(ex), _lib.stream(dev))
        ctx.save_for_backward(means, scales, quats, opacities, sh, w2c, ws, image, depth, depth_sq, normals, accum)
        ctx.cfg = (cam, int(capacity))
        ctx.mark_non_differentiable(radii, valid, ex)
        return image, depth, depth_sq, normals, accum, radii, valid, ex

    @staticmethod
    def backward(ctx, g_img, g_d, g_d2, g_n, g_a, *_):
        means, scales, quats, opacities, sh, w2c, ws, image, depth, depth_sq, normals, accum = ctx.saved_tensors
        cam, capacity = ctx.cfg
        W, H, fx, fy, cx, cy = cam
        dev = means.device
        n, k = int(means.shape[0]), int(sh.shape[1])

        def c(g):
            return None if g is None else g.contiguous().to(torch.float32)
        g_img = c(g_img) if g_img is not None else torch.zeros_like(image)
        out = [torch.empty_like(t) for t in (means, scales, quats, opacities, sh)]
        P = _lib.ptr
        _lib.call("gs_render2d_backward", P(means), P(scales), P(quats), P(opacities), P(sh), n, k, P(w2c), W, H,
                  fx, fy, cx, cy, capacity, P(ws), ws.numel(), P(image), P(depth), P(depth_sq), P(normals),
                  P(accum), P(g_img), P(c(g_d)), P(c(g_d2)), P(c(g_n)), P(c(g_a)), *[P(t) for t in out],
                  _lib.stream(dev))
        return (*out, None, None, None, None)


def render(gaussians: Gaussians2D, camera, background=None,
           capacity: Optional[int] = None) -> Tuple[torch.Tensor, Dict[str, torch.Tensor]]:
    """renderer.py (jax_2dgs):7-47. capacity bounds the (surfel, tile) pairs
    held in scratch (default N * 256, which cannot overflow)."""
    dev = gaussians.means.device
    n = int(gaussians.means.shape[0])
    args = [_f32(getattr(gaussians, f), dev) for f in ("means", "scales", "quaternions", "opacities", "sh_coeffs")]
    w2c = _f32(camera.W2C, dev)
    bg = None if background is None else _f32(background, dev).reshape(3)
    cap = int(_lib.lib().gs_default_capacity(n)) if capacity is None else int(capacity)
    cam = (int(camera.W), int(camera.H), float(camera.fx), float(camera.fy), float(camera.cx), float(camera.cy))
    image, depth, depth_sq, normals, accum, _, _, _ = _Render2DFn.apply(*args, w2c, bg, cam, cap)
    return image, {"depth": depth, "depth_sq": depth_sq, "normals": normals, "accum_weight": accum}
