"""render(): mirror of jax_gs/renderer/renderer.py:15-107.

Same signature and return value (image (H,W,3), extras dict with the keys of
renderer.py:79-90). The whole pipeline -- projection, SH colour, tile keys,
device radix sort, tile ranges, compositor -- is one gs_render_forward call;
the backward is one gs_render_backward call, wired in through
torch.autograd so that losses built on the image differentiate into the
Gaussians fields exactly as jax.value_and_grad does in trainer.py:66/137.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from gs_b200 import _lib
from gs_b200.renderer.rasterizer import (BLOCK_SIZE, MAX_TILE_CHUNKS, MAX_TILE_INTERACTIONS,  # noqa: F401
                                         OFFSET_SIZE, TILE_SIZE, _f32, _u8, num_tiles, workspace)

# GsExtras field order (include/gsb200.h).
_EXTRA_INT_FIELDS = {
    "n_interactions": 0,
    "max_interactions_per_tile": 2,
    "overflow_tiles": 3,
    "overflow_interactions": 4,
    "truncated_tiles": 5,
    "truncated_interactions": 6,
    "radius_cap_violations": 7,
    "capacity_overflow": 8,
    # not in the reference's dict: bounded device waits that gave up (the
    # outputs are then not the render; check_extras raises)
    "device_timeouts": 10,
}


def extras_dict(radii: torch.Tensor, valid: torch.Tensor, ex: torch.Tensor) -> Dict[str, torch.Tensor]:
    """renderer.py:79-90 extras from the device GsExtras block (no sync)."""
    d = {"radii": radii, "valid_mask": valid}
    for k, i in _EXTRA_INT_FIELDS.items():
        d[k] = ex[i]
    d["mean_interactions_per_tile"] = ex[1:2].view(torch.float32)[0]
    return d


def check_extras(extras: Dict[str, torch.Tensor]) -> None:
    """Raise GsError if the render behind `extras` is not valid: a bounded
    device wait gave up (GS_ERR_DEVICE_TIMEOUT; the image is then the
    background only) or pairs overflowed the capacity (GS_ERR_CAPACITY).
    Reads two device scalars (synchronises)."""
    if int(extras["device_timeouts"].max()) != 0:
        _lib.check("render", _lib.GS_ERR_DEVICE_TIMEOUT)
    if int(extras["capacity_overflow"].max()) != 0:
        _lib.check("render", _lib.GS_ERR_CAPACITY)


def _forward(entry, means, scales, quats, opacities, sh, w2c, bg, mask, cam, sh_degree, capacity):
    W, H, fx, fy, cx, cy = cam
    dev = means.device
    n = int(means.shape[0])
    k = int(sh.shape[1])
    ws = workspace(n, W, H, capacity, dev)
    image = torch.empty((H, W, 3), dtype=torch.float32, device=dev)
    radii = torch.empty((n,), dtype=torch.float32, device=dev)
    valid = torch.empty((n,), dtype=torch.uint8, device=dev)
    ex = torch.empty((16,), dtype=torch.int32, device=dev)
    _lib.call(entry, _lib.ptr(means), _lib.ptr(scales), _lib.ptr(quats),
              _lib.ptr(opacities), _lib.ptr(sh), n, k, _lib.ptr(mask), _lib.ptr(w2c), W, H, fx, fy,
              cx, cy, _lib.ptr(bg), int(sh_degree), int(capacity), _lib.ptr(ws), ws.numel(),
              _lib.ptr(image), _lib.ptr(radii), _lib.ptr(valid), _lib.ptr(ex), _lib.stream(dev))
    return ws, image, radii, valid, ex


class _RenderFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, scales, quats, opacities, sh, w2c, bg, mask, cam, sh_degree, capacity):
        ws, image, radii, valid, ex = _forward("gs_render_forward", means, scales, quats, opacities, sh,
                                               w2c, bg, mask, cam, sh_degree, capacity)
        ctx.save_for_backward(means, scales, quats, opacities, sh, w2c, bg, mask, ws)
        ctx.cfg = (cam, int(sh_degree), int(capacity))
        ctx.mark_non_differentiable(radii, valid, ex)
        return image, radii, valid, ex

    @staticmethod
    def backward(ctx, g_image, _g_radii, _g_valid, _g_ex):
        means, scales, quats, opacities, sh, w2c, bg, mask, ws = ctx.saved_tensors
        cam, sh_degree, capacity = ctx.cfg
        W, H, fx, fy, cx, cy = cam
        dev = means.device
        n = int(means.shape[0])
        k = int(sh.shape[1])
        g_image = g_image.contiguous().to(torch.float32)
        gm = torch.empty_like(means)
        gs = torch.empty_like(scales)
        gq = torch.empty_like(quats)
        go = torch.empty_like(opacities)
        gsh = torch.empty_like(sh)
        gbg = torch.empty(3, dtype=torch.float32, device=dev) if (bg is not None and ctx.needs_input_grad[6]) else None
        _lib.call("gs_render_backward", _lib.ptr(means), _lib.ptr(scales), _lib.ptr(quats),
                  _lib.ptr(opacities), _lib.ptr(sh), n, k, _lib.ptr(mask), _lib.ptr(w2c), W, H, fx, fy,
                  cx, cy, _lib.ptr(bg), sh_degree, capacity, _lib.ptr(ws), ws.numel(), _lib.ptr(g_image),
                  _lib.ptr(gm), _lib.ptr(gs), _lib.ptr(gq), _lib.ptr(go), _lib.ptr(gsh), _lib.ptr(gbg),
                  None, _lib.stream(dev))
        return gm, gs, gq, go, gsh, None, gbg, None, None, None, None


def render(gaussians, camera, background=None, fast_tpu_rasterizer: bool = False, mask=None,
           sh_degree: int = 0, capacity: Optional[int] = None) -> Tuple[torch.Tensor, Dict]:
    """Render one view (renderer.py:15-107).

    gaussians: Gaussians of CUDA float32 tensors; camera: Camera with static
    W, H, fx, fy, cx, cy and a (4,4) W2C; background (3,) or None (zeros);
    fast_tpu_rasterizer is accepted and has no effect (both reference
    rasterisers share the compositing rule); mask (N,) bool active mask or
    None; sh_degree 0..3. capacity bounds the number of (Gaussian, tile)
    pairs held in scratch (default N * 256, which can never overflow).
    """
    del fast_tpu_rasterizer
    dev = gaussians.means.device
    n = int(gaussians.means.shape[0])
    means = _f32(gaussians.means, dev)
    scales = _f32(gaussians.scales, dev)
    quats = _f32(gaussians.quaternions, dev)
    opac = _f32(gaussians.opacities, dev)
    sh = _f32(gaussians.sh_coeffs, dev)
    w2c = _f32(camera.W2C, dev)
    bg = None if background is None else _f32(background, dev).reshape(3)
    m = None if mask is None else _u8(mask, dev)
    cap = int(_lib.lib().gs_default_capacity(n)) if capacity is None else int(capacity)
    cam = (int(camera.W), int(camera.H), float(camera.fx), float(camera.fy), float(camera.cx),
           float(camera.cy))
    args = (means, scales, quats, opac, sh, w2c, bg, m, cam, int(sh_degree), cap)
    wants_grad = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (means, scales, quats, opac, sh, bg))
    if wants_grad:
        image, radii, valid, ex = _RenderFn.apply(*args)
    else:  # no backward can follow: skip its residuals (gs_render_image)
        _, image, radii, valid, ex = _forward("gs_render_image", *args)
    return image, extras_dict(radii, valid.view(torch.bool), ex)


def _extras_views(radii: torch.Tensor, valid: torch.Tensor, ex: torch.Tensor) -> Dict[str, torch.Tensor]:
    """extras_dict with a leading view axis on every entry."""
    d = {"radii": radii, "valid_mask": valid}
    for k, i in _EXTRA_INT_FIELDS.items():
        d[k] = ex[:, i]
    d["mean_interactions_per_tile"] = ex[:, 1:2].contiguous().view(torch.float32)[:, 0]
    return d


def render_views(gaussians, camera, w2cs, background=None, mask=None, sh_degree: int = 0,
                 capacity: Optional[int] = None, streams: int = 4) -> Tuple[torch.Tensor, Dict]:
    """render() over a leading view axis: the B world-to-camera matrices
    w2cs (B,4,4) share the camera's W, H, fx, fy, cx, cy (what jax.vmap of
    render over W2C gives; config 3 renders 8 views per GPU this way).
    Returns images (B,H,W,3) and the extras dict of renderer.py:79-90 with a
    leading B on every entry. Values only (gs_render_image per view).

    The views are issued round-robin on `streams` CUDA streams, each with
    its own workspace (all allocated on the current stream, which the other
    streams wait for first and which waits for them at the end), so that one
    view's pair sort overlaps another view's compositing on the GPU.
    """
    dev = gaussians.means.device
    n = int(gaussians.means.shape[0])
    means = _f32(gaussians.means, dev)
    scales = _f32(gaussians.scales, dev)
    quats = _f32(gaussians.quaternions, dev)
    opac = _f32(gaussians.opacities, dev)
    sh = _f32(gaussians.sh_coeffs, dev)
    w2cs = _f32(w2cs, dev)
    if w2cs.dim() != 3 or tuple(w2cs.shape[1:]) != (4, 4):
        raise ValueError(f"w2cs must be (B,4,4), got {tuple(w2cs.shape)}")
    B = int(w2cs.shape[0])
    bg = None if background is None else _f32(background, dev).reshape(3)
    m = None if mask is None else _u8(mask, dev)
    cap = int(_lib.lib().gs_default_capacity(n)) if capacity is None else int(capacity)
    W, H = int(camera.W), int(camera.H)
    fx, fy, cx, cy = float(camera.fx), float(camera.fy), float(camera.cx), float(camera.cy)
    k = int(sh.shape[1])
    images = torch.empty((B, H, W, 3), dtype=torch.float32, device=dev)
    radii = torch.empty((B, n), dtype=torch.float32, device=dev)
    valid = torch.empty((B, n), dtype=torch.uint8, device=dev)
    ex = torch.zeros((B, 16), dtype=torch.int32, device=dev)
    if B == 0:
        return images, _extras_views(radii, valid.view(torch.bool), ex)
    S = max(1, min(int(streams), B))
    wss = [workspace(n, W, H, cap, dev) for _ in range(S)]
    main = torch.cuda.current_stream(dev)
    side = [torch.cuda.Stream(dev) for _ in range(S - 1)]
    P = _lib.ptr
    for s2 in side:
        s2.wait_stream(main)
    try:
        for i in range(B):
            j = i % S
            st = main if j == 0 else side[j - 1]
            _lib.call("gs_render_image", P(means), P(scales), P(quats), P(opac), P(sh), n, k, P(m), P(w2cs[i]),
                      W, H, fx, fy, cx, cy, P(bg), int(sh_degree), cap, P(wss[j]), wss[j].numel(),
                      P(images[i]), P(radii[i]), P(valid[i]), P(ex[i]), st.cuda_stream)
    finally:
        for s2 in side:
            main.wait_stream(s2)
    return images, _extras_views(radii, valid.view(torch.bool), ex)
