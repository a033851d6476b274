"""Tile binning and compositing, mirror of jax_gs/renderer/rasterizer.py.

Same constant names and values (rasterizer.py:6-10) and the same function
signatures. Both functions run in libgsb200.so:
  get_tile_interactions -> gs_get_tile_interactions (key emission, device
      radix sort, tile ranges)
  render_tiles          -> gs_render_tiles / gs_render_tiles_backward
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from gs_b200 import _lib

TILE_SIZE = 16
OFFSET_SIZE = 16
BLOCK_SIZE = 512
MAX_TILE_CHUNKS = 8
MAX_TILE_INTERACTIONS = BLOCK_SIZE * MAX_TILE_CHUNKS
DEPTH_BITS = 13


def _f32(t: torch.Tensor, device) -> torch.Tensor:
    return torch.as_tensor(t, dtype=torch.float32, device=device).contiguous()


def _i32(t: torch.Tensor, device) -> torch.Tensor:
    return torch.as_tensor(t, dtype=torch.int32, device=device).contiguous()


def _u8(t: torch.Tensor, device) -> torch.Tensor:
    t = torch.as_tensor(t, device=device)
    if t.dtype == torch.bool:
        return t.contiguous().view(torch.uint8)
    return t.to(torch.uint8).contiguous()


def num_tiles(H: int, W: int) -> Tuple[int, int, int]:
    tx = (W + TILE_SIZE - 1) // TILE_SIZE
    ty = (H + TILE_SIZE - 1) // TILE_SIZE
    return tx, ty, tx * ty


def workspace(n: int, W: int, H: int, capacity: int, device) -> torch.Tensor:
    nbytes = _lib.lib().gs_workspace_bytes(int(n), int(W), int(H), int(capacity))
    if nbytes == 0:
        raise ValueError(f"invalid problem size n={n} W={W} H={H} capacity={capacity}")
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def get_tile_interactions(means2D, radii, valid_mask, depths, H, W, tile_size: int = TILE_SIZE,
                          capacity: Optional[int] = None, return_ranges: bool = False):
    """Sorted (tile, Gaussian) interactions (rasterizer.py:12-116).

    Returns (sorted_tile_ids, sorted_gaussian_ids, n_interactions) with arrays
    of length max(capacity, BLOCK_SIZE), capacity defaulting to N * 256 (the
    reference's candidate count). Entry order equals the reference's valid
    segment (stable sort by tile then 13-bit depth key, ties by Gaussian id);
    past n_interactions the arrays hold tile id num_tiles and Gaussian id 0,
    as the reference pads. The reference additionally keeps behind-camera
    candidates (tile id -1) in front of the valid segment; those carry no
    interaction and are not emitted here. With return_ranges, also returns
    the (num_tiles + 1,) searchsorted tile boundaries.
    """
    if tile_size != TILE_SIZE:
        raise ValueError("tile_size must be 16 (TILE_SIZE)")
    dev = means2D.device
    n = int(means2D.shape[0])
    cap = int(_lib.lib().gs_default_capacity(n)) if capacity is None else int(capacity)
    length = max(cap, BLOCK_SIZE)
    m2 = _f32(means2D, dev)
    r = _f32(radii, dev)
    v = _u8(valid_mask, dev)
    d = _f32(depths, dev)
    ws = workspace(n, W, H, length, dev)
    tiles = torch.empty(length, dtype=torch.int32, device=dev)
    gids = torch.empty(length, dtype=torch.int32, device=dev)
    count = torch.empty((), dtype=torch.int32, device=dev)
    _, _, T = num_tiles(H, W)
    ranges = torch.empty(T + 1, dtype=torch.int32, device=dev)
    _lib.call("gs_get_tile_interactions", _lib.ptr(m2), _lib.ptr(r), _lib.ptr(v), _lib.ptr(d), n,
              int(H), int(W), length, _lib.ptr(ws), ws.numel(), _lib.ptr(tiles), _lib.ptr(gids),
              _lib.ptr(count), _lib.ptr(ranges), _lib.stream(dev))
    if return_ranges:
        return tiles, gids, count, ranges
    return tiles, gids, count


class _RenderTilesFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means2D, cov2D, opacities, colors, tiles, gids, bg, H, W):
        dev = means2D.device
        n = int(means2D.shape[0])
        ws = workspace(n, W, H, int(tiles.numel()), dev)
        image = torch.empty((H, W, 3), dtype=torch.float32, device=dev)
        _lib.call("gs_render_tiles", _lib.ptr(means2D), _lib.ptr(cov2D), _lib.ptr(opacities),
                  _lib.ptr(colors), n, _lib.ptr(tiles), _lib.ptr(gids), int(tiles.numel()), int(H),
                  int(W), _lib.ptr(bg), _lib.ptr(ws), ws.numel(), _lib.ptr(image), _lib.stream(dev))
        ctx.save_for_backward(means2D, cov2D, opacities, colors, tiles, gids, bg)
        ctx.hw = (H, W)
        return image

    @staticmethod
    def backward(ctx, g_image):
        means2D, cov2D, opacities, colors, tiles, gids, bg = ctx.saved_tensors
        H, W = ctx.hw
        dev = means2D.device
        n = int(means2D.shape[0])
        ws = workspace(n, W, H, int(tiles.numel()), dev)
        g_image = g_image.contiguous().to(torch.float32)
        gm = torch.empty_like(means2D)
        gc = torch.empty_like(cov2D)
        go = torch.empty_like(opacities)
        gcol = torch.empty_like(colors)
        _lib.call("gs_render_tiles_backward", _lib.ptr(means2D), _lib.ptr(cov2D),
                  _lib.ptr(opacities), _lib.ptr(colors), n, _lib.ptr(tiles), _lib.ptr(gids),
                  int(tiles.numel()), int(H), int(W), _lib.ptr(bg), _lib.ptr(g_image), _lib.ptr(ws),
                  ws.numel(), _lib.ptr(gm), _lib.ptr(gc), _lib.ptr(go), _lib.ptr(gcol),
                  _lib.stream(dev))
        return gm, gc, go, gcol, None, None, None, None, None


def render_tiles(means2D, cov2D, opacities, colors, sorted_tile_ids, sorted_gaussian_ids, H, W,
                 tile_size: int = TILE_SIZE, background=None):
    """Front-to-back tile compositor (rasterizer.py:119-248).

    means2D (N,2), cov2D (N,2,2), opacities (N,1) raw logits, colors (N,3),
    sorted ids in the reference's layout (any length). Returns (H,W,3);
    differentiable w.r.t. means2D, cov2D, opacities and colors.
    """
    if tile_size != TILE_SIZE:
        raise ValueError("tile_size must be 16 (TILE_SIZE)")
    dev = means2D.device
    m2 = _f32(means2D, dev).reshape(-1, 2)
    cv = _f32(cov2D, dev).reshape(-1, 2, 2)
    op = _f32(opacities, dev).reshape(-1, 1)
    col = _f32(colors, dev).reshape(-1, 3)
    tiles = _i32(sorted_tile_ids, dev)
    gids = _i32(sorted_gaussian_ids, dev)
    bg = None if background is None else _f32(background, dev).reshape(3)
    return _RenderTilesFn.apply(m2, cv, op, col, tiles, gids, bg, int(H), int(W))
