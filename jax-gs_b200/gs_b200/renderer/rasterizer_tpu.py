"""Mirror of jax_gs/renderer/rasterizer_tpu.py:13-135.

render_tiles_tpu composites with the same per-element rule as render_tiles
(element-wise clipped gather, same alpha / transmittance rules), so on B200
both names run the same tile-parallel kernel.
"""
from __future__ import annotations

from gs_b200.renderer.rasterizer import TILE_SIZE, render_tiles


def render_tiles_tpu(means2D, cov2D, opacities, colors, sorted_tile_ids, sorted_gaussian_ids, H, W,
                     background):
    return render_tiles(means2D, cov2D, opacities, colors, sorted_tile_ids, sorted_gaussian_ids, H,
                        W, TILE_SIZE, background)
