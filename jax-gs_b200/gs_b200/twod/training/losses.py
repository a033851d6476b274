"""Mirror of jax_2dgs/training/losses.py on gs_2dgs_regularizers."""
from __future__ import annotations

import torch

from gs_b200 import _lib


class _RegFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, depth, depth_sq, normals, accum, lam_d, lam_n):
        dev = depth.device
        H, W = int(depth.shape[0]), int(depth.shape[1])
        out = torch.empty(2, dtype=torch.float32, device=dev)
        gd, gd2, gn = torch.empty_like(depth), torch.empty_like(depth_sq), torch.empty_like(normals)
        ws = torch.empty(max(256, _lib.lib().gs_2dgs_regularizers_workspace_bytes()), dtype=torch.uint8, device=dev)
        P = _lib.ptr
        _lib.call("gs_2dgs_regularizers", P(depth), P(depth_sq), P(normals), P(accum), H, W, float(lam_d),
                  float(lam_n), P(out[0:1]), P(out[1:2]), P(gd), P(gd2), P(gn), P(ws), ws.numel(), _lib.stream(dev))
        ctx.save_for_backward(gd, gd2, gn)
        return out[0], out[1]

    @staticmethod
    def backward(ctx, g_dist, g_norm):
        # the kernel's gradients are those of lam_d * dist + lam_n * normal for
        # the forward's weights; each public loss calls it with one weight 1
        # and the other 0, so each gradient pairs with its own output
        gd, gd2, gn = ctx.saved_tensors
        return gd * g_dist, gd2 * g_dist, gn * g_norm, None, None, None


def _prep(t):
    return t.contiguous().to(torch.float32)


def depth_distortion_loss(depth, depth_sq, accum_weight) -> torch.Tensor:
    """losses.py (jax_2dgs):4-32."""
    d, _ = _RegFn.apply(_prep(depth), _prep(depth_sq), torch.zeros_like(_prep(depth)).expand(
        depth.shape[0], depth.shape[1], 3).contiguous(), _prep(accum_weight).detach(), 1.0, 0.0)
    return d


def normal_consistency_loss(rendered_normals, depth_map, camera=None) -> torch.Tensor:
    """losses.py (jax_2dgs):34-78 (the camera argument is unused, as there)."""
    del camera
    d = _prep(depth_map).detach()
    _, nl = _RegFn.apply(d, torch.zeros_like(d), _prep(rendered_normals), torch.zeros_like(d), 0.0, 1.0)
    return nl
