"""Mirror of jax_gs/training/losses.py on the libgsb200 loss kernels.

l1_loss, mse_loss and d_ssim_loss are differentiable w.r.t. pred (torch
autograd) and compute value and gradient in one pass (gs_l1_loss /
gs_mse_loss / gs_dssim_loss).
"""
from __future__ import annotations

import torch

from gs_b200 import _lib


def _ws(nbytes: int, dev) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)


class _L1Fn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target):
        dev = pred.device
        loss = torch.empty((), dtype=torch.float32, device=dev)
        grad = torch.empty_like(pred)
        ws = _ws(_lib.L1_WORKSPACE_BYTES, dev)
        _lib.call("gs_l1_loss", _lib.ptr(pred), _lib.ptr(target), pred.numel(), 1.0, _lib.ptr(loss),
                  _lib.ptr(grad), _lib.ptr(ws), ws.numel(), _lib.stream(dev))
        ctx.save_for_backward(grad)
        return loss

    @staticmethod
    def backward(ctx, g):
        (grad,) = ctx.saved_tensors
        return grad * g, None


def l1_loss(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """mean |pred - target| (losses.py:4-8)."""
    pred = pred.contiguous().to(torch.float32)
    target = target.contiguous().to(torch.float32)
    return _L1Fn.apply(pred, target)


class _MseFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target):
        dev = pred.device
        loss = torch.empty((), dtype=torch.float32, device=dev)
        grad = torch.empty_like(pred)
        ws = _ws(_lib.L1_WORKSPACE_BYTES, dev)
        _lib.call("gs_mse_loss", _lib.ptr(pred), _lib.ptr(target), pred.numel(), 1.0, _lib.ptr(loss),
                  _lib.ptr(grad), _lib.ptr(ws), ws.numel(), _lib.stream(dev))
        ctx.save_for_backward(grad)
        return loss

    @staticmethod
    def backward(ctx, g):
        (grad,) = ctx.saved_tensors
        return grad * g, None


def mse_loss(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """mean (pred - target)^2 (losses.py:10-14)."""
    pred = pred.contiguous().to(torch.float32)
    target = target.contiguous().to(torch.float32)
    return _MseFn.apply(pred, target)


class _DssimFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target):
        dev = pred.device
        H, W, C = pred.shape
        loss = torch.empty((), dtype=torch.float32, device=dev)
        ssim_v = torch.empty((), dtype=torch.float32, device=dev)
        grad = torch.zeros_like(pred)
        ws = _ws(_lib.lib().gs_dssim_workspace_bytes(H, W, C), dev)
        _lib.call("gs_dssim_loss", _lib.ptr(pred), _lib.ptr(target), H, W, C, 1.0, _lib.ptr(loss),
                  _lib.ptr(ssim_v), _lib.ptr(grad), _lib.ptr(ws), ws.numel(), _lib.stream(dev))
        ctx.save_for_backward(grad)
        ctx.mark_non_differentiable(ssim_v)
        return loss, ssim_v

    @staticmethod
    def backward(ctx, g, _g_ssim):
        (grad,) = ctx.saved_tensors
        return grad * g, None


def d_ssim_loss(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """max(0, (1 - ssim) / 2) (losses.py:71-75) for (H,W,C) images."""
    pred = pred.contiguous().to(torch.float32)
    target = target.contiguous().to(torch.float32)
    return _DssimFn.apply(pred, target)[0]


def ssim(img1: torch.Tensor, img2: torch.Tensor) -> torch.Tensor:
    """Mean SSIM (losses.py:16-69, size_average=True); value only."""
    img1 = img1.contiguous().to(torch.float32)
    img2 = img2.contiguous().to(torch.float32)
    return _DssimFn.apply(img1.detach(), img2)[1]
