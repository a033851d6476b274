"""Gaussian parameter container and covariance, mirror of
jax_gs/core/gaussians.py:5-93."""
from __future__ import annotations

import dataclasses

import torch


@dataclasses.dataclass
class Gaussians:
    means: torch.Tensor  # (N, 3)
    scales: torch.Tensor  # (N, 3) log-scales
    quaternions: torch.Tensor  # (N, 4) w, x, y, z (unnormalised)
    opacities: torch.Tensor  # (N, 1) logits
    sh_coeffs: torch.Tensor  # (N, K, 3)

    def replace(self, **kw) -> "Gaussians":
        return dataclasses.replace(self, **kw)

    @property
    def n(self) -> int:
        return int(self.means.shape[0])


def init_gaussians_from_pcd(points: torch.Tensor, colors: torch.Tensor) -> Gaussians:
    """Initial Gaussians of a point cloud (gaussians.py:13-56): log-scale -3,
    identity rotation, opacity logit 0, SH degree-3 storage with the DC term
    (colour - 0.5) / C0. Colours that are all ~0 are replaced by uniform
    [0.1, 0.9] noise from a fixed generator (the reference seeds PRNGKey(42))."""
    n = points.shape[0]
    dev = points.device
    means = points.to(torch.float32)
    scales = torch.full((n, 3), -3.0, device=dev)
    quats = torch.zeros((n, 4), device=dev)
    quats[:, 0] = 1.0
    opac = torch.zeros((n, 1), device=dev)
    colors = colors.to(torch.float32)
    if float(colors.max()) < 1e-3:
        g = torch.Generator(device="cpu").manual_seed(42)
        colors = (torch.rand(colors.shape, generator=g) * 0.8 + 0.1).to(dev)
    sh = torch.zeros((n, 16, 3), device=dev)
    sh[:, 0, :] = (colors - 0.5) / 0.28209479177387814
    return Gaussians(means=means, scales=scales, quaternions=quats, opacities=opac, sh_coeffs=sh)


def get_covariance_3d(scales: torch.Tensor, quaternions: torch.Tensor) -> torch.Tensor:
    """Sigma = R S S^T R^T (gaussians.py:58-93) for scales (N,3) and
    quaternions (N,4) on the device: (N,3,3), the same bits as the covariance
    inside render() (gs_covariance_3d). Values only: render() differentiates
    through the covariance itself, so a gradient through this function is
    refused rather than silently missing."""
    from gs_b200 import _lib
    if torch.is_grad_enabled() and (scales.requires_grad or quaternions.requires_grad):
        raise NotImplementedError("get_covariance_3d has no backward here; call it under torch.no_grad() "
                                  "or on detached tensors (render() differentiates through the covariance)")
    scales = scales.detach().contiguous().to(torch.float32)
    quaternions = quaternions.detach().contiguous().to(torch.float32)
    n = scales.shape[0]
    if scales.shape != (n, 3) or quaternions.shape != (n, 4):
        raise ValueError(f"expected scales (N,3) and quaternions (N,4), got {tuple(scales.shape)} and "
                         f"{tuple(quaternions.shape)}")
    out = torch.empty((n, 3, 3), dtype=torch.float32, device=scales.device)
    _lib.call("gs_covariance_3d", _lib.ptr(scales), _lib.ptr(quaternions), n, _lib.ptr(out),
              _lib.stream(scales.device))
    return out
