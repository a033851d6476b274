"""Mirror of jax_2dgs/core/gaussians_2d.py."""
from __future__ import annotations

import dataclasses

import torch

SH_C0 = 0.28209479177387814


@dataclasses.dataclass
class Gaussians2D:
    """gaussians_2d.py:5-11."""
    means: torch.Tensor  # (N, 3)
    scales: torch.Tensor  # (N, 2) log scales of the disk
    quaternions: torch.Tensor  # (N, 4) w, x, y, z
    opacities: torch.Tensor  # (N, 1) logits
    sh_coeffs: torch.Tensor  # (N, K, 3)

    def replace(self, **kw) -> "Gaussians2D":
        return dataclasses.replace(self, **kw)


def get_tangent_vectors(quaternions: torch.Tensor):
    """gaussians_2d.py:13-54: u, v, n = the columns of the rotation of q / |q|."""
    q = quaternions / torch.linalg.norm(quaternions, dim=-1, keepdim=True)
    r, x, y, z = q.unbind(-1)
    u = torch.stack([1 - 2 * y ** 2 - 2 * z ** 2, 2 * x * y + 2 * r * z, 2 * x * z - 2 * r * y], -1)
    v = torch.stack([2 * x * y - 2 * r * z, 1 - 2 * x ** 2 - 2 * z ** 2, 2 * y * z + 2 * r * x], -1)
    n = torch.stack([2 * x * z + 2 * r * y, 2 * y * z - 2 * r * x, 1 - 2 * x ** 2 - 2 * y ** 2], -1)
    return u, v, n


def get_covariance_2d_world(scales: torch.Tensor, quaternions: torch.Tensor) -> torch.Tensor:
    """gaussians_2d.py:56-74: (N, 3, 2) matrix [s1 u | s2 v]."""
    u, v, _ = get_tangent_vectors(quaternions)
    s = torch.exp(scales)
    return torch.stack([u * s[:, 0:1], v * s[:, 1:2]], -1)


def init_gaussians_2d_from_pcd(points: torch.Tensor, colors: torch.Tensor) -> Gaussians2D:
    """gaussians_2d.py:76-115 (random colours for an all-black cloud, as there)."""
    n = points.shape[0]
    dev = points.device
    if float(colors.max()) < 1e-3:
        gen = torch.Generator(device=dev)
        gen.manual_seed(42)
        colors = torch.rand(colors.shape, generator=gen, device=dev) * 0.8 + 0.1
    sh = torch.zeros((n, 16, 3), dtype=torch.float32, device=dev)
    sh[:, 0, :] = (colors.to(torch.float32) - 0.5) / SH_C0
    return Gaussians2D(means=points.to(torch.float32).clone(),
                       scales=torch.full((n, 2), -3.0, device=dev),
                       quaternions=torch.tensor([1.0, 0.0, 0.0, 0.0], device=dev).repeat(n, 1),
                       opacities=torch.zeros((n, 1), device=dev), sh_coeffs=sh)
