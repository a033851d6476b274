"""Mirror of jax_gs/renderer/projection.py:6-79 (forward values)."""
from __future__ import annotations

import torch

from gs_b200 import _lib
from gs_b200.renderer.rasterizer import _f32, _u8


def project_gaussians(gaussians, camera, mask=None):
    """Returns (means2D (N,2), cov2D (N,2,2), radii (N,), valid_mask (N,) bool,
    z (N,)), computed by gs_project_gaussians."""
    dev = gaussians.means.device
    n = int(gaussians.means.shape[0])
    means = _f32(gaussians.means, dev)
    scales = _f32(gaussians.scales, dev)
    quats = _f32(gaussians.quaternions, dev)
    w2c = _f32(camera.W2C, dev)
    m = None if mask is None else _u8(mask, dev)
    means2D = torch.empty((n, 2), dtype=torch.float32, device=dev)
    cov2D = torch.empty((n, 2, 2), dtype=torch.float32, device=dev)
    radii = torch.empty((n,), dtype=torch.float32, device=dev)
    valid = torch.empty((n,), dtype=torch.uint8, device=dev)
    z = torch.empty((n,), dtype=torch.float32, device=dev)
    _lib.call("gs_project_gaussians", _lib.ptr(means), _lib.ptr(scales), _lib.ptr(quats), n,
              _lib.ptr(m), _lib.ptr(w2c), int(camera.W), int(camera.H), float(camera.fx),
              float(camera.fy), float(camera.cx), float(camera.cy), _lib.ptr(means2D),
              _lib.ptr(cov2D), _lib.ptr(radii), _lib.ptr(valid), _lib.ptr(z), _lib.stream(dev))
    return means2D, cov2D, radii, valid.view(torch.bool), z
