"""Camera container, mirror of jax_gs/core/camera.py:4-21."""
from __future__ import annotations

from typing import NamedTuple

import torch


class Camera(NamedTuple):
    W: int  # image width
    H: int  # image height
    fx: float
    fy: float
    cx: float
    cy: float
    W2C: torch.Tensor  # (4, 4) world-to-camera, float32
    full_proj: torch.Tensor  # unused by the renderer (kept for signature parity)

    @property
    def center(self) -> torch.Tensor:
        """Optical centre -R^T t (camera.py:14-21)."""
        R = self.W2C[:3, :3]
        t = self.W2C[:3, 3]
        return -R.T @ t


def camera_static(cam: Camera):
    """(W, H, fx, fy, cx, cy), the static tuple trainer.py:15 unpacks."""
    return (int(cam.W), int(cam.H), float(cam.fx), float(cam.fy), float(cam.cx), float(cam.cy))
