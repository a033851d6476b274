"""Mirror of jax_gs/renderer/sh.py (constants :6-23, eval_sh :25-74)."""
from __future__ import annotations

import torch

from gs_b200 import _lib
from gs_b200.renderer.rasterizer import _f32

C0 = 0.28209479177387814
C1 = 0.4886025119029199
C2 = [1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792,
      0.5462742152960396]
C3 = [-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154,
      -0.4570457994644658, 1.445305721320277, -0.5900435899266435]


def eval_sh(sh_degree: int, sh_coeffs: torch.Tensor, view_dirs: torch.Tensor) -> torch.Tensor:
    """(N,K,3) coefficients, (N,3) unit directions -> (N,3) colours (gs_eval_sh)."""
    dev = sh_coeffs.device
    sh = _f32(sh_coeffs, dev)
    d = _f32(view_dirs, dev)
    n, k = int(sh.shape[0]), int(sh.shape[1])
    out = torch.empty((n, 3), dtype=torch.float32, device=dev)
    _lib.call("gs_eval_sh", int(sh_degree), _lib.ptr(sh), n, k, _lib.ptr(d), _lib.ptr(out),
              _lib.stream(dev))
    return out
