"""Shared test helpers: seeded scenes as torch tensors for the oracle and the
CUDA path."""
from __future__ import annotations

import math

import numpy as np
import torch

from gs_b200 import synthetic


def random_scene(seed: int, n: int, W: int, H: int, sh_degree: int = 3, rotate: bool = True,
                 behind: float = 0.1, mask_frac: float = 0.0, scale_mu: float = -3.0,
                 scale_sd: float = 0.6, fov_f: float = None):
    """A small scene with a rotated camera, some Gaussians behind it and an
    optional inactive fraction; returns a dict of numpy arrays."""
    rng = np.random.default_rng(seed)
    means = np.stack([rng.uniform(-1.5, 1.5, n), rng.uniform(-1.2, 1.2, n), rng.uniform(1.0, 6.0, n)], 1)
    nb = int(behind * n)
    if nb:
        means[:nb, 2] = rng.uniform(-3.0, 0.005, nb)  # behind / at the near plane
    scales = rng.normal(scale_mu, scale_sd, (n, 3))
    q = rng.standard_normal((n, 4))
    sh = synthetic._sh(rng, n, sh_degree)
    opac = rng.normal(0.0, 1.2, (n, 1))
    if rotate:
        a, b = 0.15, -0.1
        Ry = np.array([[math.cos(a), 0, math.sin(a)], [0, 1, 0], [-math.sin(a), 0, math.cos(a)]])
        Rx = np.array([[1, 0, 0], [0, math.cos(b), -math.sin(b)], [0, math.sin(b), math.cos(b)]])
        R = Rx @ Ry
        t = np.array([0.1, -0.05, 0.3])
    else:
        R, t = np.eye(3), np.zeros(3)
    w2c = np.eye(4)
    w2c[:3, :3] = R
    w2c[:3, 3] = t
    active = rng.uniform(0, 1, n) >= mask_frac
    f = fov_f if fov_f is not None else 0.9 * W
    return dict(means=means.astype(np.float32), scales=scales.astype(np.float32),
                quats=q.astype(np.float32), opac=opac.astype(np.float32), sh=sh.astype(np.float32),
                w2c=w2c.astype(np.float32), active=active, W=W, H=H, fx=float(f), fy=float(f * 1.02),
                cx=W / 2.0 + 0.3, cy=H / 2.0 - 0.2, sh_degree=sh_degree)


def scene_from_synthetic(s: synthetic.Scene, view: int = 0):
    return dict(means=s.means, scales=s.scales, quats=s.quats, opac=s.opacities, sh=s.sh,
                w2c=s.w2cs[view], active=s.active, W=s.W, H=s.H, fx=s.fx, fy=s.fy, cx=s.cx, cy=s.cy,
                sh_degree=s.sh_degree)


def to_torch(sc: dict, device="cpu", dtype=torch.float32):
    t = lambda a: torch.as_tensor(a, dtype=dtype, device=device).contiguous()  # noqa: E731
    return dict(means=t(sc["means"]), scales=t(sc["scales"]), quats=t(sc["quats"]),
                opac=t(sc["opac"]), sh=t(sc["sh"]), w2c=t(sc["w2c"]),
                active=torch.as_tensor(sc["active"], device=device))


def oracle_render(sc: dict, dtype=torch.float32, requires_grad=False, compact_sort=True):
    from oracle import ref_restated as R
    t = to_torch(sc, "cpu", dtype)
    if requires_grad:
        for k in ("means", "scales", "quats", "opac", "sh"):
            t[k].requires_grad_(True)
    img, ex = R.render(t["means"], t["scales"], t["quats"], t["opac"], t["sh"], t["w2c"], sc["W"],
                       sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"], mask=t["active"],
                       sh_degree=sc["sh_degree"], compact_sort=compact_sort)
    return img, ex, t


def grad_errors(g, r, floor: float = 1e-2):
    """Error statistics of a gradient array g against the oracle's r: the
    largest |g - r| over max|r|, and the plain per-element relative error
    |g - r| / |r| over the entries with |r| >= floor * max|r| (maximum and
    99th percentile; their count). Entries far below the array's scale are
    left out of the relative figures, where fp32 atomics that reorder sums
    of cancelling terms make a ratio meaningless."""
    g, r = np.asarray(g, np.float64).ravel(), np.asarray(r, np.float64).ravel()
    scale = float(np.abs(r).max()) if r.size else 0.0
    err = np.abs(g - r)
    big = np.abs(r) >= floor * scale if scale > 0 else np.zeros(r.shape, bool)
    rel = err[big] / np.abs(r[big]) if big.any() else np.zeros(0)
    return {"max_err_over_scale": float(err.max() / scale) if scale > 0 else 0.0,
            "rel_max": float(rel.max()) if rel.size else 0.0,
            "rel_p99": float(np.percentile(rel, 99)) if rel.size else 0.0,
            "rel_count": int(rel.size), "scale": scale}
