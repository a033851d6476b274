"""Seeded synthetic scenes and cameras for the benchmark configurations.

The reference benchmarks on the LLFF "fern" scene, which is not available
offline; these generators stand in for it with the shapes and value
distributions of the benchmark configurations (numpy.random.default_rng(seed),
fp32). Cameras follow the look-at convention of the reference's orbit camera
(animate_ply.py:16-51): rows of R are (right, up, forward) with
up = cross(forward, right), right = cross((0,-1,0), forward).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List

import numpy as np

C0 = 0.28209479177387814


@dataclass
class Scene:
    means: np.ndarray  # (N,3)
    scales: np.ndarray  # (N,3)
    quats: np.ndarray  # (N,4)
    opacities: np.ndarray  # (N,1)
    sh: np.ndarray  # (N,K,3)
    active: np.ndarray  # (N,) bool
    sh_degree: int
    W: int
    H: int
    fx: float
    fy: float
    cx: float
    cy: float
    w2cs: List[np.ndarray]  # (4,4) each

    @property
    def n(self) -> int:
        return int(self.means.shape[0])

    def camera_static(self):
        return (self.W, self.H, self.fx, self.fy, self.cx, self.cy)


def look_at(pos, center=(0.0, 0.0, 0.0)) -> np.ndarray:
    pos = np.asarray(pos, np.float64)
    center = np.asarray(center, np.float64)
    fwd = center - pos
    fwd = fwd / np.linalg.norm(fwd)
    up = np.array([0.0, -1.0, 0.0])
    right = np.cross(up, fwd)
    nr = np.linalg.norm(right)
    if nr < 1e-9:  # looking along the up axis
        right = np.array([1.0, 0.0, 0.0])
    else:
        right = right / (nr + 1e-6)
    actual_up = np.cross(fwd, right)
    R = np.stack([right, actual_up, fwd], 0)
    w2c = np.eye(4)
    w2c[:3, :3] = R
    w2c[:3, 3] = -R @ pos
    return w2c.astype(np.float32)


def orbit_cameras(n: int, radius: float, arc_deg: float, elevation_deg: float = 0.0) -> List[np.ndarray]:
    """n cameras spread over `arc_deg` of azimuth around the y axis."""
    out = []
    for i in range(n):
        az = math.radians(-arc_deg / 2 + arc_deg * (i / max(n - 1, 1)) if arc_deg < 360
                          else 360.0 * i / n)
        el = math.radians(elevation_deg)
        pos = (radius * math.cos(el) * math.cos(az), radius * math.sin(el),
               radius * math.cos(el) * math.sin(az))
        out.append(look_at(pos))
    return out


def sphere_cameras(n: int, radius: float, seed: int = 0) -> List[np.ndarray]:
    """n views on a Fibonacci sphere (jittered by `seed`) looking at the origin."""
    rng = np.random.default_rng(seed)
    out = []
    ga = math.pi * (3.0 - math.sqrt(5.0))
    off = rng.uniform(0, 2 * math.pi)
    for i in range(n):
        y = 1 - 2 * (i + 0.5) / n
        r = math.sqrt(max(0.0, 1 - y * y))
        th = ga * i + off
        out.append(look_at((radius * r * math.cos(th), radius * y, radius * r * math.sin(th))))
    return out


def _quats(rng, n):
    q = rng.standard_normal((n, 4)).astype(np.float32)
    return (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(np.float32)


def _sh(rng, n, degree, rest_std=0.1):
    k = 16
    sh = np.zeros((n, k, 3), np.float32)
    col = np.clip(rng.normal(0.5, 0.2, (n, 3)), 0.0, 1.0)
    sh[:, 0, :] = (col - 0.5) / C0
    nk = (degree + 1) ** 2
    if nk > 1:
        sh[:, 1:nk, :] = rng.normal(0.0, rest_std, (n, nk - 1, 3))
    return sh.astype(np.float32)


def config1(seed: int = 0, n: int = 10_000, W: int = 504, H: int = 378) -> Scene:
    """Single-view fwd+bwd: fern-sized, SH degree 0."""
    rng = np.random.default_rng(seed)
    means = np.stack([rng.uniform(-1, 1, n), rng.uniform(-1, 1, n), rng.uniform(2, 6, n)], 1)
    scales = rng.normal(-4.0, 0.5, (n, 3))
    quats = _quats(rng, n)
    opac = rng.normal(0.0, 1.0, (n, 1))
    sh = _sh(rng, n, 0)
    f = 400.0 * W / 504.0
    return Scene(means.astype(np.float32), scales.astype(np.float32), quats, opac.astype(np.float32),
                 sh, np.ones(n, bool), 0, W, H, f, f, W / 2.0, H / 2.0, [np.eye(4, dtype=np.float32)])


def config2(seed: int = 0, n_active: int = 100_000, capacity: int = 200_000, W: int = 504,
            H: int = 378, n_cams: int = 20) -> Scene:
    """Data-parallel training step: SH degree 3,
    capacity 2x the active count, padded slots as init_density_state pads
    them (density.py:23-34). Log-scales ~N(-4, 0.5) and normalised N(0,1)
    quaternions (the configuration leaves both open; config 1's choice)."""
    rng = np.random.default_rng(seed)
    na = n_active
    means = np.zeros((capacity, 3), np.float32)
    scales = np.zeros((capacity, 3), np.float32)
    quats = np.zeros((capacity, 4), np.float32)
    quats[:, 0] = 1.0
    opac = np.zeros((capacity, 1), np.float32)
    sh = np.zeros((capacity, 16, 3), np.float32)
    means[:na] = 2.0 * rng.standard_normal((na, 3))
    scales[:na] = rng.normal(-4.0, 0.5, (na, 3))
    quats[:na] = _quats(rng, na)
    opac[:na] = rng.normal(-2.0, 1.0, (na, 1))
    sh[:na] = _sh(rng, na, 3)
    active = np.zeros(capacity, bool)
    active[:na] = True
    f = 400.0 * W / 504.0
    cams = orbit_cameras(n_cams, 4.0, 30.0)
    return Scene(means, scales, quats, opac, sh, active, 3, W, H, f, f, W / 2.0, H / 2.0, cams)


def config3(seed: int = 0, n: int = 1_000_000, W: int = 1920, H: int = 1080, n_views: int = 64) -> Scene:
    """Render-only throughput: 1M Gaussians, SH degree 3."""
    rng = np.random.default_rng(seed)
    means = rng.uniform(-5, 5, (n, 3))
    scales = rng.normal(-3.5, 0.7, (n, 3))
    quats = _quats(rng, n)
    opac = rng.normal(0.0, 1.5, (n, 1))
    sh = _sh(rng, n, 3)
    f = 1200.0 * W / 1920.0
    cams = sphere_cameras(n_views, 12.0, seed)
    return Scene(means.astype(np.float32), scales.astype(np.float32), quats, opac.astype(np.float32),
                 sh, np.ones(n, bool), 3, W, H, f, f, W / 2.0, H / 2.0, cams)


def config4(seed: int = 0, n: int = 4_000_000, n_active: int = 3_000_000, W: int = 1600, H: int = 1064,
            n_views: int = 200) -> Scene:
    """Large-scene training with densification: capacity
    4M with the first 3M active, means a mixture of 8 Gaussian blobs
    (sigma 1.5) with centres uniform in a 20^3 box, SH degree 3, 200 cameras
    on a 360 degree orbit at radius 15. Scales and opacities follow config 3
    (log-scale N(-3.5, 0.7), opacity logit N(0, 1.5)); fx = fy = 1000."""
    rng = np.random.default_rng(seed)
    centres = rng.uniform(-10 + 3.0, 10 - 3.0, (8, 3))
    which = rng.integers(0, 8, n)
    means = centres[which] + rng.normal(0, 1.5, (n, 3))
    means = np.clip(means, -10, 10)
    scales = rng.normal(-3.5, 0.7, (n, 3))
    quats = _quats(rng, n)
    opac = rng.normal(0.0, 1.5, (n, 1))
    sh = _sh(rng, n, 3)
    active = np.arange(n) < n_active
    cams = orbit_cameras(n_views, 15.0, 360.0)
    return Scene(means.astype(np.float32), scales.astype(np.float32), quats, opac.astype(np.float32),
                 sh, active, 3, W, H, 1000.0, 1000.0, W / 2.0, H / 2.0, cams)


def config5(seed: int = 0, n: int = 500_000, W: int = 1264, H: int = 832, n_views: int = 20) -> dict:
    """2DGS surfels: means uniform in a 6^3 box, two
    tangent log-scales N(-3.5, 0.5), normalised N(0,1) quaternions, SH
    degree 3 (the renderer uses the DC term); views on a sphere of radius 8
    looking at the origin, fx = fy = 1100."""
    rng = np.random.default_rng(seed)
    return {"means": rng.uniform(-3, 3, (n, 3)).astype(np.float32),
            "scales": rng.normal(-3.5, 0.5, (n, 2)).astype(np.float32),
            "quaternions": _quats(rng, n), "opacities": rng.normal(0.0, 1.0, (n, 1)).astype(np.float32),
            "sh_coeffs": _sh(rng, n, 3), "W": W, "H": H, "fx": 1100.0, "fy": 1100.0, "cx": W / 2.0,
            "cy": H / 2.0, "w2cs": sphere_cameras(n_views, 8.0, seed)}


def target_image(seed: int, H: int, W: int) -> np.ndarray:
    """Training target: uniform [0,1] (H,W,3)."""
    return np.random.default_rng(seed + 1000).uniform(0, 1, (H, W, 3)).astype(np.float32)
