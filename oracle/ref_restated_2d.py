"""CPU oracle for the 2DGS surfel renderer: a restatement of jax_2dgs in PyTorch.

TEST INFRASTRUCTURE ONLY. Like ref_restated.py, this module is the checker of
the CUDA path: only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline may import it; nothing in the product uses it.

It follows jax_2dgs/core/gaussians_2d.py, jax_2dgs/renderer/projection_2d.py,
jax_2dgs/renderer/rasterizer_2d.py, jax_2dgs/renderer/renderer.py and
jax_2dgs/training/losses.py function by function (citations are file:line in
the jax-gs project) in plain torch ops, so autograd gives the gradients that
jax.value_and_grad gives the reference. Pinned by the reference's own tests
(tests/test_gaussians_2d.py, restated in tests/test_oracle_2d.py) and by
finite differences.

Fixed evaluation order, as in ref_restated.py: every product that decides an
integer output (means2D, radii, depth feed the tile keys) is a sequential sum
in increasing index with one rounding per operation; the small matrix
products of the reference (W2C, J @ [u | v], M M^T) are written out that way,
and the entries that are structural zeros of J are left out (adding +0 does
not change a sum). exp(scales) and the quaternion norm are rounded once.
"""
from __future__ import annotations

from typing import Dict, Tuple

import numpy as np
import torch

from oracle.ref_restated import (TILE_SIZE, _exp_once, _sqrt, get_tile_interactions_compact,
                                 tile_ranges)

BLOCK_SIZE = 512  # rasterizer.py:8, the 2DGS compositor's per-tile cap (rasterizer_2d.py:35-37)
SH_C0 = 0.28209479177387814


def get_tangent_vectors(quaternions: torch.Tensor):
    """gaussians_2d.py:13-54: columns u, v, n of the rotation of q / |q|."""
    q = quaternions
    nrm = _sqrt(((q[:, 0] * q[:, 0] + q[:, 1] * q[:, 1]) + q[:, 2] * q[:, 2]) + q[:, 3] * q[:, 3])
    r, x, y, z = (q[:, k] / nrm for k in range(4))
    u = torch.stack([(1.0 - 2.0 * (y * y)) - 2.0 * (z * z), 2.0 * (x * y) + 2.0 * (r * z),
                     2.0 * (x * z) - 2.0 * (r * y)], -1)
    v = torch.stack([2.0 * (x * y) - 2.0 * (r * z), (1.0 - 2.0 * (x * x)) - 2.0 * (z * z),
                     2.0 * (y * z) + 2.0 * (r * x)], -1)
    n = torch.stack([2.0 * (x * z) + 2.0 * (r * y), 2.0 * (y * z) - 2.0 * (r * x),
                     (1.0 - 2.0 * (x * x)) - 2.0 * (y * y)], -1)
    return u, v, n


def init_gaussians_2d_from_pcd(points: torch.Tensor, colors: torch.Tensor) -> Dict[str, torch.Tensor]:
    """gaussians_2d.py:76-115 (colours assumed non-degenerate)."""
    n = points.shape[0]
    sh = torch.zeros((n, 16, 3))
    sh[:, 0, :] = (colors - 0.5) / SH_C0
    return {"means": points.clone(), "scales": torch.full((n, 2), -3.0),
            "quaternions": torch.tensor([1.0, 0.0, 0.0, 0.0]).repeat(n, 1),
            "opacities": torch.zeros((n, 1)), "sh_coeffs": sh}


def _rot(W: torch.Tensor, a: torch.Tensor, k: int) -> torch.Tensor:
    """(a @ W_rot^T)[:, k], sequential."""
    return (a[:, 0] * W[k, 0] + a[:, 1] * W[k, 1]) + a[:, 2] * W[k, 2]


def project_gaussians_2d(means, scales, quats, W2C, fx, fy, cx, cy):
    """projection_2d.py:6-87. Returns means2D (N,2), cov2D (N,2,2), radii (N,),
    valid (N,) bool, z (N,), normals (N,3) in camera space."""
    dt = means.dtype
    Wm = W2C.to(dt)
    m0, m1, m2 = means[:, 0], means[:, 1], means[:, 2]
    x, y, z = [((Wm[k, 0] * m0 + Wm[k, 1] * m1) + Wm[k, 2] * m2) + Wm[k, 3] for k in range(3)]  # :25-28
    valid = z > 0.01  # :31
    u, v, n = get_tangent_vectors(quats)  # :34
    u_cam = [_rot(Wm, u, k) for k in range(3)]  # :37-40
    v_cam = [_rot(Wm, v, k) for k in range(3)]
    normals = torch.stack([_rot(Wm, n, k) for k in range(3)], -1)
    fx_t, fy_t = torch.tensor(fx, dtype=dt), torch.tensor(fy, dtype=dt)
    inv_z = 1.0 / torch.maximum(z, torch.tensor(0.01, dtype=dt))  # :43-44
    inv_z2 = inv_z * inv_z
    J00, J02 = fx_t * inv_z, ((-fx_t) * x) * inv_z2  # :48-51
    J11, J12 = fy_t * inv_z, ((-fy_t) * y) * inv_z2
    s = _exp_once(scales)  # :58
    # :55 M = J @ [u | v]; :61 scaled columns
    Ms = [[(J00 * u_cam[0] + J02 * u_cam[2]) * s[:, 0], (J00 * v_cam[0] + J02 * v_cam[2]) * s[:, 1]],
          [(J11 * u_cam[1] + J12 * u_cam[2]) * s[:, 0], (J11 * v_cam[1] + J12 * v_cam[2]) * s[:, 1]]]
    # :65 cov2D = Ms Ms^T, :68-69 + 0.3 I
    cov = [[Ms[i][0] * Ms[j][0] + Ms[i][1] * Ms[j][1] for j in range(2)] for i in range(2)]
    c00, c01, c10, c11 = cov[0][0] + 0.3, cov[0][1], cov[1][0], cov[1][1] + 0.3
    cov2D = torch.stack([torch.stack([c00, c01], -1), torch.stack([c10, c11], -1)], -2)
    cx_t, cy_t = torch.tensor(cx, dtype=dt), torch.tensor(cy, dtype=dt)
    means2D = torch.stack([(fx_t * x) / z + cx_t, (fy_t * y) / z + cy_t], -1)  # :72-75
    det = c00 * c11 - c01 * c01  # :78-84
    mid = (c00 + c11) / 2.0
    term = _sqrt(torch.maximum(mid * mid - det, torch.tensor(0.0, dtype=dt)))
    radii = torch.ceil(3.0 * _sqrt(mid + term))
    return means2D, cov2D, radii, valid, z, normals


def render_tiles_2d(means2D, cov2D, opacities, colors, depths, normals, sorted_tile_ids, sorted_gaussian_ids,
                    H, W, background=None, tile_subset=None):
    """rasterizer_2d.py:6-131: colour, depth, depth^2, normal and 1 - T maps.
    Per tile the first BLOCK_SIZE sorted splats are composited (:35-37); the
    scan's transmittance is an exclusive cumprod of (1 - alpha) with alpha
    zeroed once T <= 1e-4 (:71). tile_subset (optional) composites only those
    tiles (the others stay 0), for bounded CPU timing samples."""
    dt = means2D.dtype
    if background is None:
        background = torch.zeros(3, dtype=dt)
    ntx, nty = (W + TILE_SIZE - 1) // TILE_SIZE, (H + TILE_SIZE - 1) // TILE_SIZE
    det = torch.maximum(cov2D[:, 0, 0] * cov2D[:, 1, 1] - cov2D[:, 0, 1] ** 2, torch.tensor(1e-6, dtype=dt))
    ic00, ic01, ic11 = cov2D[:, 1, 1] / det, -cov2D[:, 0, 1] / det, cov2D[:, 0, 0] / det  # :21-25
    sig = torch.sigmoid(opacities[:, 0])  # :26
    bounds = tile_ranges(np.asarray(sorted_tile_ids), ntx * nty)  # :28-29
    gids_np = np.asarray(sorted_gaussian_ids)
    py, px = np.mgrid[0:TILE_SIZE, 0:TILE_SIZE]
    out = torch.zeros((nty * TILE_SIZE, ntx * TILE_SIZE, 9), dtype=dt)
    parts = []
    for t in (range(ntx * nty) if tile_subset is None else tile_subset):
        s, e = int(bounds[t]), int(bounds[t + 1])
        count = min(e - s, BLOCK_SIZE)
        ty, tx = divmod(t, ntx)
        if count <= 0:  # :116-119 empty tile
            bg = torch.cat([background, torch.zeros(6, dtype=dt)])
            parts.append((ty, tx, bg.reshape(1, 9).expand(TILE_SIZE * TILE_SIZE, 9)))
            continue
        idx = torch.as_tensor(gids_np[s:s + count].astype(np.int64))
        gx = torch.as_tensor((tx * TILE_SIZE + px).reshape(-1), dtype=dt) + 0.5  # :54-60
        gy = torch.as_tensor((ty * TILE_SIZE + py).reshape(-1), dtype=dt) + 0.5
        mu = means2D[idx]
        dx = gx[:, None] - mu[None, :, 0]
        dy = gy[:, None] - mu[None, :, 1]
        power = -0.5 * (dx * dx * ic00[idx][None] + dx * dy * (2.0 * ic01[idx])[None]
                        + dy * dy * ic11[idx][None])  # :77
        ea = torch.exp(power) * sig[idx][None]  # :79
        a_raw = torch.where(power > -10.0, torch.minimum(torch.tensor(0.99, dtype=dt), ea),
                            torch.zeros((), dtype=dt))  # :80
        ones = torch.ones((a_raw.shape[0], 1), dtype=dt)
        with torch.no_grad():
            T_raw = torch.cat([ones, torch.cumprod(1.0 - a_raw, dim=1)[:, :-1]], dim=1)
            active = T_raw > 1e-4  # :71
        alpha = torch.where(active, a_raw, torch.zeros((), dtype=dt))
        trans = torch.cat([ones, torch.cumprod(1.0 - alpha, dim=1)], dim=1)  # :83
        w = alpha * trans[:, :-1]  # :82
        d = depths[idx]
        col = w @ colors[idx]  # :84-87
        dep = w @ d[:, None]
        dep2 = w @ (d * d)[:, None]
        nor = w @ normals[idx]
        Tf = trans[:, -1:]
        final = torch.cat([col + Tf * background[None, :], dep, dep2, nor, 1.0 - Tf], dim=1)  # :94-103
        parts.append((ty, tx, final))
    for ty, tx, val in parts:
        out[ty * TILE_SIZE:(ty + 1) * TILE_SIZE, tx * TILE_SIZE:(tx + 1) * TILE_SIZE] = \
            val.reshape(TILE_SIZE, TILE_SIZE, 9)
    full = out[:H, :W, :]  # :122-131
    return full[..., 0:3], full[..., 3:4], full[..., 4:5], full[..., 5:8], full[..., 8:9]


def render_2d(means, scales, quats, opacities, sh, W2C, W, H, fx, fy, cx, cy, background=None, tile_subset=None):
    """renderer.py (jax_2dgs):7-47: image and extras {depth, depth_sq, normals,
    accum_weight}; colours from the DC coefficient only (:27-28)."""
    means2D, cov2D, radii, valid, z, normals = project_gaussians_2d(means, scales, quats, W2C, fx, fy, cx, cy)
    colors = torch.clamp(sh[:, 0, :] * SH_C0 + 0.5, 0.0, 1.0)
    with torch.no_grad():
        tid, gid, n = get_tile_interactions_compact(means2D.detach().numpy(), radii.detach().numpy(),
                                                    valid.numpy(), z.detach().numpy(), H, W)
    image, depth, depth_sq, nmap, accum = render_tiles_2d(means2D, cov2D, opacities, colors, z, normals,
                                                           tid, gid, H, W, background, tile_subset)
    return image, {"depth": depth, "depth_sq": depth_sq, "normals": nmap, "accum_weight": accum}


def depth_distortion_loss(depth, depth_sq, accum_weight):
    """losses.py (jax_2dgs):4-32."""
    w = accum_weight.detach()
    mask = w > 1e-4
    safe_w = torch.where(mask, w, torch.ones_like(w))
    exp_d = torch.where(mask, depth / safe_w, torch.zeros_like(w))
    exp_d_sq = torch.where(mask, depth_sq / safe_w, torch.zeros_like(w))
    variance = torch.clamp(exp_d_sq - exp_d ** 2, min=0.0)
    return (variance * w).mean()


def normal_consistency_loss(rendered_normals, depth_map):
    """losses.py (jax_2dgs):34-78 (camera intrinsics unused by the reference)."""
    d = depth_map.detach()
    dz_dx = (torch.roll(d, -1, dims=1) - torch.roll(d, 1, dims=1)) / 2.0
    dz_dy = (torch.roll(d, -1, dims=0) - torch.roll(d, 1, dims=0)) / 2.0
    n_depth = torch.cat([-dz_dx, -dz_dy, torch.ones_like(d)], -1)
    n_depth = n_depth / torch.sqrt((n_depth ** 2).sum(-1, keepdim=True) + 1e-6)
    rendered_norm = torch.sqrt((rendered_normals ** 2).sum(-1, keepdim=True) + 1e-8)
    n_rendered = rendered_normals / rendered_norm
    cos_sim = (n_rendered * n_depth).sum(-1, keepdim=True)
    return ((1.0 - cos_sim) * rendered_norm.detach()).mean()


def train_loss_2d(params: Dict[str, torch.Tensor], target, W2C, W, H, fx, fy, cx, cy, tile_subset=None
                  ) -> Tuple[torch.Tensor, Dict[str, torch.Tensor]]:
    """trainer.py (jax_2dgs):24-48: (1 - 0.2) L1 + 0.2 D-SSIM + 1e-4 (distortion
    + normal consistency)."""
    from oracle import ref_restated as R
    image, ex = render_2d(params["means"], params["scales"], params["quaternions"], params["opacities"],
                          params["sh_coeffs"], W2C, W, H, fx, fy, cx, cy, tile_subset=tile_subset)
    l1 = R.l1_loss(image, target)
    ds = R.d_ssim_loss(image, target)
    l_dist = depth_distortion_loss(ex["depth"], ex["depth_sq"], ex["accum_weight"])
    l_norm = normal_consistency_loss(ex["normals"], ex["depth"])
    loss = 0.8 * l1 + 0.2 * ds + 1e-4 * l_dist + 1e-4 * l_norm
    return loss, {"l1": l1, "ssim": 1.0 - ds * 2.0, "dist_loss": l_dist, "normal_loss": l_norm}
