"""CPU oracle: a restatement of jax-gs's renderer hot path in PyTorch (CPU).

TEST INFRASTRUCTURE ONLY. This module is the checker of the CUDA path: only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
may import it. Nothing in the product (jax-gs_b200/) uses it.

It follows the reference function by function (citations are file:line in
the jax-gs project) in plain torch ops, so torch autograd yields the
per-Gaussian gradients that jax.value_and_grad gives the reference. JAX is
not installed here, so the reference cannot run; the restatement is pinned
by the reference's own known-answer tests (tests/test_renderer.py:11-33,
:53-113, :115-158; tests/test_core.py:21-38) restated in
tests/test_oracle.py, by finite differences for the gradients, and by the
golden fixtures under tests/golden/ (generated from this module).

Fixed evaluation order. The reference's 3x3 / 4x4 matrix products are XLA
dots whose summation order is backend-defined. Here every product that
decides an integer output (means2D, radii and depth feed floor / ceil / the
13-bit depth key) is written as a sequential sum in increasing index order
with one rounding per operation, and exp(scales) is rounded once from a
double evaluation. The CUDA kernels evaluate the same expressions in the same
order with FMA contraction disabled, which is what makes tile keys, sort order
and tile ranges comparable bit for bit.
"""
from __future__ import annotations

from typing import Dict, Tuple

import numpy as np
import torch

TILE_SIZE = 16  # rasterizer.py:6
OFFSET_SIZE = 16  # rasterizer.py:7
BLOCK_SIZE = 512  # rasterizer.py:8
MAX_TILE_CHUNKS = 8  # rasterizer.py:9
MAX_TILE_INTERACTIONS = BLOCK_SIZE * MAX_TILE_CHUNKS  # rasterizer.py:10
DEPTH_BITS = 13  # rasterizer.py:84

C0 = 0.28209479177387814  # sh.py:6-23
C1 = 0.4886025119029199
C2 = [1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792,
      0.5462742152960396]
C3 = [-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154,
      -0.4570457994644658, 1.445305721320277, -0.5900435899266435]


class _ExactSqrt(torch.autograd.Function):
    """IEEE correctly rounded sqrt (numpy) with the usual derivative. torch's
    CPU float32 sqrt is not always correctly rounded; CUDA's __fsqrt_rn and
    numpy are, and the radius / quaternion-norm values must match bitwise."""

    @staticmethod
    def forward(ctx, x):
        out = torch.from_numpy(np.sqrt(x.detach().cpu().numpy()))
        ctx.save_for_backward(out)
        return out

    @staticmethod
    def backward(ctx, g):
        (out,) = ctx.saved_tensors
        return g / (2.0 * out)


def _sqrt(x: torch.Tensor) -> torch.Tensor:
    return _ExactSqrt.apply(x)


def _exp_once(x: torch.Tensor) -> torch.Tensor:
    """exp rounded once to the working dtype (from a float64 evaluation)."""
    return torch.exp(x.to(torch.float64)).to(x.dtype)


def get_covariance_3d(scales: torch.Tensor, quaternions: torch.Tensor) -> torch.Tensor:
    """gaussians.py:58-93: Sigma = R S S^T R^T with R from q / |q|."""
    q = quaternions
    n2 = ((q[:, 0] * q[:, 0] + q[:, 1] * q[:, 1]) + q[:, 2] * q[:, 2]) + q[:, 3] * q[:, 3]
    nrm = _sqrt(n2)
    # :70 q / |q|, one same-shape division per component (torch's broadcast
    # division may multiply by a reciprocal, which is not the IEEE quotient)
    r, x, y, z = q[:, 0] / nrm, q[:, 1] / nrm, q[:, 2] / nrm, q[:, 3] / nrm  # :73-76
    R = torch.stack([  # :78-82
        torch.stack([1 - 2 * (y * y) - 2 * (z * z), (2 * x) * y - (2 * r) * z, (2 * x) * z + (2 * r) * y], -1),
        torch.stack([(2 * x) * y + (2 * r) * z, 1 - 2 * (x * x) - 2 * (z * z), (2 * y) * z - (2 * r) * x], -1),
        torch.stack([(2 * x) * z - (2 * r) * y, (2 * y) * z + (2 * r) * x, 1 - 2 * (x * x) - 2 * (y * y)], -1),
    ], -2)
    s = _exp_once(scales)  # :85
    M = R * s[:, None, :]  # :88
    rows = []
    for i in range(3):  # :91  M @ M^T, sequential sums
        rows.append(torch.stack([(M[:, i, 0] * M[:, j, 0] + M[:, i, 1] * M[:, j, 1]) + M[:, i, 2] * M[:, j, 2]
                                 for j in range(3)], -1))
    return torch.stack(rows, -2)


def camera_center(W2C: torch.Tensor) -> torch.Tensor:
    """camera.py:14-21: -R^T t."""
    R = W2C[:3, :3]
    t = W2C[:3, 3]
    return -(R.T @ t)


def project_gaussians(means, scales, quats, W2C, W, H, fx, fy, cx, cy, mask=None):
    """projection.py:6-79. Returns means2D (N,2), cov2D (N,2,2), radii (N,),
    valid (N,) bool, z (N,)."""
    dt = means.dtype
    Wm = W2C.to(dt)
    m0, m1, m2 = means[:, 0], means[:, 1], means[:, 2]
    # :133-134 [m, 1] @ W2C^T
    pc = [((Wm[k, 0] * m0 + Wm[k, 1] * m1) + Wm[k, 2] * m2) + Wm[k, 3] for k in range(3)]
    x, y, z = pc
    valid = z > 0.01  # :139
    if mask is not None:
        valid = valid & mask  # :141
    Sig = get_covariance_3d(scales, quats)  # :144
    fx_t = torch.tensor(fx, dtype=dt)
    fy_t = torch.tensor(fy, dtype=dt)
    safe_z = torch.maximum(z, torch.tensor(0.01, dtype=dt))  # :150
    inv_z = 1.0 / safe_z
    inv_z2 = inv_z * inv_z
    J00 = fx_t * inv_z  # :154-157
    J02 = ((-fx_t) * x) * inv_z2
    J11 = fy_t * inv_z
    J12 = ((-fy_t) * y) * inv_z2
    # :163 M = J @ W_rot (the zero entries of J contribute exact zeros)
    Mj0 = [J00 * Wm[0, k] + J02 * Wm[2, k] for k in range(3)]
    Mj1 = [J11 * Wm[1, k] + J12 * Wm[2, k] for k in range(3)]
    Mj = [Mj0, Mj1]
    # :164 cov2D = (M @ Sigma) @ M^T
    T = [[(Mj[i][0] * Sig[:, 0, k] + Mj[i][1] * Sig[:, 1, k]) + Mj[i][2] * Sig[:, 2, k] for k in range(3)]
         for i in range(2)]
    cov = [[(T[i][0] * Mj[j][0] + T[i][1] * Mj[j][1]) + T[i][2] * Mj[j][2] for j in range(2)] for i in range(2)]
    c00 = cov[0][0] + 0.3  # :168-169
    c01 = cov[0][1]
    c10 = cov[1][0]
    c11 = cov[1][1] + 0.3
    cov2D = torch.stack([torch.stack([c00, c01], -1), torch.stack([c10, c11], -1)], -2)
    cx_t = torch.tensor(cx, dtype=dt)
    cy_t = torch.tensor(cy, dtype=dt)
    means2D = torch.stack([(fx_t * x) / z + cx_t, (fy_t * y) / z + cy_t], -1)  # :172-175
    det = c00 * c11 - c01 * c01  # :178-184
    trace = c00 + c11
    mid = trace / 2.0
    term = _sqrt(torch.maximum(mid * mid - det, torch.tensor(0.0, dtype=dt)))
    lambda1 = mid + term
    radii = torch.ceil(3.0 * _sqrt(lambda1))
    return means2D, cov2D, radii, valid, z


def eval_sh(sh_degree: int, sh: torch.Tensor, dirs: torch.Tensor) -> torch.Tensor:
    """sh.py:25-74."""
    result = C0 * sh[:, 0]
    if sh_degree > 0:
        x, y, z = dirs[:, 0:1], dirs[:, 1:2], dirs[:, 2:3]
        result = result - C1 * y * sh[:, 1] + C1 * z * sh[:, 2] - C1 * x * sh[:, 3]
        if sh_degree > 1:
            xx, yy, zz = x * x, y * y, z * z
            xy, yz, xz = x * y, y * z, x * z
            result = (result + C2[0] * xy * sh[:, 4] + C2[1] * yz * sh[:, 5]
                      + C2[2] * (2.0 * zz - xx - yy) * sh[:, 6] + C2[3] * xz * sh[:, 7]
                      + C2[4] * (xx - yy) * sh[:, 8])
            if sh_degree > 2:
                result = (result + C3[0] * y * (3.0 * xx - yy) * sh[:, 9] + C3[1] * xy * z * sh[:, 10]
                          + C3[2] * y * (4.0 * zz - xx - yy) * sh[:, 11]
                          + C3[3] * z * (2.0 * zz - 3.0 * xx - 3.0 * yy) * sh[:, 12]
                          + C3[4] * x * (4.0 * zz - xx - yy) * sh[:, 13]
                          + C3[5] * z * (xx - yy) * sh[:, 14] + C3[6] * x * (xx - 3.0 * yy) * sh[:, 15])
    return result


def _clip01(x: torch.Tensor) -> torch.Tensor:
    """jnp.clip(x, 0, 1) = minimum(maximum(x, 0), 1), half gradient at ties."""
    return torch.minimum(torch.maximum(x, torch.zeros((), dtype=x.dtype)), torch.ones((), dtype=x.dtype))


def _tile_rect(means2D: np.ndarray, radii: np.ndarray, H: int, W: int):
    """rasterizer.py:36-49 (also renderer.py:63-72), float32 numpy."""
    f = np.float32
    mx, my, r = means2D[:, 0].astype(f), means2D[:, 1].astype(f), radii.astype(f)
    with np.errstate(invalid="ignore"):
        min_x = np.clip(mx - r, f(0), f(W - 1))
        max_x = np.clip(mx + r, f(0), f(W - 1))
        min_y = np.clip(my - r, f(0), f(H - 1))
        max_y = np.clip(my + r, f(0), f(H - 1))
        on_screen = (mx + r > 0) & (mx - r < W) & (my + r > 0) & (my - r < H)
    # NaNs are off-screen; give them a harmless rectangle before the int cast.
    bad = ~on_screen
    for a in (min_x, max_x, min_y, max_y):
        a[bad] = 0
    tmin_x = np.floor(min_x / f(TILE_SIZE)).astype(np.int32)
    tmax_x = np.floor(max_x / f(TILE_SIZE)).astype(np.int32)
    tmin_y = np.floor(min_y / f(TILE_SIZE)).astype(np.int32)
    tmax_y = np.floor(max_y / f(TILE_SIZE)).astype(np.int32)
    return tmin_x, tmax_x, tmin_y, tmax_y, on_screen


def _depth_key(depths: np.ndarray) -> np.ndarray:
    """rasterizer.py:93-94: bitcast(z) >> 18 (arithmetic)."""
    return depths.astype(np.float32).view(np.int32) >> (31 - DEPTH_BITS)


def get_tile_interactions(means2D, radii, valid_mask, depths, H, W):
    """rasterizer.py:12-116, literally: N*256 candidate slots, packed int32
    key, stable sort. Returns (sorted_tile_ids, sorted_gaussian_ids,
    n_valid) as numpy int32 arrays / int."""
    means2D = np.asarray(means2D, np.float32)
    radii = np.asarray(radii, np.float32)
    valid_mask = np.asarray(valid_mask, bool)
    depths = np.asarray(depths, np.float32)
    n = means2D.shape[0]
    ntx = (W + TILE_SIZE - 1) // TILE_SIZE
    nty = (H + TILE_SIZE - 1) // TILE_SIZE
    tmin_x, tmax_x, tmin_y, tmax_y, on_screen = _tile_rect(means2D, radii, H, W)
    valid = valid_mask & on_screen & (tmax_x >= tmin_x) & (tmax_y >= tmin_y)  # :51
    off_y, off_x = np.meshgrid(np.arange(OFFSET_SIZE), np.arange(OFFSET_SIZE), indexing="ij")  # :56
    off_x = off_x.reshape(-1).astype(np.int32)
    off_y = off_y.reshape(-1).astype(np.int32)
    abs_x = tmin_x[:, None] + off_x[None, :]  # :61-62
    abs_y = tmin_y[:, None] + off_y[None, :]
    in_range = (abs_x <= tmax_x[:, None]) & (abs_y <= tmax_y[:, None]) & valid[:, None]  # :65
    tile_ids = np.where(in_range, abs_y * ntx + abs_x, -1).astype(np.int32)  # :68-69
    gids = np.broadcast_to(np.arange(n, dtype=np.int32)[:, None], tile_ids.shape).reshape(-1)
    dq = np.broadcast_to(_depth_key(depths)[:, None], tile_ids.shape).reshape(-1)
    flat_tiles = tile_ids.reshape(-1)
    valid_int = flat_tiles != -1  # :79
    T = ntx * nty
    sort_tiles = np.where(valid_int, flat_tiles, T).astype(np.int32)  # :89
    key = (sort_tiles << DEPTH_BITS) | dq  # :98
    order = np.argsort(key, kind="stable")  # :101 lax.sort_key_val (stable)
    sorted_keys = key[order]
    sorted_gids = gids[order]
    sorted_tile_ids = sorted_keys >> DEPTH_BITS  # :104
    total = sorted_tile_ids.shape[0]
    padded = max(total, BLOCK_SIZE)  # :107-114
    out_t = np.full((padded,), T, np.int32)
    out_g = np.zeros((padded,), np.int32)
    out_t[:total] = sorted_tile_ids
    out_g[:total] = sorted_gids
    return out_t, out_g, int(valid_int.sum())


def get_tile_interactions_compact(means2D, radii, valid_mask, depths, H, W):
    """The valid segment of get_tile_interactions without materialising N*256
    slots: valid candidates in candidate order, then a stable sort on the same
    key. The reference's behind-camera entries (negative keys, tile -1) sort
    before and its sentinels after this segment, so the two agree on it."""
    means2D = np.asarray(means2D, np.float32)
    radii = np.asarray(radii, np.float32)
    valid_mask = np.asarray(valid_mask, bool)
    depths = np.asarray(depths, np.float32)
    ntx = (W + TILE_SIZE - 1) // TILE_SIZE
    tmin_x, tmax_x, tmin_y, tmax_y, on_screen = _tile_rect(means2D, radii, H, W)
    valid = valid_mask & on_screen & (tmax_x >= tmin_x) & (tmax_y >= tmin_y)
    nx = np.where(valid, np.minimum(tmax_x - tmin_x + 1, OFFSET_SIZE), 0).astype(np.int64)
    ny = np.where(valid, np.minimum(tmax_y - tmin_y + 1, OFFSET_SIZE), 0).astype(np.int64)
    cnt = nx * ny
    total = int(cnt.sum())
    g = np.repeat(np.arange(means2D.shape[0], dtype=np.int64), cnt)
    start = np.repeat(np.cumsum(cnt) - cnt, cnt)
    j = np.arange(total, dtype=np.int64) - start
    oy = j // nx[g]
    ox = j - oy * nx[g]
    tiles = ((tmin_y[g] + oy) * ntx + (tmin_x[g] + ox)).astype(np.int32)
    key = (tiles << DEPTH_BITS) | _depth_key(depths)[g]
    order = np.argsort(key, kind="stable")
    return (key[order] >> DEPTH_BITS).astype(np.int32), g[order].astype(np.int32), total


def tile_ranges(sorted_tile_ids: np.ndarray, num_tiles: int) -> np.ndarray:
    """rasterizer.py:159-160 / renderer.py:60: searchsorted(ids, arange(T+1))."""
    return np.searchsorted(sorted_tile_ids, np.arange(num_tiles + 1), side="left").astype(np.int32)


def render_tiles(means2D, cov2D, opacities, colors, sorted_tile_ids, sorted_gaussian_ids, H, W,
                 background=None, tile_subset=None):
    """rasterizer.py:119-248 (and rasterizer_tpu.py:13-135), differentiable in
    means2D, cov2D, opacities, colors. Per tile, all of its (<= 4096) splats
    are evaluated at once; the scan's transmittance is an exclusive cumprod of
    (1 - alpha), with alpha zeroed once T <= 1e-4 (rasterizer.py:206) -- T is
    non-increasing, so the cut found on the un-cut product is the scan's."""
    dt = means2D.dtype
    if background is None:
        background = torch.zeros(3, dtype=dt)
    ntx = (W + TILE_SIZE - 1) // TILE_SIZE
    nty = (H + TILE_SIZE - 1) // TILE_SIZE
    T_n = ntx * nty
    det = cov2D[:, 0, 0] * cov2D[:, 1, 1] - cov2D[:, 0, 1] ** 2  # :147-148
    det = torch.maximum(det, torch.tensor(1e-6, dtype=dt))
    ic00 = cov2D[:, 1, 1] / det  # :150-153
    ic01 = -cov2D[:, 0, 1] / det
    ic11 = cov2D[:, 0, 0] / det
    sig = torch.sigmoid(opacities[:, 0])  # :156
    tiles_np = np.asarray(sorted_tile_ids)
    gids_np = np.asarray(sorted_gaussian_ids)
    bounds = tile_ranges(tiles_np, T_n)  # :159-160
    py, px = np.mgrid[0:TILE_SIZE, 0:TILE_SIZE]
    out = torch.zeros((nty * TILE_SIZE, ntx * TILE_SIZE, 3), dtype=dt)
    tiles_out = []
    for t in (range(T_n) if tile_subset is None else tile_subset):
        s, e = int(bounds[t]), int(bounds[t + 1])
        count = min(e - s, MAX_TILE_INTERACTIONS)  # :171
        ty, tx = divmod(t, ntx)
        if count <= 0:  # :233-237 empty tile
            tiles_out.append((ty, tx, background.reshape(1, 3).expand(TILE_SIZE * TILE_SIZE, 3)))
            continue
        idx = torch.as_tensor(np.clip(gids_np[s:s + count], 0, means2D.shape[0] - 1).astype(np.int64))
        gx = torch.as_tensor((tx * TILE_SIZE + px).reshape(-1), dtype=dt) + 0.5  # :176-181
        gy = torch.as_tensor((ty * TILE_SIZE + py).reshape(-1), dtype=dt) + 0.5
        mu = means2D[idx]
        dx = gx[:, None] - mu[None, :, 0]
        dy = gy[:, None] - mu[None, :, 1]
        power = -0.5 * (dx * dx * ic00[idx][None] + dx * dy * (2.0 * ic01[idx])[None]
                        + dy * dy * ic11[idx][None])  # :210
        ea = torch.exp(power) * sig[idx][None]  # :211
        a_raw = torch.where(power > -10.0, torch.minimum(torch.tensor(0.99, dtype=dt), ea),
                            torch.zeros((), dtype=dt))  # :212
        ones = torch.ones((a_raw.shape[0], 1), dtype=dt)
        with torch.no_grad():
            T_raw = torch.cat([ones, torch.cumprod(1.0 - a_raw, dim=1)[:, :-1]], dim=1)
            active = T_raw > 1e-4  # :206
        alpha = torch.where(active, a_raw, torch.zeros((), dtype=dt))
        trans = torch.cat([ones, torch.cumprod(1.0 - alpha, dim=1)], dim=1)  # :213
        w = alpha * trans[:, :-1]
        col = w @ colors[idx]  # :214
        final = col + trans[:, -1:] * background[None, :]  # :230
        tiles_out.append((ty, tx, final))
    for ty, tx, val in tiles_out:
        out[ty * TILE_SIZE:(ty + 1) * TILE_SIZE, tx * TILE_SIZE:(tx + 1) * TILE_SIZE] = \
            val.reshape(TILE_SIZE, TILE_SIZE, 3)
    return out[:H, :W, :]  # :243-248


def render(means, scales, quats, opacities, sh, W2C, W, H, fx, fy, cx, cy, background=None,
           mask=None, sh_degree=0, compact_sort=True, tile_subset=None) -> Tuple[torch.Tensor, Dict]:
    """tile_subset (optional) composites only those tiles (others stay 0), to
    time a bounded sample of a large view."""
    """renderer.py:15-107. Returns (image, extras)."""
    dt = means.dtype
    if background is None:
        background = torch.zeros(3, dtype=dt)  # :31-32
    means2D, cov2D, radii, valid, z = project_gaussians(means, scales, quats, W2C, W, H, fx, fy,
                                                        cx, cy, mask)  # :36
    view_dirs = means - camera_center(W2C.to(dt))[None, :]  # :40-41
    view_dirs = view_dirs / torch.linalg.norm(view_dirs, dim=-1, keepdim=True)
    colors = _clip01(eval_sh(sh_degree, sh, view_dirs) + 0.5)  # :44-49
    m2 = means2D.detach().to(torch.float32).numpy()
    r = radii.detach().to(torch.float32).numpy()
    v = valid.numpy()
    d = z.detach().to(torch.float32).numpy()
    if compact_sort:
        tiles, gids, n_int = get_tile_interactions_compact(m2, r, v, d, H, W)
    else:
        tiles, gids, n_int = get_tile_interactions(m2, r, v, d, H, W)  # :53-55
    ntx = (W + TILE_SIZE - 1) // TILE_SIZE
    nty = (H + TILE_SIZE - 1) // TILE_SIZE
    T_n = ntx * nty
    bounds = tile_ranges(tiles, T_n)  # :60-61
    counts = (bounds[1:] - bounds[:-1]).astype(np.int64)
    tmin_x, tmax_x, tmin_y, tmax_y, on_screen = _tile_rect(m2, r, H, W)  # :63-72
    capped = ((tmax_x - tmin_x + 1) > OFFSET_SIZE) | ((tmax_y - tmin_y + 1) > OFFSET_SIZE)  # :73-74
    extras = {  # :79-90
        "radii": radii,
        "valid_mask": valid,
        "n_interactions": int(n_int),
        "mean_interactions_per_tile": float(np.float32(n_int) / np.float32(max(T_n, 1))),
        "max_interactions_per_tile": int(counts.max()) if counts.size else 0,
        "overflow_tiles": int((counts > BLOCK_SIZE).sum()),
        "overflow_interactions": int(np.maximum(counts - BLOCK_SIZE, 0).sum()),
        "truncated_tiles": int((counts > MAX_TILE_INTERACTIONS).sum()),
        "truncated_interactions": int(np.maximum(counts - MAX_TILE_INTERACTIONS, 0).sum()),
        "radius_cap_violations": int((capped & v & on_screen).sum()),
        "sorted_tile_ids": tiles,
        "sorted_gaussian_ids": gids,
        "tile_ranges": bounds,
    }
    image = render_tiles(means2D, cov2D, opacities, colors, tiles, gids, H, W, background,
                         tile_subset=tile_subset)  # :102-106
    return image, extras


# ---------------------------------------------------------------------------
# training/losses.py


def l1_loss(pred, target):
    """losses.py:4-8."""
    return torch.mean(torch.abs(pred - target))


def mse_loss(pred, target):
    """losses.py:10-14."""
    return torch.mean((pred - target) ** 2)


def _gauss_window(window_size=11, sigma=1.5, dtype=torch.float32):
    x = torch.arange(window_size, dtype=torch.float64) - window_size // 2  # losses.py:193-196
    k = torch.exp(-(x * x) / (2 * sigma ** 2)).to(dtype)
    return k / k.sum()


def ssim(img1, img2, window_size=11):
    """losses.py:16-69 (size_average=True). (H,W,C) images; separable blur,
    first along H then along W, SAME zero padding, per channel."""
    C = img1.shape[-1]
    k = _gauss_window(window_size, 1.5, img1.dtype)
    pad = window_size // 2
    wv = k.reshape(1, 1, window_size, 1).repeat(C, 1, 1, 1)
    wh = k.reshape(1, 1, 1, window_size).repeat(C, 1, 1, 1)

    def blur(img):
        x = img.permute(2, 0, 1)[None]
        x = torch.nn.functional.conv2d(x, wv, padding=(pad, 0), groups=C)
        x = torch.nn.functional.conv2d(x, wh, padding=(0, pad), groups=C)
        return x[0].permute(1, 2, 0)

    mu1, mu2 = blur(img1), blur(img2)
    mu1_sq, mu2_sq, mu1_mu2 = mu1 ** 2, mu2 ** 2, mu1 * mu2
    zero = torch.zeros((), dtype=img1.dtype)
    sigma1_sq = torch.maximum(zero, blur(img1 * img1) - mu1_sq)
    sigma2_sq = torch.maximum(zero, blur(img2 * img2) - mu2_sq)
    sigma12 = blur(img1 * img2) - mu1_mu2
    c1, c2 = 0.01 ** 2, 0.03 ** 2
    m = ((2 * mu1_mu2 + c1) * (2 * sigma12 + c2)) / ((mu1_sq + mu2_sq + c1) * (sigma1_sq + sigma2_sq + c2))
    m = torch.minimum(torch.maximum(m, torch.tensor(-1.0, dtype=m.dtype)), torch.tensor(1.0, dtype=m.dtype))
    return torch.mean(m)


def d_ssim_loss(pred, target):
    """losses.py:71-75."""
    return torch.maximum(torch.zeros((), dtype=pred.dtype), (1.0 - ssim(pred, target)) / 2.0)


# ---------------------------------------------------------------------------
# training/trainer.py + optax.adam (multi_transform of train.py:129-156)

GROUPS = ("means", "scales", "quaternions", "opacities", "sh_coeffs")


def adam_update(params: Dict[str, torch.Tensor], grads: Dict[str, torch.Tensor],
                mu: Dict[str, torch.Tensor], nu: Dict[str, torch.Tensor], count: int,
                lrs: Dict[str, float], active: torch.Tensor, b1=0.9, b2=0.999, eps=1e-8):
    """One optax.adam step per group (count = step number after increment),
    update masking of trainer.py:44-53 and apply_updates. Returns new
    (params, mu, nu)."""
    newp, newm, newv = {}, {}, {}
    # optax: 1 - decay ** count in float32 (decay a weakly typed Python float)
    f32 = lambda v: float(np.float32(v))  # noqa: E731
    bc1 = f32(1.0 - f32(f32(b1) ** count))
    bc2 = f32(1.0 - f32(f32(b2) ** count))
    for k in GROUPS:
        g = grads[k]
        m = (1 - b1) * g + b1 * mu[k]
        v = (1 - b2) * (g * g) + b2 * nu[k]
        u = -lrs[k] * ((m / bc1) / (torch.sqrt(v / bc2) + eps))
        am = active.reshape((-1,) + (1,) * (u.dim() - 1))
        u = torch.where(am, u, torch.zeros((), dtype=u.dtype))
        newp[k], newm[k], newv[k] = params[k] + u, m, v
    return newp, newm, newv


def train_step(params: Dict[str, torch.Tensor], mu, nu, count: int, lrs, active, target, W2C,
               camera_static, sh_degree=0, lambda_ssim=0.2, grad_accum=None, denom=None,
               max_radii=None, compact_sort=True, tile_subset=None):
    """trainer.py:125-169 (single device): loss, value_and_grad, Adam,
    masking, densification statistics. Returns a dict of everything.
    tile_subset (bounded CPU timing samples only) composites just those tiles."""
    W, H, fx, fy, cx, cy = camera_static
    p = {k: v.detach().clone().requires_grad_(True) for k, v in params.items()}
    image, extras = render(p["means"], p["scales"], p["quaternions"], p["opacities"], p["sh_coeffs"],
                           W2C, W, H, fx, fy, cx, cy, mask=active, sh_degree=sh_degree,
                           compact_sort=compact_sort, tile_subset=tile_subset)
    l1 = l1_loss(image, target)
    dssim = d_ssim_loss(image, target)
    loss = (1.0 - lambda_ssim) * l1 + lambda_ssim * dssim  # trainer.py:26
    loss.backward()
    grads = {k: p[k].grad.detach() for k in GROUPS}
    newp, newm, newv = adam_update(params, grads, mu, nu, count, lrs, active)
    # trainer.py:143-159
    dt = params["means"].dtype
    Wm = W2C.to(dt)
    m = params["means"]
    z = ((Wm[2, 0] * m[:, 0] + Wm[2, 1] * m[:, 1]) + Wm[2, 2] * m[:, 2]) + Wm[2, 3]
    z = torch.maximum(z, torch.tensor(0.01, dtype=dt))
    focal = (fx + fy) / 2.0
    g2d = torch.linalg.norm(grads["means"], dim=-1) * (z / focal) * (float(W) * float(H) * 3.0)
    out = {"image": image.detach(), "extras": extras, "loss": float(loss.detach()),
           "l1": float(l1.detach()), "ssim": float(1.0 - dssim.detach() * 2.0), "grads": grads, "params": newp, "mu": newm, "nu": newv,
           "grad_2d_mag": g2d}
    if grad_accum is not None:
        valid = extras["valid_mask"]
        out["grad_accum"] = grad_accum + g2d
        out["denom"] = denom + (valid & active).to(denom.dtype)
        out["max_radii"] = torch.where(valid, torch.maximum(max_radii, extras["radii"].detach()), max_radii)
    return out


def exponential_decay(init_value: float, transition_steps: int, decay_rate: float, count: int) -> float:
    """optax.exponential_decay (no staircase, no transition_begin)."""
    return init_value * decay_rate ** (count / transition_steps)


# ---------------------------------------------------------------- density control
def _stable_argsort(x: np.ndarray) -> np.ndarray:
    """jnp.argsort (stable=True by default) on a 1-D integer array."""
    return np.argsort(x, kind="stable")


def densify_and_prune(params: Dict[str, torch.Tensor], mu: Dict[str, torch.Tensor],
                      nu: Dict[str, torch.Tensor], active: np.ndarray, grad_accum: np.ndarray,
                      denom: np.ndarray, max_radii: np.ndarray, noise: np.ndarray,
                      densify_enabled: bool = True, grad_threshold: float = 0.0002,
                      min_opacity: float = 0.005, extent: float = 5.0, max_screen_size: int = 512):
    """jax_gs/training/density.py:98-211, literally (argsort-based routing).

    params / mu / nu: dicts over GROUPS of (N, ...) float32 tensors (mu / nu
    are the Adam moments of every group, reordered like the parameters,
    density.py:62-69). noise (N, 3) float32 stands for
    jax.random.normal(rng_key, (N, 3)) (density.py:188). Returns new
    (params, mu, nu, active, grad_accum, denom, max_radii, info)."""
    f32 = np.float32
    g = {k: v.detach().cpu().numpy().astype(f32) for k, v in params.items()}
    N = active.shape[0]
    # 1. prune (density.py:114-128)
    sig_ops = (1.0 / (1.0 + np.exp(-g["opacities"][:, 0].astype(np.float64)))).astype(f32)
    prune = sig_ops < f32(min_opacity)
    max_scales = np.exp(g["scales"].astype(np.float64)).astype(f32).max(axis=-1)
    # JAX compares a float32 array with the Python product 0.1 * extent as float32
    prune = prune | (max_scales > f32(0.1 * extent))
    prune = prune | (max_radii > max_screen_size)
    prune = prune & active
    active_after_prune = active & ~prune
    # 2. densify (density.py:130-135)
    with np.errstate(divide="ignore", invalid="ignore"):
        avg = np.where(denom > 0, grad_accum / np.maximum(denom, 1).astype(f32), f32(0.0)).astype(f32)
    densify = (avg >= f32(grad_threshold)) & active_after_prune
    split = densify & (max_scales > f32(0.01 * extent))
    clone = densify & ~split
    # capacity (density.py:141-151)
    will_be_empty = ~active_after_prune
    can = (int(clone.sum()) + int(split.sum()) <= int(will_be_empty.sum())) and densify_enabled
    if not can:
        clone = np.zeros_like(clone)
        split = np.zeros_like(split)
    nc, ns = int(clone.sum()), int(split.sum())
    # routing (density.py:153-169)
    empty_idx = _stable_argsort((~will_be_empty).astype(np.int8))
    clone_src = _stable_argsort((~clone).astype(np.int8))
    split_src = _stable_argsort((~split).astype(np.int8))
    idx = np.arange(N)
    is_clone_dest = idx < nc
    is_split_dest = (idx >= nc) & (idx < nc + ns)
    src = np.where(is_clone_dest, clone_src[idx], 0)
    src = np.where(is_split_dest, split_src[np.clip(idx - nc, 0, N - 1)], src)
    new_values = np.where(is_clone_dest | is_split_dest, src, empty_idx)
    gather = np.arange(N)
    gather[empty_idx] = new_values
    # data movement (density.py:171-181)
    out = {k: v[gather] for k, v in g.items()}
    mu2 = {k: v.detach().cpu().numpy()[gather] for k, v in mu.items()}
    nu2 = {k: v.detach().cpu().numpy()[gather] for k, v in nu.items()}
    # modifications (density.py:183-190)
    new_split = np.zeros(N, bool)
    new_split[empty_idx] = is_split_dest
    do_split = split | new_split
    # jnp.log(1.6) on float32(1.6), correctly rounded (numpy's float32 log is
    # one ulp off here; XLA's rounding of it is not pinned)
    log16 = f32(np.log(np.float64(f32(1.6))))
    out["scales"] = np.where(do_split[:, None], (out["scales"] - log16).astype(f32), out["scales"])
    scaled_noise = (noise.astype(f32) * np.exp(out["scales"].astype(np.float64)).astype(f32)).astype(f32)
    out["means"] = np.where(do_split[:, None], (out["means"] + scaled_noise).astype(f32), out["means"])
    # masks (density.py:192-195), accumulators (density.py:58-62, 206)
    add = np.zeros(N, bool)
    add[empty_idx] = is_clone_dest | is_split_dest
    final_active = active_after_prune | add
    t = lambda a: torch.tensor(a)  # noqa: E731
    info = {"pruned": int(prune.sum()), "clones": nc, "splits": ns, "applied": bool(nc + ns > 0)}
    return ({k: t(v) for k, v in out.items()}, {k: t(v) for k, v in mu2.items()},
            {k: t(v) for k, v in nu2.items()}, final_active, np.zeros_like(grad_accum),
            np.zeros_like(denom), max_radii.copy(), info)


def reset_opacities(params: Dict[str, torch.Tensor], active: np.ndarray, reset_val: float = 0.01):
    """density.py:76-96: active opacities set to logit(reset_val): the quotient
    in Python double, then jnp.log in float32 (correctly rounded here)."""
    inv = np.float32(np.log(np.float64(np.float32(reset_val / (1.0 - reset_val)))))
    ops = params["opacities"].detach().cpu().numpy().copy()
    ops[active, 0] = inv
    out = dict(params)
    out["opacities"] = torch.tensor(ops)
    return out
