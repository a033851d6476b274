"""The compositors skip a splat for a warp's 8x8 pixel block when
`splat_meets_rect` (jax-gs_b200/csrc/gs_common.cuh) says that its exponent
cannot exceed -10 at any pixel centre of the block. That skip is exact only if
the test never rejects a block where the compositor's own float32 exponent
(splat_q0 / splat_q1 / splat_power, gs_common.cuh) is above -10 somewhere:
there alpha would be non-zero (rasterizer.py:205-211 applies a splat where
power > -10).

This CPU test restates the device function in numpy float32 (one rounding per
operation; the device's `__fdividef` is a correctly rounded division here, a
difference the test's margin covers) and checks it against the compositor's
exponent evaluated at all 64 pixel centres, on random splats and on splats
placed so that their exponent at a block-edge pixel is within 0.05 of -10.
"""
import numpy as np

f = np.float32


def meets_rect(mx, my, ha, hb, hc, x0, x1, y0, y1):
    """splat_meets_rect, vectorised (gs_common.cuh)."""
    with np.errstate(all="ignore"):
        keep = ~((ha < 0) & (hc < 0) & (f(4) * ha * hc > hb * hb))
        keep |= ~(np.abs(mx) < f(1e30)) | ~(np.abs(my) < f(1e30))
        lx, ux, ly, uy = x0 - mx, x1 - mx, y0 - my, y1 - my
        ex = np.minimum(np.maximum(f(0), lx), ux)
        ey = np.minimum(np.maximum(f(0), ly), uy)
        inside = (ex == 0) & (ey == 0)
        best = np.full(mx.shape, -np.inf, f)
        dy = np.minimum(np.maximum((-hb * ex) / (f(2) * hc), ly), uy)
        b1 = (ha * ex + hb * dy) * ex + hc * dy * dy
        best = np.where(ex != 0, np.maximum(best, b1), best)
        dx = np.minimum(np.maximum((-hb * ey) / (f(2) * ha), lx), ux)
        b2 = (ha * dx + hb * ey) * dx + hc * ey * ey
        best = np.where(ey != 0, np.maximum(best, b2), best)
        DX = np.maximum(np.abs(lx), np.abs(ux))
        DY = np.maximum(np.abs(ly), np.abs(uy))
        mag = (np.abs(hb) * DY - ha * DX) * DX - hc * DY * DY
        slope = np.abs(hb) * (DX + DY) - f(2) * (ha * DX + hc * DY)
        ok = ~(best <= f(-10.05) - f(1e-4) * mag - f(1e-3) * slope)
    return keep | inside | ok


def _fma(a, b, c):
    """fmaf for float32 operands: the product is exact in float64, then one
    float64 rounding of the sum and one to float32."""
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(f)


def block_max_power(mx, my, ha, hb, hc, x0, y0):
    """The compositor's exponent (splat_q0, splat_q1, splat_power) maximised
    over the 64 pixel centres (x0 + i, y0 + j), i, j < 8."""
    best = np.full(mx.shape, -np.inf, f)
    for j in range(8):
        dy = (y0 + f(j)) - my
        for i in range(8):
            dx = (x0 + f(i)) - mx
            q0 = (dx * dx) * ha
            q1 = dx * hb
            best = np.maximum(best, _fma(dy, _fma(dy, hc, q1), q0))
    return best


def _conics(rng, n):
    """Halved conics (ha, hb, hc) = -(a, 2 b, c) / 2 of random 2D covariances
    (eigenvalues 0.3 .. 1.3e4 px^2, any orientation), as k_preprocess_fwd
    writes them: inverse with the det clamp, then the halving."""
    l1 = (0.3 + np.exp(rng.uniform(-1, 9.5, n))).astype(f)
    l2 = (0.3 + np.exp(rng.uniform(-1, 9.5, n))).astype(f)
    th = rng.uniform(0, np.pi, n)
    c, s = np.cos(th), np.sin(th)
    c00 = (l1 * c * c + l2 * s * s).astype(f)
    c11 = (l1 * s * s + l2 * c * c).astype(f)
    c01 = ((l1 - l2) * c * s).astype(f)
    det = np.maximum(c00 * c11 - c01 * c01, f(1e-6))
    ia, i01, ic = c11 / det, -c01 / det, c00 / det
    return f(-0.5) * ia, -i01, f(-0.5) * ic, np.maximum(l1, l2)


def _check(mx, my, ha, hb, hc, x0, y0):
    kept = meets_rect(mx, my, ha, hb, hc, x0, x0 + f(7), y0, y0 + f(7))
    mp = block_max_power(mx, my, ha, hb, hc, x0, y0)
    wrong = (~kept) & (mp > f(-10))
    assert not wrong.any(), (f"{int(wrong.sum())} blocks culled with a pixel above -10, e.g. "
                             f"mean ({mx[wrong][0]}, {my[wrong][0]}) block ({x0[wrong][0]}, {y0[wrong][0]})")
    return kept, mp


def test_random_splats_are_never_culled_wrongly():
    rng = np.random.default_rng(1)
    n = 100_000
    ha, hb, hc, lmax = _conics(rng, n)
    x0 = rng.integers(0, 4000, n).astype(f) + f(0.5)
    y0 = rng.integers(0, 4000, n).astype(f) + f(0.5)
    r = np.sqrt(20 * lmax) * 1.2 + 8
    mx = (x0 + f(3.5) + rng.uniform(-1, 1, n) * r).astype(f)
    my = (y0 + f(3.5) + rng.uniform(-1, 1, n) * r).astype(f)
    kept, mp = _check(mx, my, ha, hb, hc, x0, y0)
    # the test has teeth: many blocks are culled, and most blocks whose
    # exponent stays below -10 everywhere are
    assert (~kept).mean() > 0.2
    assert (~kept).sum() > 0.8 * (mp <= f(-10)).sum()


def test_splats_at_the_threshold_are_never_culled_wrongly():
    rng = np.random.default_rng(2)
    n = 100_000
    ha, hb, hc, _ = _conics(rng, n)
    x0 = rng.integers(0, 4000, n).astype(f) + f(0.5)
    y0 = rng.integers(0, 4000, n).astype(f) + f(0.5)
    # a pixel centre on the block's border, and a mean outside the block in a
    # random outward direction at which the exponent there is -10 + delta
    edge = rng.integers(0, 4, n)
    k = rng.integers(0, 8, n).astype(f)
    px = np.where(edge == 0, f(0), np.where(edge == 1, f(7), k)) + x0
    py = np.where(edge == 2, f(0), np.where(edge == 3, f(7), k)) + y0
    ang = rng.uniform(0, 2 * np.pi, n)
    ux, uy = np.cos(ang), np.sin(ang)
    out = np.where(edge == 0, ux < 0, np.where(edge == 1, ux > 0, np.where(edge == 2, uy < 0, uy > 0)))
    ux, uy = np.where(out, ux, -ux), np.where(out, uy, -uy)
    # power(t u) = t^2 power(u) for the mean at pixel - t u
    pu = ha.astype(np.float64) * ux * ux + hb.astype(np.float64) * ux * uy + hc.astype(np.float64) * uy * uy
    delta = rng.uniform(-0.05, 0.05, n)
    t = np.sqrt((-10.0 + delta) / pu)
    mx = (px - t * ux).astype(f)
    my = (py - t * uy).astype(f)
    kept, mp = _check(mx, my, ha, hb, hc, x0, y0)
    near = np.abs(mp + f(10)) < f(0.05)
    assert near.sum() > 1000  # the cases do sit at the threshold
