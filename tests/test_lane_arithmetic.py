"""Lane-level restatements of the warp-level and index arithmetic the kernels
rely on, checked exhaustively or on random inputs on the CPU:

* the pair emitter's tile offset j / nx by one float multiply
  (gs_sort.cu: k_emit_keys, k_emit_sorted);
* the compositors' pixel ownership (gs_raster.cu: Foot<PIX, WX>; gs_2dgs.cu:
  the same layout with k2Pix = 2, k2Wx = 8);
* the transposed warp reductions warp_sum9 (gs_raster.cu) and warp_sum16
  (gs_2dgs.cu), and the sort's same_value_lanes (gs_sort.cu), with
  __shfl_xor_sync / __ballot_sync emulated over 32 lanes.
"""
import numpy as np
import pytest

LANES = np.arange(32)


def test_emit_tile_offset_division_is_exact():
    """oy = (int)((j + 0.5f) * rcp(nx)) equals j / nx for every pair index
    j < nx * ny of a Gaussian (nx, ny <= 16), with float32 rounding of the
    reciprocal and of the product as __frcp_rn / __fmul_rn do."""
    f = np.float32
    for nx in range(1, 17):
        r = f(1) / f(nx)  # correctly rounded, as __frcp_rn
        j = np.arange(nx * 16)
        oy = ((j.astype(f) + f(0.5)) * r).astype(f).astype(np.int64)
        np.testing.assert_array_equal(oy, j // nx)
        np.testing.assert_array_equal(j - oy * nx, j % nx)


@pytest.mark.parametrize("pix,wx", [(2, 8), (1, 8), (1, 16), (2, 16), (4, 8), (4, 16)])
def test_pixel_ownership_is_a_bijection(pix, wx):
    """Foot<PIX, WX>: thread (warp, lane) owns the column col(warp, lane) and
    rows row0 .. row0 + PIX - 1 of the 16x16 tile; every pixel has exactly one
    owner, and warp w's pixels form the WX x WY block that warp_mask tests."""
    tile, nt = 16, 256 // pix
    nw, wy, wpr = nt // 32, 32 * pix // wx, tile // wx
    owner = -np.ones((tile, tile), np.int64)
    for warp in range(nw):
        for lane in range(32):
            col = (warp % wpr) * wx + lane % wx
            row0 = (warp // wpr) * wy + (lane // wx) * pix
            for i in range(pix):
                assert owner[row0 + i, col] == -1
                owner[row0 + i, col] = warp
    assert (owner >= 0).all()
    for warp in range(nw):
        ys, xs = np.nonzero(owner == warp)
        x0, y0 = (warp % wpr) * wx, (warp // wpr) * wy
        assert xs.min() == x0 and xs.max() == x0 + wx - 1
        assert ys.min() == y0 and ys.max() == y0 + wy - 1


def _shfl_xor(v, o):
    return v[LANES ^ o]


def _halve(v, n_keep, bit):
    """One transposed-reduction stage: lanes with `bit` set keep the upper
    n_keep values and send the lower ones, the others the reverse."""
    h = (LANES & bit) != 0
    out = np.empty((32, n_keep), v.dtype)
    for i in range(n_keep):
        send = np.where(h, v[:, i], v[:, i + n_keep])
        keep = np.where(h, v[:, i + n_keep], v[:, i])
        out[:, i] = keep + _shfl_xor(send, bit)
    return out


def test_warp_sum9_postcondition():
    """warp_sum9: lanes 4i .. 4i + 3 hold the total of value i (i < 8) in
    v[0]; every lane holds the total of value 8 in v[8]."""
    rng = np.random.default_rng(0)
    for _ in range(20):
        v = rng.integers(-1000, 1000, (32, 9))
        tot = v.sum(0)
        a = _halve(v[:, :8], 4, 16)
        a = _halve(a, 2, 8)
        a = _halve(a, 1, 4)[:, 0]
        a = a + _shfl_xor(a, 2)
        a = a + _shfl_xor(a, 1)
        np.testing.assert_array_equal(a, tot[LANES >> 2])
        b = v[:, 8].copy()
        for o in (16, 8, 4, 2, 1):
            b = b + _shfl_xor(b, o)
        np.testing.assert_array_equal(b, np.full(32, tot[8]))


def test_warp_sum16_postcondition():
    """warp_sum16: lane l holds the total of value l >> 1 in v[0], so the even
    lanes 2i add value i (i < 13 gradients) to the CTA's accumulator."""
    rng = np.random.default_rng(1)
    for _ in range(20):
        v = rng.integers(-1000, 1000, (32, 16))
        tot = v.sum(0)
        a = _halve(v, 8, 16)
        a = _halve(a, 4, 8)
        a = _halve(a, 2, 4)
        a = _halve(a, 1, 2)[:, 0]
        a = a + _shfl_xor(a, 1)
        np.testing.assert_array_equal(a, tot[LANES >> 1])


def _ballot(pred):
    return int(sum(1 << int(l) for l in LANES[pred]))


@pytest.mark.parametrize("nbits", [1, 5, 8, 9])
def test_same_value_lanes(nbits):
    """same_value_lanes(d, nbits): the mask of lanes holding the same d, for
    d < 2^nbits, from one ballot per bit."""
    rng = np.random.default_rng(nbits)
    for _ in range(50):
        d = rng.integers(0, 1 << nbits, 32)
        if rng.random() < 0.3:
            d = rng.integers(0, min(3, 1 << nbits), 32)  # many equal digits
        m = np.full(32, 0xFFFFFFFF, np.int64)
        for b in range(nbits):
            bit = ((d >> b) & 1).astype(bool)
            v = _ballot(bit)
            m &= np.where(bit, v, ~v & 0xFFFFFFFF)
        for lane in range(32):
            assert m[lane] == _ballot(d == d[lane])
