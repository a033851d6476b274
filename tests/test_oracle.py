"""CPU tests of the oracle (oracle/ref_restated.py).

The reference cannot run here (JAX is not installed), so the oracle is pinned
by the reference's own known-answer tests, restated against it:
tests/test_renderer.py:11-33 (projection), :35-51 (tile interactions),
:53-76 and :78-113 (red centre),
:115-158 (analytic chunked compositing, both rasterisers),
tests/test_core.py:21-38 (covariance symmetric PSD),
tests/test_training.py:9-38 (loss values) -- plus finite differences for the
gradients and the committed golden fixtures for drift.
"""
import os

import numpy as np
import pytest
import torch

from oracle import ref_restated as R
from tests.helpers import oracle_render, random_scene, to_torch

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _pcd_gaussian(mean, color):
    """init_gaussians_from_pcd for one point (gaussians.py:13-56)."""
    means = torch.tensor([mean], dtype=torch.float32)
    scales = torch.full((1, 3), -3.0)
    quats = torch.tensor([[1.0, 0.0, 0.0, 0.0]])
    opac = torch.zeros((1, 1))
    sh = torch.zeros((1, 16, 3))
    sh[:, 0, :] = (torch.tensor([color]) - 0.5) / 0.28209479177387814
    return means, scales, quats, opac, sh


def test_projection_known_answer():
    # tests/test_renderer.py:11-33
    means, scales, quats, _, _ = _pcd_gaussian([0.0, 0.0, 5.0], [1.0, 1.0, 1.0])
    m2, cov, radii, valid, z = R.project_gaussians(means, scales, quats, torch.eye(4), 100, 100, 50.0,
                                                   50.0, 50.0, 50.0)
    assert torch.allclose(m2[0], torch.tensor([50.0, 50.0]))
    assert bool(valid[0])
    assert float(z[0]) == 5.0
    assert float(radii[0]) > 0


def test_tile_interactions_known_answer():
    # tests/test_renderer.py:35-51, with the exact answer: a radius-4 splat at
    # (16, 16) covers pixels 12..20 of a 32x32 image, so all four tiles; a
    # radius-2 splat at (0, 0) covers tile 0 only; tile 0 lists the nearer
    # first; the output is padded to BLOCK_SIZE with the sentinel tile T = 4.
    t, g, n = R.get_tile_interactions(np.array([[16.0, 16.0], [0.0, 0.0]]), np.array([4, 2]),
                                      np.array([True, True]), np.array([5.0, 10.0]), 32, 32)
    assert n == 5 and len(t) == 512
    np.testing.assert_array_equal(t[:5], [0, 0, 1, 2, 3])
    np.testing.assert_array_equal(g[:5], [0, 1, 0, 0, 0])
    assert (t[5:] == 4).all()
    tc, gc, nc = R.get_tile_interactions_compact(np.array([[16.0, 16.0], [0.0, 0.0]]), np.array([4.0, 2.0]),
                                                 np.array([True, True]), np.array([5.0, 10.0]), 32, 32)
    assert nc == 5
    np.testing.assert_array_equal(np.asarray(tc)[:5], t[:5])
    np.testing.assert_array_equal(np.asarray(gc)[:5], g[:5])


def test_covariance_symmetric_psd():
    # tests/test_core.py:21-38
    rng = np.random.default_rng(0)
    scales = torch.tensor(rng.uniform(-1, 1, (10, 3)), dtype=torch.float32)
    q = torch.tensor(rng.uniform(-1, 1, (10, 4)), dtype=torch.float32)
    q = q / torch.linalg.norm(q, dim=-1, keepdim=True)
    cov = R.get_covariance_3d(scales, q)
    assert cov.shape == (10, 3, 3)
    for i in range(10):
        np.testing.assert_allclose(cov[i].numpy(), cov[i].T.numpy(), atol=1e-6)
        assert (torch.linalg.eigvalsh(cov[i].double()) >= -1e-7).all()


def test_rasterization_red_centre():
    # tests/test_renderer.py:53-76
    img = R.render_tiles(torch.tensor([[16.0, 16.0]]), torch.tensor([[[10.0, 0.0], [0.0, 10.0]]]),
                         torch.tensor([[10.0]]), torch.tensor([[1.0, 0.0, 0.0]]),
                         np.array([0, 1, 2, 3], np.int32), np.array([0, 0, 0, 0], np.int32), 32, 32,
                         torch.zeros(3))
    assert img.shape == (32, 32, 3)
    assert float(img[16, 16, 0]) > 0.5
    assert float(img[16, 16, 1]) < 0.1


def test_full_render_red_centre():
    # tests/test_renderer.py:78-113
    means, _, quats, _, sh = _pcd_gaussian([0.0, 0.0, 5.0], [1.0, 0.0, 0.0])
    img, _ = R.render(means, torch.full((1, 3), -1.0), quats, torch.tensor([[10.0]]), sh, torch.eye(4),
                      64, 64, 100.0, 100.0, 32.0, 32.0)
    u8 = (img.numpy() * 255).astype(np.uint8)
    assert u8[32, 32, 0] > 200
    assert u8[32, 32, 1] < 50


def analytic_case():
    """tests/test_renderer.py:115-158 inputs and the reference's NumPy answer."""
    n = R.BLOCK_SIZE + 8
    means2D = np.tile(np.array([[8.0, 8.0]], np.float32), (n, 1))
    cov2D = np.tile(np.array([[[6.0, 0.0], [0.0, 6.0]]], np.float32), (n, 1, 1))
    opac = np.full((n, 1), -1.5, np.float32)
    colors = np.stack([np.linspace(0, 1, n, dtype=np.float32), np.linspace(1, 0, n, dtype=np.float32),
                       np.zeros(n, np.float32)], -1)
    tiles = np.zeros(n, np.int32)
    gids = np.arange(n, dtype=np.int32)
    pixel = np.array([8.5, 8.5], np.float32)
    delta = pixel - means2D[0]
    power = -0.5 * float(delta @ np.linalg.inv(cov2D[0]) @ delta)
    alpha = min(0.99, float(np.exp(power) * (1.0 / (1.0 + np.exp(1.5)))))
    ref = np.zeros(3, np.float32)
    T = 1.0
    for c in colors:
        ref += alpha * T * c
        T *= 1.0 - alpha
    return means2D, cov2D, opac, colors, tiles, gids, ref


def test_chunked_rasterization_matches_reference():
    # tests/test_renderer.py:115-158 (render_tiles and render_tiles_tpu share the oracle)
    means2D, cov2D, opac, colors, tiles, gids, ref = analytic_case()
    img = R.render_tiles(torch.tensor(means2D), torch.tensor(cov2D), torch.tensor(opac),
                         torch.tensor(colors), tiles, gids, 16, 16, torch.zeros(3))
    np.testing.assert_allclose(img[8, 8].numpy(), ref, atol=1e-4, rtol=1e-4)


def test_losses_known_values():
    # tests/test_training.py:9-19 and :21-38
    pred = torch.tensor([1.0, 2.0, 3.0])
    target = torch.tensor([1.1, 1.9, 3.0])
    assert torch.allclose(R.l1_loss(pred, target), torch.tensor(0.06666667))
    assert torch.allclose(R.mse_loss(pred, target), torch.tensor(0.00666667))
    g = torch.Generator().manual_seed(0)
    t = torch.rand((32, 32, 3), generator=g)
    p = t + 0.1 * torch.rand((32, 32, 3), generator=g)
    s = R.ssim(p, t)
    d = R.d_ssim_loss(p, t)
    assert 0 <= float(s) <= 1 and 0 <= float(d) <= 1
    assert torch.allclose(d, (1.0 - s) / 2.0)
    assert torch.allclose(R.ssim(t, t), torch.tensor(1.0))
    assert torch.allclose(R.d_ssim_loss(t, t), torch.tensor(0.0))


@pytest.mark.parametrize("seed", [0, 1])
def test_compact_sort_equals_reference_layout(seed):
    """The compact restatement equals the literal N*256-slot sort on its valid
    segment (behind-camera entries first, sentinels last)."""
    sc = random_scene(seed, 300, 96, 80, behind=0.2, mask_frac=0.2)
    t = to_torch(sc)
    m2, _, radii, valid, z = R.project_gaussians(t["means"], t["scales"], t["quats"], t["w2c"], sc["W"],
                                                 sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"],
                                                 t["active"])
    args = (m2.numpy(), radii.numpy(), valid.numpy(), z.numpy(), sc["H"], sc["W"])
    full_t, full_g, n_full = R.get_tile_interactions(*args)
    c_t, c_g, n_c = R.get_tile_interactions_compact(*args)
    assert n_full == n_c > 0
    T = ((sc["W"] + 15) // 16) * ((sc["H"] + 15) // 16)
    seg = (full_t >= 0) & (full_t < T)
    assert seg.sum() == n_c
    lo = int(np.argmax(seg))
    np.testing.assert_array_equal(full_t[lo:lo + n_c], c_t)
    np.testing.assert_array_equal(full_g[lo:lo + n_c], c_g)
    assert (full_t[:lo] == -1).all()
    assert (full_t[lo + n_c:] == T).all()


def test_oracle_gradients_finite_differences():
    """Directional derivatives of a linear image functional, autograd (fp64)
    against central differences (fp64)."""
    sc = random_scene(3, 40, 48, 40, sh_degree=3, behind=0.0, scale_mu=-2.2, scale_sd=0.3)
    rng = np.random.default_rng(7)
    wimg = torch.tensor(rng.standard_normal((40, 48, 3)))
    img, _, t = oracle_render(sc, dtype=torch.float64, requires_grad=True)
    (img * wimg).sum().backward()
    names = ("means", "scales", "quats", "opac", "sh")
    dirs = {k: torch.tensor(rng.standard_normal(t[k].shape)) for k in names}
    ana = sum(float((t[k].grad * dirs[k]).sum()) for k in names)
    eps = 1e-6

    def f(sign):
        sc2 = dict(sc)
        for k in names:
            sc2[k] = (t[k].detach() + sign * eps * dirs[k]).numpy()
        im, _, _ = oracle_render(sc2, dtype=torch.float64)
        return float((im * wimg).sum())

    num = (f(1) - f(-1)) / (2 * eps)
    assert abs(ana - num) <= 1e-5 * max(1.0, abs(num)), (ana, num)


def test_golden_fixture_reproduces():
    """The committed golden fixture (tests/golden/make_golden.py) is reproduced."""
    path = os.path.join(GOLDEN, "scene_small.npz")
    g = np.load(path)
    sc = {k: g["in_" + k] for k in ("means", "scales", "quats", "opac", "sh", "w2c", "active")}
    for k in ("W", "H", "sh_degree"):
        sc[k] = int(g["cfg_" + k])
    for k in ("fx", "fy", "cx", "cy"):
        sc[k] = float(g["cfg_" + k])
    img, ex, t = oracle_render(sc, requires_grad=True)
    np.testing.assert_array_equal(ex["sorted_tile_ids"], g["out_tiles"])
    np.testing.assert_array_equal(ex["sorted_gaussian_ids"], g["out_gids"])
    np.testing.assert_array_equal(ex["tile_ranges"], g["out_ranges"])
    np.testing.assert_array_equal(ex["radii"].detach().numpy(), g["out_radii"])
    np.testing.assert_allclose(img.detach().numpy(), g["out_image"], atol=1e-6)
    (img * torch.tensor(g["grad_weights"])).sum().backward()
    for k in ("means", "scales", "quats", "opac", "sh"):
        ref = g["grad_" + k]
        np.testing.assert_allclose(t[k].grad.numpy(), ref, atol=1e-5 * max(1.0, float(np.abs(ref).max())))


def _numpy_projection(sc):
    """Independent float32 numpy evaluation of projection.py:21-79 in the
    oracle's fixed order (numpy rounds every operation, IEEE)."""
    f = np.float32
    q, s, m, W = (sc[k].astype(f) for k in ("quats", "scales", "means", "w2c"))
    n2 = ((q[:, 0] * q[:, 0] + q[:, 1] * q[:, 1]) + q[:, 2] * q[:, 2]) + q[:, 3] * q[:, 3]
    nr = np.sqrt(n2)
    r, x, y, z = q[:, 0] / nr, q[:, 1] / nr, q[:, 2] / nr, q[:, 3] / nr
    two, one = f(2), f(1)
    Rm = np.stack([np.stack([one - two * (y * y) - two * (z * z), (two * x) * y - (two * r) * z, (two * x) * z + (two * r) * y], -1),
                   np.stack([(two * x) * y + (two * r) * z, one - two * (x * x) - two * (z * z), (two * y) * z - (two * r) * x], -1),
                   np.stack([(two * x) * z - (two * r) * y, (two * y) * z + (two * r) * x, one - two * (x * x) - two * (y * y)], -1)], -2)
    M = Rm * np.exp(s.astype(np.float64)).astype(f)[:, None, :]
    S = np.stack([np.stack([(M[:, i, 0] * M[:, j, 0] + M[:, i, 1] * M[:, j, 1]) + M[:, i, 2] * M[:, j, 2]
                            for j in range(3)], -1) for i in range(3)], -2)
    X, Y, Z = [((W[k, 0] * m[:, 0] + W[k, 1] * m[:, 1]) + W[k, 2] * m[:, 2]) + W[k, 3] for k in range(3)]
    iz = one / np.maximum(Z, f(0.01))
    iz2 = iz * iz
    fx, fy, cx, cy = f(sc["fx"]), f(sc["fy"]), f(sc["cx"]), f(sc["cy"])
    J00, J02, J11, J12 = fx * iz, ((-fx) * X) * iz2, fy * iz, ((-fy) * Y) * iz2
    Mj = [[J00 * W[0, k] + J02 * W[2, k] for k in range(3)], [J11 * W[1, k] + J12 * W[2, k] for k in range(3)]]
    T = [[(Mj[i][0] * S[:, 0, k] + Mj[i][1] * S[:, 1, k]) + Mj[i][2] * S[:, 2, k] for k in range(3)] for i in range(2)]
    cov = [[(T[i][0] * Mj[j][0] + T[i][1] * Mj[j][1]) + T[i][2] * Mj[j][2] for j in range(2)] for i in range(2)]
    c00, c01, c10, c11 = cov[0][0] + f(0.3), cov[0][1], cov[1][0], cov[1][1] + f(0.3)
    det = c00 * c11 - c01 * c01
    mid = (c00 + c11) / f(2)
    rad = np.ceil(f(3) * np.sqrt(mid + np.sqrt(np.maximum(mid * mid - det, f(0)))))
    means2D = np.stack([(fx * X) / Z + cx, (fy * Y) / Z + cy], -1)
    return means2D, np.stack([np.stack([c00, c01], -1), np.stack([c10, c11], -1)], -2), rad, Z


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_oracle_projection_is_ieee_exact(seed):
    """The oracle's projection equals an independent numpy float32 evaluation
    bit for bit (the property the CUDA bit-exactness tests rely on)."""
    sc = random_scene(seed, 3000, 96, 80, sh_degree=3, behind=0.15, mask_frac=0.2)
    t = to_torch(sc)
    o = R.project_gaussians(t["means"], t["scales"], t["quats"], t["w2c"], sc["W"], sc["H"], sc["fx"],
                            sc["fy"], sc["cx"], sc["cy"], t["active"])
    with np.errstate(all="ignore"):
        ref = _numpy_projection(sc)
    for a, b in ((ref[0], o[0]), (ref[1], o[1]), (ref[2], o[2]), (ref[3], o[4])):
        np.testing.assert_array_equal(a, b.numpy())


def test_densify_routing_known_answer():
    """density.py:153-195 by hand on 8 slots: slots 1, 4 active and kept, 6 pruned
    (opacity), 0 and 2 clone / split sources; empty slots 3, 5, 6, 7 (index
    order) receive the clone of 0, then the split copy of 2."""
    import numpy as np
    n, K = 8, 1
    rng = np.random.default_rng(0)
    p = {"means": np.arange(n * 3, dtype=np.float32).reshape(n, 3),
         "scales": np.full((n, 3), -4.0, np.float32), "quaternions": np.tile([1, 0, 0, 0], (n, 1)).astype(np.float32),
         "opacities": np.full((n, 1), 2.0, np.float32), "sh_coeffs": rng.normal(0, 1, (n, K, 3)).astype(np.float32)}
    p["scales"][2] = -3.0  # exp(-3) = 0.0498 > 0.01 * extent (extent 4): splits
    p["opacities"][6] = -10.0  # pruned
    active = np.array([1, 1, 1, 0, 1, 0, 1, 0], bool)
    denom = np.array([1, 1, 1, 0, 1, 0, 1, 0], np.int32)
    grad = np.array([1e-3, 0, 1e-3, 0, 1e-5, 0, 1e-3, 0], np.float32)
    noise = np.ones((n, 3), np.float32)
    t = lambda d: {k: torch.tensor(v) for k, v in d.items()}  # noqa: E731
    out, mu, nu, act, ga, dn, mr, info = R.densify_and_prune(
        t(p), t(p), t(p), active, grad, denom, np.zeros(n, np.float32), noise, extent=4.0)
    assert info == {"pruned": 1, "clones": 1, "splits": 1, "applied": True}
    assert act.tolist() == [True, True, True, True, True, True, False, False]
    m = out["means"].numpy()
    np.testing.assert_array_equal(m[3], p["means"][0])  # clone of 0 in the first empty slot
    s = np.float32(-3.0) - np.float32(np.log(np.float64(np.float32(1.6))))
    e = np.float32(np.exp(np.float64(s)))
    np.testing.assert_array_equal(m[5], p["means"][2] + e)  # split copy of 2, moved by noise * exp(s)
    np.testing.assert_array_equal(m[2], p["means"][2] + e)  # the split source moves too
    assert out["scales"].numpy()[5, 0] == s and out["scales"].numpy()[2, 0] == s
    np.testing.assert_array_equal(m[7], p["means"][7])  # untouched empty slot
    np.testing.assert_array_equal(mu["means"].numpy()[3], p["means"][0])  # moments move with the row
    assert not ga.any() and not dn.any()
