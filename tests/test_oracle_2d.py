"""The 2DGS oracle (oracle/ref_restated_2d.py) against the reference's own
tests (tests/test_gaussians_2d.py, restated) and finite differences."""
import math

import numpy as np
import torch

from oracle import ref_restated_2d as R2


def test_gaussians_2d_init():
    # tests/test_gaussians_2d.py:7-15
    g = R2.init_gaussians_2d_from_pcd(torch.zeros((10, 3)), torch.ones((10, 3)))
    assert g["means"].shape == (10, 3) and g["scales"].shape == (10, 2)
    assert g["quaternions"].shape == (10, 4) and g["opacities"].shape == (10, 1)


def test_tangent_vectors():
    # tests/test_gaussians_2d.py:17-38
    u, v, n = R2.get_tangent_vectors(torch.tensor([[1.0, 0.0, 0.0, 0.0]]))
    assert torch.allclose(u, torch.tensor([[1.0, 0.0, 0.0]]), atol=1e-5)
    assert torch.allclose(v, torch.tensor([[0.0, 1.0, 0.0]]), atol=1e-5)
    assert torch.allclose(n, torch.tensor([[0.0, 0.0, 1.0]]), atol=1e-5)
    a = math.pi / 2
    u, v, n = R2.get_tangent_vectors(torch.tensor([[math.cos(a / 2), math.sin(a / 2), 0.0, 0.0]]))
    assert torch.allclose(u, torch.tensor([[1.0, 0.0, 0.0]]), atol=1e-5)
    assert torch.allclose(v, torch.tensor([[0.0, 0.0, 1.0]]), atol=1e-5)
    assert torch.allclose(n, torch.tensor([[0.0, -1.0, 0.0]]), atol=1e-5)


def test_projection_2d_known_answer():
    # tests/test_gaussians_2d.py:40-61
    g = R2.init_gaussians_2d_from_pcd(torch.tensor([[0.0, 0.0, 5.0]]), torch.ones((1, 3)))
    m2, cov, radii, valid, z, normals = R2.project_gaussians_2d(g["means"], g["scales"], g["quaternions"],
                                                                torch.eye(4), 50.0, 50.0, 50.0, 50.0)
    assert torch.allclose(m2, torch.tensor([[50.0, 50.0]]), atol=1e-5)
    assert float(z[0]) == 5.0 and bool(valid[0])
    assert torch.allclose(normals, torch.tensor([[0.0, 0.0, 1.0]]), atol=1e-5)
    assert abs(float(cov[0, 0, 0]) - 0.54) < 0.01


def _scene(seed, n=60, W=40, H=32):
    rng = np.random.default_rng(seed)
    t = lambda a: torch.tensor(a, dtype=torch.float64)  # noqa: E731
    means = np.stack([rng.uniform(-1, 1, n), rng.uniform(-0.8, 0.8, n), rng.uniform(2.5, 5, n)], 1)
    p = {"means": t(means), "scales": t(rng.normal(-2.0, 0.3, (n, 2))),
         "quaternions": t(rng.normal(0, 1, (n, 4))), "opacities": t(rng.normal(0, 1, (n, 1))),
         "sh_coeffs": t(rng.normal(0, 0.5, (n, 16, 3)))}
    return p, dict(W=W, H=H, fx=35.0, fy=36.0, cx=W / 2, cy=H / 2)


def test_render_2d_gradients_finite_differences():
    """d(sum of weighted maps)/d params by autograd against central differences
    (float64), for the image, depth, depth^2, normal and 1 - T outputs."""
    p, cam = _scene(1)
    rng = np.random.default_rng(2)
    wts = [torch.tensor(rng.normal(0, 1, s)) for s in ((cam["H"], cam["W"], 3), (cam["H"], cam["W"], 1),
                                                        (cam["H"], cam["W"], 1), (cam["H"], cam["W"], 3),
                                                        (cam["H"], cam["W"], 1))]

    def f(q):
        img, ex = R2.render_2d(q["means"], q["scales"], q["quaternions"], q["opacities"], q["sh_coeffs"],
                               torch.eye(4, dtype=torch.float64), **cam)
        maps = [img, ex["depth"], ex["depth_sq"], ex["normals"], ex["accum_weight"]]
        return sum((m * w).sum() for m, w in zip(maps, wts))

    q = {k: v.clone().requires_grad_(True) for k, v in p.items()}
    f(q).backward()
    rng = np.random.default_rng(3)
    for k in ("means", "scales", "quaternions", "opacities"):
        for _ in range(4):
            i = tuple(int(rng.integers(0, s)) for s in p[k].shape)
            h = 1e-6
            pp = {kk: vv.clone() for kk, vv in p.items()}
            pm = {kk: vv.clone() for kk, vv in p.items()}
            pp[k][i] += h
            pm[k][i] -= h
            with torch.no_grad():
                fd = (f(pp) - f(pm)) / (2 * h)
            g = float(q[k].grad[i])
            assert abs(g - float(fd)) <= 1e-4 * (1.0 + abs(float(fd))), (k, i, g, float(fd))


def test_regularizer_gradients_finite_differences():
    rng = np.random.default_rng(4)
    H, W = 9, 11
    d = torch.tensor(rng.uniform(1, 3, (H, W, 1)), requires_grad=True)
    d2 = torch.tensor((d.detach().numpy() ** 2) * rng.uniform(1.0, 1.2, (H, W, 1)), requires_grad=True)
    a = torch.tensor(rng.uniform(0, 1, (H, W, 1)))
    a[0, 0, 0] = 0.0  # below the 1e-4 mask
    n = torch.tensor(rng.normal(0, 1, (H, W, 3)), requires_grad=True)
    loss = R2.depth_distortion_loss(d, d2, a) + R2.normal_consistency_loss(n, d)
    loss.backward()
    # the reference stops the gradient of the normal loss's weight |n|: the
    # finite differences hold that weight at its value
    w0 = torch.sqrt((n.detach() ** 2).sum(-1, keepdim=True) + 1e-8)

    def total(nn):
        dd = d.detach()
        dz_dx = (torch.roll(dd, -1, dims=1) - torch.roll(dd, 1, dims=1)) / 2.0
        dz_dy = (torch.roll(dd, -1, dims=0) - torch.roll(dd, 1, dims=0)) / 2.0
        nd = torch.cat([-dz_dx, -dz_dy, torch.ones_like(dd)], -1)
        nd = nd / torch.sqrt((nd ** 2).sum(-1, keepdim=True) + 1e-6)
        nr = nn / torch.sqrt((nn ** 2).sum(-1, keepdim=True) + 1e-8)
        return R2.depth_distortion_loss(d, d2, a) + ((1.0 - (nr * nd).sum(-1, keepdim=True)) * w0).mean()

    for t, g in ((d2, d2.grad), (n, n.grad)):
        for _ in range(5):
            i = tuple(int(rng.integers(0, s)) for s in t.shape)
            h = 1e-6
            with torch.no_grad():
                t[i] += h
                up = total(n)
                t[i] -= 2 * h
                dn = total(n)
                t[i] += h
            assert abs(float(g[i]) - float(up - dn) / (2 * h)) < 1e-6


def _golden_2d_module():
    import importlib.util
    import os
    path = os.path.join(os.path.dirname(__file__), "golden", "make_golden.py")
    spec = importlib.util.spec_from_file_location("make_golden", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod, os.path.join(os.path.dirname(path), "scene_small_2d.npz")


def test_golden_2d_fixture_reproduces():
    """The committed 2DGS golden fixture (tests/golden/make_golden.py 2d): the
    oracle reproduces its five maps and the gradients of their weighted sum."""
    mg, path = _golden_2d_module()
    g = np.load(path)
    p = {k: g["in_" + k] for k in ("means", "scales", "quaternions", "opacities", "sh_coeffs")}
    cam = {k: (int if k in ("W", "H") else float)(g["cfg_" + k]) for k in ("W", "H", "fx", "fy", "cx", "cy")}
    weights = [g["grad_weights_%d" % i] for i in range(5)]
    img, ex, t = mg.render_2d_golden(p, g["in_w2c"], cam, weights)
    np.testing.assert_allclose(img.detach().numpy(), g["out_image"], atol=1e-6)
    for k in mg.MAPS_2D:
        np.testing.assert_allclose(ex[k].detach().numpy(), g["out_" + k], atol=1e-5, rtol=1e-6)
    for k in p:
        ref = g["grad_" + k]
        np.testing.assert_allclose(t[k].grad.numpy(), ref, atol=1e-5 * max(1.0, float(np.abs(ref).max())))
    # the fixture exercises the renderer: visible surfels, non-trivial maps
    assert float(g["out_accum_weight"].max()) > 0.5
    assert np.count_nonzero(g["grad_means"]) > 300
