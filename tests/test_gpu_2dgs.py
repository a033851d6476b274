"""2DGS surfel renderer (jax_2dgs) on the device against the oracle
(oracle/ref_restated_2d.py): projection, the five compositor maps, their
gradients, the regularisers and the training loss."""
import numpy as np
import pytest
import torch

from oracle import ref_restated as R
from oracle import ref_restated_2d as R2

pytestmark = pytest.mark.gpu
IMG_TOL = 1e-4


def _scene(seed, n=600, W=72, H=56, spread=1.2, scale_mu=-2.6, crowd=0):
    rng = np.random.default_rng(seed)
    means = np.stack([rng.uniform(-spread, spread, n), rng.uniform(-spread * 0.8, spread * 0.8, n),
                      rng.uniform(2.0, 6.0, n)], 1)
    if crowd:  # many surfels on one tile: the 512 cap
        means[:crowd, 0] = rng.normal(0, 0.01, crowd)
        means[:crowd, 1] = rng.normal(0, 0.01, crowd)
    means[: n // 20, 2] = rng.uniform(-2, 0.005, n // 20)  # behind / at the near plane
    p = {"means": means, "scales": rng.normal(scale_mu, 0.4, (n, 2)), "quaternions": rng.normal(0, 1, (n, 4)),
         "opacities": rng.normal(0, 1.2, (n, 1)), "sh_coeffs": rng.normal(0, 0.5, (n, 16, 3))}
    p = {k: v.astype(np.float32) for k, v in p.items()}
    a, b = 0.12, -0.08
    Ry = np.array([[np.cos(a), 0, np.sin(a)], [0, 1, 0], [-np.sin(a), 0, np.cos(a)]])
    Rx = np.array([[1, 0, 0], [0, np.cos(b), -np.sin(b)], [0, np.sin(b), np.cos(b)]])
    w2c = np.eye(4, dtype=np.float32)
    w2c[:3, :3] = Rx @ Ry
    w2c[:3, 3] = [0.05, -0.02, 0.2]
    cam = dict(W=W, H=H, fx=0.9 * W, fy=0.92 * W, cx=W / 2 + 0.3, cy=H / 2 - 0.2)
    return p, w2c, cam


def _gpu(p, w2c, cam, requires_grad=False, background=None):
    from gs_b200.core.camera import Camera
    from gs_b200.twod.core.gaussians_2d import Gaussians2D
    from gs_b200.twod.renderer.renderer import render
    t = {k: torch.tensor(v, device="cuda", requires_grad=requires_grad) for k, v in p.items()}
    g = Gaussians2D(t["means"], t["scales"], t["quaternions"], t["opacities"], t["sh_coeffs"])
    c = Camera(cam["W"], cam["H"], cam["fx"], cam["fy"], cam["cx"], cam["cy"], torch.tensor(w2c, device="cuda"), None)
    img, ex = render(g, c, background=background)
    return img, ex, t


def _oracle(p, w2c, cam, requires_grad=False, background=None):
    t = {k: torch.tensor(v, requires_grad=requires_grad) for k, v in p.items()}
    img, ex = R2.render_2d(t["means"], t["scales"], t["quaternions"], t["opacities"], t["sh_coeffs"],
                           torch.tensor(w2c), cam["W"], cam["H"], cam["fx"], cam["fy"], cam["cx"], cam["cy"],
                           background)
    return img, ex, t


def _np(x):
    return x.detach().cpu().numpy()


CASES = [("random", lambda: _scene(1)), ("crowded_512", lambda: _scene(2, n=900, crowd=700, scale_mu=-3.0)),
         ("big", lambda: _scene(3, n=150, scale_mu=-1.2))]


@pytest.mark.parametrize("name,make", CASES)
def test_render2d_matches_oracle(name, make):
    p, w2c, cam = make()
    img, ex, _ = _gpu(p, w2c, cam)
    oimg, oex, _ = _oracle(p, w2c, cam)
    assert np.abs(_np(img) - _np(oimg)).max() <= IMG_TOL
    for k in ("depth", "depth_sq", "normals", "accum_weight"):
        r = _np(oex[k])
        assert np.abs(_np(ex[k]) - r).max() <= IMG_TOL * max(1.0, np.abs(r).max()), k


def test_render2d_projection_bit_exact():
    """radii and valid (which decide the tile keys) equal the oracle's bits."""
    from gs_b200 import _lib
    from gs_b200.twod.renderer.renderer import workspace2d
    p, w2c, cam = _scene(4)
    n, W, H = p["means"].shape[0], cam["W"], cam["H"]
    t = {k: torch.tensor(v, device="cuda") for k, v in p.items()}
    ws = workspace2d(n, W, H, n * 256, "cuda")
    f = dict(dtype=torch.float32, device="cuda")
    maps = [torch.empty(s, **f) for s in ((H, W, 3), (H, W, 1), (H, W, 1), (H, W, 3), (H, W, 1))]
    radii, valid = torch.empty(n, **f), torch.empty(n, dtype=torch.uint8, device="cuda")
    ex = torch.empty(16, dtype=torch.int32, device="cuda")
    P = _lib.ptr
    _lib.call("gs_render2d_forward", P(t["means"]), P(t["scales"]), P(t["quaternions"]), P(t["opacities"]),
              P(t["sh_coeffs"]), n, 16, P(torch.tensor(w2c, device="cuda")), W, H, cam["fx"], cam["fy"], cam["cx"],
              cam["cy"], None, n * 256, P(ws), ws.numel(), *[P(m) for m in maps], P(radii), P(valid), P(ex),
              _lib.stream(torch.device("cuda")))
    m2, cov, orad, oval, z, nor = R2.project_gaussians_2d(*(torch.tensor(p[k]) for k in ("means", "scales",
                                                                                        "quaternions")),
                                                         torch.tensor(w2c), cam["fx"], cam["fy"], cam["cx"],
                                                         cam["cy"])
    np.testing.assert_array_equal(_np(radii), _np(orad))
    np.testing.assert_array_equal(_np(valid).astype(bool), _np(oval))
    tid, gid, nv = R.get_tile_interactions_compact(_np(m2), _np(orad), _np(oval), _np(z), H, W)
    assert int(ex[0]) == nv


@pytest.mark.parametrize("name,make", CASES[:2])
def test_render2d_backward_matches_oracle(name, make):
    p, w2c, cam = make()
    rng = np.random.default_rng(7)
    H, W = cam["H"], cam["W"]
    wts = [rng.normal(0, 1, s).astype(np.float32) for s in ((H, W, 3), (H, W, 1), (H, W, 1), (H, W, 3), (H, W, 1))]
    img, ex, t = _gpu(p, w2c, cam, requires_grad=True)
    maps = [img, ex["depth"], ex["depth_sq"], ex["normals"], ex["accum_weight"]]
    sum((m * torch.tensor(w, device="cuda")).sum() for m, w in zip(maps, wts)).backward()
    oimg, oex, ot = _oracle(p, w2c, cam, requires_grad=True)
    omaps = [oimg, oex["depth"], oex["depth_sq"], oex["normals"], oex["accum_weight"]]
    sum((m * torch.tensor(w)).sum() for m, w in zip(omaps, wts)).backward()
    for k in ("means", "scales", "quaternions", "opacities", "sh_coeffs"):
        g, r = _np(t[k].grad).astype(np.float64), _np(ot[k].grad).astype(np.float64)
        assert np.all(np.abs(g - r) <= 1e-3 * (np.abs(r) + np.abs(r).max())), k
    assert not _np(t["sh_coeffs"].grad)[:, 1:].any()


def test_regularizers_match_oracle():
    from gs_b200.twod.training.losses import depth_distortion_loss, normal_consistency_loss
    rng = np.random.default_rng(8)
    H, W = 37, 45
    d = rng.uniform(1, 3, (H, W, 1)).astype(np.float32)
    d2 = (d ** 2 * rng.uniform(1.0, 1.2, (H, W, 1))).astype(np.float32)
    a = rng.uniform(0, 1, (H, W, 1)).astype(np.float32)
    a[:3, :3] = 0.0
    n = rng.normal(0, 1, (H, W, 3)).astype(np.float32)
    td, td2, tn = (torch.tensor(x, device="cuda", requires_grad=True) for x in (d, d2, n))
    ta = torch.tensor(a, device="cuda")
    ld = depth_distortion_loss(td, td2, ta)
    ln = normal_consistency_loss(tn, td)
    (ld + 2.0 * ln).backward()
    od, od2, on = (torch.tensor(x, requires_grad=True) for x in (d, d2, n))
    old = R2.depth_distortion_loss(od, od2, torch.tensor(a))
    oln = R2.normal_consistency_loss(on, od)
    (old + 2.0 * oln).backward()
    assert float(ld.detach()) == pytest.approx(float(old.detach()), rel=1e-4, abs=1e-7)
    assert float(ln.detach()) == pytest.approx(float(oln.detach()), rel=1e-4, abs=1e-7)
    for g, r in ((td.grad, od.grad), (td2.grad, od2.grad), (tn.grad, on.grad)):
        g, r = _np(g), _np(r)
        assert np.abs(g - r).max() <= 1e-3 * np.abs(r).max() + 1e-9


def test_train_step_2d_loss_and_gradients_match_oracle():
    from gs_b200.twod.core.gaussians_2d import Gaussians2D
    from gs_b200.twod.training.trainer import State2D, train_step
    p, w2c, cam = _scene(9, n=500)
    rng = np.random.default_rng(10)
    target = rng.uniform(0, 1, (cam["H"], cam["W"], 3)).astype(np.float32)
    t = {k: torch.tensor(v, device="cuda") for k, v in p.items()}
    st = State2D(Gaussians2D(t["means"], t["scales"], t["quaternions"], t["opacities"], t["sh_coeffs"]))
    before = st.params.clone()
    st, loss, metrics = train_step(st, torch.tensor(target), torch.tensor(w2c),
                                   (cam["W"], cam["H"], cam["fx"], cam["fy"], cam["cx"], cam["cy"]))
    ot = {k: torch.tensor(v, requires_grad=True) for k, v in p.items()}
    oloss, om = R2.train_loss_2d(ot, torch.tensor(target), torch.tensor(w2c), cam["W"], cam["H"], cam["fx"],
                                 cam["fy"], cam["cx"], cam["cy"])
    oloss.backward()
    assert float(loss) == pytest.approx(float(oloss), rel=1e-4)
    for key in ("l1", "ssim", "dist_loss", "normal_loss"):
        assert float(metrics[key]) == pytest.approx(float(om[key]), rel=1e-3, abs=1e-6), key
    gf = st.grad_fields
    for k, f in (("means", "means"), ("scales", "scales"), ("quaternions", "quaternions"),
                 ("opacities", "opacities"), ("sh_coeffs", "sh_coeffs")):
        g = _np(getattr(gf, f)).astype(np.float64)
        r = _np(ot[k].grad).astype(np.float64)
        assert np.all(np.abs(g - r) <= 1e-3 * (np.abs(r) + np.abs(r).max())), k
    assert not torch.equal(before, st.params)  # Adam moved the parameters


def test_captured_2d_step_replays_the_eager_step():
    """CapturedStep2D (a CUDA graph with the optax count on the device) gives
    the eager train_step's parameters, moments and count over three steps."""
    from gs_b200.twod.core.gaussians_2d import Gaussians2D
    from gs_b200.twod.training.trainer import CapturedStep2D, State2D, train_step
    p, w2c, cam = _scene(12, n=700)
    camera = (cam["W"], cam["H"], cam["fx"], cam["fy"], cam["cx"], cam["cy"])
    rng = np.random.default_rng(13)
    targets = [torch.tensor(rng.uniform(0, 1, (cam["H"], cam["W"], 3)).astype(np.float32)) for _ in range(3)]
    views = []
    for i in range(3):
        w = np.array(w2c, dtype=np.float32)
        w[0, 3] += 0.03 * i
        views.append(torch.tensor(w))

    def state():
        t = {k: torch.tensor(v, device="cuda") for k, v in p.items()}
        return State2D(Gaussians2D(t["means"], t["scales"], t["quaternions"], t["opacities"], t["sh_coeffs"]))

    eager, graphed = state(), state()
    for i in range(3):
        train_step(eager, targets[i].cuda(), views[i].cuda(), camera)
    cap = CapturedStep2D(graphed, targets[0].cuda(), views[0].cuda(), camera)  # trains step 0
    for i in (1, 2):
        cap(targets[i].pin_memory(), views[i].pin_memory())  # host inputs through the stager
    torch.cuda.synchronize()
    assert int(eager.adam_state[0]) == 3 and int(graphed.adam_state[0]) == 3
    assert eager.count == graphed.count == 3
    for name, rtol in (("params", 1e-4), ("mu", 1e-3), ("nu", 2e-3)):
        a, r = _np(getattr(graphed, name)), _np(getattr(eager, name))
        # compositor atomics may order the gradient sums differently: the
        # moments carry the gradient's rounding (mu ~ g, nu ~ g^2), so their
        # bar is the renderer's gradient bar (1e-3 relative; 2e-3 for g^2)
        np.testing.assert_allclose(a, r, rtol=rtol, atol=1e-6 * (np.abs(r).max() + 1e-30), err_msg=name)
