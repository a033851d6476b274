"""GPU parity of the training-step kernels (losses, Adam, densification
statistics) and of a whole train step against the CPU oracle."""
import numpy as np
import pytest
import torch

from oracle import ref_restated as R
from tests.helpers import random_scene, to_torch

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("H,W", [(378, 504), (37, 53)])
def test_l1_and_dssim_match_oracle(H, W):
    from gs_b200.training.losses import d_ssim_loss, l1_loss, ssim
    rng = np.random.default_rng(H)
    tgt = rng.uniform(0, 1, (H, W, 3)).astype(np.float32)
    pred = np.clip(tgt + rng.normal(0, 0.2, tgt.shape), 0, 1).astype(np.float32)
    p = torch.tensor(pred, device="cuda", requires_grad=True)
    t = torch.tensor(tgt, device="cuda")
    l1 = l1_loss(p, t)
    ds = d_ssim_loss(p, t)
    (0.8 * l1 + 0.2 * ds).backward()
    po = torch.tensor(pred, requires_grad=True)
    to = torch.tensor(tgt)
    l1o = R.l1_loss(po, to)
    dso = R.d_ssim_loss(po, to)
    (0.8 * l1o + 0.2 * dso).backward()
    assert float(l1) == pytest.approx(float(l1o), rel=1e-5)
    assert float(ds) == pytest.approx(float(dso), rel=1e-4, abs=1e-6)
    assert float(ssim(p, t)) == pytest.approx(float(R.ssim(po, to)), rel=1e-4)
    g, r = _np(p.grad), _np(po.grad)
    assert np.abs(g - r).max() <= 1e-3 * np.abs(r).max()


@pytest.mark.parametrize("H,W,C", [(378, 504, 3), (37, 53, 3), (16, 40, 1), (5, 7, 2)])
def test_fused_l1_dssim_matches_oracle(H, W, C):
    """gs_l1_dssim_loss: trainer.py:18-26's (1 - 0.2) L1 + 0.2 D-SSIM in one
    call, its parts and its image gradient, against the oracle."""
    from gs_b200 import _lib
    rng = np.random.default_rng(H * 7 + C)
    tgt = rng.uniform(0, 1, (H, W, C)).astype(np.float32)
    pred = np.clip(tgt + rng.normal(0, 0.2, tgt.shape), 0, 1).astype(np.float32)
    pred[0, 0, 0] = tgt[0, 0, 0]  # a zero difference: L1's gradient is 0 there
    p = torch.tensor(pred, device="cuda")
    t = torch.tensor(tgt, device="cuda")
    out = torch.full((4,), float("nan"), device="cuda")
    grad = torch.full_like(p, float("nan"))
    ws = torch.empty(_lib.lib().gs_l1_dssim_workspace_bytes(H, W, C), dtype=torch.uint8, device="cuda")
    for _ in range(2):  # the reduction state resets itself between calls
        _lib.call("gs_l1_dssim_loss", _lib.ptr(p), _lib.ptr(t), H, W, C, 0.2, _lib.ptr(out[0:1]),
                  _lib.ptr(out[1:2]), _lib.ptr(out[2:3]), _lib.ptr(out[3:4]), _lib.ptr(grad), _lib.ptr(ws),
                  ws.numel(), _lib.stream(p.device))
    po = torch.tensor(pred, requires_grad=True)
    to = torch.tensor(tgt)
    l1o = R.l1_loss(po, to)
    dso = R.d_ssim_loss(po, to)
    loss_o = 0.8 * l1o + 0.2 * dso
    loss_o.backward()
    o = out.cpu().numpy()
    assert o[0] == pytest.approx(float(l1o), rel=1e-5)
    assert o[1] == pytest.approx(float(dso), rel=1e-4, abs=1e-6)
    assert o[2] == pytest.approx(float(R.ssim(po.detach(), to)), rel=1e-4)
    assert o[3] == pytest.approx(float(loss_o), rel=1e-4, abs=1e-6)
    g, r = _np(grad), _np(po.grad)
    assert np.isfinite(g).all()
    assert np.abs(g - r).max() <= 1e-3 * np.abs(r).max()


def test_dssim_identical_images():
    from gs_b200.training.losses import d_ssim_loss, ssim
    t = torch.rand((32, 32, 3), device="cuda")
    assert float(ssim(t, t)) == pytest.approx(1.0, abs=1e-6)
    assert float(d_ssim_loss(t, t)) == pytest.approx(0.0, abs=1e-6)


def test_adam_step_matches_optax_restatement():
    from gs_b200 import _lib
    import ctypes
    n, k = 1000, 16
    rng = np.random.default_rng(0)
    sizes = [3 * n, 3 * n, 4 * n, n, 3 * k * n]
    tot = sum(sizes)
    params = rng.standard_normal(tot).astype(np.float32)
    mu = (0.01 * rng.standard_normal(tot)).astype(np.float32)
    nu = (0.001 * rng.uniform(0, 1, tot)).astype(np.float32)
    active = rng.uniform(0, 1, n) > 0.3
    lrs = [1e-3, 5e-3, 1e-3, 5e-2, 2.5e-3]
    P, M, V = (torch.tensor(a, device="cuda") for a in (params, mu, nu))
    op = {}
    off = 0
    shapes = [(n, 3), (n, 3), (n, 4), (n, 1), (n, k, 3)]
    for name, sz, shp in zip(R.GROUPS, sizes, shapes):
        op[name] = (slice(off, off + sz), shp)
        off += sz
    p_o = {nm: torch.tensor(params[s]).reshape(shp) for nm, (s, shp) in op.items()}
    m_o = {nm: torch.tensor(mu[s]).reshape(shp) for nm, (s, shp) in op.items()}
    v_o = {nm: torch.tensor(nu[s]).reshape(shp) for nm, (s, shp) in op.items()}
    act_d = torch.tensor(active, device="cuda").view(torch.uint8)
    for step in (1, 2, 3):
        grads = rng.standard_normal(tot).astype(np.float32)
        G = torch.tensor(grads, device="cuda")
        arr = (ctypes.c_float * 5)(*lrs)
        _lib.call("gs_adam_step", _lib.ptr(P), _lib.ptr(G), _lib.ptr(M), _lib.ptr(V), n, k, _lib.ptr(act_d),
                  ctypes.cast(arr, ctypes.c_void_p), step, 0.9, 0.999, 1e-8, _lib.stream(P.device))
        g_o = {nm: torch.tensor(grads[s]).reshape(shp) for nm, (s, shp) in op.items()}
        p_o, m_o, v_o = R.adam_update(p_o, g_o, m_o, v_o, step, dict(zip(R.GROUPS, lrs)),
                                      torch.tensor(active))
    for nm, (s, shp) in op.items():
        np.testing.assert_allclose(_np(P)[s].reshape(shp), p_o[nm].numpy(), rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(_np(M)[s].reshape(shp), m_o[nm].numpy(), rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(_np(V)[s].reshape(shp), v_o[nm].numpy(), rtol=1e-5, atol=1e-9)
    # inactive Gaussians: parameters untouched, moments still updated
    s, shp = op["means"]
    np.testing.assert_array_equal(_np(P)[s].reshape(shp)[~active], params[s].reshape(shp)[~active])


def _state_from_scene(sc, device="cuda"):
    from gs_b200.core.gaussians import Gaussians
    from gs_b200.training.trainer import AdamConfig, init_density_state
    t = to_torch(sc, device)
    na = int(sc["active"].sum())
    g = Gaussians(means=t["means"][:na], scales=t["scales"][:na], quaternions=t["quats"][:na],
                  opacities=t["opac"][:na], sh_coeffs=t["sh"][:na])
    opt = AdamConfig.from_extent(3.0, 30000)
    return init_density_state(g, opt, sc["means"].shape[0]), opt


def test_train_step_matches_oracle():
    from gs_b200.training.trainer import train_step
    sc = random_scene(21, 1200, 96, 80, sh_degree=3, behind=0.05)
    na = 900
    sc["active"] = np.arange(1200) < na
    state, opt = _state_from_scene(sc)
    rng = np.random.default_rng(1)
    target = rng.uniform(0, 1, (80, 96, 3)).astype(np.float32)
    cam = (sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"])
    p0 = {k: v.detach().clone().cpu() for k, v in vars(state.gaussians).items()}
    state, loss, metrics = train_step(state, torch.tensor(target, device="cuda"),
                                      torch.tensor(sc["w2c"], device="cuda"), cam, opt, sh_degree=3)
    torch.cuda.synchronize()
    # oracle on the padded state
    params = {"means": p0["means"], "scales": p0["scales"], "quaternions": p0["quaternions"],
              "opacities": p0["opacities"], "sh_coeffs": p0["sh_coeffs"]}
    zeros = {k: torch.zeros_like(v) for k, v in params.items()}
    lrs = dict(zip(R.GROUPS, opt.lrs(0)))
    act = torch.tensor(sc["active"])
    o = R.train_step(params, zeros, dict(zeros), 1, lrs, act, torch.tensor(target), torch.tensor(sc["w2c"]),
                     cam, sh_degree=3, grad_accum=torch.zeros(1200), denom=torch.zeros(1200, dtype=torch.int32),
                     max_radii=torch.zeros(1200))
    assert float(loss) == pytest.approx(o["loss"], rel=1e-4)
    assert float(metrics["l1"]) == pytest.approx(o["l1"], rel=1e-5)
    assert float(metrics["ssim"]) == pytest.approx(o["ssim"], rel=1e-4, abs=1e-5)
    assert float(metrics["n_interactions"]) == o["extras"]["n_interactions"]
    from tests.test_gpu_parity import _grad_close
    gf = state.grad_fields
    for f in R.GROUPS:
        _grad_close(_np(getattr(gf, f))[:na], np.nan_to_num(o["grads"][f].numpy()[:na]), f)
    # parameters: padded untouched; active updated where the gradient is
    # clearly non-zero (Adam's first step moves by ~lr * sign(g))
    g1 = state.gaussians
    for f in R.GROUPS:
        new = _np(getattr(g1, f))
        np.testing.assert_array_equal(new[na:], p0[f].numpy()[na:])
        ref = o["params"][f].numpy()
        gr = np.abs(o["grads"][f].numpy())
        sig = gr > 1e-2 * gr.max()
        sig[na:] = False
        np.testing.assert_allclose(new[sig], ref[sig], rtol=1e-4, atol=1e-6)
    np.testing.assert_array_equal(_np(state.denom), o["denom"].numpy())
    np.testing.assert_array_equal(_np(state.max_radii), o["max_radii"].numpy())
    ga, gr2 = _np(state.grad_accum), o["grad_accum"].numpy()
    assert np.abs(ga - gr2).max() <= 1e-3 * (np.abs(gr2).max() + 1e-12)


def test_padded_gaussians_untouched_and_active_change():
    """tests/test_training.py:40-68 intent: one step changes active means and
    leaves padded ones bit-identical. (The reference places its points at the
    camera centre, where its gradients are NaN; here they sit in front.)"""
    from gs_b200.core.gaussians import init_gaussians_from_pcd
    from gs_b200.training.trainer import AdamConfig, init_density_state, train_step
    rng = np.random.default_rng(0)
    pts = torch.tensor(np.stack([rng.uniform(-0.3, 0.3, 10), rng.uniform(-0.3, 0.3, 10), np.full(10, 3.0)], 1),
                       dtype=torch.float32, device="cuda")
    g = init_gaussians_from_pcd(pts, torch.full((10, 3), 0.7, device="cuda"))
    opt = AdamConfig(means_lr_init=1e-3, means_lr_end=1e-3)
    st = init_density_state(g, opt, 20)
    before = st.gaussians.means.clone()
    st, loss, m = train_step(st, torch.zeros((16, 16, 3), device="cuda"), torch.eye(4, device="cuda"),
                             (16, 16, 10.0, 10.0, 8.0, 8.0), opt)
    after = st.gaussians.means
    assert not torch.allclose(after[:10], before[:10])
    assert torch.equal(after[10:], before[10:])


def test_adam_scheduled_matches_host_adam():
    """gs_adam_step_scheduled (schedule evaluated on the device from a device
    step counter, for graph replay) equals gs_adam_step with host-side
    learning rates over several steps, and advances the counter."""
    import ctypes
    from gs_b200 import _lib
    from gs_b200.training.trainer import AdamConfig
    n, k = 1000, 16
    rng = np.random.default_rng(3)
    tot = n * (11 + 3 * k)
    opt = AdamConfig(means_lr_init=1e-2, means_lr_end=1e-4, transition_steps=10)
    p0 = rng.standard_normal(tot).astype(np.float32)
    bufs = [torch.tensor(p0, device="cuda") for _ in range(2)]
    mus = [torch.zeros(tot, device="cuda") for _ in range(2)]
    nus = [torch.zeros(tot, device="cuda") for _ in range(2)]
    act = torch.tensor(rng.uniform(0, 1, n) > 0.2, device="cuda").view(torch.uint8)
    state = torch.zeros(2, dtype=torch.int32, device="cuda")
    sched = opt.schedule()
    st = _lib.stream(torch.device("cuda"))
    for step in range(4):
        g = torch.tensor(rng.standard_normal(tot).astype(np.float32), device="cuda")
        arr = (ctypes.c_float * 5)(*opt.lrs(step))
        _lib.call("gs_adam_step", _lib.ptr(bufs[0]), _lib.ptr(g), _lib.ptr(mus[0]), _lib.ptr(nus[0]), n, k,
                  _lib.ptr(act), ctypes.cast(arr, ctypes.c_void_p), step + 1, opt.b1, opt.b2, opt.eps, st)
        _lib.call("gs_adam_step_scheduled", _lib.ptr(bufs[1]), _lib.ptr(g), _lib.ptr(mus[1]), _lib.ptr(nus[1]),
                  n, k, _lib.ptr(act), ctypes.byref(sched), _lib.ptr(state), st)
    torch.cuda.synchronize()
    assert int(state[0]) == 4 and int(state[1]) == 0
    np.testing.assert_allclose(_np(bufs[1]), _np(bufs[0]), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(_np(mus[1]), _np(mus[0]), rtol=1e-6, atol=1e-9)


def test_captured_step_matches_eager():
    """A CUDA-graph replay of the train step produces the eager step's losses
    and parameters (up to the reordering of fp32 atomics)."""
    from gs_b200.training.trainer import CapturedStep, train_step
    sc = random_scene(31, 1500, 96, 80, sh_degree=3, behind=0.05)
    sc["active"] = np.arange(1500) < 1100
    rng = np.random.default_rng(2)
    targets = [torch.tensor(rng.uniform(0, 1, (80, 96, 3)).astype(np.float32), device="cuda") for _ in range(3)]
    w2c = torch.tensor(sc["w2c"], device="cuda")
    cam = (sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"])
    sa, opt = _state_from_scene(sc)
    sb, _ = _state_from_scene(sc)
    la = []
    for t in targets:
        sa, loss, _ = train_step(sa, t, w2c, cam, opt, sh_degree=3)
        la.append(float(loss))
    cs = CapturedStep(sb, targets[0], w2c, cam, opt, sh_degree=3)
    lb = [float(sb.tail[0] * 0.8 + sb.tail[1] * 0.2)]
    for t in targets[1:]:
        _, loss, metrics = cs(t, w2c)
        lb.append(float(loss))
    np.testing.assert_allclose(lb, la, rtol=1e-5)
    assert int(sb.adam_state[0]) == int(sa.adam_state[0]) == 3
    for f in ("means", "scales", "quaternions", "opacities", "sh_coeffs"):
        a, b = _np(getattr(sa.gaussians, f)), _np(getattr(sb.gaussians, f))
        assert np.abs(a - b).max() <= 3 * 2 * 0.05 + 1e-6, f
        assert np.median(np.abs(a - b)) <= 1e-6, f


def test_mse_loss_matches_oracle():
    """mse_loss (losses.py:10-14): the reference's known answer
    (tests/test_training.py:9-19), and value and gradient against the oracle."""
    from gs_b200.training.losses import mse_loss
    pred = torch.tensor([1.0, 2.0, 3.0], device="cuda")
    target = torch.tensor([1.1, 1.9, 3.0], device="cuda")
    assert float(mse_loss(pred, target)) == pytest.approx(0.00666667, rel=1e-4)
    rng = np.random.default_rng(5)
    tgt = rng.uniform(0, 1, (61, 47, 3)).astype(np.float32)
    prd = (tgt + rng.normal(0, 0.1, tgt.shape)).astype(np.float32)
    p = torch.tensor(prd, device="cuda", requires_grad=True)
    loss = mse_loss(p, torch.tensor(tgt, device="cuda"))
    loss.backward()
    po = torch.tensor(prd, requires_grad=True)
    lo = R.mse_loss(po, torch.tensor(tgt))
    lo.backward()
    assert float(loss) == pytest.approx(float(lo), rel=1e-5)
    np.testing.assert_allclose(_np(p.grad), _np(po.grad), rtol=1e-5, atol=1e-10)


def test_covariance_3d_matches_oracle():
    """get_covariance_3d (gaussians.py:58-93): bit-exact against the oracle
    (the arithmetic of the projection's covariance), symmetric and positive
    semi-definite (tests/test_core.py:21-38)."""
    from gs_b200.core.gaussians import get_covariance_3d
    rng = np.random.default_rng(9)
    n = 1000
    scales = rng.uniform(-5, 1, (n, 3)).astype(np.float32)
    quats = rng.normal(0, 1, (n, 4)).astype(np.float32)
    with torch.no_grad():
        cov = _np(get_covariance_3d(torch.tensor(scales, device="cuda"), torch.tensor(quats, device="cuda")))
    ref = R.get_covariance_3d(torch.tensor(scales), torch.tensor(quats)).numpy()
    assert cov.shape == (n, 3, 3)
    np.testing.assert_array_equal(cov, ref)
    np.testing.assert_array_equal(cov, cov.transpose(0, 2, 1))
    ev = np.linalg.eigvalsh(cov.astype(np.float64))
    assert (ev >= -1e-6 * np.abs(ev).max(axis=1, keepdims=True)).all()


@pytest.mark.parametrize("deg", [0, 1, 2, 3])
def test_eval_sh_entry_matches_oracle(deg):
    """gs_eval_sh on its own (sh.py:25-74): every degree, K = 16 stored
    coefficients, unit directions, against the oracle's eval_sh."""
    from gs_b200.renderer.sh import eval_sh
    rng = np.random.default_rng(40 + deg)
    n = 5000
    sh = rng.normal(0, 0.5, (n, 16, 3)).astype(np.float32)
    d = rng.standard_normal((n, 3))
    d = (d / np.linalg.norm(d, axis=1, keepdims=True)).astype(np.float32)
    got = eval_sh(deg, torch.tensor(sh, device="cuda"), torch.tensor(d, device="cuda")).cpu().numpy()
    ref = R.eval_sh(deg, torch.tensor(sh), torch.tensor(d)).numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)


def test_density_step_stats_equals_the_two_calls():
    """gs_density_step_stats (one kernel) gives the bits of
    gs_grad2d_magnitude followed by gs_accumulate_density_stats."""
    from gs_b200 import _lib
    rng = np.random.default_rng(12)
    n = 20000
    t = lambda a, dt=torch.float32: torch.tensor(a, device="cuda", dtype=dt)  # noqa: E731
    gmeans = t(rng.normal(0, 1e-3, (n, 3)))
    means = t(rng.normal(0, 2, (n, 3)))
    w2c = t(np.array([[1, 0, 0, 0.1], [0, 1, 0, -0.2], [0, 0, 1, 4.0], [0, 0, 0, 1]]))
    radii = t(rng.uniform(0, 30, n))
    valid = t(rng.uniform(0, 1, n) < 0.6, torch.uint8)
    active = t(rng.uniform(0, 1, n) < 0.8, torch.uint8)
    acc0, den0, mr0 = t(rng.uniform(0, 1, n)), t(rng.integers(0, 9, n), torch.int32), t(rng.uniform(0, 40, n))
    P = _lib.ptr
    st = _lib.stream(gmeans.device)
    a1, d1, m1, g1 = acc0.clone(), den0.clone(), mr0.clone(), torch.empty(n, device="cuda")
    _lib.call("gs_density_step_stats", P(gmeans), P(means), P(w2c), n, 400.0, 410.0, 504, 378, P(radii), P(valid),
              P(active), P(a1), P(d1), P(m1), P(g1), st)
    a2, d2, m2, g2 = acc0.clone(), den0.clone(), mr0.clone(), torch.empty(n, device="cuda")
    _lib.call("gs_grad2d_magnitude", P(gmeans), P(means), P(w2c), n, 400.0, 410.0, 504, 378, P(g2), st)
    _lib.call("gs_accumulate_density_stats", P(g2), P(radii), P(valid), P(valid), P(active), n, P(a2), P(d2), P(m2),
              st)
    torch.cuda.synchronize()
    for x, y in ((a1, a2), (d1, d2), (m1, m2), (g1, g2)):
        assert torch.equal(x, y)
