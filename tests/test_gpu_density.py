"""densify_and_prune / reset_opacities (jax_gs/training/density.py:76-211)
on the device against the oracle's literal (argsort-routed) restatement."""
import numpy as np
import pytest
import torch

from oracle import ref_restated as R

pytestmark = pytest.mark.gpu

K = 16
SIZES = {"means": 3, "scales": 3, "quaternions": 4, "opacities": 1, "sh_coeffs": 3 * K}


def _random_state(seed, n, active_frac=0.7, hot_frac=0.08):
    rng = np.random.default_rng(seed)
    p = {
        "means": rng.normal(0, 1, (n, 3)),
        "scales": rng.normal(-3.5, 1.0, (n, 3)),
        "quaternions": rng.normal(0, 1, (n, 4)),
        "opacities": rng.normal(-1.0, 2.5, (n, 1)),
        "sh_coeffs": rng.normal(0, 0.2, (n, K, 3)),
    }
    p = {k: v.astype(np.float32) for k, v in p.items()}
    mu = {k: rng.normal(0, 1e-3, v.shape).astype(np.float32) for k, v in p.items()}
    nu = {k: rng.uniform(0, 1e-5, v.shape).astype(np.float32) for k, v in p.items()}
    active = rng.uniform(0, 1, n) < active_frac
    denom = rng.integers(0, 20, n).astype(np.int32)
    grad_accum = (rng.uniform(0, 1, n) * denom * 2e-4).astype(np.float32)
    hot = rng.uniform(0, 1, n) < hot_frac
    grad_accum[hot] *= 20
    max_radii = rng.uniform(0, 600, n).astype(np.float32)
    noise = rng.normal(0, 1, (n, 3)).astype(np.float32)
    return p, mu, nu, active, grad_accum, denom, max_radii, noise


def _device_state(p, mu, nu, active, grad_accum, denom, max_radii):
    from gs_b200.training.trainer import DensityState
    n = active.shape[0]
    st = DensityState(n, K, "cuda")
    for buf, src in ((st.params, p), (st.mu, mu), (st.nu, nu)):
        flat = torch.cat([torch.tensor(src[k]).reshape(-1) for k in R.GROUPS])
        buf.copy_(flat)
    st.active_mask.copy_(torch.tensor(active))
    st.grad_accum.copy_(torch.tensor(grad_accum))
    st.denom.copy_(torch.tensor(denom))
    st.max_radii.copy_(torch.tensor(max_radii))
    return st


def _split_fields(buf, n):
    out, off = {}, 0
    for k in R.GROUPS:
        w = SIZES[k]
        out[k] = buf[off:off + n * w].reshape((n, w) if k != "sh_coeffs" else (n, K, 3)).cpu().numpy()
        off += n * w
    return out


@pytest.mark.parametrize("case", ["normal", "no_room", "disabled", "prune_only"])
def test_densify_and_prune_matches_oracle(case):
    from gs_b200.training.density import densify_and_prune
    n = 3000
    args = dict(grad_threshold=0.0002, min_opacity=0.005, extent=5.0, max_screen_size=512)
    if case == "no_room":
        p, mu, nu, active, ga, dn, mr, noise = _random_state(1, n, active_frac=0.995, hot_frac=0.3)
    else:
        p, mu, nu, active, ga, dn, mr, noise = _random_state(0, n)
    enabled = case != "disabled"
    if case == "prune_only":
        ga[:] = 0.0
    st = _device_state(p, mu, nu, active, ga, dn, mr)
    densify_and_prune(st, densify_enabled=enabled, noise=torch.tensor(noise), **args)
    t = lambda d: {k: torch.tensor(v) for k, v in d.items()}  # noqa: E731
    rp, rmu, rnu, ract, rga, rdn, rmr, info = R.densify_and_prune(
        t(p), t(mu), t(nu), active.copy(), ga.copy(), dn.copy(), mr.copy(), noise, densify_enabled=enabled, **args)
    got_info = st.densify_info.cpu().numpy()
    assert got_info[0] == info["pruned"] and got_info[1] == info["clones"] and got_info[2] == info["splits"]
    assert bool(got_info[3]) == info["applied"]
    if case == "normal":
        assert info["clones"] > 0 and info["splits"] > 0 and info["pruned"] > 0
    if case in ("no_room", "disabled", "prune_only"):
        assert not info["applied"]
    np.testing.assert_array_equal(st.active_mask.cpu().numpy(), ract)
    gp, gmu, gnu = (_split_fields(b, n) for b in (st.params, st.mu, st.nu))
    for k in R.GROUPS:
        np.testing.assert_array_equal(gp[k], rp[k].numpy(), err_msg=k)
        np.testing.assert_array_equal(gmu[k], rmu[k].numpy(), err_msg=k)
        np.testing.assert_array_equal(gnu[k], rnu[k].numpy(), err_msg=k)
    assert not st.grad_accum.any() and not st.denom.any()
    np.testing.assert_array_equal(st.max_radii.cpu().numpy(), rmr)


def test_densify_large_capacity_counts():
    """A config-4-sized capacity (4M, 75 % active): counts agree with a numpy
    evaluation of the masks and the active count changes by clones + splits
    - pruned."""
    from gs_b200.training.density import densify_and_prune
    from gs_b200.training.trainer import DensityState
    n = 4_000_000
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    st = DensityState(n, K, "cuda")
    fields = st.gaussians
    fields.means.normal_(0, 1, generator=g)
    fields.scales.normal_(-3.5, 1.0, generator=g)
    fields.quaternions.normal_(0, 1, generator=g)
    fields.opacities.normal_(-1.0, 2.5, generator=g)
    st.active_mask.copy_(torch.rand(n, generator=g, device="cuda") < 0.75)
    st.denom.copy_(torch.randint(0, 20, (n,), generator=g, device="cuda", dtype=torch.int32))
    st.grad_accum.copy_(torch.rand(n, generator=g, device="cuda") * st.denom * 2.1e-4)
    st.max_radii.copy_(torch.rand(n, generator=g, device="cuda") * 600)
    before = int(st.active_mask.sum())
    densify_and_prune(st, rng_key=7)
    pruned, clones, splits, applied = (int(x) for x in st.densify_info.cpu())
    assert applied == 1 and clones > 0 and splits > 0
    assert int(st.active_mask.sum()) == before - pruned + clones + splits


def test_reset_opacities_matches_oracle():
    from gs_b200.training.density import reset_opacities
    n = 1000
    p, mu, nu, active, ga, dn, mr, _ = _random_state(5, n)
    st = _device_state(p, mu, nu, active, ga, dn, mr)
    reset_opacities(st, 0.01)
    ref = R.reset_opacities({k: torch.tensor(v) for k, v in p.items()}, active, 0.01)
    np.testing.assert_array_equal(_split_fields(st.params, n)["opacities"], ref["opacities"].numpy())
