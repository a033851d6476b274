"""Data-parallel host logic (trainer.py:69-71, :97, :108-113) on two CPU
ranks over gloo: the gradient buffer (with its loss / metric tail) is
averaged, grad_2d averaged, radii / visibility max-reduced, and every rank
ends with identical state."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "jax-gs_b200"), root]
    from gs_b200.training.trainer import pmean_gradients, pmean_grad2d_pmax_radii
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    g = torch.Generator().manual_seed(100 + rank)
    n = 50
    grads = torch.randn(59 * n + 16, generator=g)
    tail = grads[59 * n:]
    tail[:3] = torch.tensor([0.1 * (rank + 1), 0.2 * (rank + 1), 0.3])
    extras = torch.zeros(16, dtype=torch.int32)
    extras[0] = 1000 * (rank + 1)
    extras[1:2].view(torch.float32)[0] = 2.5 * (rank + 1)
    extras[2] = 7 + rank
    before = grads.clone()
    pmean_gradients(grads, tail, extras, dist.group.WORLD)
    g2d = torch.randn(n, generator=g).abs()
    g2d_before = g2d.clone()
    radii = torch.randint(0, 50, (n,), generator=g).float()
    valid = (torch.rand(n, generator=g) > 0.5).to(torch.uint8)
    r_max, v_any = pmean_grad2d_pmax_radii(g2d, radii, valid, dist.group.WORLD)
    out[rank] = dict(before=before, after=grads.clone(), g2d_before=g2d_before, g2d=g2d.clone(),
                     radii=radii, valid=valid, r_max=r_max, v_any=v_any)
    dist.barrier()
    dist.destroy_process_group()


def test_data_parallel_reductions_two_ranks():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    a, b = out[0], out[1]
    n = 50
    mean = (a["before"][:59 * n] + b["before"][:59 * n]) / 2
    for r in (a, b):
        torch.testing.assert_close(r["after"][:59 * n], mean)
        t = r["after"][59 * n:]
        torch.testing.assert_close(t[:3], torch.tensor([0.15, 0.3, 0.3]))
        assert float(t[3]) == pytest.approx(1500.0)  # n_interactions averaged
        assert float(t[4]) == pytest.approx(3.75)    # mean_interactions_per_tile (a float field)
        assert float(t[5]) == pytest.approx(7.5)
        torch.testing.assert_close(r["g2d"], (a["g2d_before"] + b["g2d_before"]) / 2)
        masked = lambda q: torch.where(q["valid"].bool(), q["radii"], torch.zeros(()))  # noqa: E731
        torch.testing.assert_close(r["r_max"], torch.maximum(masked(a), masked(b)))
        assert torch.equal(r["v_any"], ((a["valid"] + b["valid"]) > 0).to(torch.uint8))
    assert torch.equal(a["after"], b["after"])


K_SH = 16
_WIDTHS = {"means": 3, "scales": 3, "quaternions": 4, "opacities": 1, "sh_coeffs": 3 * K_SH}


def _flat_to_groups(buf, n):
    from oracle import ref_restated as R
    out, off = {}, 0
    for k in R.GROUPS:
        w = _WIDTHS[k]
        shape = (n, K_SH, 3) if k == "sh_coeffs" else (n, w)
        out[k] = buf[off:off + n * w].reshape(shape).clone()
        off += n * w
    return out


def _groups_to_flat(d):
    from oracle import ref_restated as R
    return torch.cat([torch.as_tensor(d[k]).reshape(-1) for k in R.GROUPS])


def _density_inputs(n):
    """The replicated state of the ranks (identical parameters, mask and
    statistics; rank-specific denominators) and the true Adam moments."""
    g = torch.Generator().manual_seed(11)
    size = 59 * n
    params = torch.randn(size, generator=g)
    params[3 * n:6 * n] = params[3 * n:6 * n] * 0.8 - 3.5  # log scales around -3.5
    params[10 * n:11 * n] = params[10 * n:11 * n] * 2.5 - 1.0  # opacity logits
    mu = torch.randn(size, generator=g) * 1e-3
    nu = torch.rand(size, generator=g) * 1e-5
    active = torch.rand(n, generator=g) < 0.7
    grad_accum = torch.rand(n, generator=g) * 6e-3
    max_radii = torch.rand(n, generator=g) * 600
    noise = torch.randn(n, 3, generator=g)
    return params, mu, nu, active, grad_accum, max_radii, noise


def _denom(rank, n):
    return torch.randint(0, 30, (n,), generator=torch.Generator().manual_seed(200 + rank), dtype=torch.int32)


def _densify_worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "jax-gs_b200"), root]
    from gs_b200.training.density import update_from_rank0
    from gs_b200.training.trainer import DensityState, dp_owner
    from oracle import ref_restated as R
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    n = 400
    params, mu, nu, active, grad_accum, max_radii, noise = _density_inputs(n)
    st = DensityState(n, K_SH, "cpu")
    st.params.copy_(params)
    st.active_mask.copy_(active)
    st.grad_accum.copy_(grad_accum)
    st.max_radii.copy_(max_radii)
    st.denom.copy_(_denom(rank, n))
    # sliced moments, as the fused update leaves them: current on this
    # rank's slice of every group, stale (here: rank-specific junk) elsewhere
    junk = torch.Generator().manual_seed(300 + rank)
    st.mu.copy_(torch.randn(59 * n, generator=junk))
    st.nu.copy_(torch.randn(59 * n, generator=junk))
    own = dp_owner(n, world) == rank
    for (a, b), w in zip(st.segments, [3, 3, 4, 1, 3 * K_SH]):
        st.mu[a:b].view(n, w)[own] = mu[a:b].view(n, w)[own]
        st.nu[a:b].view(n, w)[own] = nu[a:b].view(n, w)[own]

    def oracle_update(s):
        p, m, v, act, ga, dn, mr, info = R.densify_and_prune(
            _flat_to_groups(s.params, n), _flat_to_groups(s.mu, n), _flat_to_groups(s.nu, n),
            s.active_mask.numpy().copy(), s.grad_accum.numpy().copy(), s.denom.numpy().copy(),
            s.max_radii.numpy().copy(), noise.numpy(), extent=5.0)
        s.params.copy_(_groups_to_flat(p))
        s.mu.copy_(_groups_to_flat(m))
        s.nu.copy_(_groups_to_flat(v))
        s.active_mask.copy_(torch.as_tensor(act))
        s.grad_accum.copy_(torch.as_tensor(ga))
        s.denom.copy_(torch.as_tensor(dn))
        s.max_radii.copy_(torch.as_tensor(mr))
        s.densify_info = torch.tensor([info["pruned"], info["clones"], info["splits"], int(info["applied"])],
                                      dtype=torch.int32)

    update_from_rank0(st, dist.group.WORLD, oracle_update, fused=True)
    out[rank] = {k: getattr(st, k).clone() for k in ("params", "mu", "nu", "active_mask", "grad_accum", "denom",
                                                     "max_radii", "densify_info")}
    dist.barrier()
    dist.destroy_process_group()


def test_densify_on_rank0_is_copied_to_every_rank():
    """train_parallel.py:269-283 on two gloo ranks: the density step runs on
    rank 0's state (rank 0's denominators, the moments gathered from their
    slice owners) and every rank ends with exactly that result."""
    from oracle import ref_restated as R
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_densify_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    n = 400
    params, mu, nu, active, grad_accum, max_radii, noise = _density_inputs(n)
    p, m, v, act, ga, dn, mr, info = R.densify_and_prune(
        _flat_to_groups(params, n), _flat_to_groups(mu, n), _flat_to_groups(nu, n), active.numpy().copy(),
        grad_accum.numpy().copy(), _denom(0, n).numpy(), max_radii.numpy().copy(), noise.numpy(), extent=5.0)
    assert info["applied"] and info["clones"] > 0 and info["splits"] > 0 and info["pruned"] > 0
    want = {"params": _groups_to_flat(p), "mu": _groups_to_flat(m), "nu": _groups_to_flat(v),
            "active_mask": torch.as_tensor(act), "grad_accum": torch.as_tensor(ga), "denom": torch.as_tensor(dn),
            "max_radii": torch.as_tensor(mr)}
    for r in (0, 1):
        for k, w in want.items():
            assert torch.equal(out[r][k], w.to(out[r][k].dtype)), (r, k)
        assert out[r]["densify_info"].tolist() == [info["pruned"], info["clones"], info["splits"], 1]
    # rank 1's own denominators would have routed differently
    p1 = R.densify_and_prune(
        _flat_to_groups(params, n), _flat_to_groups(mu, n), _flat_to_groups(nu, n), active.numpy().copy(),
        grad_accum.numpy().copy(), _denom(1, n).numpy(), max_radii.numpy().copy(), noise.numpy(), extent=5.0)[0]
    assert not torch.equal(_groups_to_flat(p1), want["params"])
