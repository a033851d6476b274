"""gs_dp_barrier's bounded wait, on one GPU: a rank whose peer never arrives
gets a counted timeout instead of a hang, and the context stays usable
(failure detection without a GPU fault: the flag that nothing sets)."""
import ctypes
import time

import pytest
import torch

from gs_b200 import _lib

pytestmark = pytest.mark.gpu


def _peer_set(flags):
    ps = _lib.GsPeerSet()
    ps.world, ps.rank = len(flags), 0
    for r, f in enumerate(flags):
        ps.flags[r] = f.data_ptr()
    return ps


def test_barrier_times_out_when_a_rank_never_arrives():
    dev = torch.device("cuda", 0)
    mine = torch.zeros(8, dtype=torch.int32, device=dev)    # this rank's rendezvous words
    absent = torch.zeros(8, dtype=torch.int32, device=dev)  # stands in for the missing rank's words
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ps = _peer_set([mine, absent])
    st = _lib.stream(dev)
    t0 = time.perf_counter()
    _lib.call("gs_dp_barrier", ctypes.byref(ps), _lib.ptr(epoch), _lib.ptr(status), st)
    torch.cuda.synchronize(dev)
    waited = time.perf_counter() - t0
    assert int(status.item()) == 1
    assert int(epoch.item()) == 1
    assert int(mine[0].item()) == 1 and int(absent[0].item()) == 1  # this rank raised its word everywhere
    assert int(mine[1].item()) == 0
    assert waited < 30.0
    # the context is still usable
    assert float(torch.ones(16, device=dev).sum().item()) == 16.0
    # the peer "arrives" at the next epoch: no further timeout
    mine[1] = 2
    torch.cuda.synchronize(dev)
    _lib.call("gs_dp_barrier", ctypes.byref(ps), _lib.ptr(epoch), _lib.ptr(status), st)
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 1
    assert int(epoch.item()) == 2


def test_barrier_single_rank_passes():
    dev = torch.device("cuda", 0)
    mine = torch.zeros(8, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ps = _peer_set([mine])
    for _ in range(3):
        _lib.call("gs_dp_barrier", ctypes.byref(ps), _lib.ptr(epoch), _lib.ptr(status), _lib.stream(dev))
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 0 and int(epoch.item()) == 3 and int(mine[0].item()) == 3


def test_update_after_a_timed_out_rendezvous_touches_no_peer():
    """After a rendezvous gave up, gs_dp_update must not read or write the
    absent rank's buffers (its process may be gone) nor change this rank's
    state; gs_train_step_metrics reports the expired wait."""
    dev = torch.device("cuda", 0)
    n, k = 64, 16
    rec = 11 + 3 * k
    st = _lib.stream(dev)
    g = torch.Generator(device=dev).manual_seed(5)

    def rank_buffers(fill):
        f = dict(device=dev, dtype=torch.float32)
        return {"params": torch.randn(rec * n, generator=g, **f), "grads": torch.randn(rec * n + 16, generator=g, **f),
                "radii": torch.full((n,), fill, **f), "valid": torch.ones(n, dtype=torch.uint8, device=dev),
                "w2c": torch.eye(4, **f), "grad_accum": torch.full((n,), fill, **f),
                "denom": torch.full((n,), 7, dtype=torch.int32, device=dev), "max_radii": torch.full((n,), fill, **f),
                "flags": torch.zeros(8, dtype=torch.int32, device=dev)}

    mine, absent = rank_buffers(1.0), rank_buffers(-3.0)
    ps = _lib.GsPeerSet()
    ps.world, ps.rank = 2, 0
    for r, b in enumerate((mine, absent)):
        for key in ("params", "grads", "radii", "valid", "w2c", "grad_accum", "denom", "max_radii", "flags"):
            getattr(ps, key)[r] = b[key].data_ptr()
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.call("gs_dp_barrier", ctypes.byref(ps), _lib.ptr(epoch), _lib.ptr(status), st)  # rank 1 never arrives
    mu = torch.randn(rec * n, generator=g, device=dev)
    nu = torch.rand(rec * n, generator=g, device=dev)
    adam_state = torch.zeros(2, dtype=torch.int32, device=dev)
    tail_out = torch.full((16,), 9.0, device=dev)
    before = {name: {key: t.clone() for key, t in b.items()} for name, b in (("mine", mine), ("absent", absent))}
    mu0, nu0 = mu.clone(), nu.clone()
    from gs_b200.training.trainer import AdamConfig
    sched = AdamConfig().schedule()
    _lib.call("gs_dp_update", ctypes.byref(ps), _lib.ptr(mu), _lib.ptr(nu), n, k, None, ctypes.byref(sched),
              _lib.ptr(adam_state), 100.0, 100.0, 64, 48, 16, _lib.ptr(tail_out), _lib.ptr(status), st)
    out = torch.zeros(12, device=dev)
    ex = torch.zeros(16, dtype=torch.int32, device=dev)
    _lib.call("gs_train_step_metrics", _lib.ptr(tail_out), _lib.ptr(ex), 0.2, _lib.ptr(status), _lib.ptr(out), st)
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 1
    for name, b in (("mine", mine), ("absent", absent)):
        for key, t in b.items():
            if key == "flags":
                continue  # the barrier itself raised this rank's word everywhere
            assert torch.equal(t, before[name][key]), (name, key)
    assert torch.equal(mu, mu0) and torch.equal(nu, nu0)
    assert adam_state.tolist() == [0, 0]  # no optax count advanced
    assert torch.all(tail_out == 9.0)
    assert float(out[11]) == 1.0  # the step reports the expired wait
    # with a clean status word the same call does update (and reads the "peer")
    status.zero_()
    _lib.call("gs_dp_update", ctypes.byref(ps), _lib.ptr(mu), _lib.ptr(nu), n, k, None, ctypes.byref(sched),
              _lib.ptr(adam_state), 100.0, 100.0, 64, 48, 16, _lib.ptr(tail_out), _lib.ptr(status), st)
    torch.cuda.synchronize(dev)
    assert adam_state.tolist()[0] == 1
    assert not torch.equal(mine["params"], before["mine"]["params"])
    # rank 0 owns the first stripe of 32 Gaussians (of 64): their new values
    # are written to every replica, the other stripe is left to rank 1
    from gs_b200.training.trainer import dp_owner
    own_g = dp_owner(n, 2, dev) == 0
    assert own_g[:32].all() and not own_g[32:].any()
    off = 0
    for w in (3, 3, 4, 1, 3 * k):
        seg = slice(off, off + w * n)
        m_new, a_new = mine["params"][seg].view(n, w), absent["params"][seg].view(n, w)
        a_old = before["absent"]["params"][seg].view(n, w)
        assert torch.equal(m_new[own_g], a_new[own_g])
        assert torch.equal(a_new[~own_g], a_old[~own_g])
        off += w * n
