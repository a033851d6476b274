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
