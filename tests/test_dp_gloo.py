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
