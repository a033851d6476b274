"""Two-GPU data-parallel step: the fused peer-memory path (gs_dp_update over
CUDA IPC) against the NCCL all-reduce path, as two spawned NCCL ranks.
Skipped where fewer than two GPUs are visible (the round-end GPU test box
has one)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "jax-gs_b200"), root]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from tests.helpers import random_scene, to_torch
        from gs_b200.core.gaussians import Gaussians
        from gs_b200.training.trainer import AdamConfig, init_density_state, train_step_internal
        sc = random_scene(41, 3000, 96, 80, sh_degree=3, behind=0.05)
        na = 2200
        t = to_torch(sc, "cuda")
        g = Gaussians(means=t["means"][:na], scales=t["scales"][:na], quaternions=t["quats"][:na],
                      opacities=t["opac"][:na], sh_coeffs=t["sh"][:na])
        opt = AdamConfig.from_extent(3.0, 100)
        states = {f: init_density_state(g, opt, 3000) for f in (True, False)}
        cam = (sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"])
        rng = np.random.default_rng(rank)
        losses = {True: [], False: []}
        for step in range(3):
            w2c = torch.tensor(sc["w2c"], device="cuda")
            w2c[0, 3] += 0.05 * (rank - 0.5) + 0.01 * step  # a different view per rank and step
            tgt = torch.tensor(rng.uniform(0, 1, (sc["H"], sc["W"], 3)).astype(np.float32), device="cuda")
            for fused, st in states.items():
                _, loss, _ = train_step_internal(st, tgt, w2c, cam, opt, sh_degree=3, group=dist.group.WORLD,
                                                 fused=fused)
                losses[fused].append(float(loss))
        torch.cuda.synchronize()
        out = {}
        for fused, st in states.items():
            for name in ("params", "grad_accum", "max_radii", "denom"):
                buf = getattr(st, name).contiguous()
                allb = [torch.empty_like(buf) for _ in range(world)]
                dist.all_gather(allb, buf)
                out[(fused, name)] = [b.cpu().numpy() for b in allb]
        out["losses"] = losses
        out["count"] = [int(st.adam_state[0]) for st in states.values()]
        peer_sets = [v for v in states[True]._buffers.values() if hasattr(v, "timeouts")]
        out["barrier"] = [(v.device_barrier, v.timeouts()) for v in peer_sets]
        if rank == 0:
            q.put(out)
        dist.barrier()
    finally:
        for st in locals().get("states", {}).values():
            for v in st._buffers.values():
                if hasattr(v, "close"):
                    v.close()
        dist.destroy_process_group()


def test_fused_dp_update_matches_nccl_path():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    import queue
    import time
    out, t0 = None, time.time()
    while out is None and time.time() - t0 < 300:
        try:
            out = q.get(timeout=2)
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert out is not None
    assert out["count"] == [3, 3]
    # the fused path's rendezvous ran over peer memory and never timed out
    assert out["barrier"] and all(dev and t == 0 for dev, t in out["barrier"]), out["barrier"]
    np.testing.assert_allclose(out["losses"][True], out["losses"][False], rtol=1e-5)
    for name in ("params", "grad_accum", "max_radii", "denom"):
        fused, ref = out[(True, name)], out[(False, name)]
        # replicas stay identical across ranks (denom counts each rank's own view)
        if name != "denom":
            assert np.array_equal(fused[0], fused[1]), name
            assert np.array_equal(ref[0], ref[1]), name
        for r in range(2):
            if name in ("denom", "max_radii"):
                np.testing.assert_array_equal(fused[r], ref[r], err_msg=name)
            elif name == "grad_accum":
                np.testing.assert_allclose(fused[r], ref[r], rtol=1e-4, atol=1e-6 * np.abs(ref[r]).max())
            else:
                d = np.abs(fused[r] - ref[r])
                assert np.median(d) <= 1e-6 and d.max() <= 3 * 2 * 0.05 + 1e-6, name
