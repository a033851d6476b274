"""Two-GPU data-parallel step: the fused peer-memory path (gs_dp_update over
CUDA IPC) against the NCCL all-reduce path and the oracle's mean-of-views
step, and the density step on rank 0's authoritative state copied to every
rank, as two spawned NCCL ranks. Skipped where fewer than two GPUs are
visible."""
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
        from gs_b200.training import trainer as T
        from gs_b200.training.trainer import AdamConfig, init_density_state, train_step_internal
        sc = random_scene(41, 3000, 96, 80, sh_degree=3, behind=0.05)
        na = 2200
        t = to_torch(sc, "cuda")
        g = Gaussians(means=t["means"][:na], scales=t["scales"][:na], quaternions=t["quats"][:na],
                      opacities=t["opac"][:na], sh_coeffs=t["sh"][:na])
        opt = AdamConfig.from_extent(3.0, 100)
        # True: the fused peer-memory path; False: the NCCL path; "skip": the
        # fused path with untouched gradient rows skipped (published flags),
        # which two ranks use only when asked
        states = {f: init_density_state(g, opt, 3000) for f in (True, False, "skip")}
        skip_default = T.DP_SKIP_MIN_RANKS
        cam = (sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"])
        rng = np.random.default_rng(rank)
        losses = {True: [], False: [], "skip": []}
        metrics = {}
        for step in range(3):
            w2c = torch.tensor(sc["w2c"], device="cuda")
            w2c[0, 3] += 0.05 * (rank - 0.5) + 0.01 * step  # a different view per rank and step
            tgt = torch.tensor(rng.uniform(0, 1, (sc["H"], sc["W"], 3)).astype(np.float32), device="cuda")
            for fused, st in states.items():
                T.DP_SKIP_MIN_RANKS = 1 if fused == "skip" else skip_default
                _, loss, m = train_step_internal(st, tgt, w2c, cam, opt, sh_degree=3, group=dist.group.WORLD,
                                                 fused=fused is not False)
                losses[fused].append(float(loss))
                metrics[fused] = {k: float(v) for k, v in m.items()}
            T.DP_SKIP_MIN_RANKS = skip_default
            if step == 0:
                # the first Adam moment after one step is (1 - b1) times the
                # averaged gradient: made whole over the slice owners, it
                # shows the fused path's mean-of-views gradient
                from gs_b200.training.density import gather_moments
                gather_moments(states[True], dist.group.WORLD)
                mu1 = states[True].mu.detach().cpu().clone()
        torch.cuda.synchronize()
        out = {"mu_step1": mu1}
        for fused, st in states.items():
            for name in ("params", "grad_accum", "max_radii", "denom"):
                buf = getattr(st, name).contiguous()
                allb = [torch.empty_like(buf) for _ in range(world)]
                dist.all_gather(allb, buf)
                out[(fused, name)] = [b.cpu().numpy() for b in allb]
        out["losses"] = losses
        out["metrics"] = metrics
        out["count"] = [int(st.adam_state[0]) for st in states.values()]
        peer_sets = [v for k in (True, "skip") for v in states[k]._buffers.values() if hasattr(v, "timeouts")]
        out["barrier"] = [(v.device_barrier, v.timeouts()) for v in peer_sets]
        out["skip_on"] = [v.skip_untouched for v in peer_sets]
        if rank == 0:
            q.put(out)
        dist.barrier()
    finally:
        for st in locals().get("states", {}).values():
            for v in st._buffers.values():
                if hasattr(v, "close"):
                    v.close()
        dist.destroy_process_group()


def _check_mean_of_views_gradient(mu1):
    """trainer.py:69: the step's gradient is the mean over the ranks of each
    rank's own view gradient. The oracle computes both views' gradients (the
    inputs of _worker's first step) and their mean; the fused step's first
    moment divided by (1 - b1) must match it at the renderer's gradient bar."""
    from oracle import ref_restated as R
    from tests.helpers import random_scene
    from gs_b200.core.gaussians import Gaussians
    from gs_b200.training.trainer import AdamConfig, init_density_state
    sc = random_scene(41, 3000, 96, 80, sh_degree=3, behind=0.05)
    na, n = 2200, 3000
    t = {k: torch.as_tensor(sc[k]) for k in ("means", "scales", "quats", "opac", "sh")}
    g = Gaussians(means=t["means"][:na], scales=t["scales"][:na], quaternions=t["quats"][:na],
                  opacities=t["opac"][:na], sh_coeffs=t["sh"][:na])
    opt = AdamConfig.from_extent(3.0, 100)
    st = init_density_state(g, opt, n)  # CPU tensors: the padded state of the workers
    fields = st.gaussians
    params = {"means": fields.means, "scales": fields.scales, "quaternions": fields.quaternions,
              "opacities": fields.opacities, "sh_coeffs": fields.sh_coeffs}
    zeros = {k: torch.zeros_like(v) for k, v in params.items()}
    cam = (sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"])
    mean = None
    for r in range(2):
        w2c = torch.tensor(sc["w2c"])
        w2c[0, 3] += 0.05 * (r - 0.5) + 0.01 * 0
        tgt = torch.tensor(np.random.default_rng(r).uniform(0, 1, (sc["H"], sc["W"], 3)).astype(np.float32))
        o = R.train_step(params, zeros, zeros, 1, dict(zip(R.GROUPS, opt.lrs(0))), st.active_mask, tgt, w2c, cam,
                         sh_degree=3)
        gr = torch.cat([o["grads"][k].reshape(-1) for k in R.GROUPS])
        mean = gr if mean is None else (mean + gr)
    mean = mean / 2
    got = mu1 / np.float32(1.0 - 0.9)
    act = st.active_mask.numpy()
    off = 0
    for k, w in zip(R.GROUPS, (3, 3, 4, 1, 48)):
        a = got[off:off + n * w].reshape(n, w).numpy()[act]
        r_ = np.nan_to_num(mean[off:off + n * w].reshape(n, w).numpy()[act])
        off += n * w
        scale = float(np.abs(r_).max())
        d = np.abs(a - r_)
        assert (d <= 1e-3 * (np.abs(r_) + scale) + 1e-12).all(), (k, float(d.max()), scale)
        big = np.abs(r_) > 1e-2 * scale  # per-element relative error where the gradient is not tiny
        if big.any():
            assert float((d[big] / np.abs(r_[big])).max()) <= 2e-2, k


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
    assert out["count"] == [3, 3, 3]
    assert out["skip_on"] == [False, True]
    # the fused path's rendezvous ran over peer memory and never timed out
    assert out["barrier"] and all(dev and t == 0 for dev, t in out["barrier"]), out["barrier"]
    np.testing.assert_allclose(out["losses"][True], out["losses"][False], rtol=1e-5)
    # the render counters averaged over the ranks: the fused paths read them
    # from every rank's extras, the NCCL path all-reduces them in the tail
    for path in (True, "skip"):
        for k, v in out["metrics"][False].items():
            assert out["metrics"][path][k] == pytest.approx(v, rel=1e-5, abs=1e-6), (path, k)
    assert out["metrics"][True]["n_interactions"] > 0 and out["metrics"][True]["device_timeouts"] == 0
    # skipping exact-zero gradient rows adds nothing but +0 less: the same
    # step as the fused path's, up to the compositor's atomic sums (whose
    # order changes from run to run); the same bars as against the NCCL path
    np.testing.assert_allclose(out["losses"]["skip"], out["losses"][True], rtol=1e-5)
    for name in ("params", "grad_accum", "max_radii", "denom"):
        skip, fused = out[("skip", name)], out[(True, name)]
        if name != "denom":
            assert np.array_equal(skip[0], skip[1]), name
        for r in range(2):
            if name in ("denom", "max_radii"):
                np.testing.assert_array_equal(skip[r], fused[r], err_msg=name)
            elif name == "grad_accum":
                np.testing.assert_allclose(skip[r], fused[r], rtol=1e-4, atol=1e-6 * np.abs(fused[r]).max())
            else:
                d = np.abs(skip[r] - fused[r])
                assert np.median(d) <= 1e-6 and d.max() <= 3 * 2 * 0.05 + 1e-6, name
    _check_mean_of_views_gradient(out["mu_step1"])
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


def _densify_worker(rank, world, port, q):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "jax-gs_b200"), root]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    st = None
    try:
        from tests.helpers import random_scene, to_torch
        from gs_b200.core.gaussians import Gaussians
        from gs_b200.training.density import densify_and_prune_parallel, gather_moments
        from gs_b200.training.trainer import AdamConfig, init_density_state, train_step_internal
        sc = random_scene(43, 3000, 96, 80, sh_degree=3, behind=0.05)
        na = 2200
        t = to_torch(sc, "cuda")
        g = Gaussians(means=t["means"][:na], scales=t["scales"][:na], quaternions=t["quats"][:na],
                      opacities=t["opac"][:na], sh_coeffs=t["sh"][:na])
        opt = AdamConfig.from_extent(3.0, 100)
        st = init_density_state(g, opt, 3000)
        cam = (sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"])
        rng = np.random.default_rng(rank)
        for step in range(4):
            w2c = torch.tensor(sc["w2c"], device="cuda")
            w2c[0, 3] += 0.2 * (rank - 0.5) + 0.01 * step  # each rank sees its own views
            tgt = torch.tensor(rng.uniform(0, 1, (sc["H"], sc["W"], 3)).astype(np.float32), device="cuda")
            train_step_internal(st, tgt, w2c, cam, opt, sh_degree=3, group=dist.group.WORLD, fused=True)
        torch.cuda.synchronize()
        # rank 0's pre-densify state, moments made whole (what the step gathers)
        gather_moments(st, dist.group.WORLD)
        torch.cuda.synchronize()
        pre = {k: getattr(st, k).detach().cpu().clone() for k in
               ("params", "mu", "nu", "active_mask", "grad_accum", "denom", "max_radii")}
        # a threshold that selects about a fifth of rank 0's visible Gaussians
        avg = pre["grad_accum"] / pre["denom"].clamp(min=1).float()
        thr = torch.tensor([float(torch.quantile(avg[pre["denom"] > 0], 0.8))], device="cuda")
        dist.broadcast(thr, src=0)
        noise = torch.randn((3000, 3), generator=torch.Generator().manual_seed(9)).cuda()
        densify_and_prune_parallel(st, dist.group.WORLD, grad_threshold=float(thr), extent=3.0, noise=noise)
        torch.cuda.synchronize()
        out = {"pre": pre, "thr": float(thr), "noise": noise.cpu()}
        for name in ("params", "mu", "nu", "active_mask", "grad_accum", "denom", "max_radii", "densify_info"):
            buf = getattr(st, name).contiguous()
            if buf.dtype == torch.bool:
                buf = buf.to(torch.uint8)
            allb = [torch.empty_like(buf) for _ in range(world)]
            dist.all_gather(allb, buf)
            out[name] = [b.cpu() for b in allb]
        if rank == 0:
            q.put(out)
        dist.barrier()
    finally:
        if st is not None:
            for v in st._buffers.values():
                if hasattr(v, "close"):
                    v.close()
        dist.destroy_process_group()


def test_parallel_densify_runs_on_rank0_and_replicates():
    """train_parallel.py:269-283: after steps in which the ranks saw different
    views (so their denominators differ), the density step applied to rank
    0's state is what every rank holds afterwards, bit for bit, and equals
    the oracle's densify_and_prune of rank 0's pre-densify state."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from oracle import ref_restated as R
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_densify_worker, args=(r, 2, port, q)) for r in range(2)]
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
    for name in ("params", "mu", "nu", "active_mask", "grad_accum", "denom", "max_radii", "densify_info"):
        assert torch.equal(out[name][0], out[name][1]), name
    n, K = 3000, 16
    pre = out["pre"]
    widths = {"means": 3, "scales": 3, "quaternions": 4, "opacities": 1, "sh_coeffs": 3 * K}

    def groups(buf):
        d, off = {}, 0
        for k in R.GROUPS:
            w = widths[k]
            d[k] = buf[off:off + n * w].reshape((n, K, 3) if k == "sh_coeffs" else (n, w)).clone()
            off += n * w
        return d

    p, m, v, act, ga, dn, mr, info = R.densify_and_prune(
        groups(pre["params"]), groups(pre["mu"]), groups(pre["nu"]), pre["active_mask"].numpy().copy(),
        pre["grad_accum"].numpy().copy(), pre["denom"].numpy().copy(), pre["max_radii"].numpy().copy(),
        out["noise"].numpy(), grad_threshold=out["thr"], extent=3.0)
    assert info["applied"] and info["clones"] + info["splits"] > 0
    assert out["densify_info"][0].tolist() == [info["pruned"], info["clones"], info["splits"], 1]
    flat = lambda d: torch.cat([torch.as_tensor(d[k]).reshape(-1) for k in R.GROUPS])  # noqa: E731
    assert torch.equal(out["params"][0], flat(p))
    assert torch.equal(out["mu"][0], flat(m))
    assert torch.equal(out["nu"][0], flat(v))
    assert torch.equal(out["active_mask"][0], torch.as_tensor(act).to(torch.uint8))
    assert not out["grad_accum"][0].any() and not out["denom"][0].any()
    assert torch.equal(out["max_radii"][0], torch.as_tensor(mr))
