"""bench.py's reference arm runs on the host alone: one bounded oracle step of
the default workload prints one JSON line with the contract's keys."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, cwd=ROOT, env=env, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    rec = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in rec, key
    assert rec["impl"] == "reference" and rec["value"] > 0
    assert rec["cpu_baseline"]["kind"] in ("port", "reference")
    assert rec["e2e"]["h2d_bytes_per_step"] == 0 and rec["e2e"]["d2h_bytes_per_step"] == 0
    # the same config object and warm-up count as the GPU arm's line
    sys.path.insert(0, ROOT)
    import bench
    assert rec["config"] == bench.static_config("train", 1)
    assert rec["warmup"] == 1 and rec["steps"] == 1


def test_reference_arm_config1_workload():
    """BASELINE config 1 (single-view fwd+bwd) on the host: its own metric,
    the warm-up count asked for, and the GPU arm's config object."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                          "config1", "--steps", "2", "--warmup", "2"], capture_output=True, text=True, cwd=ROOT,
                         env=env, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    rec = json.loads(lines[0])
    sys.path.insert(0, ROOT)
    import bench
    assert rec["metric"] == bench.METRICS["config1"][0] and rec["unit"] == "views/s"
    assert rec["config"] == bench.static_config("config1", 1)
    assert rec["warmup"] == 2 and rec["steps"] == 2 and rec["value"] > 0


def test_reference_arm_under_torchrun_prints_once_from_rank_0():
    """Launched as the driver launches N > 1 (torchrun, one process per
    rank), the reference arm runs on rank 0 alone: one JSON line, every rank
    exits 0 and the line reports the world size."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="4")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"),
           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1"]
    out = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, env=env, timeout=900)
    assert out.returncode == 0, out.stderr[-3000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and rec["n_gpus"] == 2 and rec["value"] > 0
