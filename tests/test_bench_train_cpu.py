"""bench_train.py's contract on CPU (tiny model, gloo): one JSON line with the training
throughput fields, for one rank and for two FSDP2 ranks."""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.timeout(600)
@pytest.mark.parametrize("world", [1, 2])
def test_bench_train_tiny(world):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), "bench_train.py",
           "--tiny", "--steps", "1", "--warmup", "1", "--gpus", str(world)]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=580)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    out = json.loads(lines[0])
    assert out["n_gpus"] == world and out["steps"] == 1 and out["value"] > 0
    assert out["higher_is_better"] is True and out["loss"] == out["loss"]


@pytest.mark.timeout(600)
@pytest.mark.parametrize("world,kernels", [(1, "on"), (2, "off")])
def test_bench_train_dmd_tiny(world, kernels):
    """--stage dmd times DMD2 sub-iterations on the 1:5 turn schedule and reports each turn
    kind and the cycle rate; --kernels off (the labelled baseline arm) runs the same loop."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), "bench_train.py",
           "--tiny", "--stage", "dmd", "--steps", "2", "--warmup", "2", "--gpus", str(world),
           "--kernels", kernels]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=580)
    assert r.returncode == 0, r.stderr[-3000:]
    out = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][0])
    assert "Stage DMD" in out["metric"] and out["kernels"] == kernels
    assert len(out["step_ms"]) == 2 and out["generator_turn_ms"] > 0 and out["fake_turn_ms"] > 0
    assert out["cycle_samples_per_s"] > 0 and len(out["rollout_k"]) == 2
