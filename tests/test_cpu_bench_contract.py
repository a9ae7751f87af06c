"""The benchmark's CPU reference arm keeps the JSON-line contract the round-end
driver reads: one line, impl "reference", the CUDA arm's metric and workload,
at least three warm-up steps, a cpu_baseline describing this run and an e2e
object that moves no bytes between host and device.  It times the C++
restatement of the reference decoder (the C# reference cannot run here), so it
needs no GPU and never loads the product library."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ)
    env.pop("CUDA_VISIBLE_DEVICES", None)
    # bench.py runs as __main__ in a child that then reports whether the
    # product library is mapped into it
    script = ("import runpy, sys\n"
              "sys.argv = ['bench.py', '--impl', 'reference', '--config', 'bs1_100', '--steps', '2', '--warmup', '1']\n"
              "runpy.run_path('bench.py', run_name='__main__')\n"
              "print('MAPPED', open('/proc/self/maps').read().count('libfunasr_cuda'))\n")
    out = subprocess.run([sys.executable, "-c", script], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["metric"] == "decode tokens/sec (Qwen3-0.6B Q8_0 bs1)" and d["unit"] == "tokens/s"
    assert d["n_gpus"] == 1 and d["steps"] == 2 and d["warmup"] == 3  # warm-up is raised to the minimum of 3
    assert d["value"] > 0 and d["higher_is_better"] is True and d["vs_baseline"] is None
    assert abs(d["ms_per_step"] - 1000.0 / d["value"]) < 1e-9 * d["ms_per_step"] + 1e-12
    assert d["config"]["workload"] == "qwen3-0.6b-q8_0 bs1 prefix 100+8, greedy 128"
    assert d["config"]["timed_positions"] == [108, 110]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["unit"] == "tokens/s"
    assert "2 decode steps after the 108-frame prefill" in cb["sample"]
    # the product library stayed unloaded
    assert "MAPPED 0" in out.stdout.splitlines(), out.stdout[-500:]


def test_reference_arm_under_torchrun_prints_once():
    """Launched like the CUDA arm at N > 1 (torchrun, one process per GPU),
    rank 0 alone runs the CPU reference and prints; the other rank exits 0
    without work and without a process group."""
    env = dict(os.environ)
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
           "--gpus", "2", "--config", "bs1_100", "--steps", "2", "--warmup", "3"]
    out = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["config"]["parallelism"] == "replicas x2"
