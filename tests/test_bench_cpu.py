"""bench.py's reference arm under torchrun, on CPU.

The arm times the reference's algorithm (the C restatement of ternary-rows)
on the host cores.  Launched like the GPU arm, with one process per GPU, rank
0 alone runs it and prints the one JSON line; the other ranks print nothing
and exit 0.
"""
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_reference_arm_under_torchrun_two_ranks():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    j = json.loads(lines[0])
    assert j["impl"] == "reference" and j["n_gpus"] == 2
    assert j["unit"] == "GB/s" and j["higher_is_better"] is True and j["value"] > 0
    assert j["steps"] == 1 and j["warmup"] == 3
    assert j["e2e"] == {"value": j["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    cpu = j["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == j["value"]
    assert j["config"]["workload"].startswith("ternary GEMV")
