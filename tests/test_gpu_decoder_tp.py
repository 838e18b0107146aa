"""The tensor-parallel decoder on 2 GPUs (NCCL all-reduce of the O and down
projections, vocab-split LM head with a max all-reduce of argmax keys)
against the CPU model: tests/tp_decoder_check.py under torchrun.  Skipped on
a machine with fewer than two GPUs."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _gpu_count():
    r = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True)
    return sum(1 for line in r.stdout.splitlines() if line.startswith("GPU "))


def test_decoder_tp2_matches_cpu_model():
    if _gpu_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29533", os.path.join(HERE, "tp_decoder_check.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TP_OK 2" in r.stdout
