"""The tensor-parallel decoder on 2, 4 and 8 GPUs (peer exchange of the O and
down projections, vocab-split LM head with a max of the argmax keys) against
the CPU model: tests/tp_decoder_check.py under torchrun; and the report of a
peer wait that gives up.  Each case is skipped on a machine with fewer GPUs."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _gpu_count():
    r = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True)
    return sum(1 for line in r.stdout.splitlines() if line.startswith("GPU "))


def _torchrun(n, port, *args):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", str(n), "--master-addr", "127.0.0.1",
           "--master-port", str(port), os.path.join(HERE, "tp_decoder_check.py"), *args]
    return subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)


@pytest.mark.parametrize("n,extra", [(2, ()), (2, ("--uneven",)), (4, ()), (8, ())])
def test_decoder_tp_matches_cpu_model(n, extra):
    if _gpu_count() < n:
        pytest.skip(f"needs {n} GPUs")
    r = _torchrun(n, 29533 + n + 10 * len(extra), *extra)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert f"TP_OK {n}" in r.stdout


def test_decoder_tp2_peer_wait_timeout_is_reported():
    """One rank stops early; the other's bounded peer waits give up and its
    generate returns the error (no GPU fault, the context stays usable)."""
    if _gpu_count() < 2:
        pytest.skip("needs two GPUs")
    r = _torchrun(2, 29543, "--peer-timeout")
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TIMEOUT_OK 2" in r.stdout
