"""The N-sharded GEMM across real GPUs (2, and every GPU of the node up to 8):
every rank's C after the fused all-gather equals the single-GPU GEMM bit for
bit (tests/nsharded_worker.py under torchrun). Skipped with fewer GPUs."""
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _run(world, port):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "60", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "tests", "nsharded_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=420)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
    assert r.stdout.count(": ok") == world


def test_two_rank_fused_allgather_bitwise(cuda):
    n = cuda.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    _run(2, 29517)


def test_all_gpus_fused_allgather_bitwise(cuda):
    """Every GPU of the node (up to the kernel's 8 peers) as one N-sharded GEMM."""
    n = min(8, cuda.cuda.device_count())
    if n < 3:
        pytest.skip("needs more than 2 GPUs")
    _run(n, 29518)
