"""The N-sharded GEMM across real GPUs (2 or more on one node): every rank's
C after the fused all-gather equals the single-GPU GEMM bit for bit
(tests/nsharded_worker.py under torchrun). Skipped with fewer than 2 GPUs."""
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def test_two_rank_fused_allgather_bitwise(cuda):
    n = cuda.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "60", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", "29517",
           os.path.join(ROOT, "tests", "nsharded_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=420)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
    assert r.stdout.count(": ok") == world
