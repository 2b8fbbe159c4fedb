"""Shared test setup.

Markers: `gpu` tests need a CUDA device (a B200: the library ships sm_100a
code only); everything else runs on a CPU-only machine. The GPU tests call
the kernels only through the C ABI (libaegis_capi.so via aegis_capi.py) and
compare them with the CPU oracle (oracle/, test infrastructure).
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
for sub in ("aegis-core_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def golden_cases():
    return sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz") and f != "config1_512.npz")


def load_golden(name):
    import oracle_py as op
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    M, N, K, la, lb, lda, ldb, ldc, batch, sa, sb, sc = (int(v) for v in z["desc"])
    alpha, beta = (float(v) for v in z["alpha_beta"])
    d = op.make_desc(M, N, K, la, lb, lda, ldb, ldc, alpha, beta, batch, sa, sb, sc, "f16")
    return d, z["A"], z["B"], z["C0"], z["ref"], float(z["ref_tol"])


@pytest.fixture(scope="session")
def cuda():
    """torch with a CUDA device, or skip (GPU tests only)."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch
