"""The C++ drop-in: tests/matmul_test.cpp, a program on the reference's C++ API
(aegis::matmul in its f16 pointer form and its GemmParams form, matmul_choice,
gemm::registry / find), linked statically against libaegis.a and run on the
GPU, as the reference's tests/test_matmul.cu runs against its libaegis.a. Its
outputs are checked against the FP64 oracle under both bounds."""
import json
import subprocess

import numpy as np
import pytest

import aegis_capi as ac
import oracle_py as op
from cpp_build import build_matmul_test
from gpu_util import check, context

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(512, 512, 512), (300, 1000, 777)])
def test_cpp_program_against_the_oracle(cuda, tmp_path, shape):
    M, N, K = shape
    exe = tmp_path / "matmul_test"
    r = build_matmul_test(str(exe))
    assert r.returncode == 0, r.stderr[-3000:]
    out = subprocess.run([str(exe), str(tmp_path / "c"), str(M), str(N), str(K)], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-3000:]
    facts = json.loads(out.stdout.strip().splitlines()[-1])
    ctx = context(cuda)
    assert facts["registry"] == len(ctx.registry()) and facts["find_pair"] and facts["invalid_refused"]
    assert facts["choice_f16"] == ctx.plan(M, N, K, None, ac.DTYPE_F16)["impl"]
    assert facts["choice_bf16"] == ctx.plan(M, N, K, None, ac.DTYPE_BF16)["impl"]
    for dtype in ("f16", "bf16"):
        g = ac.Generator(0)  # std::mt19937(0), uniform[-1, 1], A then B: the program's own draws
        A, B = g.uniform(M * K, dtype), g.uniform(K * N, dtype)
        got = np.fromfile(tmp_path / f"c.{dtype}", dtype=np.uint16)
        d = op.make_desc(M, N, K, dtype=dtype)
        check(d, A, B, None, got, op.gemm_ref(d, A, B), name=f"C++ aegis::matmul {dtype} {shape}")
