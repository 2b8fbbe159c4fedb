"""Builds tests/matmul_test.cpp against the static archive libaegis.a with the
host C++ compiler (the C++ drop-in path: a program written against the
reference's C++ API, linked with no nvcc step)."""
import os
import shutil
import subprocess

from conftest import ROOT

ARCHIVE = os.path.join(ROOT, "aegis-core_b200", "build", "libaegis.a")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build_matmul_test(out_path: str) -> subprocess.CompletedProcess:
    cxx = shutil.which("g++") or shutil.which("c++")
    cmd = [cxx, "-std=c++20", "-O2", f"-I{ROOT}/include", f"-I{CUDA}/include",
           os.path.join(ROOT, "tests", "matmul_test.cpp"), "-L" + os.path.dirname(ARCHIVE), "-laegis",
           f"-L{CUDA}/lib64", "-lcudart_static", "-lpthread", "-ldl", "-lrt", "-o", out_path]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=300)
