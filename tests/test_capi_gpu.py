"""The C ABI test program (tests/capi_test.c, strict C11) built and run on
the GPU, as the reference runs its tests/capi_test.c under ctest."""
import os
import subprocess

import pytest

import aegis_capi as ac
from conftest import ROOT

pytestmark = pytest.mark.gpu


def test_capi_program(cuda, tmp_path):
    exe = tmp_path / "capi_test"
    libdir = os.path.dirname(ac.LIB_PATH)
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    "-I" + os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "capi_test.c"),
                    "-L" + libdir, "-laegis_capi", "-lm", "-Wl,-rpath," + libdir, "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    print(r.stdout[-4000:])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "capi_test: all passed" in r.stdout
