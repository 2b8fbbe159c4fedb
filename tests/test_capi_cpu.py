"""C ABI checks that need no GPU: the shared library loads, exports exactly
the functions include/aegis.h declares (the reference's
tests/test_capi_exports.sh rule: only aegis_* symbols, all declared), the
test program compiles as strict C11 against the drop-in include path, and
the argument checks that run before any CUDA call behave."""
import ctypes
import os
import re
import subprocess

import pytest

import aegis_capi as ac
from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "aegis.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^AEGIS_API [^(]*?\b(aegis_[a-z0-9_]+)\s*\(", src, re.M)))


def exported():
    out = subprocess.run(["nm", "-D", "--defined-only", ac.LIB_PATH], check=True, capture_output=True, text=True)
    return sorted({line.split()[-1] for line in out.stdout.splitlines() if line.strip()})


def test_exports_exactly_the_declared_abi():
    decl, exp = declared(), exported()
    assert len(decl) == 34
    assert [s for s in exp if not s.startswith("aegis_")] == []
    assert exp == decl


def test_every_declared_symbol_resolves():
    lib = ac.load()
    for name in declared():
        assert getattr(lib, name) is not None
    assert set(declared()) == set(ac._SIGNATURES)  # the Python binding declares every entry point


def test_abi_1_3_entry_points_kept():
    names = set(declared())
    for n in ["aegis_abi_version", "aegis_status_string", "aegis_last_error_string", "aegis_create",
              "aegis_destroy", "aegis_set_stream", "aegis_synchronize", "aegis_last_error", "aegis_device_alloc",
              "aegis_device_free", "aegis_copy_to_device", "aegis_copy_to_host", "aegis_gemm_f16",
              "aegis_gemm_f16_ex", "aegis_gemm_f16_strided_batched", "aegis_gemm_choice", "aegis_device_manifest",
              "aegis_hw_info_json", "aegis_hw_gpu", "aegis_hw_cpu"]:
        assert n in names


def test_struct_layouts_match_the_reference_abi():
    class Gpu(ctypes.Structure):
        _fields_ = [("struct_size", ctypes.c_uint32), ("present", ctypes.c_int32), ("device", ctypes.c_int32),
                    ("arch", ctypes.c_int32), ("sm_count", ctypes.c_int32), ("regs_per_sm", ctypes.c_int32),
                    ("smem_per_sm", ctypes.c_int64), ("smem_per_block", ctypes.c_int64),
                    ("smem_per_block_optin", ctypes.c_int64), ("l2_bytes", ctypes.c_int64),
                    ("memory_bytes", ctypes.c_int64), ("unified", ctypes.c_int32), ("tma_hardware", ctypes.c_int32),
                    ("tma_built", ctypes.c_int32), ("nvml", ctypes.c_int32), ("max_sm_clock_mhz", ctypes.c_int32),
                    ("max_mem_clock_mhz", ctypes.c_int32), ("power_limit_w", ctypes.c_double),
                    ("name", ctypes.c_char * 128)]
    prog = r'''
#include <stdio.h>
#include <stddef.h>
#include "aegis/aegis.h"
int main(void){printf("%zu %zu %zu\n", sizeof(aegis_hw_gpu_info), offsetof(aegis_hw_gpu_info, power_limit_w),
 sizeof(aegis_hw_cpu_info));return 0;}'''
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "s.c")
        open(c, "w").write(prog)
        exe = os.path.join(d, "s")
        subprocess.run(["gcc", "-std=c11", "-I" + os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        got = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split()
    assert int(got[0]) == ctypes.sizeof(Gpu) and int(got[1]) == Gpu.power_limit_w.offset

    class Cpu(ctypes.Structure):
        _fields_ = [("struct_size", ctypes.c_uint32), ("logical_cpus", ctypes.c_int32), ("clusters", ctypes.c_int32),
                    ("core_types", ctypes.c_int32), ("performance_cores", ctypes.c_int32),
                    ("performance_max_khz", ctypes.c_int64)] + [(f, ctypes.c_int32) for f in
                                                                ("neon", "fp16", "dotprod", "sve", "sve2", "i8mm",
                                                                 "bf16")]
    assert int(got[2]) == ctypes.sizeof(Cpu) == 64


def test_capi_test_compiles_as_strict_c11(tmp_path):
    exe = tmp_path / "capi_test"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    "-I" + os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "capi_test.c"),
                    "-L" + os.path.dirname(ac.LIB_PATH), "-laegis_capi", "-lm", "-o", str(exe)], check=True)
    assert exe.exists()


def test_host_side_argument_checks_without_gpu():
    lib = ac.load()
    assert lib.aegis_abi_version() == 1004
    assert lib.aegis_status_string(ac.AEGIS_ERR_CUDA).decode() != "unknown status"
    assert lib.aegis_status_string(12345).decode() == "unknown status"
    assert lib.aegis_create(None, 0) == ac.AEGIS_ERR_INVALID_ARGUMENT
    assert lib.aegis_gemm_f16(None, None, None, None, 4, 4, 4) == ac.AEGIS_ERR_INVALID_ARGUMENT
    assert "NULL" in ac.last_error_string()
    assert lib.aegis_destroy(None) == ac.AEGIS_OK
    assert lib.aegis_gemm_choice(None, 0, 4, 4, None, 0, None) == ac.AEGIS_ERR_INVALID_ARGUMENT
    assert lib.aegis_watchdog_selftest(None, 10) == ac.AEGIS_ERR_INVALID_ARGUMENT
    info = ac.hw_info(-1)  # host only: makes no CUDA call
    assert info["schema"] == "aegis-hw/1" and info["cpu"]["logical_cpus"] >= 1 and "core_types" in info["cpu"]
    assert "nvdec" in info["video"] and info["gpu"]["present"] is False


@pytest.mark.skipif(os.environ.get("CUDA_VISIBLE_DEVICES", None) != "" and
                    __import__("torch").cuda.is_available(), reason="checks the no-GPU answers")
def test_no_device_answers():
    lib = ac.load()
    ctx = ctypes.c_void_p()
    assert lib.aegis_create(ctypes.byref(ctx), 0) == ac.AEGIS_ERR_NO_DEVICE
    assert lib.aegis_hw_info_json(0, None, 0, None) == ac.AEGIS_ERR_NO_DEVICE
    assert lib.aegis_device_manifest(0, None, 0, None) == ac.AEGIS_ERR_NO_DEVICE


def test_static_archive_exports_the_cpp_api():
    """libaegis.a carries the reference's C++ entry points (include/aegis/matmul.h:
    112-123, include/aegis/gemm.h registry) with their C++ signatures."""
    from cpp_build import ARCHIVE
    out = subprocess.run(["nm", "-C", "--defined-only", ARCHIVE], capture_output=True, text=True, check=True).stdout
    for sym in ["aegis::matmul(__half const*, __half const*, __half*, int, int, int, CUstream_st*)",
                "aegis::matmul(aegis::gemm::GemmParams const&, CUstream_st*)",
                "aegis::matmul_choice(int, int, int)", "aegis::matmul_last_error()",
                "aegis::gemm::registry()", "aegis::gemm::find(std::basic_string_view<char, std::char_traits<char> >)",
                "aegis_gemm_f16"]:
        assert re.search(r" T " + re.escape(sym) + r"$", out, re.M), sym


def test_cpp_program_links_against_the_static_archive(tmp_path):
    from cpp_build import build_matmul_test
    exe = tmp_path / "matmul_test"
    r = build_matmul_test(str(exe))
    assert r.returncode == 0, r.stderr[-3000:]
    assert exe.exists()
