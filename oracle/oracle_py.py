"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of the checkers.

Loads oracle/liboracle.so (oracle.c, the C restatement of the reference's
FP64 GEMM oracle, tolerance and comparer) and, when it was built here,
oracle/_ref/libaegis_ref.so (the reference's own src/bench/reference.cu).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
this module; the product path never does.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_double, c_float, c_int, c_longlong, c_size_t, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libaegis_ref.so")


class Desc(ctypes.Structure):
    """oracle_gemm in oracle.c (and ref_gemm in ref_shim.cu)."""
    _fields_ = [("M", c_int), ("N", c_int), ("K", c_int), ("layout_a", c_int), ("layout_b", c_int),
                ("lda", c_longlong), ("ldb", c_longlong), ("ldc", c_longlong), ("alpha", c_float),
                ("beta", c_float), ("batch", c_int), ("stride_a", c_longlong), ("stride_b", c_longlong),
                ("stride_c", c_longlong), ("dtype", c_int)]


class Result(ctypes.Structure):
    _fields_ = [("pass_", c_int), ("checked", c_longlong), ("nan_mismatch", c_longlong),
                ("inf_mismatch", c_longlong), ("out_of_tol", c_longlong), ("max_err", c_double),
                ("max_ratio", c_double), ("first_index", c_longlong), ("first_got", c_double),
                ("first_want", c_double)]


_oracle = None
_ref = None


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            raise FileNotFoundError(f"{ORACLE_SO} not built: run `make -C oracle`")
        lib = ctypes.CDLL(ORACLE_SO)
        lib.oracle_gemm_ref.restype = c_int
        lib.oracle_gemm_ref.argtypes = [POINTER(Desc), c_void_p, c_void_p, c_void_p, c_void_p, c_int]
        lib.oracle_gemm_ref_rows.restype = c_int
        lib.oracle_gemm_ref_rows.argtypes = [POINTER(Desc), c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                             c_int]
        lib.oracle_tolerance.restype = c_double
        lib.oracle_tolerance.argtypes = [POINTER(Desc), c_void_p, c_size_t, c_void_p, c_size_t, c_void_p, c_size_t,
                                         c_double, c_int]
        lib.oracle_compare.restype = c_int
        lib.oracle_compare.argtypes = [POINTER(Desc), c_void_p, c_size_t, c_void_p, c_void_p, c_double,
                                       POINTER(Result)]
        lib.oracle_decode.restype = c_double
        lib.oracle_decode.argtypes = [ctypes.c_uint16, c_int]
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        lib = ctypes.CDLL(REF_SO)
        lib.ref_cpu_reference.restype = c_int
        lib.ref_cpu_reference.argtypes = [POINTER(Desc), c_void_p, c_size_t, c_void_p, c_size_t, c_void_p, c_size_t,
                                          c_void_p]
        lib.ref_tolerance.restype = c_double
        lib.ref_tolerance.argtypes = [POINTER(Desc), c_void_p, c_size_t, c_void_p, c_size_t, c_void_p, c_size_t,
                                      c_double]
        _ref = lib
    return _ref


def make_desc(M, N, K, layout_a=0, layout_b=0, lda=None, ldb=None, ldc=None, alpha=1.0, beta=0.0, batch=1,
              stride_a=0, stride_b=0, stride_c=0, dtype="f16") -> Desc:
    if lda is None:
        lda = K if layout_a == 0 else M
    if ldb is None:
        ldb = N if layout_b == 0 else K
    if ldc is None:
        ldc = N
    return Desc(M, N, K, layout_a, layout_b, lda, ldb, ldc, alpha, beta, batch, stride_a, stride_b, stride_c,
                1 if dtype == "bf16" else 0)


def spans(d: Desc) -> tuple[int, int, int]:
    """Elements each batched operand spans (reference src/bench/reference.cu:41-60)."""
    if d.M == 0 or d.N == 0 or d.K == 0 or d.batch == 0:
        return 0, 0, 0
    one_a = (d.M - 1) * d.lda + d.K if d.layout_a == 0 else (d.K - 1) * d.lda + d.M
    one_b = (d.K - 1) * d.ldb + d.N if d.layout_b == 0 else (d.N - 1) * d.ldb + d.K
    one_c = (d.M - 1) * d.ldc + d.N
    return ((d.batch - 1) * d.stride_a + one_a, (d.batch - 1) * d.stride_b + one_b,
            (d.batch - 1) * d.stride_c + one_c)


def _u16(x):
    return None if x is None else np.ascontiguousarray(x, dtype=np.uint16)


def gemm_ref(d: Desc, A, B, C0=None, nthreads: int | None = None) -> np.ndarray:
    """FP64 reference, shape (batch, M, N)."""
    A, B, C0 = _u16(A), _u16(B), _u16(C0)
    out = np.zeros((d.batch, d.M, d.N), dtype=np.float64)
    nt = nthreads or min(16, os.cpu_count() or 1)
    rc = oracle_lib().oracle_gemm_ref(ctypes.byref(d), A.ctypes.data, B.ctypes.data,
                                      C0.ctypes.data if C0 is not None else None, out.ctypes.data, nt)
    if rc != 0:
        raise RuntimeError("oracle_gemm_ref failed")
    return out


def gemm_ref_rows(d: Desc, A, B, r0: int, r1: int, C0=None, nthreads: int | None = None) -> np.ndarray:
    """FP64 reference of rows [r0, r1) of every batch, shape (batch, r1-r0, N)."""
    A, B, C0 = _u16(A), _u16(B), _u16(C0)
    out = np.zeros((d.batch, r1 - r0, d.N), dtype=np.float64)
    nt = nthreads or min(16, os.cpu_count() or 1)
    rc = oracle_lib().oracle_gemm_ref_rows(ctypes.byref(d), A.ctypes.data, B.ctypes.data,
                                           C0.ctypes.data if C0 is not None else None, out.ctypes.data, r0, r1, nt)
    if rc != 0:
        raise RuntimeError("oracle_gemm_ref_rows failed")
    return out


def tolerance(d: Desc, A, B, C0=None, c: float = 2.0, kind: str = "reference") -> float:
    """kind "reference": c*sqrt(K)*eps*max|A|*max|B|*|alpha| + eps*|beta|*max|C0|
    (reference.cu:186-194); kind "north_star": eps*K*max|A|*max|B|*|alpha| (+ beta term), eps = 2^-10
    for f16 outputs (the bound as stated) and 2^-7 for bf16 outputs (the output type's eps)."""
    A, B, C0 = _u16(A), _u16(B), _u16(C0)
    return oracle_lib().oracle_tolerance(ctypes.byref(d), A.ctypes.data, A.size, B.ctypes.data, B.size,
                                         C0.ctypes.data if C0 is not None else None,
                                         C0.size if C0 is not None else 0, c, 1 if kind == "north_star" else 0)


def compare(d: Desc, out, ref, C0=None, allowed: float = 0.0) -> dict:
    out, C0 = _u16(out), _u16(C0)
    ref = np.ascontiguousarray(ref, dtype=np.float64)
    r = Result()
    oracle_lib().oracle_compare(ctypes.byref(d), out.ctypes.data, out.size, ref.ctypes.data,
                                C0.ctypes.data if C0 is not None else None, allowed, ctypes.byref(r))
    return {"pass": bool(r.pass_), "checked": r.checked, "nan_mismatch": r.nan_mismatch,
            "inf_mismatch": r.inf_mismatch, "out_of_tol": r.out_of_tol, "max_err": r.max_err,
            "max_ratio": r.max_ratio, "first_index": r.first_index, "first_got": r.first_got,
            "first_want": r.first_want}


def ref_cpu_reference(d: Desc, A, B, C0=None) -> np.ndarray:
    """The reference's own aegis::bench::cpu_reference (f16 only)."""
    A, B, C0 = _u16(A), _u16(B), _u16(C0)
    out = np.zeros((d.batch, d.M, d.N), dtype=np.float64)
    rc = ref_lib().ref_cpu_reference(ctypes.byref(d), A.ctypes.data, A.size, B.ctypes.data, B.size,
                                     C0.ctypes.data if C0 is not None else None,
                                     C0.size if C0 is not None else 0, out.ctypes.data)
    if rc != 0:
        raise RuntimeError("ref_cpu_reference failed")
    return out


def ref_tolerance(d: Desc, A, B, C0=None, c: float = 2.0) -> float:
    A, B, C0 = _u16(A), _u16(B), _u16(C0)
    return ref_lib().ref_tolerance(ctypes.byref(d), A.ctypes.data, A.size, B.ctypes.data, B.size,
                                   C0.ctypes.data if C0 is not None else None, C0.size if C0 is not None else 0, c)
