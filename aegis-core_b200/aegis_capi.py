"""ctypes binding of libaegis_capi.so (include/aegis.h) and libaegis_datagen.so.

The reference exposes its C ABI to Rust through bindgen (rust/aegis-sys); this
module is the equivalent binding for Python callers: tests, bench.py and the
tuner reach the kernels only through these C entry points. Operand pointers are
device addresses as Python ints (e.g. ``torch.Tensor.data_ptr()``).

Nothing here falls back to another implementation: if the shared library is
missing, ``load()`` raises.
"""
from __future__ import annotations

import ctypes
import json
import os
from ctypes import (POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_uint, c_void_p)

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "libaegis_capi.so")
DATAGEN_PATH = os.path.join(HERE, "build", "libaegis_datagen.so")

AEGIS_OK = 0
AEGIS_ERR_INVALID_ARGUMENT = -1
AEGIS_ERR_CUDA = -2
AEGIS_ERR_BUFFER_TOO_SMALL = -3
AEGIS_ERR_NO_DEVICE = -4
AEGIS_ERR_OUT_OF_MEMORY = -5
AEGIS_ERR_LAUNCH_FAILED = -6
ROW_MAJOR, COL_MAJOR = 0, 1
DTYPE_F16, DTYPE_BF16 = 0, 1
IPC_HANDLE_BYTES = 64
CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy

_lib = None
_datagen_lib = None

# name -> (restype, argtypes); every function declared in include/aegis.h.
_SIGNATURES = {
    "aegis_abi_version": (c_int, []),
    "aegis_status_string": (c_char_p, [c_int]),
    "aegis_last_error_string": (c_char_p, []),
    "aegis_create": (c_int, [POINTER(c_void_p), c_int]),
    "aegis_destroy": (c_int, [c_void_p]),
    "aegis_set_stream": (c_int, [c_void_p, c_void_p]),
    "aegis_synchronize": (c_int, [c_void_p]),
    "aegis_last_error": (c_char_p, [c_void_p]),
    "aegis_device_alloc": (c_int, [c_void_p, c_size_t, POINTER(c_void_p)]),
    "aegis_device_free": (c_int, [c_void_p, c_void_p]),
    "aegis_copy_to_device": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t]),
    "aegis_copy_to_host": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t]),
    "aegis_gemm_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int]),
    "aegis_gemm_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int]),
    "aegis_gemm_f16_ex": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p, c_int64,
                                  c_void_p, c_int64, c_float, c_void_p, c_int64]),
    "aegis_gemm_bf16_ex": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p, c_int64,
                                   c_void_p, c_int64, c_float, c_void_p, c_int64]),
    "aegis_gemm_f16_strided_batched": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p,
                                               c_int64, c_int64, c_void_p, c_int64, c_int64, c_float, c_void_p,
                                               c_int64, c_int64, c_int]),
    "aegis_gemm_bf16_strided_batched": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p,
                                                c_int64, c_int64, c_void_p, c_int64, c_int64, c_float, c_void_p,
                                                c_int64, c_int64, c_int]),
    "aegis_gemm_choice": (c_int, [c_void_p, c_int, c_int, c_int, c_char_p, c_size_t, POINTER(c_size_t)]),
    "aegis_device_manifest": (c_int, [c_int, c_char_p, c_size_t, POINTER(c_size_t)]),
    "aegis_hw_info_json": (c_int, [c_int, c_char_p, c_size_t, POINTER(c_size_t)]),
    "aegis_hw_gpu": (c_int, [c_int, c_void_p]),
    "aegis_hw_cpu": (c_int, [c_void_p]),
    "aegis_gemm_bf16_nsharded": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int64, c_void_p, c_int64,
                                         POINTER(c_void_p), c_int64, c_int, c_int]),
    "aegis_gemm_f16_nsharded": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int64, c_void_p, c_int64,
                                        POINTER(c_void_p), c_int64, c_int, c_int]),
    "aegis_ipc_get_handle": (c_int, [c_void_p, c_void_p, c_void_p]),
    "aegis_ipc_open_handle": (c_int, [c_void_p, c_void_p, POINTER(c_void_p)]),
    "aegis_ipc_close_handle": (c_int, [c_void_p, c_void_p]),
    "aegis_gemm_impl": (c_int, [c_void_p, c_char_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p,
                                c_int64, c_int64, c_void_p, c_int64, c_int64, c_float, c_void_p, c_int64, c_int64,
                                c_int]),
    "aegis_registry_json": (c_int, [c_void_p, c_char_p, c_size_t, POINTER(c_size_t)]),
    "aegis_gemm_plan_json": (c_int, [c_void_p, c_char_p, c_int, c_int, c_int, c_int, c_char_p, c_size_t,
                                     POINTER(c_size_t)]),
    "aegis_plan_simulated_json": (c_int, [c_int, c_int, c_char_p, c_int, c_int, c_int, c_int, c_char_p, c_size_t,
                                          POINTER(c_size_t)]),
    "aegis_gemv_noalloc": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p, c_int64,
                                   c_void_p, c_int64, c_float, c_void_p, c_int64]),
    "aegis_watchdog_selftest": (c_int, [c_void_p, c_int64]),
}


class AegisError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str):
        super().__init__(f"{where}: status {status} ({status_string(status)}): {detail}")
        self.status = status
        self.detail = detail


def load(path: str | None = None) -> ctypes.CDLL:
    """Load libaegis_capi.so (once) and declare every C signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise FileNotFoundError(f"{p} is not built: run `make -C aegis-core_b200` (or __graft_entry__.build())")
    lib = ctypes.CDLL(p)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def status_string(s: int) -> str:
    return load().aegis_status_string(s).decode()


def last_error_string() -> str:
    return load().aegis_last_error_string().decode()


def check(status: int, where: str) -> None:
    if status != AEGIS_OK:
        raise AegisError(status, where, last_error_string())


def _query_string(fn, *args) -> str:
    needed = c_size_t(0)
    check(fn(*args, None, 0, ctypes.byref(needed)), fn.__name__)
    buf = ctypes.create_string_buffer(needed.value)
    check(fn(*args, buf, needed.value, ctypes.byref(needed)), fn.__name__)
    return buf.value.decode()


def plan_simulated(M: int, N: int, K: int, impl: str | None = None, dtype: int = DTYPE_F16, arch: int = 100,
                   sm_count: int = 148) -> dict:
    """The dispatcher's choice and the launch plan on a simulated device (no
    GPU needed): {"impl", "splits", "k_chunk", "tiles", "grid", "dispatch",
    "kind"} (aegis_plan_simulated_json)."""
    lib = load()
    return json.loads(_query_string(lib.aegis_plan_simulated_json, arch, sm_count,
                                    impl.encode() if impl else None, dtype, M, N, K))


class Context:
    """One device + one stream (aegis_context). The stream may be a caller's
    cudaStream_t (e.g. ``torch.cuda.current_stream().cuda_stream``)."""

    def __init__(self, device: int = 0):
        self.lib = load()
        self.ptr = c_void_p()
        check(self.lib.aegis_create(ctypes.byref(self.ptr), device), "aegis_create")
        self.device = device

    def close(self) -> None:
        if self.ptr:
            check(self.lib.aegis_destroy(self.ptr), "aegis_destroy")
            self.ptr = c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_stream(self, stream: int | None) -> None:
        """Queue this context's work on `stream` (a cudaStream_t as int).
        0 is the legacy default stream (torch's default stream reports
        handle 0): it is passed as cudaStreamLegacy, because a NULL stream in
        the C ABI means the context's own stream. None: the context's own."""
        handle = CUDA_STREAM_LEGACY if stream == 0 else (stream or 0)
        check(self.lib.aegis_set_stream(self.ptr, c_void_p(handle)), "aegis_set_stream")

    def synchronize(self) -> None:
        check(self.lib.aegis_synchronize(self.ptr), "aegis_synchronize")

    def gemm(self, A: int, B: int, C: int, M: int, N: int, K: int, dtype: int = DTYPE_F16) -> None:
        fn = self.lib.aegis_gemm_bf16 if dtype == DTYPE_BF16 else self.lib.aegis_gemm_f16
        check(fn(self.ptr, c_void_p(A), c_void_p(B), c_void_p(C), M, N, K), fn.__name__)

    def gemm_ex(self, layout_a, layout_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, dtype=DTYPE_F16) -> None:
        fn = self.lib.aegis_gemm_bf16_ex if dtype == DTYPE_BF16 else self.lib.aegis_gemm_f16_ex
        check(fn(self.ptr, layout_a, layout_b, M, N, K, alpha, c_void_p(A), lda, c_void_p(B), ldb, beta,
                 c_void_p(C), ldc), fn.__name__)

    def gemm_strided_batched(self, layout_a, layout_b, M, N, K, alpha, A, lda, sa, B, ldb, sb, beta, C, ldc, sc,
                             batch, dtype=DTYPE_F16) -> None:
        fn = (self.lib.aegis_gemm_bf16_strided_batched if dtype == DTYPE_BF16
              else self.lib.aegis_gemm_f16_strided_batched)
        check(fn(self.ptr, layout_a, layout_b, M, N, K, alpha, c_void_p(A), lda, sa, c_void_p(B), ldb, sb, beta,
                 c_void_p(C), ldc, sc, batch), fn.__name__)

    def gemm_impl(self, impl, dtype, layout_a, layout_b, M, N, K, alpha, A, lda, sa, B, ldb, sb, beta, C, ldc, sc,
                  batch) -> None:
        check(self.lib.aegis_gemm_impl(self.ptr, impl.encode(), dtype, layout_a, layout_b, M, N, K, alpha,
                                       c_void_p(A), lda, sa, c_void_p(B), ldb, sb, beta, c_void_p(C), ldc, sc,
                                       batch), f"aegis_gemm_impl({impl})")

    def choice(self, M: int, N: int, K: int) -> str:
        return _query_string(self.lib.aegis_gemm_choice, self.ptr, M, N, K)

    def registry(self) -> list:
        return json.loads(_query_string(self.lib.aegis_registry_json, self.ptr))

    def plan(self, M: int, N: int, K: int, impl: str | None = None, dtype: int = DTYPE_F16) -> dict:
        return json.loads(_query_string(self.lib.aegis_gemm_plan_json, self.ptr,
                                        impl.encode() if impl else None, dtype, M, N, K))

    def nsharded(self, M, N, K, A, lda, B_shard, ldb, c_ranks, ldc, nranks, rank, dtype=DTYPE_BF16) -> None:
        arr = (c_void_p * nranks)(*[c_void_p(p) for p in c_ranks])
        fn = self.lib.aegis_gemm_bf16_nsharded if dtype == DTYPE_BF16 else self.lib.aegis_gemm_f16_nsharded
        check(fn(self.ptr, M, N, K, c_void_p(A), lda, c_void_p(B_shard), ldb, arr, ldc, nranks, rank), fn.__name__)

    def ipc_get_handle(self, dptr: int) -> bytes:
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        check(self.lib.aegis_ipc_get_handle(self.ptr, c_void_p(dptr), buf), "aegis_ipc_get_handle")
        return buf.raw

    def ipc_open_handle(self, handle: bytes) -> int:
        out = c_void_p()
        buf = ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES)
        check(self.lib.aegis_ipc_open_handle(self.ptr, buf, ctypes.byref(out)), "aegis_ipc_open_handle")
        return out.value

    def ipc_close_handle(self, dptr: int) -> None:
        check(self.lib.aegis_ipc_close_handle(self.ptr, c_void_p(dptr)), "aegis_ipc_close_handle")

    def gemv_noalloc(self, dtype, layout_a, layout_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc) -> None:
        """aegis_gemv_noalloc: the decode GEMV with its scratch in the library's
        fixed device array (no allocation on any call)."""
        check(self.lib.aegis_gemv_noalloc(self.ptr, dtype, layout_a, layout_b, M, N, K, alpha, c_void_p(A), lda,
                                          c_void_p(B), ldb, beta, c_void_p(C), ldc), "aegis_gemv_noalloc")

    def watchdog_selftest(self, timeout_ns: int) -> int:
        return self.lib.aegis_watchdog_selftest(self.ptr, timeout_ns)


def device_manifest(device: int = 0) -> dict:
    return json.loads(_query_string(load().aegis_device_manifest, device))


def hw_info(device: int = -1) -> dict:
    return json.loads(_query_string(load().aegis_hw_info_json, device))


# ----------------------------------------------------------------- host data
def _datagen() -> ctypes.CDLL:
    global _datagen_lib
    if _datagen_lib is None:
        if not os.path.exists(DATAGEN_PATH):
            raise FileNotFoundError(f"{DATAGEN_PATH} is not built: run `make -C aegis-core_b200`")
        d = ctypes.CDLL(DATAGEN_PATH)
        d.datagen_engine_new.restype = c_void_p
        d.datagen_engine_new.argtypes = [c_uint]
        d.datagen_engine_free.restype = None
        d.datagen_engine_free.argtypes = [c_void_p]
        d.datagen_fill.restype = c_int
        d.datagen_fill.argtypes = [c_void_p, c_int, c_float, c_float, c_int, c_void_p, c_size_t]
        d.datagen_f32_to_16.restype = None
        d.datagen_f32_to_16.argtypes = [c_void_p, c_void_p, c_size_t, c_int]
        _datagen_lib = d
    return _datagen_lib


class Generator:
    """std::mt19937(seed) shared by successive draws, as the reference's
    harness draws A then B from one engine (src/bench/harness.cu:48-54)."""

    def __init__(self, seed: int):
        self.d = _datagen()
        self.eng = self.d.datagen_engine_new(seed)

    def __del__(self):
        if getattr(self, "eng", None):
            self.d.datagen_engine_free(self.eng)
            self.eng = None

    def _fill(self, kind, p0, p1, n, dtype):
        if dtype == "f32":
            out = np.empty(n, dtype=np.float32)
            code = 2
        else:
            out = np.empty(n, dtype=np.uint16)
            code = DTYPE_BF16 if dtype == "bf16" else DTYPE_F16
        if self.d.datagen_fill(self.eng, kind, p0, p1, code, out.ctypes.data, n) != 0:
            raise RuntimeError("datagen_fill failed")
        return out

    def uniform(self, n: int, dtype: str = "f16", lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
        """std::uniform_real_distribution<float>(lo, hi), rounded to 16 bits (RNE)."""
        return self._fill(0, lo, hi, n, dtype)

    def normal(self, n: int, dtype: str = "f16", mean: float = 0.0, std: float = 1.0) -> np.ndarray:
        """std::normal_distribution<float>(mean, std), rounded to 16 bits (RNE)."""
        return self._fill(1, mean, std, n, dtype)


def f32_to_16(x: np.ndarray, bf16: bool) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    _datagen().datagen_f32_to_16(x.ctypes.data, out.ctypes.data, x.size, 1 if bf16 else 0)
    return out


def to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    """16-bit patterns (uint16) -> float32, exactly."""
    bits = np.asarray(bits, dtype=np.uint16)
    if dtype == "bf16":
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits.view(np.float16).astype(np.float32)
