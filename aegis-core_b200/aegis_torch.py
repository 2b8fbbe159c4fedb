"""torch.ops.aegis.matmul: the library's GEMM as a PyTorch operator.

    import aegis_torch  # registers the op
    C = torch.ops.aegis.matmul(A, B)      # A [M, K], B [K, N], both f16 or both bf16, on one CUDA device

The op calls the C ABI (aegis_gemm_f16_ex / aegis_gemm_bf16_ex through
aegis_capi) on torch's current stream, so it orders with the surrounding torch
work. The dispatcher picks the kernel: the tuned winner for the shape, else
the built-in rule. Operands may be row-major (contiguous) or column-major
(transposed views). Any other stride pattern is copied to a contiguous tensor
first. C is a new row-major tensor of the inputs' dtype (FP32 accumulation).
A fake implementation gives shapes under meta and fake tensors.

It is the Python-side counterpart of the reference's C++ aegis::matmul and
only plumbing: the GEMM is the same C-ABI call every other caller makes.
"""
from __future__ import annotations

import threading

import torch
from torch.library import custom_op

import aegis_capi as ac

_lock = threading.Lock()
_contexts: dict[int, ac.Context] = {}


def _context(device: int) -> ac.Context:
    with _lock:
        ctx = _contexts.get(device)
        if ctx is None:
            ctx = ac.Context(device)
            _contexts[device] = ctx
        return ctx


def _operand(t: torch.Tensor):
    """(tensor, layout, ld) for a 2-D operand: row-major if rows are
    contiguous, column-major if columns are, else a contiguous copy."""
    r, c = t.shape
    if t.stride(1) == 1 and (r <= 1 or t.stride(0) >= c):
        return t, ac.ROW_MAJOR, max(t.stride(0), c, 1)
    if t.stride(0) == 1 and (c <= 1 or t.stride(1) >= r):
        return t, ac.COL_MAJOR, max(t.stride(1), r, 1)
    t = t.contiguous()
    return t, ac.ROW_MAJOR, max(c, 1)


@custom_op("aegis::matmul", mutates_args=())
def matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("aegis::matmul takes 2-D operands")
    if a.shape[1] != b.shape[0]:
        raise ValueError(f"aegis::matmul: inner sizes differ ({tuple(a.shape)} x {tuple(b.shape)})")
    if a.dtype != b.dtype or a.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("aegis::matmul: both operands float16 or both bfloat16")
    if not (a.is_cuda and b.is_cuda) or a.device != b.device:
        raise ValueError("aegis::matmul: both operands on one CUDA device")
    M, K = a.shape
    N = b.shape[1]
    out = torch.empty((M, N), dtype=a.dtype, device=a.device)
    if M == 0 or N == 0:
        return out
    if K == 0:
        return out.zero_()
    a_, la, lda = _operand(a)
    b_, lb, ldb = _operand(b)
    dtype = ac.DTYPE_BF16 if a.dtype == torch.bfloat16 else ac.DTYPE_F16
    ctx = _context(a.device.index if a.device.index is not None else torch.cuda.current_device())
    with torch.cuda.device(a.device):
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        ctx.gemm_ex(la, lb, M, N, K, 1.0, a_.data_ptr(), lda, b_.data_ptr(), ldb, 0.0, out.data_ptr(), N, dtype)
    return out


@matmul.register_fake
def _(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    torch._check(a.dim() == 2 and b.dim() == 2, lambda: "aegis::matmul takes 2-D operands")
    torch._check(a.shape[1] == b.shape[0], lambda: "aegis::matmul: inner sizes differ")
    return a.new_empty((a.shape[0], b.shape[1]))
