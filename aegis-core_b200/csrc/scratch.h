#pragma once
// Library-owned device scratch for split-K: FP32 partial tiles and the
// per-tile ticket counters of the ordered fix-up.
//
// The rules callers rely on (the promises the reference library makes for
// its per-stream workspace, src/gemm/workspace.h:1-24 and
// include/aegis/matmul.h:26-31 there):
//   - Scratch is keyed by (host thread, device, stream, kind, size class).
//     Size classes are powers of two, 64 KiB and up.
//   - The first request for a key allocates the class with cudaMalloc and
//     zero-fills it on `stream`; later requests return the same buffer, so a
//     call sequence allocates nothing after its first call per key. Buffers
//     live until the process exits.
//   - A first request made while `stream` is being captured into a CUDA graph
//     allocates nothing and returns cudaErrorStreamCaptureUnsupported: make
//     the first call per (stream, size class) before capturing.
//   - Kernels that take tickets leave every counter at zero when they finish,
//     so a counter buffer reads zero at each launch.
#include <cuda_runtime.h>

#include <cstddef>

namespace aegis::scratch {

enum class Kind : unsigned char { Tickets = 0, Partials = 1 };

cudaError_t acquire(cudaStream_t stream, size_t bytes, Kind kind, void** out);

// Buffers this host thread holds (tests check that warm calls add none).
size_t held();

}  // namespace aegis::scratch
