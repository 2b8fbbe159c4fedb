#pragma once
// Per-stream device workspace for split-K partials and tickets.
// Contract (same as the reference's src/gemm/workspace.h:1-40):
//   - one buffer per (host thread, device, stream, use, size class); size
//     classes are powers of two from 64 KiB;
//   - a buffer is allocated and zeroed (on its stream) on the first request of
//     its class and then reused as is: never resized, never freed;
//   - a first request while `stream` is capturing returns
//     cudaErrorStreamCaptureUnsupported and touches nothing, so make the first
//     call per (stream, size class) outside capture;
//   - ticket counters are returned to zero by the kernel that used them, so a
//     counter buffer reads zero at every launch.
#include <cuda_runtime.h>

#include <cstddef>

namespace aegis::ws {

enum class Use : int { SplitKCounters = 0, SplitKPartials = 1 };

cudaError_t get(cudaStream_t stream, size_t bytes, void** out, Use use);
// Buffers allocated by this host thread (tests: nothing allocates after warm-up).
size_t allocations();

}  // namespace aegis::ws
