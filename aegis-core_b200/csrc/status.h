#pragma once
// Per-device status word written by kernel watchdogs. Every wait inside this
// library's kernels is bounded (mbarrier waits, see ptx.cuh); a wait that
// runs out sets a bit here (kStatus* in common.cuh), the kernel skips the rest
// of its work, releases what it holds (TMEM, in-flight copies) and returns.
// aegis_synchronize() reads and clears the word and turns a set bit into
// AEGIS_ERR_CUDA. Allocated (and zeroed) on the first launch per device,
// which therefore must come before any stream capture.
#include <cuda_runtime.h>

namespace aegis::status {

// Device pointer of the current device's status word (4 unsigned; word 0 is
// the OR of the bits, word 1 the first failing block index + 1).
cudaError_t word(unsigned** out);
// Reads and clears the current device's status (synchronous). *bits = 0 if
// the word was never allocated.
cudaError_t take(unsigned* bits, unsigned* block);

}  // namespace aegis::status
