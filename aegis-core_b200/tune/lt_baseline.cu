// C entry points over LtSweep (lt_best.h) for bench.py's "cublaslt_best"
// baseline: build the heuristic sweep for a row-major problem, describe a
// candidate, run a candidate on the caller's stream. bench.py times every
// candidate with the same graph-captured, cold-L2 protocol it uses for its own
// kernels and keeps the fastest that passes the check. Built into
// build/libaegis_ltbase.so; baseline code, not part of libaegis_capi.
#include <cstring>

#include "lt_best.h"

#define LTB_API extern "C" __attribute__((visibility("default")))

using aegis::tune::LtSweep;

// 0 on success; *n = candidates kept (FP32 reductions only), *dropped = those
// the heuristic offered with reduced-precision split-K partials.
LTB_API int ltb_create(int bf16, int M, int N, int K, size_t max_workspace, void** out, int* n, int* dropped) {
  *out = nullptr;
  auto* s = new LtSweep(bf16 != 0, M, N, K, max_workspace);
  if (!s->ok()) {
    delete s;
    return -1;
  }
  *out = s;
  *n = s->size();
  *dropped = s->dropped();
  return 0;
}

LTB_API void ltb_destroy(void* h) { delete static_cast<LtSweep*>(h); }

LTB_API int ltb_describe(void* h, int i, char* buf, size_t len) {
  const auto* s = static_cast<LtSweep*>(h);
  if (i < 0 || i >= s->size() || len == 0) return -1;
  const std::string d = s->describe(i);
  std::strncpy(buf, d.c_str(), len - 1);
  buf[len - 1] = 0;
  return 0;
}

LTB_API size_t ltb_workspace(void* h, int i) {
  const auto* s = static_cast<LtSweep*>(h);
  return i >= 0 && i < s->size() ? s->algo(i).workspace : 0;
}

LTB_API int ltb_run(void* h, int i, const void* A, const void* B, void* C, void* ws, size_t ws_bytes,
                    cudaStream_t stream) {
  const auto* s = static_cast<LtSweep*>(h);
  if (i < 0 || i >= s->size()) return -1;
  return int(s->run(i, A, B, C, ws, ws_bytes, stream));
}
