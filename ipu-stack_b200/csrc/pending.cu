// Entry points whose kernels are not built yet: they fail loudly with
// IPUC_ERR_UNSUPPORTED (no fallback path).
#include "common.cuh"

using namespace ipuc;

extern "C" uint64_t ipuc_gemm_f32_workspace_bytes(int64_t m, int64_t n, int64_t k) { return 0; }
extern "C" ipuc_status ipuc_gemm_f32(float *, const float *, const float *, int64_t, int64_t, int64_t, int64_t,
                                     int64_t, int64_t, uint32_t, void *, uint64_t, ipuc_stream) {
  return fail(IPUC_ERR_UNSUPPORTED, "gemm_f32: not built");
}
