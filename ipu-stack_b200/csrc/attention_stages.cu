// Staged attention kernels for the Materialized strategy and for per-stage
// parity: the per-key-block softmax (device/attention_softmax_f16.cpp:63-139,
// device/attention_stages_f16.S:54-695) and the online merge
// (device/attention_stages_f16.S:698-855).  The fused tensor-core flash
// attention (flash_attention.cu) does the same arithmetic in registers; these
// keep the reference's memory formats for graphs that schedule the stages
// separately.  Both are small, memory-bound kernels.
#include <math.h>

#include "common.cuh"

namespace ipuc {
namespace {

// One thread per query row.  Row r's 16 scores of panel p sit at
// p*Q*16 + r*16, so a warp reads 32 consecutive rows = 1 KB contiguous per panel.
__global__ void __launch_bounds__(128) softmax_kernel(uint16_t *__restrict__ weights, const uint16_t *__restrict__ scores,
                                                      int64_t Q, int64_t key_rows, int64_t KB, float scale) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= Q) return;
  const int64_t panels = KB / 16;
  float maximum = -65504.0f;  // attention_softmax_f16.cpp:94
  for (int64_t p = 0; p < panels; ++p) {
    const uint16_t *src = scores + p * Q * 16 + row * 16;
    uint4 v[2] = {reinterpret_cast<const uint4 *>(src)[0], reinterpret_cast<const uint4 *>(src)[1]};
    const uint16_t *h = reinterpret_cast<const uint16_t *>(v);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (p * 16 + j < key_rows) maximum = fmaxf(maximum, h2f(h[j]));
  }
  const float smax = maximum * scale;
  float denominator = 0.0f;
  for (int64_t p = 0; p < panels; ++p) {
    const uint16_t *src = scores + p * Q * 16 + row * 16;
    uint4 v[2] = {reinterpret_cast<const uint4 *>(src)[0], reinterpret_cast<const uint4 *>(src)[1]};
    const uint16_t *h = reinterpret_cast<const uint16_t *>(v);
    uint4 o[2];
    uint16_t *w = reinterpret_cast<uint16_t *>(o);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const bool valid = p * 16 + j < key_rows;
      const float normalized = valid ? h2f(h[j]) * scale - smax : -65504.0f;
      // The reference rounds the argument to f16 and exponentiates in f16.
      const float arg = __half2float(__float2half_rn(normalized));
      w[j] = f2h(expf(arg));
      if (valid) denominator += h2f(w[j]);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(weights + p * Q * 16 + row * 16);
    dst[0] = o[0];
    dst[1] = o[1];
  }
  float *maxima = reinterpret_cast<float *>(weights + Q * KB);
  maxima[row] = smax;
  maxima[Q + row] = denominator;
}

// One warp per query row; lanes stride the value columns.
__global__ void __launch_bounds__(256) merge_kernel(float *__restrict__ acc, const uint16_t *__restrict__ block,
                                                    const float *__restrict__ state, int64_t Q, int64_t V,
                                                    int64_t Vp, int initial, int final_block) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= Q) return;
  float *a = acc + row * Vp;
  const float mb = state[row], lb = state[Q + row];
  float s_old = 0.0f, s_new = 1.0f, m_new = mb, l_new = lb;
  if (!initial) {
    const float m = a[V], l = a[V + 1];
    m_new = fmaxf(m, mb);
    s_old = expf(m - m_new);
    s_new = expf(mb - m_new);
    l_new = l * s_old + lb * s_new;
  }
  const float rcp = final_block ? 1.0f / l_new : 1.0f;
  for (int64_t c = lane; c < V; c += 32) {
    const float pv = h2f(block[(c / 16) * Q * 16 + row * 16 + (c % 16)]);
    float v = initial ? pv : a[c] * s_old + pv * s_new;
    if (final_block) v *= rcp;
    a[c] = v;
  }
  __syncwarp();
  if (lane == 0) {
    a[V] = m_new;
    a[V + 1] = l_new;
  }
}

}  // namespace
}  // namespace ipuc

using namespace ipuc;

extern "C" ipuc_status ipuc_attention_softmax_f16(void *weights, const void *scores, int64_t query_rows,
                                                  int64_t key_rows, int64_t key_block_columns,
                                                  int64_t head_dimension, ipuc_stream stream) {
  IPUC_CHECK_ARG(query_rows >= 0 && key_rows >= 0 && head_dimension > 0, "attention_softmax: bad extents");
  IPUC_CHECK_ARG(key_block_columns > 0 && key_block_columns % 16 == 0,
                 "attention_softmax: key block columns must be a positive multiple of 16");
  IPUC_CHECK_ARG(key_rows <= key_block_columns, "attention_softmax: key rows exceed the key block");
  if (query_rows == 0) return IPUC_OK;
  IPUC_CHECK_ALIGN(aligned(weights, 16) && aligned(scores, 16), "attention_softmax: pointers must be 16-byte aligned");
  const float scale = 1.0f / sqrtf((float)head_dimension);
  const unsigned grid = (unsigned)((query_rows + 127) / 128);
  softmax_kernel<<<grid, 128, 0, stream>>>((uint16_t *)weights, (const uint16_t *)scores, query_rows, key_rows,
                                           key_block_columns, scale);
  return check_launch("softmax_kernel");
}

extern "C" ipuc_status ipuc_attention_merge_f16(float *acc, const void *block, const float *state,
                                                int64_t query_rows, int64_t value_dimension,
                                                int64_t padded_value_dimension, int initial, int final_block,
                                                ipuc_stream stream) {
  IPUC_CHECK_ARG(query_rows >= 0 && value_dimension > 0, "attention_merge: bad extents");
  IPUC_CHECK_ARG(padded_value_dimension >= value_dimension + 2,
                 "attention_merge: padded value dimension must hold the two state words (attention_stages_f16.S:773)");
  if (query_rows == 0) return IPUC_OK;
  IPUC_CHECK_ARG(acc && block && state, "attention_merge: null pointer");
  const int64_t threads = query_rows * 32;
  const unsigned grid = (unsigned)((threads + 255) / 256);
  merge_kernel<<<grid, 256, 0, stream>>>(acc, (const uint16_t *)block, state, query_rows, value_dimension,
                                         padded_value_dimension, initial, final_block);
  return check_launch("merge_kernel");
}
