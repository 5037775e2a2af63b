// Shared host/device helpers for libipuc.so: status plumbing, argument checks,
// f16 helpers and the device error word used by bounded waits.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/ipuc.h"

namespace ipuc {

// Thread-local last-error text (ipuc_last_error_string).
void set_error(const std::string &msg);
ipuc_status fail(ipuc_status st, const std::string &msg);
ipuc_status cuda_fail(cudaError_t err, const char *what);

// Launch epilogue: turn a launch error into IPUC_ERR_CUDA.
inline ipuc_status check_launch(const char *what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(err, what);
  return IPUC_OK;
}

inline bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Number of SMs on the current device (cached per device).
int sm_count();

// Device error word.  Kernels that spin on an mbarrier give up after a bounded
// time, record a code in this word and return; ipuc_device_status() reads and
// clears it.  Codes: (kernel id << 16) | site.  Returns the word's device
// address on the current device (nullptr if it cannot be resolved).
uint32_t *device_error_word();

enum : uint32_t {
  ERR_SITE_PRODUCER = 1,
  ERR_SITE_MMA = 2,
  ERR_SITE_EPILOGUE = 3,
  ERR_KERNEL_GEMM_F16 = 1u << 16,
  ERR_KERNEL_GEMM_F32 = 2u << 16,
  ERR_KERNEL_ATTENTION = 3u << 16,
  ERR_KERNEL_SELFTEST = 4u << 16,
  ERR_KERNEL_LAYOUT = 5u << 16,
};

__device__ __forceinline__ void record_device_error(uint32_t *word, uint32_t code) {
  if (word) atomicCAS(word, 0u, code);
}

// ---- f16 helpers -----------------------------------------------------------
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  return (uint32_t)f2h(lo) | ((uint32_t)f2h(hi) << 16);
}

// tanh-approximation GELU, 0.5x(1+tanh(u)) with u = 0.7978846(x + 0.044715x^3)
// (crates/ipu-tests/src/main.rs:1985-1987), evaluated through the identity
// 0.5(1+tanh(u)) = 1/(1+exp(-2u)) with two MUFU instructions: ex2.approx
// (exp(y) = 2^(y*log2(e))) and rcp.approx, each within ~2^-22 relative, far
// below the f16 rounding of the result.  The reciprocal of +inf is 0, so large
// negative x gives -0 as the formula's limit.
__device__ __forceinline__ float gelu_f32(float x) {
  // -2 log2(e) u = x (k0 + k1 x^2), k0 = -2 log2(e) 0.7978846, k1 = k0 0.044715
  constexpr float k0 = -2.0f * 1.4426950408889634f * 0.7978846f, k1 = k0 * 0.044715f;
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * fmaf(k1, x * x, k0)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return x * r;
}

// GELU on a pair of f16 values in f16x2 arithmetic, the way the reference's
// tile kernel evaluates it (device/gelu_f16.S:14-25: f16v2mul/add/tanh):
// y = x/2 * (1 + tanh(0.7978846 * (x + 0.044715 x^3))), tanh from the
// hardware tanh.approx.f16x2.  Used by the GEMM epilogue, where the f32
// formula's extra MUFU work would otherwise dominate.  For |x| large enough
// that x^3 overflows, tanh saturates to +-1 and the result is x or 0.
__device__ __forceinline__ uint32_t gelu_h2(uint32_t xh) {
  const __half2 x = *reinterpret_cast<const __half2 *>(&xh);
  const __half2 x2 = __hmul2(x, x);
  const __half2 inner = __hfma2(__hmul2(x2, x), __float2half2_rn(0.044715f), x);
  const __half2 u = __hmul2(inner, __float2half2_rn(0.7978846f));
  uint32_t ub = *reinterpret_cast<const uint32_t *>(&u), tb;
  asm("tanh.approx.f16x2 %0, %1;" : "=r"(tb) : "r"(ub));
  const __half2 t = *reinterpret_cast<const __half2 *>(&tb);
  const __half2 hx = __hmul2(x, __float2half2_rn(0.5f));
  const __half2 y = __hfma2(hx, t, hx);
  return *reinterpret_cast<const uint32_t *>(&y);
}

}  // namespace ipuc

#define IPUC_CHECK_ARG(cond, msg)                                   \
  do {                                                              \
    if (!(cond)) return ::ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, msg); \
  } while (0)
#define IPUC_CHECK_ALIGN(cond, msg)                           \
  do {                                                        \
    if (!(cond)) return ::ipuc::fail(IPUC_ERR_ALIGNMENT, msg); \
  } while (0)
#define IPUC_CUDA(call)                                      \
  do {                                                       \
    cudaError_t _e = (call);                                 \
    if (_e != cudaSuccess) return ::ipuc::cuda_fail(_e, #call); \
  } while (0)
