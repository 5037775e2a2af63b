/* A C program that uses libipuc.so through include/ipuc.h alone, as a host
 * binding of the reference (a Rust/cgo/JNI FFI) would: no Python, no torch.
 * Runs one f16 GEMM, one flash-attention call and one spec-driven launch on
 * device buffers it allocates itself, and checks the GEMM against a host loop.
 * Exit status 0 on success. */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ipuc.h"

static uint16_t f2h(float f) { /* round to nearest even; normal range only */
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  int32_t e = (int32_t)((x >> 23) & 0xff) - 127 + 15;
  uint32_t m = x & 0x7fffffu;
  if (e <= 0) return (uint16_t)sign;
  uint32_t h = sign | ((uint32_t)e << 10) | (m >> 13);
  uint32_t rest = m & 0x1fffu;
  if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)h;
}
static float h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff, x;
  if (e == 0) { float v = ldexpf((float)m, -24); return sign ? -v : v; }
  x = sign | ((e - 15 + 127) << 23) | (m << 13);
  float f;
  memcpy(&f, &x, 4);
  return f;
}

#define CHECK(call)                                                                               \
  do {                                                                                            \
    ipuc_status st_ = (call);                                                                     \
    if (st_ != IPUC_OK) {                                                                         \
      fprintf(stderr, "%s: %s (%s)\n", #call, ipuc_status_string(st_), ipuc_last_error_string()); \
      return 1;                                                                                   \
    }                                                                                             \
  } while (0)

int main(void) {
  const int64_t m = 256, n = 192, k = 128;
  printf("%s\n", ipuc_version());
  uint16_t *ha = malloc(m * k * 2), *hb = malloc(k * n * 2), *hc = malloc(m * n * 2);
  for (int64_t i = 0; i < m * k; ++i) ha[i] = f2h((float)((i * 37) % 17 - 8) * 0.0625f);
  for (int64_t i = 0; i < k * n; ++i) hb[i] = f2h((float)((i * 11) % 13 - 6) * 0.125f);
  void *da, *db, *dc;
  if (cudaMalloc(&da, m * k * 2) || cudaMalloc(&db, k * n * 2) || cudaMalloc(&dc, m * n * 4)) return 2;
  cudaMemcpy(da, ha, m * k * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(db, hb, k * n * 2, cudaMemcpyHostToDevice);
  CHECK(ipuc_gemm_f16(dc, da, db, m, n, k, k, n, n, 0, NULL));
  CHECK(ipuc_device_status(NULL));
  cudaMemcpy(hc, dc, m * n * 2, cudaMemcpyDeviceToHost);
  double worst = 0.0;
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c) {
      double acc = 0.0;
      for (int64_t i = 0; i < k; ++i) acc += (double)h2f(ha[r * k + i]) * h2f(hb[i * n + c]);
      const double err = fabs(h2f(hc[r * n + c]) - acc) / (fabs(acc) + 1.0);
      if (err > worst) worst = err;
    }
  printf("gemm_f16 %lldx%lldx%lld: max relative error %.2e\n", (long long)m, (long long)n, (long long)k, worst);
  if (worst > 2e-3) return 3;

  /* Flash attention on 2 streams x 128 rows x 64 head dim (Q = K = V = A's rows). */
  CHECK(ipuc_flash_attention_f16(dc, IPUC_F32, da, da, da, 2, 128, 128, 64, 0.0f, NULL));
  CHECK(ipuc_device_status(NULL));

  /* The same GEMM through the spec-driven entry, accumulating onto C. */
  ipuc_kernel_spec spec;
  memset(&spec, 0, sizeof spec);
  spec.kind = IPUC_KERNEL_GEMM;
  spec.gemm.multiply = IPUC_F16;
  spec.gemm.accumulate = IPUC_F32;
  spec.gemm.mode = 0;
  ipuc_kernel_abi abi;
  CHECK(ipuc_query_abi(&spec, IPUC_F16, &abi));
  printf("spec gemm -> %s (replaces %s), %d inputs, %d scalars\n", abi.symbol, abi.reference_symbol,
         abi.input_count, abi.scalar_count);
  ipuc_tensor out = {dc, IPUC_F16, 2, {m, n, 0, 0}};
  ipuc_tensor in[2] = {{da, IPUC_F16, 2, {m, k, 0, 0}}, {db, IPUC_F16, 2, {k, n, 0, 0}}};
  CHECK(ipuc_launch(&spec, &out, in, 2, NULL, 0, NULL, 0, NULL));
  CHECK(ipuc_device_status(NULL));
  uint16_t *hc2 = malloc(m * n * 2);
  cudaMemcpy(hc2, dc, m * n * 2, cudaMemcpyDeviceToHost);
  if (memcmp(hc, hc2, m * n * 2) != 0) return 4; /* same call, same bits */

  /* A rejected run: GELU with an odd element count, as validate_kernel_run rejects it. */
  spec.kind = IPUC_KERNEL_GELU;
  ipuc_tensor g = {dc, IPUC_F16, 1, {7, 0, 0, 0}};
  uint32_t count = 7;
  ipuc_status st = ipuc_launch(&spec, &g, &g, 1, &count, 1, NULL, 0, NULL);
  printf("odd GELU: %s: %s\n", ipuc_status_string(st), ipuc_last_error_string());
  if (st != IPUC_ERR_INVALID_ARGUMENT) return 5;
  printf("ok\n");
  return 0;
}
