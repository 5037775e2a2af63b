/* A C program that drives the graph entry (include/ipug.h) alone, as a Rust
 * or other FFI caller of the reference's ComputeGraph API would: it builds
 * two GEMM-GELU-GEMM blocks as a Repeat over value sequences of weights
 * (the SiglipMlpBenchmark graph shape), prints the lowered plan and rank 1's
 * shard of a 2-GPU split, opens a session with every value kept (fuse = 0),
 * runs it, checks the output against a host evaluation that rounds every op
 * result to f16 (the reference evaluator's rule), and walks the per-op
 * diagnostic.  Exit status 0 on success. */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ipug.h"

enum { T = 64, D = 64, F = 128, BLOCKS = 2 };

static float q16(float f) { /* round to f16 (nearest even) and back: cuda_fp16 is not C */
  if (f == 0.0f || !isfinite(f)) return f;
  int e;
  frexpf(f, &e);               /* |f| in [2^(e-1), 2^e) */
  int q = e - 11;               /* 11 significant bits */
  if (q < -24) q = -24;         /* subnormal spacing */
  return ldexpf(nearbyintf(ldexpf(f, -q)), q);
}
static uint16_t f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  int32_t e = (int32_t)((x >> 23) & 0xff) - 127 + 15;
  uint32_t m = x & 0x7fffffu;
  if (e <= 0) { /* subnormal half */
    float a = fabsf(f);
    uint32_t v = (uint32_t)nearbyintf(a * 16777216.0f);
    return (uint16_t)(sign | v);
  }
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
static float gelu(float x) { return 0.5f * x * (1.0f + tanhf(0.7978846f * (x + 0.044715f * x * x * x))); }

#define CHECK(call)                                                                               \
  do {                                                                                            \
    ipuc_status st_ = (call);                                                                     \
    if (st_ != IPUC_OK) {                                                                         \
      fprintf(stderr, "%s: %s (%s)\n", #call, ipuc_status_string(st_), ipuc_last_error_string()); \
      return 1;                                                                                   \
    }                                                                                             \
  } while (0)
#define CHECKV(v)                                                                     \
  do {                                                                                \
    if ((v) < 0) {                                                                    \
      fprintf(stderr, "%s failed: %s\n", #v, ipuc_last_error_string());               \
      return 1;                                                                       \
    }                                                                                 \
  } while (0)

static void gemm(const float *a, const float *b, float *c, int m, int n, int k) {
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j) {
      float s = 0.0f;
      for (int e = 0; e < k; ++e) s += a[i * k + e] * b[e * n + j];
      c[i * n + j] = q16(s);
    }
}

int main(int argc, char **argv) {
  const int run = argc < 2 || strcmp(argv[1], "--plan-only") != 0;
  ipug_graph *g = ipug_graph_create();
  const uint32_t xs[3] = {1, T, D}, us[3] = {1, D, F}, ds[3] = {1, F, D};
  int32_t x = ipug_host_input(g, "left", xs, 3), up[BLOCKS], down[BLOCKS];
  CHECKV(x);
  char name[32];
  for (int i = 0; i < BLOCKS; ++i) {
    snprintf(name, sizeof name, "up%d", i);
    CHECKV(up[i] = ipug_parameter(g, name, us, 3));
    snprintf(name, sizeof name, "down%d", i);
    CHECKV(down[i] = ipug_parameter(g, name, ds, 3));
  }
  int32_t seqs[2];
  CHECKV(seqs[0] = ipug_value_sequence(g, "MLP up weights", up, BLOCKS));
  CHECKV(seqs[1] = ipug_value_sequence(g, "MLP down weights", down, BLOCKS));
  int32_t args[3], result;
  CHECK(ipug_repeat_begin(g, BLOCKS, &x, 1, NULL, 0, seqs, 2, args));
  int32_t h;
  CHECKV(h = ipug_gemm(g, args[0], args[1], 0, 0));
  CHECKV(h = ipug_gelu(g, h));
  CHECKV(h = ipug_gemm(g, h, args[2], 0, 0));
  if (ipug_repeat_end(g, &h, 1, &result) != 1) {
    fprintf(stderr, "repeat_end: %s\n", ipuc_last_error_string());
    return 1;
  }
  CHECK(ipug_set_outputs(g, &result, 1));

  static char buf[1 << 16];
  uint64_t need = 0;
  CHECK(ipug_graph_plan(g, buf, sizeof buf, &need));
  printf("plan:\n%s", buf);
  CHECK(ipug_graph_shard_json(g, 1, 2, buf, sizeof buf, &need));
  printf("rank 1 of 2: %.60s...\n", buf);
  if (!strstr(buf, "\"all_reduce\"")) {
    fprintf(stderr, "expected an all-reduce in the 2-GPU shard\n");
    return 1;
  }
  if (!run) {
    printf("ok\n");
    return 0;
  }

  /* inputs: deterministic values, rounded to f16 */
  float *hx = malloc(sizeof(float) * T * D), *hu[BLOCKS], *hd[BLOCKS];
  uint16_t *bits = malloc(2 * F * D > 2 * T * D ? 2 * F * D : 2 * T * D);
  for (int i = 0; i < T * D; ++i) hx[i] = q16(sinf(0.37f * i) * 1.5f);
  ipug_session_options o = {0, 0, 1, NULL, 0};
  ipuc_status st = IPUC_OK;
  ipug_session *s = ipug_session_open_ex(g, &o, &st);
  if (!s) {
    fprintf(stderr, "session_open: %s\n", ipuc_last_error_string());
    return 1;
  }
  for (int i = 0; i < T * D; ++i) bits[i] = f2h(hx[i]);
  CHECK(ipug_session_write(s, x, bits, 2ull * T * D, 0));
  for (int b = 0; b < BLOCKS; ++b) {
    hu[b] = malloc(sizeof(float) * D * F);
    hd[b] = malloc(sizeof(float) * F * D);
    for (int i = 0; i < D * F; ++i) {
      hu[b][i] = q16(cosf(0.11f * i + b) * 0.15f);
      hd[b][i] = q16(sinf(0.07f * i - b) * 0.12f);
    }
    for (int i = 0; i < D * F; ++i) bits[i] = f2h(hu[b][i]);
    CHECK(ipug_session_write(s, up[b], bits, 2ull * D * F, 0));
    for (int i = 0; i < D * F; ++i) bits[i] = f2h(hd[b][i]);
    CHECK(ipug_session_write(s, down[b], bits, 2ull * D * F, 0));
  }
  CHECK(ipug_session_run(s, 0));
  if (cudaDeviceSynchronize() != cudaSuccess) return 1;
  uint16_t *out = malloc(2ull * T * D);
  CHECK(ipug_session_read(s, result, out, 2ull * T * D, 0));

  /* host evaluation (f16 rounding after every op) */
  float *cur = malloc(sizeof(float) * T * D), *hid = malloc(sizeof(float) * T * F), *nxt = malloc(sizeof(float) * T * D);
  memcpy(cur, hx, sizeof(float) * T * D);
  for (int b = 0; b < BLOCKS; ++b) {
    gemm(cur, hu[b], hid, T, F, D);
    for (int i = 0; i < T * F; ++i) hid[i] = q16(gelu(hid[i]));
    gemm(hid, hd[b], nxt, T, D, F);
    memcpy(cur, nxt, sizeof(float) * T * D);
  }
  double err = 0.0, mx = 0.0, e2 = 0.0, r2 = 0.0;
  for (int i = 0; i < T * D; ++i) {
    const double d = (double)h2f(out[i]) - cur[i];
    err = fmax(err, fabs(d));
    mx = fmax(mx, fabs(cur[i]));
    e2 += d * d;
    r2 += (double)cur[i] * cur[i];
  }
  printf("max|err| %.3g of max|ref| %.3g, rel-L2 %.3g\n", err, mx, sqrt(e2 / r2));
  if (!(err <= 2e-2 * mx && sqrt(e2 / r2) <= 5e-3)) return 1;

  /* per-op diagnostic against the host value of the result */
  const float *ref = cur;
  ipug_value_report rep;
  CHECK(ipug_session_diagnose(s, &result, &ref, 1, &rep, 0));
  printf("diagnose v%d: available %d, rel-L2 %.3g\n", rep.value, rep.available, rep.rel_l2);
  if (!rep.available || rep.rel_l2 > 5e-3) return 1;
  ipug_session_close(s);
  ipug_graph_destroy(g);
  printf("ok\n");
  return 0;
}
