/*
 * CPU oracle for the ipu-stack operator-catalog hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is a plain-C restatement of the
 * reference's host-side evaluator and of its layout index maps.  It is the
 * checker for the CUDA kernels in ipu-stack_b200/csrc and the timed CPU
 * baseline in bench.py; no product code path may call it.
 *
 * Every function cites the reference source (paths relative to the
 * osmarks/ipu-stack checkout) whose behaviour it restates.
 *
 * Parity pinning: the reference is Rust and cannot be compiled here, so this
 * restatement is pinned against the known-answer checks held in the
 * reference's own tests (tests/test_oracle_kat.py lists them with file:line).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* IEEE binary16 conversion, round to nearest even.                          */
/* The reference uses the `half` crate 2.7.1 (Cargo.lock:288-290) through     */
/* f32_to_half / half_to_f32 (crates/ipu-tests/src/main.rs:2040-2046).        */
/* ------------------------------------------------------------------------ */

static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t oracle_f32_to_half(float value) {
  uint32_t x = f32_bits(value);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xffu) { /* inf / nan */
    if (man == 0) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | 0x7e00u | (man >> 13));
  }
  int32_t e = (int32_t)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u); /* overflow -> inf */
  if (e <= 0) {
    /* subnormal half (or zero) */
    if (e < -10) return (uint16_t)sign;
    uint32_t m = man | 0x800000u;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t half_man = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (half_man & 1u))) half_man++;
    return (uint16_t)(sign | half_man);
  }
  uint32_t half_man = man >> 13;
  uint32_t rem = man & 0x1fffu;
  uint32_t out = sign | ((uint32_t)e << 10) | half_man;
  if (rem > 0x1000u || (rem == 0x1000u && (half_man & 1u))) out++; /* carries into exp ok */
  return (uint16_t)out;
}

float oracle_half_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    if (man == 0) return bits_f32(sign);
    /* subnormal: value = man * 2^-24 */
    float v = (float)man * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  if (exp == 31) return bits_f32(sign | 0x7f800000u | (man << 13));
  return bits_f32(sign | ((exp - 15 + 127) << 23) | (man << 13));
}

/* quantize(value, F16): crates/ipu-tests/src/diagnostic.rs:841-847 */
float oracle_quantize_f16(float v) { return oracle_half_to_f32(oracle_f32_to_half(v)); }

void oracle_f32_to_half_array(const float *in, uint16_t *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f32_to_half(in[i]);
}
void oracle_half_to_f32_array(const uint16_t *in, float *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_half_to_f32(in[i]);
}

/* ------------------------------------------------------------------------ */
/* Layout index maps: crates/ipu-codegen/src/storage.rs                      */
/* Orders (include/ipuc.h numbering):                                         */
/*   0 row-major, 1 AMP-Left, 2 AMP-TransposedLeft, 3 AMP-TransposedRight,    */
/*   4 AMP-Output, 5 AMP-TransposedOutput, 6 BlockMajor, 7 BlockMajor^T       */
/* micro = 16 for F16 (storage.rs:784-790).  Return -1 on an invalid view.     */
/* ------------------------------------------------------------------------ */

enum { ORD_ROW = 0, ORD_AMP_LEFT = 1, ORD_AMP_TLEFT = 2, ORD_AMP_TRIGHT = 3,
       ORD_AMP_OUTPUT = 4, ORD_AMP_TOUTPUT = 5, ORD_BLOCK = 6, ORD_BLOCK_T = 7 };

/* storage.rs:353-371 right_matrix_index */
static int64_t right_index(int64_t micro, int64_t rows, int64_t cols, int64_t r, int64_t c) {
  if (r >= rows || c >= cols || rows % micro || cols % 16) return -1;
  int64_t panel = (c / 16) * (rows / micro) + r / micro;
  return panel * micro * 16 + (c % 16) * micro + r % micro;
}

/* storage.rs:301-351 amp_matrix_index */
int64_t oracle_amp_index(int order, int64_t micro, int64_t rows, int64_t cols, int64_t r, int64_t c) {
  if (r < 0 || c < 0 || r >= rows || c >= cols) return -1;
  switch (order) {
  case ORD_AMP_LEFT:
    if (cols % micro) return -1;
    return (c / micro) * rows * micro + r * micro + c % micro;
  case ORD_AMP_TRIGHT:
    return right_index(micro, cols, rows, c, r);
  case ORD_AMP_TLEFT:
    return oracle_amp_index(ORD_AMP_LEFT, micro, cols, rows, c, r);
  case ORD_AMP_OUTPUT: {
    if (cols % 16) return -1;
    int64_t logical_pair = c % 16 / 2;
    int64_t physical_pair = logical_pair % 4 * 2 + logical_pair / 4;
    int64_t physical_column = physical_pair * 2 + c % 2;
    return (c / 16) * rows * 16 + r * 16 + physical_column;
  }
  case ORD_AMP_TOUTPUT:
    return oracle_amp_index(ORD_AMP_OUTPUT, micro, cols, rows, c, r);
  default:
    return -1;
  }
}

/* storage.rs:372-426 block_major_matrix_index */
int64_t oracle_block_major_index(int transposed, int64_t micro, int64_t row_block, int64_t column_block,
                                 int64_t rows, int64_t cols, int64_t r, int64_t c) {
  if (transposed)
    return oracle_block_major_index(0, micro, row_block, column_block, cols, rows, c, r);
  if (r < 0 || c < 0 || r >= rows || c >= cols || row_block == 0 || column_block == 0 ||
      rows % row_block || cols % column_block || row_block % micro)
    return -1;
  int64_t row_groups = row_block / micro;
  int64_t panel = (r / row_block) * (cols / column_block) * row_groups +
                  (c / column_block) * row_groups + (r % row_block) / micro;
  return panel * micro * column_block + (c % column_block) * micro + r % micro;
}

/* Unified physical index of logical (r, c) in a [rows x cols] physical matrix. */
int64_t oracle_layout_index(int order, int64_t row_block, int64_t column_block,
                            int64_t rows, int64_t cols, int64_t r, int64_t c) {
  switch (order) {
  case ORD_ROW:
    if (r < 0 || c < 0 || r >= rows || c >= cols) return -1;
    return r * cols + c;
  case ORD_BLOCK: return oracle_block_major_index(0, 16, row_block, column_block, rows, cols, r, c);
  case ORD_BLOCK_T: return oracle_block_major_index(1, 16, row_block, column_block, rows, cols, r, c);
  default: return oracle_amp_index(order, 16, rows, cols, r, c);
  }
}

/* storage.rs:656-705 amp_matrix_coordinates, storage.rs:706-727
 * right_matrix_coordinates, storage.rs:729-782 block_major_matrix_coordinates.
 * Writes (row, col); returns 0 on success, -1 on an invalid view. */
int oracle_layout_coordinates(int order, int64_t row_block, int64_t column_block,
                              int64_t rows, int64_t cols, int64_t linear, int64_t *row, int64_t *col) {
  const int64_t micro = 16;
  switch (order) {
  case ORD_ROW:
    *row = linear / cols; *col = linear % cols; return 0;
  case ORD_AMP_LEFT: {
    if (cols % micro) return -1;
    int64_t pe = rows * micro, panel = linear / pe, off = linear % pe;
    *row = off / micro; *col = panel * micro + off % micro; return 0;
  }
  case ORD_AMP_TLEFT:
    return oracle_layout_coordinates(ORD_AMP_LEFT, 0, 0, cols, rows, linear, col, row);
  case ORD_AMP_TRIGHT: {
    /* right_matrix_coordinates(columns, rows) then swap */
    int64_t rr = cols, cc = rows; /* rows/cols of the right matrix */
    if (rr % micro || cc % 16) return -1;
    int64_t pe = micro * 16, panel = linear / pe, off = linear % pe;
    int64_t groups = rr / micro, cg = panel / groups, ig = panel % groups;
    int64_t right_row = ig * micro + off % micro;
    int64_t right_col = cg * 16 + off / micro;
    *row = right_col; *col = right_row; return 0;
  }
  case ORD_AMP_OUTPUT: {
    if (cols % 16) return -1;
    int64_t pe = rows * 16, panel = linear / pe, off = linear % pe;
    int64_t pc = off % 16, pp = pc / 2, lp = (pp % 2) * 4 + pp / 2;
    *row = off / 16; *col = panel * 16 + lp * 2 + pc % 2; return 0;
  }
  case ORD_AMP_TOUTPUT:
    return oracle_layout_coordinates(ORD_AMP_OUTPUT, 0, 0, cols, rows, linear, col, row);
  case ORD_BLOCK_T:
    return oracle_layout_coordinates(ORD_BLOCK, row_block, column_block, cols, rows, linear, col, row);
  case ORD_BLOCK: {
    if (!row_block || !column_block || rows % row_block || cols % column_block || row_block % micro)
      return -1;
    int64_t pe = micro * column_block, panel = linear / pe, off = linear % pe;
    int64_t rg = row_block / micro, cgs = cols / column_block, per = cgs * rg;
    int64_t rbi = panel / per, within = panel % per, cgi = within / rg, rgi = within % rg;
    *row = rbi * row_block + rgi * micro + off % micro;
    *col = cgi * column_block + off / micro;
    return 0;
  }
  default:
    return -1;
  }
}

/* ------------------------------------------------------------------------ */
/* Rearrange row-major -> {AMP-Left, AMP-TransposedRight, BlockMajor}, f16.  */
/* device/rearrange_f16.cpp:36-155 (generic), device/rearrange_amp_left_f16.S */
/* device/rearrange_transposed_right_f16.S, device/rearrange_block_major_f16.S */
/* Source: `matrices` row-major [R x C] matrices (row stride C).  Destination: */
/* `matrices` physical [Rp x Cp] matrices; padding is zero.                   */
/* target_order uses the codelet numbering of crates/ipu-codegen/src/         */
/* kernel.rs:363-498: 0 AMP-Left, 1 AMP-TransposedRight, 2 BlockMajor.        */
/* Returns 0, or -1 for an unsupported geometry.                              */
/* ------------------------------------------------------------------------ */
int oracle_rearrange_f16(uint16_t *dst, const uint16_t *src, int64_t matrices,
                         int64_t R, int64_t Rp, int target, int64_t C, int64_t Cp,
                         int64_t row_block, int64_t column_block) {
  if (R > Rp || C > Cp || C % 2) return -1;
  for (int64_t m = 0; m < matrices; ++m) {
    const uint16_t *s = src + m * R * C;
    uint16_t *d = dst + m * Rp * Cp;
    for (int64_t r = 0; r < Rp; ++r) {
      for (int64_t c = 0; c < Cp; ++c) {
        int64_t idx;
        if (target == 0) {
          if (Cp % 16) return -1;
          idx = (c / 16) * Rp * 16 + r * 16 + c % 16;
        } else if (target == 1) {
          /* rearrange_f16.cpp:74-91, columnBlock rows per panel, 16 columns */
          if (Cp % 16 || Rp % column_block) return -1;
          int64_t panel = (r / column_block) * (Cp / 16) + c / 16;
          idx = panel * 16 * column_block + (r % column_block) * 16 + c % 16;
        } else if (target == 2) {
          idx = oracle_block_major_index(0, 16, row_block, column_block, Rp, Cp, r, c);
          if (idx < 0) return -1;
        } else {
          return -1;
        }
        d[idx] = (r < R && c < C) ? s[r * C + c] : 0;
      }
    }
  }
  return 0;
}

/* Unpack AMP-Output (order 0) / AMP-TransposedLeft (order 1) -> row-major.  */
/* device/unpack_amp_f16.cpp:40-81.  Destination is row-major [Rp x Cp] per   */
/* matrix with zeros outside the logical [R x C] region.                      */
int oracle_unpack_f16(uint16_t *dst, const uint16_t *src, int source_order, int64_t matrices,
                      int64_t R, int64_t Rp, int64_t C, int64_t Cp) {
  if (source_order == 0 && Cp % 16) return -1;
  if (source_order == 1 && Rp % 16) return -1;
  if (Cp % 2 || R > Rp || C > Cp) return -1;
  int64_t me = Rp * Cp;
  for (int64_t m = 0; m < matrices; ++m) {
    for (int64_t r = 0; r < Rp; ++r) {
      for (int64_t c = 0; c < Cp; ++c) {
        uint16_t v = 0;
        if (r < R && c < C) {
          int64_t phys;
          if (source_order == 0) {
            int64_t lp = c % 16 / 2, pp = lp % 4 * 2 + lp / 4, pc = pp * 2 + c % 2;
            phys = (c / 16) * Rp * 16 + r * 16 + pc;
          } else {
            phys = (r / 16) * Cp * 16 + c * 16 + r % 16;
          }
          v = src[m * me + phys];
        }
        dst[m * me + r * Cp + c] = v;
      }
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* GELU: gelu_reference, crates/ipu-tests/src/main.rs:1985-1987 (f32 math).   */
/* ------------------------------------------------------------------------ */
float oracle_gelu(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978846f * (x + 0.044715f * (x * x * x))));
}

/* Map unary GELU then quantise to f16 (diagnostic.rs:433-436, :454-460). */
void oracle_gelu_f16(uint16_t *out, const uint16_t *in, int64_t n) {
  for (int64_t i = 0; i < n; ++i)
    out[i] = oracle_f32_to_half(oracle_gelu(oracle_half_to_f32(in[i])));
}

/* ------------------------------------------------------------------------ */
/* reduce_add: out = p0 + sum_i p_i (device/reduce_add_f16.S:7-72; ABI       */
/* crates/ipu-codegen/src/kernel.rs:1264-1274).  The host evaluator has no    */
/* reduction (split-K is a lowering artefact), so the sum is taken in f32 and */
/* quantised once, which is the evaluator's per-op-result rule.               */
/* in_f32 != 0: partials are f32; else f16.                                    */
/* ------------------------------------------------------------------------ */
void oracle_reduce_sum(uint16_t *out, const void *initial, const void *remote,
                       int64_t num_remote, int64_t n, int in_f32) {
  for (int64_t i = 0; i < n; ++i) {
    float acc;
    if (in_f32) {
      acc = ((const float *)initial)[i];
      for (int64_t p = 0; p < num_remote; ++p) acc += ((const float *)remote)[p * n + i];
    } else {
      acc = oracle_half_to_f32(((const uint16_t *)initial)[i]);
      for (int64_t p = 0; p < num_remote; ++p)
        acc += oracle_half_to_f32(((const uint16_t *)remote)[p * n + i]);
    }
    out[i] = oracle_f32_to_half(acc);
  }
}

/* ------------------------------------------------------------------------ */
/* GEMM scalar reference: the check that pins the BLAS path,                 */
/* diagnostic.rs:855-907 randomized_blas_gemm_matches_scalar_reference.       */
/* Row-major; ta/tb select transposed storage.  f32 accumulation.             */
/* The bulk oracle GEMM is cblas_sgemm via numpy (oracle.py), as in            */
/* diagnostic.rs:581-654.                                                      */
/* ------------------------------------------------------------------------ */
void oracle_sgemm_scalar(float *out, const float *a, const float *b, int64_t M, int64_t N, int64_t K,
                         int ta, int tb) {
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      float s = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        float av = ta ? a[k * M + i] : a[i * K + k];
        float bv = tb ? b[j * K + k] : b[k * N + j];
        s += av * bv;
      }
      out[i * N + j] = s;
    }
}

/* ------------------------------------------------------------------------ */
/* Attention: diagnostic.rs:711-780.  Q[S][Sq][D], K[S][Sk][D], V[S][Sk][Dv]  */
/* f32 values (already quantised by the caller), f32 output.  Non-causal      */
/* unless causal != 0.  Streams [s0, s1) only, so callers can time a subset   */
/* and thread over streams with identical per-row arithmetic.                 */
/* ------------------------------------------------------------------------ */
static void attention_streams(float *out, const float *q, const float *k, const float *v,
                              int64_t s0, int64_t s1, int64_t Sq, int64_t Sk, int64_t D, int64_t Dv,
                              float scale, int causal, float *logits) {
  for (int64_t s = s0; s < s1; ++s) {
    for (int64_t row = 0; row < Sq; ++row) {
      int64_t allowed = causal ? ((row + 1) < Sk ? (row + 1) : Sk) : Sk;
      for (int64_t col = 0; col < allowed; ++col) {
        float dot = 0.0f;
        const float *qr = q + (s * Sq + row) * D;
        const float *kr = k + (s * Sk + col) * D;
        for (int64_t i = 0; i < D; ++i) dot += qr[i] * kr[i];
        logits[col] = dot * scale;
      }
      float maximum = -INFINITY;
      for (int64_t col = 0; col < allowed; ++col) maximum = fmaxf(maximum, logits[col]);
      float sum = 0.0f;
      for (int64_t col = 0; col < allowed; ++col) {
        logits[col] = expf(logits[col] - maximum);
        sum += logits[col];
      }
      for (int64_t c = 0; c < Dv; ++c) {
        float result = 0.0f;
        for (int64_t i = 0; i < allowed; ++i)
          result += logits[i] / sum * v[(s * Sk + i) * Dv + c];
        out[(s * Sq + row) * Dv + c] = result;
      }
    }
  }
}

typedef struct {
  float *out; const float *q, *k, *v;
  int64_t s0, s1, Sq, Sk, D, Dv; float scale; int causal;
} attn_job;

static void *attn_worker(void *p) {
  attn_job *j = (attn_job *)p;
  float *logits = (float *)malloc(sizeof(float) * (size_t)(j->Sk > 0 ? j->Sk : 1));
  attention_streams(j->out, j->q, j->k, j->v, j->s0, j->s1, j->Sq, j->Sk, j->D, j->Dv, j->scale,
                    j->causal, logits);
  free(logits);
  return NULL;
}

/* threads <= 1: the reference's single-threaded loop. */
void oracle_attention(float *out, const float *q, const float *k, const float *v,
                      int64_t streams, int64_t Sq, int64_t Sk, int64_t D, int64_t Dv,
                      float scale, int causal, int threads) {
  if (threads <= 1 || streams < 2) {
    attn_job j = {out, q, k, v, 0, streams, Sq, Sk, D, Dv, scale, causal};
    attn_worker(&j);
    return;
  }
  if (threads > streams) threads = (int)streams;
  pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
  attn_job *jobs = (attn_job *)malloc(sizeof(attn_job) * (size_t)threads);
  for (int t = 0; t < threads; ++t) {
    int64_t s0 = streams * t / threads, s1 = streams * (t + 1) / threads;
    attn_job j = {out, q, k, v, s0, s1, Sq, Sk, D, Dv, scale, causal};
    jobs[t] = j;
    pthread_create(&tid[t], NULL, attn_worker, &jobs[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
  free(tid);
  free(jobs);
}

/* ------------------------------------------------------------------------ */
/* Flash (online) attention vertex: device/flash_attention_online_f16.cpp:   */
/* 61-143.  f16 inputs, f32 online max/sum/accumulator, key block 32,         */
/* f32 output.                                                                */
/* ------------------------------------------------------------------------ */
void oracle_flash_attention_online(float *out, const uint16_t *q, const uint16_t *k, const uint16_t *v,
                                   int64_t matrices, int64_t Sq, int64_t Sk, int64_t D, int64_t Dv,
                                   float scale, int64_t key_block) {
  float *scores = (float *)malloc(sizeof(float) * (size_t)key_block);
  for (int64_t m = 0; m < matrices; ++m) {
    for (int64_t row = 0; row < Sq; ++row) {
      const uint16_t *qv = q + (m * Sq + row) * D;
      float *dst = out + (m * Sq + row) * Dv;
      for (int64_t c = 0; c < Dv; ++c) dst[c] = 0.0f;
      float maximum = -INFINITY, denominator = 0.0f;
      for (int64_t ks = 0; ks < Sk; ks += key_block) {
        int64_t rows = Sk - ks < key_block ? Sk - ks : key_block;
        float bmax = -INFINITY;
        for (int64_t br = 0; br < rows; ++br) {
          const uint16_t *kv = k + (m * Sk + ks + br) * D;
          float s = 0.0f;
          for (int64_t i = 0; i < D; ++i) s += oracle_half_to_f32(qv[i]) * oracle_half_to_f32(kv[i]);
          scores[br] = s * scale;
          bmax = fmaxf(bmax, scores[br]);
        }
        float next = fmaxf(maximum, bmax);
        float prev_scale = maximum == -INFINITY ? 0.0f : expf(maximum - next);
        denominator *= prev_scale;
        for (int64_t c = 0; c < Dv; ++c) dst[c] *= prev_scale;
        for (int64_t br = 0; br < rows; ++br) {
          float w = expf(scores[br] - next);
          denominator += w;
          const uint16_t *vv = v + (m * Sk + ks + br) * Dv;
          for (int64_t c = 0; c < Dv; ++c) dst[c] += oracle_half_to_f32(vv[c]) * w;
        }
        maximum = next;
      }
      float rcp = 1.0f / denominator;
      for (int64_t c = 0; c < Dv; ++c) dst[c] *= rcp;
    }
  }
  free(scores);
}

/* ------------------------------------------------------------------------ */
/* Attention softmax stage: device/attention_softmax_f16.cpp:63-139.          */
/* scores: f16 panels [KB/16][Q][16]; key_rows valid keys of KB (KB % 16 == 0)*/
/* weights: f16 in the same order, followed by Q f32 maxima (scaled) and Q    */
/* f32 denominators (written into `state`).  exp is evaluated from the f16-   */
/* rounded argument and rounded to f16 (the reference's f16v2exp).            */
/* ------------------------------------------------------------------------ */
void oracle_attention_softmax(uint16_t *weights, float *state, const uint16_t *scores,
                              int64_t Q, int64_t key_rows, int64_t KB, int64_t head_dim) {
  const float scale = 1.0f / sqrtf((float)head_dim);
  for (int64_t row = 0; row < Q; ++row) {
    float maximum = -65504.0f;
    for (int64_t c = 0; c < key_rows; ++c) {
      int64_t src = (c / 16) * Q * 16 + row * 16 + c % 16;
      maximum = fmaxf(maximum, oracle_half_to_f32(scores[src]));
    }
    float smax = maximum * scale;
    float denominator = 0.0f;
    for (int64_t c = 0; c < KB; ++c) {
      int64_t idx = (c / 16) * Q * 16 + row * 16 + c % 16;
      float normalized = -65504.0f;
      if (c < key_rows) normalized = oracle_half_to_f32(scores[idx]) * scale - smax;
      float arg = oracle_quantize_f16(normalized);
      uint16_t w = oracle_f32_to_half(expf(arg));
      weights[idx] = w;
      if (c < key_rows) denominator += oracle_half_to_f32(w);
    }
    state[row] = smax;
    state[Q + row] = denominator;
  }
}

/* ------------------------------------------------------------------------ */
/* Attention merge stage: device/attention_stages_f16.S:698-855.              */
/* acc: f32 rows of stride Vp; the row's {max, denominator} live at acc[V],   */
/* acc[V+1] (stages.S:773).  block: f16 PV panels [ceil(V/16)][Q][16].        */
/* state: Q maxima then Q denominators (the softmax stage's output).          */
/* ------------------------------------------------------------------------ */
void oracle_attention_merge(float *acc, const uint16_t *block, const float *state, int64_t Q,
                            int64_t V, int64_t Vp, int initial, int final_block) {
  for (int64_t r = 0; r < Q; ++r) {
    float *a = acc + r * Vp;
    float mb = state[r], lb = state[Q + r];
    if (initial) {
      a[V] = mb;
      a[V + 1] = lb;
      for (int64_t c = 0; c < V; ++c) a[c] = oracle_half_to_f32(block[(c / 16) * Q * 16 + r * 16 + c % 16]);
    } else {
      float m = a[V], l = a[V + 1];
      float mn = fmaxf(m, mb);
      float s_old = expf(m - mn), s_new = expf(mb - mn);
      a[V] = mn;
      a[V + 1] = l * s_old + lb * s_new;
      for (int64_t c = 0; c < V; ++c)
        a[c] = a[c] * s_old + oracle_half_to_f32(block[(c / 16) * Q * 16 + r * 16 + c % 16]) * s_new;
    }
    if (final_block) {
      float rcp = 1.0f / a[V + 1];
      for (int64_t c = 0; c < V; ++c) a[c] *= rcp;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* SplitHeads: diagnostic.rs:685-709, [b, r, h*c] -> [b*h, r, c].             */
/* Add with NumPy broadcasting: diagnostic.rs:673-683 (restated for the       */
/* row-broadcast case used by bias/residual adds: right repeats every         */
/* `right_period` elements, 0 = same shape).                                  */
/* ------------------------------------------------------------------------ */
void oracle_split_heads(uint16_t *out, const uint16_t *in, int64_t batch, int64_t rows,
                        int64_t heads, int64_t channels) {
  int64_t width = heads * channels;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t h = 0; h < heads; ++h)
      for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < channels; ++c)
          out[((b * heads + h) * rows + r) * channels + c] = in[(b * rows + r) * width + h * channels + c];
}

void oracle_add_f16(uint16_t *out, const uint16_t *left, const uint16_t *right, int64_t n,
                    int64_t left_period, int64_t right_period) {
  for (int64_t i = 0; i < n; ++i) {
    float l = oracle_half_to_f32(left[left_period ? i % left_period : i]);
    float r = oracle_half_to_f32(right[right_period ? i % right_period : i]);
    out[i] = oracle_f32_to_half(l + r);
  }
}
