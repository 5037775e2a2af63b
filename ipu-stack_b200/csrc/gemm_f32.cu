// FP32 GEMM: the B200 counterpart of the reference's gemm_f32_64_amp tile
// kernels (device/gemm_f32_64_amp.S:129-385, f32 multiply, f32 accumulate).
//
// fp32 accuracy on the tensor cores by a three-pass f16 split: every row of A
// and column of B is scaled by a power of two (below), every scaled operand
// x = hi + lo with hi = f16(x) and lo = f16(x - hi), and
//   A.B ~= A_hi.B_hi + A_hi.B_lo + A_lo.B_hi
// (the dropped lo.lo term is ~2^-22 relative), accumulated in fp32 in TMEM.
// f16 carries the same 10 explicit mantissa bits as TF32, and kind::f16 MMAs
// run at twice the kind::tf32 rate with half the operand bytes, so this split
// matches the classic 3xTF32 one in accuracy at twice its MMA throughput.
// Long chains of MMAs into one accumulator lose precision, so each tile's K
// loop runs in chunks of 256: every chunk accumulates into a fresh TMEM
// buffer (two, ping-ponged) and the epilogue warps sum the chunk partials in
// fp32 registers.
// Prepass kernels find the row maxima of A and the column maxima of B and
// write the scaled hi/lo planes (B transposed to K-major when it is row-major
// [k x n]) into the caller's workspace; the main kernel is the same
// warp-specialised persistent tcgen05 pipeline as the FP16 GEMM (TMA producer
// / single-thread MMA issuer / 8 epilogue warps, double-buffered 128x256
// accumulators, CTA pairs when there is a wave of 256x256 tiles) issuing
// three kind::f16 MMAs per K16 step, and its epilogue removes the scaling.
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <cstdlib>
#include <cstring>
#include <mutex>

namespace ipuc {
namespace {

using namespace sm100;

// A k-block is one 128-byte swizzle row of each plane: 64 f16 or 32 TF32
// elements; an MMA k-step (K16 f16, K8 TF32) is 32 bytes of it either way, so
// stage sizes and descriptor offsets are the same for both splits.
constexpr int BM = 128, BN = 256, BK_BYTES = 128, STAGES = 2;
constexpr int A_BYTES = BM * BK_BYTES;  // 16 KB per plane
constexpr int B_BYTES = BN * BK_BYTES;  // 32 KB per plane
constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;  // 96 KB
constexpr int TMEM_COLS = 2 * BN;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int GROUP_M = 16;
constexpr int CHUNK_K = 256;     // K per TMEM accumulation chunk
template <bool kF16> struct Split {
  static constexpr int BK = kF16 ? 64 : 32;            // elements per k-block
  static constexpr int KC = CHUNK_K / BK;               // k-blocks per chunk
  static constexpr uint32_t kFormat = kF16 ? 0u : 2u;   // instruction-descriptor A/B format
};
constexpr int EPI_THREADS = 256; // 8 epilogue warps
constexpr int NUM_THREADS = 64 + EPI_THREADS;

// Round to TF32 (10 explicit mantissa bits), nearest, ties away from zero.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// 3xTF32 (IPUC_GEMM_F32_SPLIT_TF32): hi/lo planes of a row-major [rows x cols]
// matrix with leading dimension ld into dense [rows x cols] fp32 planes, with
// hi = tf32(x) and lo = tf32(x - hi); no scaling (TF32 has fp32's exponent).
__global__ void __launch_bounds__(256) split_tf32_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                         int64_t ld, float *__restrict__ hi, float *__restrict__ lo) {
  const int64_t total4 = rows * cols / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += stride) {
    const int64_t e = i * 4, r = e / cols, c = e % cols;
    const float4 x = *reinterpret_cast<const float4 *>(src + r * ld + c);
    float4 h, l;
    h.x = to_tf32(x.x); l.x = to_tf32(x.x - h.x);
    h.y = to_tf32(x.y); l.y = to_tf32(x.y - h.y);
    h.z = to_tf32(x.z); l.z = to_tf32(x.z - h.z);
    h.w = to_tf32(x.w); l.w = to_tf32(x.w - h.w);
    reinterpret_cast<float4 *>(hi)[i] = h;
    reinterpret_cast<float4 *>(lo)[i] = l;
  }
}

// hi/lo planes of B^T: B is row-major [rows x cols] (ld); the planes are dense
// [cols x rows], so the MMA reads B K-major.  64x64 tiles through shared memory,
// 16-byte loads and stores (each thread moves 16 elements each way) so that
// enough bytes are in flight per SM to run near HBM bandwidth; the padded tile
// row (65 floats) keeps the column reads conflict-free.  Vector accesses need
// rows, cols and ld to be multiples of 4 (the gemm_f32 entry requires that);
// ragged 64x64 tiles fall back to scalar accesses.
__global__ void __launch_bounds__(256) split_tf32_transpose_kernel(const float *__restrict__ src, int64_t rows,
                                                                   int64_t cols, int64_t ld, float *__restrict__ hi,
                                                                   float *__restrict__ lo) {
  __shared__ float tile[64][65];
  const int64_t tr = (rows + 63) / 64, tc = (cols + 63) / 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads, 4 consecutive elements each
  for (int64_t t = blockIdx.x; t < tr * tc; t += gridDim.x) {
    const int64_t r0 = (t / tc) * 64, c0 = (t % tc) * 64;
    const bool full = r0 + 64 <= rows && c0 + 64 <= cols;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = ty + 16 * i, cc = tx * 4;
      const int64_t r = r0 + rr, c = c0 + cc;
      float4 v;
      if (full) {
        v = *reinterpret_cast<const float4 *>(src + r * ld + c);
      } else {
        v.x = (r < rows && c < cols) ? src[r * ld + c] : 0.0f;
        v.y = (r < rows && c + 1 < cols) ? src[r * ld + c + 1] : 0.0f;
        v.z = (r < rows && c + 2 < cols) ? src[r * ld + c + 2] : 0.0f;
        v.w = (r < rows && c + 3 < cols) ? src[r * ld + c + 3] : 0.0f;
      }
      tile[rr][cc] = v.x;
      tile[rr][cc + 1] = v.y;
      tile[rr][cc + 2] = v.z;
      tile[rr][cc + 3] = v.w;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int oc = ty + 16 * i, orr = tx * 4;  // output row = source column c0 + oc
      const int64_t c = c0 + oc, r = r0 + orr;
      float x[4], h[4], l[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        x[e] = tile[orr + e][oc];
        h[e] = to_tf32(x[e]);
        l[e] = to_tf32(x[e] - h[e]);
      }
      if (full) {
        *reinterpret_cast<float4 *>(hi + c * rows + r) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4 *>(lo + c * rows + r) = make_float4(l[0], l[1], l[2], l[3]);
      } else if (c < cols) {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (r + e < rows) {
            hi[c * rows + r + e] = h[e];
            lo[c * rows + r + e] = l[e];
          }
      }
    }
  }
}

// ---- 3xF16 split with power-of-two row/column scaling ----
// f16 has TF32's 10 explicit mantissa bits but only a 5-bit exponent, so each
// row of A and each column of B is first scaled by an exact power of two 2^e
// that puts its largest magnitude in [2^14, 2^15): then hi = f16(x 2^e) and
// lo = f16(x 2^e - hi) carry 22 bits for every element within 2^17 of the
// row's maximum (smaller ones keep an absolute error below 2^-39 of it), and
// the MMA products of the scaled planes equal the TF32 split's to the bit
// budget.  The epilogue multiplies C by 2^-(e_row + e_col).  Maxima are kept
// as the bits of |x| compared as integers: non-negative floats order like
// their bit patterns, and +inf and NaN sort above every finite value, so a
// maximum >= 0x7f800000 marks a row or column holding a non-finite value.
//
// Elements more than 2^17 below their row's (column's) maximum keep fewer
// than 22 bits (their lo part falls into f16 subnormals).  The prepass counts
// them per row and column ("tiny" counts; a non-finite row or column gets
// kTinyAll).  With T tiny elements in row i and column j together, the lost
// bits add at most T * 2^-10 to the scaled product sum C_s (each such operand
// is off by at most 2^-25 and its partner is below 2^15).  The epilogue keeps
// C_s only where that bound is below 2^-23 |C_s|; otherwise it leaves the
// element alone and marks it in a bitmap, and a fix-up kernel recomputes the
// marked elements with plain fp32 FMAs from A and B (which also gives the
// IEEE inf/NaN pattern of a non-finite input element by element).  Rows of
// everyday data (normal or uniform values, K in the thousands) hold at most a
// few tiny elements and mark nothing or next to nothing.

// e such that mx * 2^e lies in [2^14, 2^15); 0 for zero, inf and NaN rows;
// at most 126 so that 2^e and 2^-e are normal floats.
__host__ __device__ __forceinline__ int split_exponent(uint32_t max_bits) {
  const uint32_t f = max_bits >> 23;
  if (max_bits == 0 || f >= 255) return 0;
#ifdef __CUDA_ARCH__
  const int lz = __clz(max_bits);
#else
  const int lz = __builtin_clz(max_bits);
#endif
  const int ex = f ? (int)f - 127 : (31 - lz) - 149;  // floor(log2(mx))
  const int e = 14 - ex;
  return e < 126 ? e : 126;
}

__device__ __forceinline__ float pow2(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

constexpr int32_t kTinyAll = 1 << 24;           // tiny count of a row/column with a non-finite value
__device__ __forceinline__ uint32_t abs_bits(float x) { return __float_as_uint(x) & 0x7fffffffu; }
// A scaled element that keeps fewer than 22 bits in hi + lo.
// (|xs| bits - 1) < bits(0.125) - 1 as unsigned: nonzero and below 2^-3.
__device__ __forceinline__ int is_tiny(float xs) {
  return ((__float_as_uint(xs) & 0x7fffffffu) - 1u) < 0x3dffffffu;
}
// True where the tiny elements of the element's row and column (`tiny`
// together) may have moved the scaled sum v by more than 2^-23 |v| (or v is
// not finite while a non-finite input is involved).
__device__ __forceinline__ bool needs_fixup(float v, int tiny) {
  return tiny != 0 && !(fabsf(v) * 0x1p-13f >= (float)tiny);
}

__device__ __forceinline__ void split_f16(float x, float scale, __half &h, __half &l) {
  const float xs = x * scale;
  h = __float2half_rn(xs);
  l = __float2half_rn(xs - __half2float(h));
}

// Largest |x| of every column of a row-major [rows x cols] matrix into out
// (zeroed by the caller).  A CTA covers 128 columns x COLMAX_ROWS rows: 8 row
// lanes of 32 threads, each thread 4 columns with four 16-byte loads in
// flight; the 8 row lanes merge through shared memory and one atomicMax per
// column and CTA (on the float bits) merges the CTAs.
constexpr int COLMAX_ROWS = 128;
__global__ void __launch_bounds__(256) col_absmax_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                         int64_t ld, uint32_t *__restrict__ out) {
  __shared__ uint4 part[8][32];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t col_tiles = (cols + 127) / 128, bands = (rows + COLMAX_ROWS - 1) / COLMAX_ROWS;
  for (int64_t t = blockIdx.x; t < col_tiles * bands; t += gridDim.x) {
    const int64_t c = (t % col_tiles) * 128 + 4 * tx;
    const int64_t r0 = (t / col_tiles) * COLMAX_ROWS, r1 = min(rows, r0 + COLMAX_ROWS);
    uint4 mx = make_uint4(0u, 0u, 0u, 0u);
    if (c < cols) {
      for (int64_t r = r0 + ty; r < r1; r += 32) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          v[u] = r + 8 * u < r1 ? __ldg(reinterpret_cast<const float4 *>(src + (r + 8 * u) * ld + c))
                                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          mx.x = max(mx.x, abs_bits(v[u].x)); mx.y = max(mx.y, abs_bits(v[u].y));
          mx.z = max(mx.z, abs_bits(v[u].z)); mx.w = max(mx.w, abs_bits(v[u].w));
        }
      }
    }
    __syncthreads();
    part[ty][tx] = mx;
    __syncthreads();
    if (ty == 0 && c < cols) {
#pragma unroll
      for (int y = 1; y < 8; ++y) {
        const uint4 o = part[y][tx];
        mx.x = max(mx.x, o.x); mx.y = max(mx.y, o.y); mx.z = max(mx.z, o.z); mx.w = max(mx.w, o.w);
      }
      atomicMax(out + c, mx.x);
      atomicMax(out + c + 1, mx.y);
      atomicMax(out + c + 2, mx.z);
      atomicMax(out + c + 3, mx.w);
    }
  }
}

// Row exponents and f16 hi/lo planes [rows x ldp] of a row-major [rows x
// cols] matrix with one read of the matrix: one CTA per row holds the row in
// registers (ROW_CACHE float4 per thread: rows up to 4096 floats; longer rows
// re-read their remainder, from L2), reduces the row's largest |x| through
// shared memory, stores the row's split exponent to rexp for the epilogue and
// writes the row scaled and split.  Pad columns [cols, ldp) are zero.  cols
// and ld are multiples of 4.
constexpr int ROW_CACHE = 4;
__global__ void __launch_bounds__(256) split_f16_rows_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                             int64_t ld, int32_t *__restrict__ rexp, int64_t ldp,
                                                             __half *__restrict__ hi, __half *__restrict__ lo,
                                                             int32_t *__restrict__ tiny, uint32_t *__restrict__ fixrow) {
  __shared__ uint32_t red[8];
  __shared__ int cnt[8];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t q = cols / 4, qp = ldp / 4;
  const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  auto amax4 = [](uint32_t m, float4 x) {
    return max(max(m, max(abs_bits(x.x), abs_bits(x.y))), max(abs_bits(x.z), abs_bits(x.w)));
  };
  auto put = [&](int64_t r, int64_t c, float4 x, float scale) {
    __half h[4], l[4];
    split_f16(x.x, scale, h[0], l[0]);
    split_f16(x.y, scale, h[1], l[1]);
    split_f16(x.z, scale, h[2], l[2]);
    split_f16(x.w, scale, h[3], l[3]);
    *reinterpret_cast<uint2 *>(hi + r * ldp + 4 * c) = *reinterpret_cast<const uint2 *>(h);
    *reinterpret_cast<uint2 *>(lo + r * ldp + 4 * c) = *reinterpret_cast<const uint2 *>(l);
    return is_tiny(x.x * scale) + is_tiny(x.y * scale) + is_tiny(x.z * scale) + is_tiny(x.w * scale);
  };
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float4 *row = reinterpret_cast<const float4 *>(src + r * ld);
    float4 v[ROW_CACHE];
    uint32_t mx = 0;
#pragma unroll
    for (int u = 0; u < ROW_CACHE; ++u) {
      const int64_t c = tid + u * 256;
      v[u] = c < q ? row[c] : zero;
      mx = amax4(mx, v[u]);
    }
    for (int64_t c = tid + ROW_CACHE * 256; c < q; c += 256) mx = amax4(mx, row[c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[wid] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = max(mx, red[w]);
    const int e = split_exponent(mx);
    if (tid == 0) {
      rexp[r] = e;
      if (fixrow) fixrow[r] = 0u;  // the epilogue raises it where a row needs the fix-up
    }
    const float scale = pow2(e);
    int t = 0;
#pragma unroll
    for (int u = 0; u < ROW_CACHE; ++u) {
      const int64_t c = tid + u * 256;
      if (c < qp) t += put(r, c, v[u], scale);
    }
    for (int64_t c = tid + ROW_CACHE * 256; c < qp; c += 256) t += put(r, c, c < q ? row[c] : zero, scale);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) cnt[wid] = t;
    __syncthreads();
    if (tid == 0) {
      int total = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) total += cnt[w];
      tiny[r] = mx >= 0x7f800000u ? kTinyAll : total;
    }
    __syncthreads();  // red and cnt are rewritten for the next row
  }
}

// f16 hi/lo planes of B^T: B row-major [rows x cols] (ld) -> planes
// [cols x ldp] (K-major), source column c scaled by 2^split_exponent(cmax[c]);
// the tiles of the first row band also store the column exponents to cexp.
// 64x64 tiles through shared memory (16-byte loads; the padded tile row of 65
// floats keeps the column reads conflict-free); pad elements [rows, ldp) of
// each plane row are zero.  Full 64x64 tiles need rows, cols and ld multiples
// of 4 (the gemm_f32 entry requires that); ragged tiles use scalar loads.
__global__ void __launch_bounds__(256, 8) split_f16_transpose_kernel(const float *__restrict__ src, int64_t rows,
                                                                  int64_t cols, int64_t ld,
                                                                  const uint32_t *__restrict__ cmax, int64_t ldp,
                                                                  __half *__restrict__ hi, __half *__restrict__ lo,
                                                                  int32_t *__restrict__ cexp, int32_t *__restrict__ tiny) {
  __shared__ float tile[64][65];
  const int64_t tr = (ldp + 63) / 64, tc = (cols + 63) / 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  for (int64_t t = blockIdx.x; t < tr * tc; t += gridDim.x) {
    const int64_t r0 = (t / tc) * 64, c0 = (t % tc) * 64;
    const bool full = r0 + 64 <= rows && c0 + 64 <= cols;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = ty + 16 * i, cc = tx * 4;
      const int64_t r = r0 + rr, c = c0 + cc;
      float4 v;
      if (full) {
        v = *reinterpret_cast<const float4 *>(src + r * ld + c);
      } else {
        v.x = (r < rows && c < cols) ? src[r * ld + c] : 0.0f;
        v.y = (r < rows && c + 1 < cols) ? src[r * ld + c + 1] : 0.0f;
        v.z = (r < rows && c + 2 < cols) ? src[r * ld + c + 2] : 0.0f;
        v.w = (r < rows && c + 3 < cols) ? src[r * ld + c + 3] : 0.0f;
      }
      tile[rr][cc] = v.x;
      tile[rr][cc + 1] = v.y;
      tile[rr][cc + 2] = v.z;
      tile[rr][cc + 3] = v.w;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int oc = ty + 16 * i, orr = tx * 4;  // plane row = source column c0 + oc
      const int64_t c = c0 + oc, r = r0 + orr;
      if (c < cols && r < ldp) {
        int t = 0;
        const uint32_t mx = cmax[c];
        const int ce = split_exponent(mx);
        if (r0 == 0 && tx == 0) {
          cexp[c] = ce;
          if (mx >= 0x7f800000u) tiny[c] = kTinyAll;
        }
        const float scale = pow2(ce);
        __half h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = tile[orr + e][oc];
          split_f16(x, scale, h[e], l[e]);
          t += is_tiny(x * scale);
        }
        *reinterpret_cast<uint2 *>(hi + c * ldp + r) = *reinterpret_cast<const uint2 *>(h);
        *reinterpret_cast<uint2 *>(lo + c * ldp + r) = *reinterpret_cast<const uint2 *>(l);
        // tiny elements are rare: one atomic where a thread holds some
        if (t > 0 && mx < 0x7f800000u) atomicAdd(tiny + c, t);
      }
    }
  }
}

struct Gemm32Params {
  float *c;
  int64_t m, n, k;
  int64_t ldc;
  int32_t tiles_m, tiles_n, k_blocks;
  int64_t num_tiles;
  uint32_t flags;
  uint32_t *err;
  const int32_t *ea, *eb;  // split exponents of the rows of A and the columns of B
  const int32_t *ta, *tb;  // tiny counts of the rows of A and the columns of B
  uint32_t *fixmap;        // [m][fix_words] bitmap of C elements left to the fix-up kernel
  uint32_t *fixrow;        // [m] nonzero where a row has a marked element
  int64_t fix_words;
  // Work units of the CTA-pair kernel: units [0, split_from) are whole tiles;
  // every tile t >= split_from (the last, partial wave) is two units, one per
  // half of its K chunks, whose epilogues add their partial sums into C
  // (zeroed beforehand) with atomics.  No split: split_from = num_units = num_tiles.
  int64_t num_units, split_from;
};

// C element scale 2^-(e_row + e_col) of the 3xF16 split, exact unless C itself
// over- or underflows.
__device__ __forceinline__ float unscale(float v, int e_row, int e_col) {
  const int e = e_row + e_col;
  if (e >= -126 && e <= 126) return v * pow2(-e);
  return (v * pow2(-e_row)) * pow2(-e_col);
}

// Writes one 32-column word of the fix-up bitmap (3xF16).  A whole tile's
// epilogue owns its words, so it stores them outright (no clearing needed);
// the two K halves of a split tile OR theirs into words the zeroing kernel
// cleared.
__device__ __forceinline__ void put_fix_word(const Gemm32Params &p, int64_t row, int64_t col, uint32_t word,
                                             bool split) {
  uint32_t *w = p.fixmap + row * p.fix_words + (col >> 5);
  if (split) {
    if (word) atomicOr(w, word);
  } else {
    *w = word;
  }
  if (word) p.fixrow[row] = 1u;
}

// Epilogue store of the scaled sums v of C[row][col .. col+3] (cp points at
// C[row][col]): unscaled (3xF16), then added atomically (a K-split half),
// added to C (IPUC_GEMM_ACCUMULATE) or stored.  Elements that need the fix-up
// are left alone; the returned 4-bit mask names them.
template <bool kF16>
__device__ __forceinline__ uint32_t store_c4(const Gemm32Params &p, float *cp, int64_t col, float4 v, int er, int tr,
                                             bool split, bool accumulate) {
  if constexpr (kF16) {
    const int4 ec = __ldg(reinterpret_cast<const int4 *>(p.eb + col));
    const int4 tc = __ldg(reinterpret_cast<const int4 *>(p.tb + col));
    const uint32_t f = (needs_fixup(v.x, tr + tc.x) ? 1u : 0u) | (needs_fixup(v.y, tr + tc.y) ? 2u : 0u) |
                       (needs_fixup(v.z, tr + tc.z) ? 4u : 0u) | (needs_fixup(v.w, tr + tc.w) ? 8u : 0u);
    v.x = unscale(v.x, er, ec.x);
    v.y = unscale(v.y, er, ec.y);
    v.z = unscale(v.z, er, ec.z);
    v.w = unscale(v.w, er, ec.w);
    if (f) {
      const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (f & (1u << e)) continue;
        if (split) atomicAdd(cp + e, x[e]);
        else cp[e] = accumulate ? cp[e] + x[e] : x[e];
      }
      return f;
    }
  }
  float4 *c4 = reinterpret_cast<float4 *>(cp);
  if (split) {
    atomicAdd(c4, v);
    return 0u;
  }
  if (accumulate) {
    const float4 o = *c4;
    v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
  }
  *c4 = v;
  return 0u;
}

template <bool kF16>
__device__ __forceinline__ uint32_t store_c1(const Gemm32Params &p, float *cp, int64_t col, float x, int er, int tr,
                                             bool split, bool accumulate) {
  if constexpr (kF16) {
    if (needs_fixup(x, tr + p.tb[col])) return 1u;
    x = unscale(x, er, p.eb[col]);
  }
  if (split) atomicAdd(cp, x);
  else *cp = accumulate ? *cp + x : x;
  return 0u;
}

// The epilogue of one thread's row segment (BN / 2 columns from col_base).
template <bool kF16>
__device__ __forceinline__ void store_row(const Gemm32Params &p, const float (&acc)[BN / 2], int64_t row,
                                          int64_t col_base, bool vec_ok, bool split, bool accumulate) {
  const int er = kF16 ? p.ea[row] : 0, tr = kF16 ? p.ta[row] : 0;
  float *cp = p.c + row * p.ldc + col_base;
  uint32_t word = 0;
  if (vec_ok && col_base + BN / 2 <= p.n) {
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
      word |= store_c4<kF16>(p, cp + 4 * j, col_base + 4 * j,
                             make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]), er, tr, split,
                             accumulate)
              << ((4 * j) & 31);
      if (kF16 && (4 * j + 4) % 32 == 0) {
        put_fix_word(p, row, col_base + 4 * j - 28, word, split);
        word = 0;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < BN / 2; ++j) {
      if (col_base + j < p.n)
        word |= store_c1<kF16>(p, cp + j, col_base + j, acc[j], er, tr, split, accumulate) << (j & 31);
      if (kF16 && (j & 31) == 31) {
        if (col_base + j - 31 < p.n) put_fix_word(p, row, col_base + j - 31, word, split);
        word = 0;
      }
    }
  }
}

__device__ __forceinline__ void tile_coords(const Gemm32Params &p, int64_t t, int &mt, int &nt) {
  const int64_t in_group = (int64_t)GROUP_M * p.tiles_n;
  const int64_t g = t / in_group;
  const int first = (int)(g * GROUP_M);
  const int gs = min(p.tiles_m - first, GROUP_M);
  const int64_t w = t % in_group;
  mt = first + (int)(w % gs);
  nt = (int)(w / gs);
}

struct WorkUnit {
  int64_t tile;
  int c0, c1;   // K chunks [c0, c1)
  bool split;   // one of two halves: the epilogue adds into C
};
__device__ __forceinline__ WorkUnit work_unit(const Gemm32Params &p, int64_t u, int chunks) {
  if (u < p.split_from) return {u, 0, chunks, false};
  const int64_t v = u - p.split_from;
  const int mid = chunks / 2;
  return {p.split_from + v / 2, (v & 1) ? mid : 0, (v & 1) ? chunks : mid, true};
}

// Zeroes the C regions of the split tiles (blockIdx.y = tile - split_from)
// and, for 3xF16, their words of the fix-up bitmap (the two halves OR into them).
__global__ void __launch_bounds__(256) zero_split_tiles_kernel(const Gemm32Params p, int pair_bm) {
  int mt, nt;
  tile_coords(p, p.split_from + blockIdx.y, mt, nt);
  const int64_t r0 = (int64_t)mt * pair_bm, c0 = (int64_t)nt * BN;
  // one float4 of C per thread and step (ldc and n are multiples of 4)
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < pair_bm * BN / 4; idx += gridDim.x * blockDim.x) {
    const int64_t r = r0 + idx / (BN / 4), c = c0 + 4 * (idx % (BN / 4));
    if (r < p.m && c < p.n) {
      *reinterpret_cast<float4 *>(p.c + r * p.ldc + c) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (p.fixmap && (c & 31) == 0) p.fixmap[r * p.fix_words + (c >> 5)] = 0u;
    }
  }
}

template <bool kF16>
__device__ __forceinline__ void mma_split(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  if constexpr (kF16) mma_f16_ss(d, a, b, idesc, acc);
  else mma_tf32_ss(d, a, b, idesc, acc);
}
template <bool kF16>
__device__ __forceinline__ void mma_split_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  if constexpr (kF16) mma_f16_ss_pair(d, a, b, idesc, acc);
  else mma_tf32_ss_pair(d, a, b, idesc, acc);
}

template <bool kF16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_split3_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                       const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
                       const Gemm32Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *acc_full = empty + STAGES;
  uint64_t *acc_empty = acc_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_THREADS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  constexpr int BK = Split<kF16>::BK, KC = Split<kF16>::KC;
  const int chunks = (p.k_blocks + KC - 1) / KC;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int mt, nt;
        tile_coords(p, t, mt, nt);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *st = smem + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tma_load_3d(st, &tmAh, &full[s], kb * BK, mt * BM, 0);
          tma_load_3d(st + A_BYTES, &tmAl, &full[s], kb * BK, mt * BM, 0);
          uint8_t *bh = st + 2 * A_BYTES, *bl = bh + B_BYTES;
          tma_load_3d(bh, &tmBh, &full[s], kb * BK, nt * BN, 0);
          tma_load_3d(bl, &tmBl, &full[s], kb * BK, nt * BN, 0);
        }
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F32 | ERR_SITE_PRODUCER);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(BM, BN, Split<kF16>::kFormat, false, false);
      uint32_t it = 0, g = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        for (int c = 0; c < chunks && ok; ++c, ++g) {
          const uint32_t buf = g & 1u, use = g >> 1;
          if (!mbar_wait_bounded(&acc_empty[buf], (use & 1u) ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * BN;
          const int kb_end = min(p.k_blocks, (c + 1) * KC);
          for (int kb = c * KC; kb < kb_end; ++kb, ++it) {
            const int s = it % STAGES;
            const uint32_t ph = (it / STAGES) & 1u;
            if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t ah = smem_u32(smem + s * STAGE_BYTES), al = ah + A_BYTES;
            const uint32_t bh = ah + 2 * A_BYTES, bl = bh + B_BYTES;
#pragma unroll
            for (int k = 0; k < BK_BYTES / 32; ++k) {  // 32-byte k-steps
              const uint64_t dah = make_smem_desc(ah + k * 32, 16, 1024, kSwizzle128B);
              const uint64_t dal = make_smem_desc(al + k * 32, 16, 1024, kSwizzle128B);
              const uint64_t dbh = make_smem_desc(bh + k * 32, 16, 1024, kSwizzle128B);
              const uint64_t dbl = make_smem_desc(bl + k * 32, 16, 1024, kSwizzle128B);
              // Small terms first, then the dominant hi.hi product.
              mma_split<kF16>(d_tmem, dal, dbh, idesc, (kb != c * KC || k != 0) ? 1u : 0u);
              mma_split<kF16>(d_tmem, dah, dbl, idesc, 1u);
              mma_split<kF16>(d_tmem, dah, dbh, idesc, 1u);
            }
            mma_commit(&empty[s]);
          }
          if (!ok) break;
          mma_commit(&acc_full[buf]);
        }
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F32 | ERR_SITE_MMA);
        *abort_flag = 1;
      }
    }
  } else {
    // 8 epilogue warps: warp w owns TMEM lanes of quarter w%4 and the column
    // half (w-2)/4 of the 256-wide tile.  Each K chunk's partial product is
    // drained from TMEM and summed in fp32 registers, so no tensor-core
    // accumulation chain is longer than one chunk.
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const bool accumulate = (p.flags & IPUC_GEMM_ACCUMULATE) != 0;
    const bool vec_ok = (p.ldc % 4 == 0);
    uint32_t g = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
      float acc[BN / 2];
#pragma unroll
      for (int i = 0; i < BN / 2; ++i) acc[i] = 0.0f;
      for (int c = 0; c < chunks; ++c, ++g) {
        const uint32_t buf = g & 1u, use = g >> 1;
        if (!mbar_wait_bounded(&acc_full[buf], use & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int ch = 0; ch < BN / 64; ++ch) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + buf * BN + half * (BN / 2) + ch * 32 + ((uint32_t)(quarter * 32) << 16), r);
          tmem_wait_ld(r);
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[ch * 32 + i] += __uint_as_float(r[i]);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
      }
      if (!ok) break;
      int mt, nt;
      tile_coords(p, t, mt, nt);
      const int64_t row = (int64_t)mt * BM + quarter * 32 + lane;
      const int64_t col_base = (int64_t)nt * BN + half * (BN / 2);
      if (row < p.m) store_row<kF16>(p, acc, row, col_base, vec_ok, false, accumulate);
    }
    if (!ok) {
      record_device_error(p.err, ERR_KERNEL_GEMM_F32 | ERR_SITE_EPILOGUE);
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// CTA-pair form (cluster of 2, tcgen05.mma.cta_group::2): a 256x256 tile per
// pair, each CTA loading its own 128 rows of the A planes and 128 rows of the
// K-major B planes, the leader issuing M256 N256 K8 MMAs.  Per CTA this halves
// the shared-memory traffic of B (TMA fill + operand reads), which bounds the
// single-CTA kernel.
constexpr int P_STAGE_BYTES = 2 * A_BYTES + 2 * A_BYTES;  // A hi/lo + half of B hi/lo: 64 KB
constexpr int P_STAGES = 3;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256;
constexpr int PAIR_BM = 2 * BM;

template <bool kF16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_split3_pair_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                            const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
                            const Gemm32Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + P_STAGES * P_STAGE_BYTES);
  uint64_t *empty = full + P_STAGES;
  uint64_t *acc_full = empty + P_STAGES;
  uint64_t *acc_empty = acc_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);   // the leader's arrive_expect_tx; both CTAs' bytes land on it
      mbar_init(&empty[s], 1);  // one multicast commit per stage use
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * (EPI_THREADS / 32));  // lane 0 of every epilogue warp of both CTAs
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  constexpr int BK = Split<kF16>::BK, KC = Split<kF16>::KC;
  const int chunks = (p.k_blocks + KC - 1) / KC;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t u = pair; u < p.num_units && ok; u += pairs) {
        const WorkUnit w = work_unit(p, u, chunks);
        int mt, nt;
        tile_coords(p, w.tile, mt, nt);  // mt counts 256-row pair tiles
        const int32_t arow = mt * PAIR_BM + (int32_t)rank * BM, brow = nt * BN + (int32_t)rank * (BN / 2);
        const int kb_end = min(p.k_blocks, w.c1 * KC);
        for (int kb = w.c0 * KC; kb < kb_end; ++kb, ++it) {
          const int s = it % P_STAGES;
          const uint32_t ph = (it / P_STAGES) & 1u;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *st = smem + s * P_STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * P_STAGE_BYTES);
          tma_load_3d_pair(st, &tmAh, &full[s], kb * BK, arow, 0);
          tma_load_3d_pair(st + A_BYTES, &tmAl, &full[s], kb * BK, arow, 0);
          tma_load_3d_pair(st + 2 * A_BYTES, &tmBh, &full[s], kb * BK, brow, 0);
          tma_load_3d_pair(st + 3 * A_BYTES, &tmBl, &full[s], kb * BK, brow, 0);
        }
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F32 | ERR_SITE_PRODUCER);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = make_idesc(PAIR_BM, BN, Split<kF16>::kFormat, false, false);
      // Descriptors built once; stages and k-steps add offsets in 16-byte units.
      const uint64_t d0 = make_smem_desc(smem_u32(smem), 16, 1024, kSwizzle128B);
      uint32_t it = 0, g = 0;
      bool ok = true;
      for (int64_t u = pair; u < p.num_units && ok; u += pairs) {
        const WorkUnit w = work_unit(p, u, chunks);
        for (int c = w.c0; c < w.c1 && ok; ++c, ++g) {
          const uint32_t buf = g & 1u, use = g >> 1;
          if (!mbar_wait_bounded(&acc_empty[buf], (use & 1u) ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * BN;
          const int kb_end = min(p.k_blocks, (c + 1) * KC);
          for (int kb = c * KC; kb < kb_end; ++kb, ++it) {
            const int s = it % P_STAGES;
            const uint32_t ph = (it / P_STAGES) & 1u;
            if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t dah = d0 + (uint64_t)(s * (P_STAGE_BYTES >> 4));
            const uint64_t dal = dah + (uint64_t)(A_BYTES >> 4);
            const uint64_t dbh = dah + (uint64_t)((2 * A_BYTES) >> 4);
            const uint64_t dbl = dah + (uint64_t)((3 * A_BYTES) >> 4);
#pragma unroll
            for (int k = 0; k < BK_BYTES / 32; ++k) {  // 32-byte k-steps
              const uint64_t o = (uint64_t)((k * 32) >> 4);
              // Small terms first, then the dominant hi.hi product.
              mma_split_pair<kF16>(d_tmem, dal + o, dbh + o, idesc, (kb != c * KC || k != 0) ? 1u : 0u);
              mma_split_pair<kF16>(d_tmem, dah + o, dbl + o, idesc, 1u);
              mma_split_pair<kF16>(d_tmem, dah + o, dbh + o, idesc, 1u);
            }
            mma_commit_pair(&empty[s], 0x3);
          }
          if (!ok) break;
          mma_commit_pair(&acc_full[buf], 0x3);
        }
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F32 | ERR_SITE_MMA);
        *abort_flag = 1;
      }
    }
  } else if (warp >= 2) {
    // 8 epilogue warps per CTA, as in the single-CTA kernel: warp w owns TMEM
    // lanes of quarter w%4 (this CTA's 128 rows) and the column half (w-2)/4.
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const bool accumulate = (p.flags & IPUC_GEMM_ACCUMULATE) != 0;
    const bool vec_ok = (p.ldc % 4 == 0);
    uint32_t g = 0;
    bool ok = true;
    for (int64_t u = pair; u < p.num_units && ok; u += pairs) {
      const WorkUnit w = work_unit(p, u, chunks);
      float acc[BN / 2];
#pragma unroll
      for (int i = 0; i < BN / 2; ++i) acc[i] = 0.0f;
      for (int c = w.c0; c < w.c1; ++c, ++g) {
        const uint32_t buf = g & 1u, use = g >> 1;
        if (!mbar_wait_bounded(&acc_full[buf], use & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int ch = 0; ch < BN / 64; ++ch) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + buf * BN + half * (BN / 2) + ch * 32 + ((uint32_t)(quarter * 32) << 16), r);
          tmem_wait_ld(r);
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[ch * 32 + i] += __uint_as_float(r[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_leader(&acc_empty[buf]);
      }
      if (!ok) break;
      int mt, nt;
      tile_coords(p, w.tile, mt, nt);
      const int64_t row = (int64_t)mt * PAIR_BM + (int64_t)rank * BM + quarter * 32 + lane;
      const int64_t col_base = (int64_t)nt * BN + half * (BN / 2);
      if (row < p.m) store_row<kF16>(p, acc, row, col_base, vec_ok, w.split, accumulate);
    }
    if (!ok) {
      record_device_error(p.err, ERR_KERNEL_GEMM_F32 | ERR_SITE_EPILOGUE);
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

inline uint64_t round256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

// Recomputes the C elements the 3xF16 epilogue marked (tiny or non-finite
// operands, see above) as fp32 FMA dot products: C = (IPUC_GEMM_ACCUMULATE ?
// C : 0) + sum_k A[r][k] B[k][j].  One warp per marked element: lane l sums
// k = l, l + 32, ... (32 loads in flight instead of a k-long chain of
// dependent ones), then the lanes' sums are added in a fixed butterfly order.
// CTA b owns rows b, b + grid, b + 2 grid, ...; it reads 256 of their flags at
// once (one load per thread) and its 8 warps share the marked rows' words.
__global__ void __launch_bounds__(256) gemm_f32_fixup_kernel(const float *__restrict__ a, const float *__restrict__ b,
                                                             float *__restrict__ c, int64_t m, int64_t n, int64_t k,
                                                             int64_t lda, int64_t ldb, int64_t ldc, int bt,
                                                             int accumulate, const uint32_t *__restrict__ fixmap,
                                                             const uint32_t *__restrict__ fixrow, int64_t words) {
  __shared__ int64_t marked[256];
  __shared__ int count;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t g = gridDim.x;
  for (int64_t base = blockIdx.x; base < m; base += 256 * g) {
    if (threadIdx.x == 0) count = 0;
    __syncthreads();
    const int64_t r = base + (int64_t)threadIdx.x * g;
    if (r < m && fixrow[r]) marked[atomicAdd(&count, 1)] = r;
    __syncthreads();
    for (int q = 0; q < count; ++q) {
      const int64_t row = marked[q];
      const uint32_t *map = fixmap + row * words;
      const float *ar = a + row * lda;
      for (int64_t wd = warp; wd < words; wd += 8) {
        uint32_t bits = map[wd];
        while (bits) {
          const int bit = __ffs(bits) - 1;
          bits &= bits - 1;
          const int64_t j = wd * 32 + bit;
          if (j >= n) break;
          float sum = 0.0f;
          if (bt) {
            const float *bc = b + j * ldb;
#pragma unroll 4
            for (int64_t e = lane; e < k; e += 32) sum = fmaf(ar[e], bc[e], sum);
          } else {
#pragma unroll 4
            for (int64_t e = lane; e < k; e += 32) sum = fmaf(ar[e], b[e * ldb + j], sum);
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
          if (lane == 0) {
            float *cp = c + row * ldc + j;
            *cp = accumulate ? *cp + sum : sum;
          }
        }
      }
    }
    __syncthreads();  // count and marked are rewritten for the next group
  }
}

// Workspace, 3xF16: A_hi, A_lo [m x kp] and B_hi, B_lo [n x kp] f16 (kp = k
// rounded up to 8, so that plane rows are 16-byte multiples for TMA), then the
// split exponents of A's rows [m] and B's columns [n] (int32), B's column
// maxima [n] (u32 |x| bits, row-major B only), the tiny counts of B's columns
// [n] and A's rows [m], the fix-up row flags [m] and the fix-up bitmap
// [m x ceil(n / 32)] (u32), each 256-byte aligned.
// 3xTF32: A_hi, A_lo [m x k] and B_hi, B_lo [n x k] fp32.  The workspace size
// is the larger of the two.
int64_t f16_pitch(int64_t k) { return (k + 7) & ~int64_t(7); }
uint64_t tf32_workspace(int64_t m, int64_t n, int64_t k) {
  return 2 * round256((uint64_t)m * k * 4) + 2 * round256((uint64_t)k * n * 4);
}

template <bool kF16>
ipuc_status launch_main(const CUtensorMap &tah, const CUtensorMap &tal, void *bh, void *bl, int64_t m, int64_t n,
                        int64_t k, int64_t ldp, Gemm32Params &p, cudaStream_t stream) {
  constexpr int BK = Split<kF16>::BK;
  const auto dt = kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const size_t eb = kF16 ? 2 : 4;
  ipuc_status st;
  p.tiles_n = (int32_t)((n + BN - 1) / BN);
  p.k_blocks = (int32_t)((k + BK - 1) / BK);
  const int sms = sm_count();
  const int64_t pair_tiles = ((m + PAIR_BM - 1) / PAIR_BM) * (int64_t)p.tiles_n;
  if (m > BM && sms >= 2 && pair_tiles >= sms / 2) {
    // CTA pairs (at least one full wave of 256x256 tiles; below that the
    // single-CTA kernel spreads the work over more SMs): A boxes of 128 rows
    // per CTA, B boxes of 128 rows (half of BN).
    CUtensorMap pbh, pbl;
    if ((st = make_map_3d(&pbh, dt, eb, bh, k, n, 1, ldp, 0, BK, BN / 2)) != IPUC_OK) return st;
    if ((st = make_map_3d(&pbl, dt, eb, bl, k, n, 1, ldp, 0, BK, BN / 2)) != IPUC_OK) return st;
    p.tiles_m = (int32_t)((m + PAIR_BM - 1) / PAIR_BM);
    p.num_tiles = (int64_t)p.tiles_m * p.tiles_n;
    const int64_t pairs = p.num_tiles < sms / 2 ? p.num_tiles : sms / 2;
    // A last wave at most half full runs as two K halves per tile (two units
    // each), so that it takes about half a wave-time; C must not be an
    // accumulation target (two atomic adds onto zero are order-independent).
    const int chunks = (p.k_blocks + Split<kF16>::KC - 1) / Split<kF16>::KC;
    const int64_t tail = p.num_tiles % pairs;
    p.split_from = p.num_units = p.num_tiles;
    if (tail > 0 && 2 * tail <= pairs && chunks >= 2 && !(p.flags & IPUC_GEMM_ACCUMULATE)) {
      p.split_from = p.num_tiles - tail;
      p.num_units = p.num_tiles + tail;
      zero_split_tiles_kernel<<<dim3(64, (unsigned)tail), 256, 0, stream>>>(p, PAIR_BM);
      if ((st = check_launch("zero_split_tiles_kernel")) != IPUC_OK) return st;
    }
    IPUC_CUDA(cudaFuncSetAttribute(gemm_split3_pair_kernel<kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   P_SMEM_BYTES));
    gemm_split3_pair_kernel<kF16><<<(unsigned)(2 * pairs), NUM_THREADS, P_SMEM_BYTES, stream>>>(tah, tal, pbh, pbl, p);
    return check_launch("gemm_split3_pair_kernel");
  }
  CUtensorMap tbh, tbl;
  if ((st = make_map_3d(&tbh, dt, eb, bh, k, n, 1, ldp, 0, BK, BN)) != IPUC_OK) return st;
  if ((st = make_map_3d(&tbl, dt, eb, bl, k, n, 1, ldp, 0, BK, BN)) != IPUC_OK) return st;
  p.tiles_m = (int32_t)((m + BM - 1) / BM);
  p.num_tiles = (int64_t)p.tiles_m * p.tiles_n;
  p.split_from = p.num_units = p.num_tiles;
  const int grid = (int)(p.num_tiles < sms ? p.num_tiles : sms);
  IPUC_CUDA(cudaFuncSetAttribute(gemm_split3_kernel<kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  gemm_split3_kernel<kF16><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(tah, tal, tbh, tbl, p);
  return check_launch("gemm_split3_kernel");
}

}  // namespace

// Bytes of workspace the split named by `flags` uses.
uint64_t gemm_f32_workspace_for(int64_t m, int64_t n, int64_t k, uint32_t flags) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  if (flags & IPUC_GEMM_F32_SPLIT_TF32) return tf32_workspace(m, n, k);
  const uint64_t kp = (uint64_t)f16_pitch(k);
  const uint64_t words = ((uint64_t)n + 31) / 32;
  return 2 * round256((uint64_t)m * kp * 2) + 2 * round256((uint64_t)n * kp * 2) + 3 * round256((uint64_t)m * 4) +
         3 * round256((uint64_t)n * 4) + round256((uint64_t)m * words * 4);
}

// ipuc_gemm_f32_workspace_bytes: enough for either split.
uint64_t gemm_f32_workspace(int64_t m, int64_t n, int64_t k) {
  const uint64_t a = gemm_f32_workspace_for(m, n, k, 0), b = gemm_f32_workspace_for(m, n, k, IPUC_GEMM_F32_SPLIT_TF32);
  return a > b ? a : b;
}

ipuc_status gemm_f32_launch(float *c, const float *a, const float *b, int64_t m, int64_t n, int64_t k, int64_t lda,
                            int64_t ldb, int64_t ldc, uint32_t flags, void *workspace, uint64_t workspace_bytes,
                            cudaStream_t stream) {
  IPUC_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "gemm_f32: negative extent");
  IPUC_CHECK_ARG((flags & ~(uint32_t)(IPUC_GEMM_ACCUMULATE | IPUC_GEMM_B_TRANSPOSED | IPUC_GEMM_F32_SPLIT_TF32)) == 0,
                 "gemm_f32: only IPUC_GEMM_ACCUMULATE, IPUC_GEMM_B_TRANSPOSED and IPUC_GEMM_F32_SPLIT_TF32 apply");
  if (m == 0 || n == 0) return IPUC_OK;
  IPUC_CHECK_ARG(k > 0, "gemm_f32: k must be positive");
  IPUC_CHECK_ARG(a && b && c, "gemm_f32: null pointer");
  const bool bt = (flags & IPUC_GEMM_B_TRANSPOSED) != 0;
  IPUC_CHECK_ARG(lda >= k && ldc >= n && ldb >= (bt ? k : n), "gemm_f32: leading dimension too small");
  IPUC_CHECK_ALIGN(aligned(a, 16) && aligned(b, 16) && aligned(c, 16), "gemm_f32: pointers must be 16-byte aligned");
  IPUC_CHECK_ALIGN(lda % 4 == 0 && ldb % 4 == 0 && k % 4 == 0 && n % 4 == 0,
                   "gemm_f32: lda, ldb, k and n must be multiples of 4 elements");
  IPUC_CHECK_ARG(m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), "gemm_f32: extent too large");
  const uint64_t need = gemm_f32_workspace_for(m, n, k, flags);
  IPUC_CHECK_ARG(workspace != nullptr && workspace_bytes >= need,
                 "gemm_f32: workspace smaller than ipuc_gemm_f32_workspace_bytes()");
  IPUC_CHECK_ALIGN(aligned(workspace, 256), "gemm_f32: workspace must be 256-byte aligned");
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const int cap = sm_count() * 8;

  Gemm32Params p;
  p.c = c;
  p.m = m; p.n = n; p.k = k;
  p.ldc = ldc;
  p.flags = flags;
  p.err = device_error_word();
  p.ea = p.eb = p.ta = p.tb = nullptr;
  p.fixmap = p.fixrow = nullptr;
  p.fix_words = 0;
  ipuc_status st;
  CUtensorMap tah, tal;

  if (!(flags & IPUC_GEMM_F32_SPLIT_TF32)) {
    const int64_t kp = f16_pitch(k);
    __half *ah = reinterpret_cast<__half *>(ws);
    __half *al = reinterpret_cast<__half *>(ws + round256((uint64_t)m * kp * 2));
    uint8_t *bbase = ws + 2 * round256((uint64_t)m * kp * 2);
    __half *bh = reinterpret_cast<__half *>(bbase);
    __half *bl = reinterpret_cast<__half *>(bbase + round256((uint64_t)n * kp * 2));
    uint8_t *mbase = bbase + 2 * round256((uint64_t)n * kp * 2);
    const uint64_t m4 = round256((uint64_t)m * 4), n4 = round256((uint64_t)n * 4);
    const int64_t words = (n + 31) / 32;
    int32_t *ea = reinterpret_cast<int32_t *>(mbase);
    int32_t *eb = reinterpret_cast<int32_t *>(mbase + m4);
    uint32_t *bmax = reinterpret_cast<uint32_t *>(mbase + m4 + n4);
    int32_t *tb = reinterpret_cast<int32_t *>(mbase + m4 + 2 * n4);  // right after bmax: one memset clears both
    int32_t *ta = reinterpret_cast<int32_t *>(mbase + m4 + 3 * n4);
    uint32_t *fixrow = reinterpret_cast<uint32_t *>(mbase + 2 * m4 + 3 * n4);
    uint32_t *fixmap = reinterpret_cast<uint32_t *>(mbase + 3 * m4 + 3 * n4);
    split_f16_rows_kernel<<<(unsigned)(m < cap ? m : cap), 256, 0, stream>>>(a, m, k, lda, ea, kp, ah, al, ta,
                                                                               fixrow);
    if (bt) {
      split_f16_rows_kernel<<<(unsigned)(n < cap ? n : cap), 256, 0, stream>>>(b, n, k, ldb, eb, kp, bh, bl, tb,
                                                                               nullptr);
    } else {
      IPUC_CUDA(cudaMemsetAsync(bmax, 0, 2 * n4, stream));
      const int64_t col_ctas = ((n + 127) / 128) * ((k + COLMAX_ROWS - 1) / COLMAX_ROWS);
      col_absmax_kernel<<<(unsigned)(col_ctas < cap ? col_ctas : cap), 256, 0, stream>>>(b, k, n, ldb, bmax);
      const int64_t tiles = ((kp + 63) / 64) * ((n + 63) / 64);
      split_f16_transpose_kernel<<<(unsigned)(tiles < cap ? tiles : cap), 256, 0, stream>>>(b, k, n, ldb, bmax, kp,
                                                                                            bh, bl, eb, tb);
    }
    if ((st = check_launch("gemm_f32 split (3xF16)")) != IPUC_OK) return st;
    const auto f16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if ((st = make_map_3d(&tah, f16, 2, ah, k, m, 1, kp, 0, Split<true>::BK, BM)) != IPUC_OK) return st;
    if ((st = make_map_3d(&tal, f16, 2, al, k, m, 1, kp, 0, Split<true>::BK, BM)) != IPUC_OK) return st;
    p.ea = ea;
    p.eb = eb;
    p.ta = ta;
    p.tb = tb;
    p.fixmap = fixmap;
    p.fixrow = fixrow;
    p.fix_words = words;
    if ((st = launch_main<true>(tah, tal, bh, bl, m, n, k, kp, p, stream)) != IPUC_OK) return st;
    gemm_f32_fixup_kernel<<<(unsigned)(m < cap ? m : cap), 256, 0, stream>>>(
        a, b, c, m, n, k, lda, ldb, ldc, bt ? 1 : 0, (flags & IPUC_GEMM_ACCUMULATE) ? 1 : 0, fixmap, fixrow, words);
    return check_launch("gemm_f32_fixup_kernel");
  }

  // 3xTF32: unscaled TF32 hi/lo planes, fp32 storage.
  float *ah = reinterpret_cast<float *>(ws);
  float *al = reinterpret_cast<float *>(ws + round256((uint64_t)m * k * 4));
  float *bh = reinterpret_cast<float *>(ws + 2 * round256((uint64_t)m * k * 4));
  float *bl = reinterpret_cast<float *>(ws + 2 * round256((uint64_t)m * k * 4) + round256((uint64_t)k * n * 4));
  auto grid_of = [&](int64_t threads) {
    const int64_t g = (threads + 255) / 256;
    return (unsigned)(g < cap ? (g < 1 ? 1 : g) : cap);
  };
  split_tf32_kernel<<<grid_of(m * k / 4), 256, 0, stream>>>(a, m, k, lda, ah, al);
  if (bt) {
    split_tf32_kernel<<<grid_of(n * k / 4), 256, 0, stream>>>(b, n, k, ldb, bh, bl);
  } else {
    const int64_t tiles = ((k + 63) / 64) * ((n + 63) / 64);
    split_tf32_transpose_kernel<<<(unsigned)(tiles < cap ? tiles : cap), 256, 0, stream>>>(b, k, n, ldb, bh, bl);
  }
  if ((st = check_launch("gemm_f32 split (3xTF32)")) != IPUC_OK) return st;
  const auto f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if ((st = make_map_3d(&tah, f32, 4, ah, k, m, 1, k, 0, Split<false>::BK, BM)) != IPUC_OK) return st;
  if ((st = make_map_3d(&tal, f32, 4, al, k, m, 1, k, 0, Split<false>::BK, BM)) != IPUC_OK) return st;
  return launch_main<false>(tah, tal, bh, bl, m, n, k, k, p, stream);
}

}  // namespace ipuc

using namespace ipuc;

extern "C" uint64_t ipuc_gemm_f32_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  return gemm_f32_workspace(m, n, k);
}

extern "C" ipuc_status ipuc_gemm_f32(float *c, const float *a, const float *b, int64_t m, int64_t n, int64_t k,
                                     int64_t lda, int64_t ldb, int64_t ldc, uint32_t flags, void *workspace,
                                     uint64_t workspace_bytes, ipuc_stream stream) {
  return gemm_f32_launch(c, a, b, m, n, k, lda, ldb, ldc, flags, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of ipuc_gemm_f32.
//
// Some callers cannot allocate device memory at the point where they need an
// FP32 GEMM: a plug-in loaded into a host framework that owns the device
// allocator and forbids cudaMalloc from library code, code running in a host
// callback, or a real-time path whose memory budget is fixed up front.  They get ipuc_gemm_f32_noalloc: the same kernels, with the
// hi/lo f16 split planes placed in a fixed file-scope device array instead
// of a caller-provided workspace.
//
// The array is a device symbol, so on the host its name is only a stand-in:
// its device address is resolved once per device with cudaGetSymbolAddress
// (during the first call on that device, with that device current) and cached
// together with the current context, so that a call after cudaDeviceReset or
// under another context resolves it again.
// Every GPU that loads libipuc.so holds the array until the process exits.
// All calls share it: two calls that overlap on the GPU (different streams, or
// the same call issued concurrently from two host threads) race on it.  The
// split kernels rewrite every byte the GEMM reads, so nothing needs clearing
// between calls.
// ---------------------------------------------------------------------------
namespace ipuc {
namespace {

constexpr uint64_t kNoAllocScratchBytes = 64ull << 20;  // 64 MiB
static __device__ __align__(256) uint8_t g_gemm_f32_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
// Cached device address of the array per device, with the context it was
// resolved in: a module reloaded into a new context (after cudaDeviceReset, or
// under a caller's non-primary context) places the array elsewhere, so a
// context change re-resolves it.
struct ScratchSlot {
  void *ctx = nullptr;
  void *ptr = nullptr;
};
ScratchSlot g_scratch_slot[64];

using CtxGetCurrentFn = int (*)(void **);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

ipuc_status scratch_address(void **out) {
  int dev = 0;
  IPUC_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(IPUC_ERR_UNSUPPORTED, "gemm_f32_noalloc: device index above 63");
  CtxGetCurrentFn get = ctx_get_current();
  if (!get) return fail(IPUC_ERR_CUDA, "gemm_f32_noalloc: cuCtxGetCurrent is unavailable");
  void *ctx = nullptr;
  if (get(&ctx) != 0) return fail(IPUC_ERR_CUDA, "gemm_f32_noalloc: cuCtxGetCurrent failed");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot &slot = g_scratch_slot[dev];
  if (!ctx || !slot.ptr || slot.ctx != ctx) {
    // With no context current yet, this runtime call makes the primary one
    // current; the context is read again afterwards.
    void *p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_gemm_f32_scratch);
    if (err != cudaSuccess) return cuda_fail(err, "gemm_f32_noalloc: cudaGetSymbolAddress(scratch)");
    if (!ctx && (get(&ctx) != 0 || !ctx)) return fail(IPUC_ERR_CUDA, "gemm_f32_noalloc: no current context");
    slot.ctx = ctx;
    slot.ptr = p;
  }
  *out = slot.ptr;
  return IPUC_OK;
}

}  // namespace
}  // namespace ipuc

extern "C" ipuc_status ipuc_gemm_f32_noalloc(float *c, const float *a, const float *b, int64_t m, int64_t n,
                                             int64_t k, int64_t lda, int64_t ldb, int64_t ldc, uint32_t flags,
                                             ipuc_stream stream) {
  const uint64_t need = ipuc::gemm_f32_workspace_for(m, n, k, flags);
  if (need > ipuc::kNoAllocScratchBytes) {
    char buf[320];
    snprintf(buf, sizeof(buf),
             "gemm_f32_noalloc: m=%lld n=%lld k=%lld needs %llu scratch bytes, above the fixed %llu-byte array "
             "(about 4*(m + n)*k, or 8*(m + n)*k with IPUC_GEMM_F32_SPLIT_TF32, <= 64 MiB); use ipuc_gemm_f32 "
             "with a workspace",
             (long long)m, (long long)n, (long long)k, (unsigned long long)need,
             (unsigned long long)ipuc::kNoAllocScratchBytes);
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, buf);
  }
  void *scratch = nullptr;
  if (need > 0) {
    const ipuc_status st = ipuc::scratch_address(&scratch);
    if (st != IPUC_OK) return st;
  }
  return ipuc::gemm_f32_launch(c, a, b, m, n, k, lda, ldb, ldc, flags, scratch, ipuc::kNoAllocScratchBytes, stream);
}
