// FP32 GEMM: the B200 counterpart of the reference's gemm_f32_64_amp tile
// kernels (device/gemm_f32_64_amp.S:129-385, f32 multiply, f32 accumulate).
//
// fp32 accuracy on the tensor cores by three-pass TF32 splitting: every
// operand x = hi + lo with hi = tf32(x) and lo = tf32(x - hi), and
//   A.B ~= A_hi.B_hi + A_hi.B_lo + A_lo.B_hi
// (the dropped lo.lo term is ~2^-22 relative), accumulated in fp32 in TMEM.
// The tensor core's fp32 accumulation loses precision over long chains of
// MMAs into one accumulator, so each tile's K loop runs in chunks of 256:
// every chunk accumulates into a fresh TMEM buffer (two, ping-ponged) and the
// epilogue warps sum the chunk partials in fp32 registers.
// A prepass kernel writes the hi/lo planes of A and of B (transposed to
// K-major when B is row-major [k x n]) into the caller's workspace; the main
// kernel is the same warp-specialised persistent tcgen05
// pipeline as the FP16 GEMM (TMA producer / single-thread MMA issuer /
// 4 epilogue warps, double-buffered 128x256 accumulators) issuing
// kind::tf32 MMAs, three per 8-wide k step.
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <mutex>

namespace ipuc {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 32, STAGES = 2;
constexpr int A_BYTES = BM * BK * 4;  // 16 KB per plane
constexpr int B_BYTES = BN * BK * 4;  // 32 KB per plane
constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;  // 96 KB
constexpr int TMEM_COLS = 2 * BN;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int GROUP_M = 16;
constexpr int KC = 8;            // k-blocks (of 32) per TMEM accumulation chunk
constexpr int EPI_THREADS = 256; // 8 epilogue warps
constexpr int NUM_THREADS = 64 + EPI_THREADS;

// Round to TF32 (10 explicit mantissa bits), nearest, ties away from zero.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi/lo planes of a row-major [rows x cols] matrix with leading dimension ld
// into dense [rows x cols] planes.
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

struct Gemm32Params {
  float *c;
  int64_t m, n, k;
  int64_t ldc;
  int32_t tiles_m, tiles_n, k_blocks;
  int64_t num_tiles;
  uint32_t flags;
  uint32_t *err;
};

__device__ __forceinline__ void tile_coords(const Gemm32Params &p, int64_t t, int &mt, int &nt) {
  const int64_t in_group = (int64_t)GROUP_M * p.tiles_n;
  const int64_t g = t / in_group;
  const int first = (int)(g * GROUP_M);
  const int gs = min(p.tiles_m - first, GROUP_M);
  const int64_t w = t % in_group;
  mt = first + (int)(w % gs);
  nt = (int)(w / gs);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
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
        record_device_error(p.err, ERR_KERNEL_GEMM_TF32 | ERR_SITE_PRODUCER);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(BM, BN, /*tf32*/ 2, false, false);
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
            for (int k = 0; k < BK / 8; ++k) {
              const uint64_t dah = make_smem_desc(ah + k * 32, 16, 1024, kSwizzle128B);
              const uint64_t dal = make_smem_desc(al + k * 32, 16, 1024, kSwizzle128B);
              const uint64_t dbh = make_smem_desc(bh + k * 32, 16, 1024, kSwizzle128B);
              const uint64_t dbl = make_smem_desc(bl + k * 32, 16, 1024, kSwizzle128B);
              // Small terms first, then the dominant hi.hi product.
              mma_tf32_ss(d_tmem, dal, dbh, idesc, (kb != c * KC || k != 0) ? 1u : 0u);
              mma_tf32_ss(d_tmem, dah, dbl, idesc, 1u);
              mma_tf32_ss(d_tmem, dah, dbh, idesc, 1u);
            }
            mma_commit(&empty[s]);
          }
          if (!ok) break;
          mma_commit(&acc_full[buf]);
        }
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_TF32 | ERR_SITE_MMA);
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
      if (row < p.m) {
        float *cp = p.c + row * p.ldc + col_base;
        if (vec_ok && col_base + BN / 2 <= p.n) {
          float4 *c4 = reinterpret_cast<float4 *>(cp);
#pragma unroll
          for (int j = 0; j < BN / 8; ++j) {
            float4 v = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
            if (accumulate) {
              const float4 o = c4[j];
              v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
            }
            c4[j] = v;
          }
        } else {
#pragma unroll
          for (int j = 0; j < BN / 2; ++j) {
            if (col_base + j < p.n) {
              float x = acc[j];
              if (accumulate) x += cp[j];
              cp[j] = x;
            }
          }
        }
      }
    }
    if (!ok) {
      record_device_error(p.err, ERR_KERNEL_GEMM_TF32 | ERR_SITE_EPILOGUE);
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

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_tf32x3_pair_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
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
  const int chunks = (p.k_blocks + KC - 1) / KC;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t t = pair; t < p.num_tiles && ok; t += pairs) {
        int mt, nt;
        tile_coords(p, t, mt, nt);  // mt counts 256-row pair tiles
        const int32_t arow = mt * PAIR_BM + (int32_t)rank * BM, brow = nt * BN + (int32_t)rank * (BN / 2);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
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
        record_device_error(p.err, ERR_KERNEL_GEMM_TF32 | ERR_SITE_PRODUCER);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = make_idesc(PAIR_BM, BN, /*tf32*/ 2, false, false);
      // Descriptors built once; stages and k-steps add offsets in 16-byte units.
      const uint64_t d0 = make_smem_desc(smem_u32(smem), 16, 1024, kSwizzle128B);
      uint32_t it = 0, g = 0;
      bool ok = true;
      for (int64_t t = pair; t < p.num_tiles && ok; t += pairs) {
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
            for (int k = 0; k < BK / 8; ++k) {
              const uint64_t o = (uint64_t)((k * 32) >> 4);
              // Small terms first, then the dominant hi.hi product.
              mma_tf32_ss_pair(d_tmem, dal + o, dbh + o, idesc, (kb != c * KC || k != 0) ? 1u : 0u);
              mma_tf32_ss_pair(d_tmem, dah + o, dbl + o, idesc, 1u);
              mma_tf32_ss_pair(d_tmem, dah + o, dbh + o, idesc, 1u);
            }
            mma_commit_pair(&empty[s], 0x3);
          }
          if (!ok) break;
          mma_commit_pair(&acc_full[buf], 0x3);
        }
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_TF32 | ERR_SITE_MMA);
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
    for (int64_t t = pair; t < p.num_tiles && ok; t += pairs) {
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
        __syncwarp();
        if (lane == 0) mbar_arrive_leader(&acc_empty[buf]);
      }
      if (!ok) break;
      int mt, nt;
      tile_coords(p, t, mt, nt);
      const int64_t row = (int64_t)mt * PAIR_BM + (int64_t)rank * BM + quarter * 32 + lane;
      const int64_t col_base = (int64_t)nt * BN + half * (BN / 2);
      if (row < p.m) {
        float *cp = p.c + row * p.ldc + col_base;
        if (vec_ok && col_base + BN / 2 <= p.n) {
          float4 *c4 = reinterpret_cast<float4 *>(cp);
#pragma unroll
          for (int j = 0; j < BN / 8; ++j) {
            float4 v = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
            if (accumulate) {
              const float4 o = c4[j];
              v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
            }
            c4[j] = v;
          }
        } else {
#pragma unroll
          for (int j = 0; j < BN / 2; ++j) {
            if (col_base + j < p.n) {
              float x = acc[j];
              if (accumulate) x += cp[j];
              cp[j] = x;
            }
          }
        }
      }
    }
    if (!ok) {
      record_device_error(p.err, ERR_KERNEL_GEMM_TF32 | ERR_SITE_EPILOGUE);
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

}  // namespace

// Workspace: A_hi, A_lo [m x k] and B_hi, B_lo (B's shape), dense fp32.
uint64_t gemm_f32_workspace(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  return 2 * round256((uint64_t)m * k * 4) + 2 * round256((uint64_t)k * n * 4);
}

ipuc_status gemm_f32_launch(float *c, const float *a, const float *b, int64_t m, int64_t n, int64_t k, int64_t lda,
                            int64_t ldb, int64_t ldc, uint32_t flags, void *workspace, uint64_t workspace_bytes,
                            cudaStream_t stream) {
  IPUC_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "gemm_f32: negative extent");
  IPUC_CHECK_ARG((flags & ~(uint32_t)(IPUC_GEMM_ACCUMULATE | IPUC_GEMM_B_TRANSPOSED)) == 0,
                 "gemm_f32: only IPUC_GEMM_ACCUMULATE and IPUC_GEMM_B_TRANSPOSED apply");
  if (m == 0 || n == 0) return IPUC_OK;
  IPUC_CHECK_ARG(k > 0, "gemm_f32: k must be positive");
  IPUC_CHECK_ARG(a && b && c, "gemm_f32: null pointer");
  const bool bt = (flags & IPUC_GEMM_B_TRANSPOSED) != 0;
  IPUC_CHECK_ARG(lda >= k && ldc >= n && ldb >= (bt ? k : n), "gemm_f32: leading dimension too small");
  IPUC_CHECK_ALIGN(aligned(a, 16) && aligned(b, 16) && aligned(c, 16), "gemm_f32: pointers must be 16-byte aligned");
  IPUC_CHECK_ALIGN(lda % 4 == 0 && ldb % 4 == 0 && k % 4 == 0 && n % 4 == 0,
                   "gemm_f32: lda, ldb, k and n must be multiples of 4 elements");
  IPUC_CHECK_ARG(m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), "gemm_f32: extent too large");
  const uint64_t need = gemm_f32_workspace(m, n, k);
  IPUC_CHECK_ARG(workspace != nullptr && workspace_bytes >= need,
                 "gemm_f32: workspace smaller than ipuc_gemm_f32_workspace_bytes()");
  IPUC_CHECK_ALIGN(aligned(workspace, 256), "gemm_f32: workspace must be 256-byte aligned");
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  float *ah = reinterpret_cast<float *>(ws);
  float *al = reinterpret_cast<float *>(ws + round256((uint64_t)m * k * 4));
  float *bh = reinterpret_cast<float *>(ws + 2 * round256((uint64_t)m * k * 4));
  float *bl = reinterpret_cast<float *>(ws + 2 * round256((uint64_t)m * k * 4) + round256((uint64_t)k * n * 4));
  const int64_t brows = bt ? n : k, bcols = bt ? k : n;
  const int cap = sm_count() * 8;
  auto grid_of = [&](int64_t elems) {
    int64_t g = (elems / 4 + 255) / 256;
    return (unsigned)(g < cap ? (g < 1 ? 1 : g) : cap);
  };
  split_tf32_kernel<<<grid_of(m * k), 256, 0, stream>>>(a, m, k, lda, ah, al);
  if (bt) {
    split_tf32_kernel<<<grid_of(brows * bcols), 256, 0, stream>>>(b, brows, bcols, ldb, bh, bl);
  } else {
    const int64_t tiles = ((k + 63) / 64) * ((n + 63) / 64);
    const unsigned g = (unsigned)(tiles < cap ? tiles : cap);
    split_tf32_transpose_kernel<<<g, 256, 0, stream>>>(b, k, n, ldb, bh, bl);
  }
  ipuc_status st = check_launch("split_tf32_kernel");
  if (st != IPUC_OK) return st;

  CUtensorMap tah, tal, tbh, tbl;
  const auto f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if ((st = make_map_3d(&tah, f32, 4, ah, k, m, 1, k, 0, BK, BM)) != IPUC_OK) return st;
  if ((st = make_map_3d(&tal, f32, 4, al, k, m, 1, k, 0, BK, BM)) != IPUC_OK) return st;
  // Both B layouts arrive as dense K-major [n x k] planes.
  if ((st = make_map_3d(&tbh, f32, 4, bh, k, n, 1, k, 0, BK, BN)) != IPUC_OK) return st;
  if ((st = make_map_3d(&tbl, f32, 4, bl, k, n, 1, k, 0, BK, BN)) != IPUC_OK) return st;
  Gemm32Params p;
  p.c = c;
  p.m = m; p.n = n; p.k = k;
  p.ldc = ldc;
  p.tiles_n = (int32_t)((n + BN - 1) / BN);
  p.k_blocks = (int32_t)((k + BK - 1) / BK);
  p.flags = flags;
  p.err = device_error_word();
  const int sms = sm_count();
  const int64_t pair_tiles = ((m + PAIR_BM - 1) / PAIR_BM) * (int64_t)p.tiles_n;
  if (m > BM && sms >= 2 && pair_tiles >= sms / 2) {
    // CTA pairs (at least one full wave of 256x256 tiles; below that the
    // single-CTA kernel spreads the work over more SMs): A boxes of 128 rows
    // per CTA, B boxes of 128 rows (half of BN).
    CUtensorMap pbh, pbl;
    if ((st = make_map_3d(&pbh, f32, 4, bh, k, n, 1, k, 0, BK, BN / 2)) != IPUC_OK) return st;
    if ((st = make_map_3d(&pbl, f32, 4, bl, k, n, 1, k, 0, BK, BN / 2)) != IPUC_OK) return st;
    p.tiles_m = (int32_t)((m + PAIR_BM - 1) / PAIR_BM);
    p.num_tiles = (int64_t)p.tiles_m * p.tiles_n;
    const int64_t pairs = p.num_tiles < sms / 2 ? p.num_tiles : sms / 2;
    IPUC_CUDA(cudaFuncSetAttribute(gemm_tf32x3_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES));
    gemm_tf32x3_pair_kernel<<<(unsigned)(2 * pairs), NUM_THREADS, P_SMEM_BYTES, stream>>>(tah, tal, pbh, pbl, p);
    return check_launch("gemm_tf32x3_pair_kernel");
  }
  p.tiles_m = (int32_t)((m + BM - 1) / BM);
  p.num_tiles = (int64_t)p.tiles_m * p.tiles_n;
  const int grid = (int)(p.num_tiles < sms ? p.num_tiles : sms);
  IPUC_CUDA(cudaFuncSetAttribute(gemm_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  gemm_tf32x3_kernel<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(tah, tal, tbh, tbl, p);
  return check_launch("gemm_tf32x3_kernel");
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
// hi/lo TF32 split planes placed in a fixed file-scope device array instead
// of a caller-provided workspace.
//
// The array is a device symbol, so on the host its name is only a stand-in:
// its device address is resolved once per device with cudaGetSymbolAddress
// (during the first call on that device, with that device current) and cached.
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
void *g_scratch_ptr[64] = {};

ipuc_status scratch_address(void **out) {
  int dev = 0;
  IPUC_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(IPUC_ERR_UNSUPPORTED, "gemm_f32_noalloc: device index above 63");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_gemm_f32_scratch);
    if (err != cudaSuccess) return cuda_fail(err, "gemm_f32_noalloc: cudaGetSymbolAddress(scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return IPUC_OK;
}

}  // namespace
}  // namespace ipuc

extern "C" ipuc_status ipuc_gemm_f32_noalloc(float *c, const float *a, const float *b, int64_t m, int64_t n,
                                             int64_t k, int64_t lda, int64_t ldb, int64_t ldc, uint32_t flags,
                                             ipuc_stream stream) {
  const uint64_t need = ipuc::gemm_f32_workspace(m, n, k);
  if (need > ipuc::kNoAllocScratchBytes) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "gemm_f32_noalloc: m=%lld n=%lld k=%lld needs %llu scratch bytes, above the fixed %llu-byte array "
             "(2*4*(m*k + k*n) <= 64 MiB); use ipuc_gemm_f32 with a workspace",
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
