// FP16 GEMM on the 5th-generation tensor cores: the B200 counterpart of the
// reference's gemm_f16_amp tile kernels (device/gemm_f16_amp.S:186-440; spec
// TileKernelSpec::Gemm, crates/ipu-codegen/src/operator.rs:59-66).
//
// Design (one persistent CTA per SM, warp-specialised):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [64 x 256] per
//               k-block into a 4-stage shared-memory ring (128-byte swizzle).
//   warp 1      MMA issuer: allocates 512 TMEM columns (two 128x256 f32
//               accumulators), issues tcgen05.mma M=128 N=256 K=16 from one
//               thread, commits stage releases and accumulator-ready signals.
//   warps 2-5   epilogue: tcgen05.ld the accumulator (each warp owns its
//               32-lane TMEM quarter), optional accumulate with C, rounding,
//               fused tanh-GELU (f16x2, as the reference kernel), f16 or f32 stores.  Double-buffered TMEM lets
//               the epilogue of tile i overlap the MMAs of tile i+1.
// The whole K loop accumulates in TMEM (fp32), so the reference's f16 partial
// round trip between 64-wide K blocks (gemm_f16_amp.S:363-437) disappears.
// Every mbarrier wait is bounded; on timeout the kernel records an error word
// and all roles drain to the teardown (no trap).
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace ipuc {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;          // 16 KB
constexpr int B_BYTES = BN * BK * 2;          // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;             // 512
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int GROUP_M = 16;

struct GemmParams {
  void *c;
  const void *add;          // what IPUC_GEMM_ACCUMULATE adds: C itself, or a separate addend
  int64_t ld_add, stride_add;
  int64_t m, n, k, batch;
  int64_t ldc, stride_c;
  int32_t tiles_m, tiles_n, k_blocks;
  int64_t num_tiles;
  uint32_t flags;
  uint32_t *err;
};

__device__ __forceinline__ void tile_coords(const GemmParams &p, int64_t t, int &b, int &mt, int &nt) {
  const int64_t per = (int64_t)p.tiles_m * p.tiles_n;
  b = (int)(t / per);
  const int64_t r = t % per;
  const int64_t in_group = (int64_t)GROUP_M * p.tiles_n;
  const int64_t g = r / in_group;
  const int first = (int)(g * GROUP_M);
  const int gs = min(p.tiles_m - first, GROUP_M);
  const int64_t w = r % in_group;
  mt = first + (int)(w % gs);
  nt = (int)(w / gs);
}

// Epilogue for one 32-column chunk of one accumulator row: optional
// accumulate with C, rounding to C's precision, fused GELU, vector stores.
__device__ __forceinline__ void store_chunk(const GemmParams &p, int b, int64_t row, int64_t col0,
                                            const uint32_t (&r)[32], bool vec_ok, bool out_f32, bool accumulate,
                                            bool gelu) {
  const bool full_chunk = vec_ok && (col0 + 32 <= p.n);
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (out_f32) {
    float *cp = static_cast<float *>(p.c) + b * p.stride_c + row * p.ldc + col0;
    const float *ap = static_cast<const float *>(p.add) + b * p.stride_add + row * p.ld_add + col0;
    if (full_chunk) {
      float4 *c4 = reinterpret_cast<float4 *>(cp);
      if (accumulate) {
        const float4 *a4 = reinterpret_cast<const float4 *>(ap);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 o = a4[j];
          v[4 * j] += o.x; v[4 * j + 1] += o.y; v[4 * j + 2] += o.z; v[4 * j + 3] += o.w;
        }
      }
      if (gelu) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = gelu_f32(v[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) c4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
      for (int j = 0; j < 32 && col0 + j < p.n; ++j) {
        float x = v[j];
        if (accumulate) x += ap[j];
        if (gelu) x = gelu_f32(x);
        cp[j] = x;
      }
    }
  } else {
    uint16_t *cp = static_cast<uint16_t *>(p.c) + b * p.stride_c + row * p.ldc + col0;
    const uint16_t *ap = static_cast<const uint16_t *>(p.add) + b * p.stride_add + row * p.ld_add + col0;
    if (full_chunk) {
      uint4 *c4 = reinterpret_cast<uint4 *>(cp);
      if (accumulate) {
        const uint4 *a4 = reinterpret_cast<const uint4 *>(ap);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 o = a4[j];
          const uint16_t *h = reinterpret_cast<const uint16_t *>(&o);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[8 * j + e] += h2f(h[e]);
        }
      }
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        packed[j] = pack_h2(v[2 * j], v[2 * j + 1]);  // the GEMM result rounded to f16
        if (gelu) packed[j] = gelu_h2(packed[j]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        c4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
    } else {
      for (int j = 0; j < 32 && col0 + j < p.n; ++j) {
        float x = v[j];
        if (accumulate) x += h2f(ap[j]);
        uint32_t h = f2h(x);
        if (gelu) h = gelu_h2(h) & 0xffffu;
        cp[j] = (uint16_t)h;
      }
    }
  }
}

template <bool kAKMajor, bool kBKMajor>
__global__ void __launch_bounds__(192, 1)
    gemm_f16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *tmem_full = empty + STAGES;
  uint64_t *tmem_empty = tmem_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tmem_empty + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int b, mt, nt;
        tile_coords(p, t, b, mt, nt);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *a_s = smem + s * STAGE_BYTES;
          uint8_t *b_s = a_s + A_BYTES;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          if (kAKMajor) {
            tma_load_3d(a_s, &tmA, &full[s], kb * BK, mt * BM, b);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_3d(a_s + j * 8192, &tmA, &full[s], mt * BM + j * 64, kb * BK, b);
          }
          if (kBKMajor) {
            tma_load_3d(b_s, &tmB, &full[s], kb * BK, nt * BN, b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_3d(b_s + j * 8192, &tmB, &full[s], nt * BN + j * 64, kb * BK, b);
          }
        }
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F16 | ERR_SITE_PRODUCER);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(BM, BN, /*f16*/ 0, !kAKMajor, !kBKMajor);
      uint32_t it = 0, local = 0;
      bool ok = true;
      const uint64_t a_desc0 = make_smem_desc(smem_u32(smem), kAKMajor ? 16 : 8192, 1024, kSwizzle128B);
      const uint64_t b_desc0 = make_smem_desc(smem_u32(smem) + A_BYTES, kBKMajor ? 16 : 8192, 1024, kSwizzle128B);
      for (int64_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++local) {
        const uint32_t buf = local & 1u, use = local >> 1;
        if (!mbar_wait_bounded(&tmem_empty[buf], (use & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Stage descriptors = base + stage offset; k-steps add compile-time
          // offsets (16-byte units), keeping the issuing thread ahead of the pipe.
          const uint64_t ad = a_desc0 + (uint64_t)(s * (STAGE_BYTES >> 4));
          const uint64_t bd = b_desc0 + (uint64_t)(s * (STAGE_BYTES >> 4));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = ad + (uint64_t)((kAKMajor ? k * 32 : k * 2048) >> 4);
            const uint64_t bdesc = bd + (uint64_t)((kBKMajor ? k * 32 : k * 2048) >> 4);
            mma_f16_ss(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&tmem_full[buf]);
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F16 | ERR_SITE_MMA);
        *abort_flag = 1;
      }
    }
  } else {
    // Epilogue: 128 threads; warp w owns TMEM lanes [32*(w%4), 32*(w%4)+32).
    const int quarter = warp & 3;
    const bool out_f32 = (p.flags & IPUC_GEMM_OUT_F32) != 0;
    const bool accumulate = (p.flags & IPUC_GEMM_ACCUMULATE) != 0;
    const bool gelu = (p.flags & IPUC_GEMM_EPILOGUE_GELU) != 0;
    const bool vec_ok = (p.ldc % 8 == 0) && (p.stride_c % 8 == 0) && (p.ld_add % 8 == 0) && (p.stride_add % 8 == 0);
    uint32_t local = 0;
    for (int64_t t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++local) {
      const uint32_t buf = local & 1u, use = local >> 1;
      if (!mbar_wait_bounded(&tmem_full[buf], use & 1u, abort_flag)) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F16 | ERR_SITE_EPILOGUE);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      int b, mt, nt;
      tile_coords(p, t, b, mt, nt);
      const int64_t row = (int64_t)mt * BM + quarter * 32 + lane;
      const bool row_ok = row < p.m;
      for (int chunk = 0; chunk < BN / 32; ++chunk) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + buf * BN + chunk * 32 + ((uint32_t)(quarter * 32) << 16), r);
        tmem_wait_ld(r);
        const int64_t col0 = (int64_t)nt * BN + chunk * 32;
        if (!row_ok || col0 >= p.n) continue;
        store_chunk(p, b, row, col0, r, vec_ok, out_f32, accumulate, gelu);
      }
      tc_fence_before();
      mbar_arrive(&tmem_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// CTA-pair variant (cluster of 2, tcgen05 cta_group::2).  A pair computes a
// 256 x 256 tile: each CTA loads its own 128 rows of A and its own 128 columns
// of B (non-multicast TMA, completion counted on the leader's barrier), the
// leader issues M=256 N=256 MMAs that read both CTAs' shared memory, and each
// CTA's TMEM receives its 128 accumulator rows.  Per CTA this halves the B
// traffic through shared memory compared with the single-CTA kernel, which is
// what keeps the tensor pipe fed (TMA fill + MMA operand reads stay under the
// shared-memory bandwidth).
constexpr int PB_N = 128;                      // B columns per CTA
constexpr int P_A_BYTES = BM * BK * 2;         // 16 KB
constexpr int P_B_BYTES = PB_N * BK * 2;       // 16 KB
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_STAGES = 6;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256;
constexpr int PAIR_BM = 2 * BM;                // 256 rows per pair tile

template <bool kAKMajor, bool kBKMajor>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_f16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + P_STAGES * P_STAGE_BYTES);
  uint64_t *empty = full + P_STAGES;
  uint64_t *tmem_full = empty + P_STAGES;
  uint64_t *tmem_empty = tmem_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tmem_empty + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);   // leader: its own arrive_expect_tx; peers only add bytes
      mbar_init(&empty[s], 1);  // one multicast commit per stage use
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 8);  // lane 0 of the 4 epilogue warps of both CTAs
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t t = pair; t < p.num_tiles && ok; t += pairs) {
        int b, mt, nt;
        tile_coords(p, t, b, mt, nt);  // mt counts 256-row pair tiles
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % P_STAGES;
          const uint32_t ph = (it / P_STAGES) & 1u;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *a_s = smem + s * P_STAGE_BYTES;
          uint8_t *b_s = a_s + P_A_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * P_STAGE_BYTES);
          if (kAKMajor) {
            tma_load_3d_pair(a_s, &tmA, &full[s], kb * BK, mt * PAIR_BM + (int)rank * BM, b);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_3d_pair(a_s + j * 8192, &tmA, &full[s], mt * PAIR_BM + (int)rank * BM + j * 64, kb * BK, b);
          }
          if (kBKMajor) {
            tma_load_3d_pair(b_s, &tmB, &full[s], kb * BK, nt * BN + (int)rank * PB_N, b);
          } else {
#pragma unroll
            for (int j = 0; j < PB_N / 64; ++j)
              tma_load_3d_pair(b_s + j * 8192, &tmB, &full[s], nt * BN + (int)rank * PB_N + j * 64, kb * BK, b);
          }
        }
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F16 | ERR_SITE_PRODUCER);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = make_idesc(PAIR_BM, BN, /*f16*/ 0, !kAKMajor, !kBKMajor);
      uint32_t it = 0, local = 0;
      bool ok = true;
      const uint64_t a_desc0 = make_smem_desc(smem_u32(smem), kAKMajor ? 16 : 8192, 1024, kSwizzle128B);
      const uint64_t b_desc0 = make_smem_desc(smem_u32(smem) + P_A_BYTES, kBKMajor ? 16 : 8192, 1024, kSwizzle128B);
      for (int64_t t = pair; t < p.num_tiles && ok; t += pairs, ++local) {
        const uint32_t buf = local & 1u, use = local >> 1;
        if (!mbar_wait_bounded(&tmem_empty[buf], (use & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % P_STAGES;
          const uint32_t ph = (it / P_STAGES) & 1u;
          if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Stage descriptors = base + stage offset; k-steps add compile-time
          // offsets (16-byte units), keeping the issuing thread ahead of the pipe.
          const uint64_t ad = a_desc0 + (uint64_t)(s * (P_STAGE_BYTES >> 4));
          const uint64_t bd = b_desc0 + (uint64_t)(s * (P_STAGE_BYTES >> 4));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = ad + (uint64_t)((kAKMajor ? k * 32 : k * 2048) >> 4);
            const uint64_t bdesc = bd + (uint64_t)((kBKMajor ? k * 32 : k * 2048) >> 4);
            mma_f16_ss_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit_pair(&empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair(&tmem_full[buf], 0x3);
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F16 | ERR_SITE_MMA);
        *abort_flag = 1;
      }
    }
  } else {
    const int quarter = warp & 3;
    const bool out_f32 = (p.flags & IPUC_GEMM_OUT_F32) != 0;
    const bool accumulate = (p.flags & IPUC_GEMM_ACCUMULATE) != 0;
    const bool gelu = (p.flags & IPUC_GEMM_EPILOGUE_GELU) != 0;
    const bool vec_ok = (p.ldc % 8 == 0) && (p.stride_c % 8 == 0) && (p.ld_add % 8 == 0) && (p.stride_add % 8 == 0);
    uint32_t local = 0;
    for (int64_t t = pair; t < p.num_tiles; t += pairs, ++local) {
      const uint32_t buf = local & 1u, use = local >> 1;
      if (!mbar_wait_bounded(&tmem_full[buf], use & 1u, abort_flag)) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F16 | ERR_SITE_EPILOGUE);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      int b, mt, nt;
      tile_coords(p, t, b, mt, nt);
      const int64_t row = (int64_t)mt * PAIR_BM + (int64_t)rank * BM + quarter * 32 + lane;
      const bool row_ok = row < p.m;
      for (int chunk = 0; chunk < BN / 32; ++chunk) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + buf * BN + chunk * 32 + ((uint32_t)(quarter * 32) << 16), r);
        tmem_wait_ld(r);
        const int64_t col0 = (int64_t)nt * BN + chunk * 32;
        if (!row_ok || col0 >= p.n) continue;
        store_chunk(p, b, row, col0, r, vec_ok, out_f32, accumulate, gelu);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(&tmem_empty[buf]);
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

// ---------------------------------------------------------------------------
// Latency form for small GEMMs (config 1, 256^3: 8 tiles of 128 x 64): one
// 128 x 64 tile per CTA over a 4-stage K ring, a 64-column TMEM accumulator,
// and programmatic dependent launch, so that the CTA's prologue (barrier
// setup, TMEM allocation, descriptor prefetch) overlaps the previous kernel's
// tail and only the loads wait for it.
constexpr int SBN = 64, S_STAGES = 4;
constexpr int S_A_BYTES = BM * BK * 2;   // 16 KB
constexpr int S_B_BYTES = SBN * BK * 2;  // 8 KB
constexpr int S_STAGE_BYTES = S_A_BYTES + S_B_BYTES;
constexpr int S_SMEM_BYTES = S_STAGES * S_STAGE_BYTES + 1024 + 256;

template <bool kAKMajor, bool kBKMajor>
__global__ void __launch_bounds__(192, 1)
    gemm_f16_small_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S_STAGES * S_STAGE_BYTES);
  uint64_t *empty = full + S_STAGES;
  uint64_t *done = empty + S_STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, SBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  int b, mt, nt;
  {
    const int64_t per = (int64_t)p.tiles_m * p.tiles_n;
    b = (int)(blockIdx.x / per);
    const int64_t r = blockIdx.x % per;
    mt = (int)(r % p.tiles_m);
    nt = (int)(r / p.tiles_m);
  }
  griddep_wait();  // inputs (and C) belong to the previous kernel until here
  griddep_launch_dependents();
  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      for (int kb = 0; kb < p.k_blocks && ok; ++kb) {
        const int s = kb % S_STAGES;
        if (!mbar_wait_bounded(&empty[s], ((kb / S_STAGES) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t *a_s = smem + s * S_STAGE_BYTES, *b_s = a_s + S_A_BYTES;
        mbar_arrive_expect_tx(&full[s], S_STAGE_BYTES);
        if (kAKMajor) {
          tma_load_3d(a_s, &tmA, &full[s], kb * BK, mt * BM, b);
        } else {
#pragma unroll
          for (int j = 0; j < BM / 64; ++j) tma_load_3d(a_s + j * 8192, &tmA, &full[s], mt * BM + j * 64, kb * BK, b);
        }
        if (kBKMajor) tma_load_3d(b_s, &tmB, &full[s], kb * BK, nt * SBN, b);
        else tma_load_3d(b_s, &tmB, &full[s], nt * SBN, kb * BK, b);
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F16 | ERR_SITE_PRODUCER);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(BM, SBN, /*f16*/ 0, !kAKMajor, !kBKMajor);
      const uint64_t a_desc0 = make_smem_desc(smem_u32(smem), kAKMajor ? 16 : 8192, 1024, kSwizzle128B);
      const uint64_t b_desc0 = make_smem_desc(smem_u32(smem) + S_A_BYTES, kBKMajor ? 16 : 8192, 1024, kSwizzle128B);
      bool ok = true;
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        const int s = kb % S_STAGES;
        if (!mbar_wait_bounded(&full[s], (kb / S_STAGES) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = a_desc0 + (uint64_t)(s * (S_STAGE_BYTES >> 4));
        const uint64_t bd = b_desc0 + (uint64_t)(s * (S_STAGE_BYTES >> 4));
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          mma_f16_ss(tmem_base, ad + (uint64_t)((kAKMajor ? k * 32 : k * 2048) >> 4),
                     bd + (uint64_t)((kBKMajor ? k * 32 : k * 2048) >> 4), idesc, (kb | k) != 0 ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      if (ok) mma_commit(done);
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_GEMM_F16 | ERR_SITE_MMA);
        *abort_flag = 1;
      }
    }
  } else {
    const int quarter = warp & 3;
    const bool out_f32 = (p.flags & IPUC_GEMM_OUT_F32) != 0;
    const bool accumulate = (p.flags & IPUC_GEMM_ACCUMULATE) != 0;
    const bool gelu = (p.flags & IPUC_GEMM_EPILOGUE_GELU) != 0;
    const bool vec_ok = (p.ldc % 8 == 0) && (p.stride_c % 8 == 0) && (p.ld_add % 8 == 0) && (p.stride_add % 8 == 0);
    if (!mbar_wait_bounded(done, 0, abort_flag)) {
      record_device_error(p.err, ERR_KERNEL_GEMM_F16 | ERR_SITE_EPILOGUE);
      *abort_flag = 1;
    } else {
      tc_fence_after();
      const int64_t row = (int64_t)mt * BM + quarter * 32 + lane;
#pragma unroll
      for (int chunk = 0; chunk < SBN / 32; ++chunk) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + chunk * 32 + ((uint32_t)(quarter * 32) << 16), r);
        tmem_wait_ld(r);
        const int64_t col0 = (int64_t)nt * SBN + chunk * 32;
        if (row < p.m && col0 < p.n) store_chunk(p, b, row, col0, r, vec_ok, out_f32, accumulate, gelu);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, SBN);
  }
}

ipuc_status launch_gemm_f16(void *c, const void *a, const void *b, int64_t batch, int64_t m, int64_t n, int64_t k,
                            int64_t lda, int64_t ldb, int64_t ldc, int64_t sa, int64_t sb, int64_t sc,
                            uint32_t flags, cudaStream_t stream, const void *addend = nullptr, int64_t ld_add = 0) {
  IPUC_CHECK_ARG(m >= 0 && n >= 0 && k >= 0 && batch >= 0, "gemm_f16: negative extent");
  IPUC_CHECK_ARG((flags & ~(uint32_t)(IPUC_GEMM_ACCUMULATE | IPUC_GEMM_B_TRANSPOSED | IPUC_GEMM_OUT_F32 |
                                       IPUC_GEMM_EPILOGUE_GELU | IPUC_GEMM_A_TRANSPOSED)) == 0,
                 "gemm_f16: unknown flag");
  if (m == 0 || n == 0 || batch == 0) return IPUC_OK;
  IPUC_CHECK_ARG(k > 0, "gemm_f16: k must be positive");
  IPUC_CHECK_ARG(a && b && c, "gemm_f16: null pointer");
  const bool bt = (flags & IPUC_GEMM_B_TRANSPOSED) != 0, at = (flags & IPUC_GEMM_A_TRANSPOSED) != 0;
  IPUC_CHECK_ARG(lda >= (at ? m : k) && ldc >= n && ldb >= (bt ? k : n), "gemm_f16: leading dimension too small");
  IPUC_CHECK_ALIGN(aligned(a, 16) && aligned(b, 16) && aligned(c, 16), "gemm_f16: pointers must be 16-byte aligned");
  IPUC_CHECK_ALIGN(lda % 8 == 0 && ldb % 8 == 0 && k % 8 == 0 && (!at || m % 8 == 0),
                   "gemm_f16: lda, ldb and k (m too with IPUC_GEMM_A_TRANSPOSED) must be multiples of 8 elements "
                   "(16-byte TMA rows)");
  IPUC_CHECK_ALIGN(batch == 1 || (sa % 8 == 0 && sb % 8 == 0), "gemm_f16: batch strides must be multiples of 8");
  IPUC_CHECK_ARG(m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31) && batch < (1ll << 31), "gemm_f16: extent too large");
  if (batch > 1 && (sa == 0 || sb == 0 || sc == 0)) {
    // An operand shared by every batch entry (stride 0): a tensor map cannot
    // repeat a tensor with stride 0.  With K-major A rows, B shared and the
    // batches of A and C back to back, the batch is just more rows of one GEMM;
    // otherwise each entry runs as its own GEMM.
    IPUC_CHECK_ARG(sc != 0, "gemm_f16: batched C needs a nonzero stride");
    const bool add_batched = addend == nullptr;  // the C-accumulate source follows C's stride
    if (sb == 0 && sa != 0 && !at && sa == m * lda && sc == m * ldc && add_batched)
      return launch_gemm_f16(c, a, b, 1, m * batch, n, k, lda, ldb, ldc, 0, 0, 0, flags, stream);
    const size_t esz = (flags & IPUC_GEMM_OUT_F32) ? 4 : 2;
    for (int64_t i = 0; i < batch; ++i) {
      const ipuc_status st = launch_gemm_f16(static_cast<uint8_t *>(c) + i * sc * esz,
                                             static_cast<const uint16_t *>(a) + i * sa,
                                             static_cast<const uint16_t *>(b) + i * sb, 1, m, n, k, lda, ldb, ldc, 0,
                                             0, 0, flags, stream, addend, ld_add);
      if (st != IPUC_OK) return st;
    }
    return IPUC_OK;
  }
  CUtensorMap ta, tb;
  // A: K-major [m x k] tiles of 128 x 64, or with IPUC_GEMM_A_TRANSPOSED
  // M-major ([k x m] rows, 64-row boxes of 64 k).
  auto map_a = [&](CUtensorMap *map) {
    return at ? make_map_3d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, m, k, batch, lda, batch > 1 ? sa : 0, 64, BK)
              : make_map_3d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, k, m, batch, lda, batch > 1 ? sa : 0, BK, BM);
  };
  ipuc_status st = map_a(&ta);
  if (st != IPUC_OK) return st;
  if (bt) st = make_map_3d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, k, n, batch, ldb, batch > 1 ? sb : 0, BK, BN);
  else st = make_map_3d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, n, k, batch, ldb, batch > 1 ? sb : 0, 64, BK);
  if (st != IPUC_OK) return st;
  GemmParams p;
  p.c = c;
  p.add = addend ? addend : c;
  p.ld_add = addend ? ld_add : ldc;
  p.stride_add = addend ? 0 : (batch > 1 ? sc : 0);
  p.m = m; p.n = n; p.k = k; p.batch = batch;
  p.ldc = ldc;
  p.stride_c = batch > 1 ? sc : 0;
  p.tiles_n = (int32_t)((n + BN - 1) / BN);
  p.k_blocks = (int32_t)((k + BK - 1) / BK);
  p.flags = flags;
  p.err = device_error_word();
  const int sms = sm_count();
  // Small problems (at most a quarter wave of 128 x 256 tiles): the latency
  // form, 128 x 64 tiles, one per CTA, with programmatic dependent launch.
  const int64_t big_tiles = ((m + BM - 1) / BM) * ((n + BN - 1) / BN) * batch;
  if (4 * big_tiles <= sms) {
    CUtensorMap tbs;
    if (bt) st = make_map_3d(&tbs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, k, n, batch, ldb, batch > 1 ? sb : 0, BK, SBN);
    else st = make_map_3d(&tbs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, n, k, batch, ldb, batch > 1 ? sb : 0, 64, BK);
    if (st != IPUC_OK) return st;
    p.tiles_m = (int32_t)((m + BM - 1) / BM);
    p.tiles_n = (int32_t)((n + SBN - 1) / SBN);
    p.num_tiles = (int64_t)p.tiles_m * p.tiles_n * batch;
    auto go = [&](auto kernel) -> ipuc_status {
      IPUC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S_SMEM_BYTES));
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)p.num_tiles);
      cfg.blockDim = dim3(192);
      cfg.dynamicSmemBytes = S_SMEM_BYTES;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      IPUC_CUDA(cudaLaunchKernelEx(&cfg, kernel, ta, tbs, p));
      return check_launch("gemm_f16_small_kernel");
    };
    if (at) return bt ? go(gemm_f16_small_kernel<false, true>) : go(gemm_f16_small_kernel<false, false>);
    return bt ? go(gemm_f16_small_kernel<true, true>) : go(gemm_f16_small_kernel<true, false>);
  }
  // CTA pairs once there are at least two 128-row tiles of work per pair slot.
  const bool use_pair = m > BM && sms >= 2;
  if (use_pair) {
    p.tiles_m = (int32_t)((m + PAIR_BM - 1) / PAIR_BM);
    p.num_tiles = (int64_t)p.tiles_m * p.tiles_n * batch;
    const int64_t pairs = p.num_tiles < sms / 2 ? p.num_tiles : sms / 2;
    CUtensorMap tap, tbp;
    st = map_a(&tap);
    if (st != IPUC_OK) return st;
    if (bt) st = make_map_3d(&tbp, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, k, n, batch, ldb, batch > 1 ? sb : 0, BK, PB_N);
    else st = make_map_3d(&tbp, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, n, k, batch, ldb, batch > 1 ? sb : 0, 64, BK);
    if (st != IPUC_OK) return st;
    auto go = [&](auto kernel) -> ipuc_status {
      IPUC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES));
      kernel<<<(unsigned)(2 * pairs), 192, P_SMEM_BYTES, stream>>>(tap, tbp, p);
      return check_launch("gemm_f16_pair_kernel");
    };
    if (at) return bt ? go(gemm_f16_pair_kernel<false, true>) : go(gemm_f16_pair_kernel<false, false>);
    return bt ? go(gemm_f16_pair_kernel<true, true>) : go(gemm_f16_pair_kernel<true, false>);
  }
  p.tiles_m = (int32_t)((m + BM - 1) / BM);
  p.num_tiles = (int64_t)p.tiles_m * p.tiles_n * batch;
  const int grid = (int)(p.num_tiles < sms ? p.num_tiles : sms);
  auto go = [&](auto kernel) -> ipuc_status {
    IPUC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    kernel<<<grid, 192, SMEM_BYTES, stream>>>(ta, tb, p);
    return check_launch("gemm_f16_kernel");
  };
  if (at) return bt ? go(gemm_f16_kernel<false, true>) : go(gemm_f16_kernel<false, false>);
  return bt ? go(gemm_f16_kernel<true, true>) : go(gemm_f16_kernel<true, false>);
}

}  // namespace
}  // namespace ipuc

using namespace ipuc;

extern "C" ipuc_status ipuc_gemm_f16(void *c, const void *a, const void *b, int64_t m, int64_t n, int64_t k,
                                     int64_t lda, int64_t ldb, int64_t ldc, uint32_t flags, ipuc_stream stream) {
  return launch_gemm_f16(c, a, b, 1, m, n, k, lda, ldb, ldc, 0, 0, 0, flags, stream);
}

extern "C" ipuc_status ipuc_gemm_f16_addend(void *c, const void *a, const void *b, int64_t m, int64_t n, int64_t k,
                                            int64_t lda, int64_t ldb, int64_t ldc, uint32_t flags,
                                            const void *addend, int64_t ld_addend, ipuc_stream stream) {
  IPUC_CHECK_ARG(addend != nullptr, "gemm_f16_addend: null addend");
  IPUC_CHECK_ARG(ld_addend >= n, "gemm_f16_addend: addend leading dimension too small");
  IPUC_CHECK_ALIGN(aligned(addend, 16), "gemm_f16_addend: addend must be 16-byte aligned");
  return launch_gemm_f16(c, a, b, 1, m, n, k, lda, ldb, ldc, 0, 0, 0, flags | IPUC_GEMM_ACCUMULATE, stream, addend,
                         ld_addend);
}

extern "C" ipuc_status ipuc_gemm_f16_batched(void *c, const void *a, const void *b, int64_t batch, int64_t m,
                                             int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                                             int64_t stride_a, int64_t stride_b, int64_t stride_c, uint32_t flags,
                                             ipuc_stream stream) {
  return launch_gemm_f16(c, a, b, batch, m, n, k, lda, ldb, ldc, stride_a, stride_b, stride_c, flags, stream);
}
