// Fused non-causal flash attention on the tcgen05 tensor cores: the B200
// counterpart of flash_attention_online_f16 (device/flash_attention_online_f16.
// cpp:61-143) and of the reference's four-launches-per-key-block staged loop
// (crates/ipu-codegen/src/low.rs:2272-2510: QK^T GEMM -> softmax -> PV GEMM ->
// merge, with the exact online max/denominator recurrence of
// device/attention_stages_f16.S:803-849).
//
// One CTA owns 256 query rows of one stream as two 128-row tiles (Q0, Q1) and
// streams 128-key K/V tiles through 2-stage TMA rings (K stages are released
// as soon as both tiles' QK^T products finish, V stages after PV).  Warp roles:
//   warp 0      TMA loads (Q once; K_j, V_j per key tile)
//   warp 1      MMA issue: S_t = Q_t K_j^T into TMEM, then O_t += P_t V_j with
//               P_t read straight from TMEM (it aliases S_t as packed f16)
//   warps 2-17  softmax: 8 warps per Q tile, two per TMEM lane quarter, each
//               thread owning 64 of its query row's 128 scores
// The two tiles ping-pong so the tensor core computes one tile's products
// while the other tile's softmax runs.  TMEM: S0 | S1 | O0 | O1 (4 x 128 cols).
// The softmax keeps an fp32 running max and denominator per row; the O rescale
// (the merge stage's acc*e^{m-m'}) is applied only when a row's max grows by
// more than 2^8 in the exponent, which keeps P <= 256 and is exact because
// the final 1/denominator uses the same stale max.
// Head dims up to 128 (multiple of 8) are zero-padded to 128 by the TMA; key
// and query tails are masked.  Every wait is bounded (error word, no trap).
//
// Launch partition: from 512 query rows up, persistent CTA pairs
// (cta_group::2, M = 256 over the pair, each CTA loading half of every K and
// V tile) loop over 512-row units in whole waves: the next unit's Q lands in
// a second Q buffer while the current unit runs, and its first QK^T products
// queue behind the current unit's last PV products while the softmax warps
// store the finished O (the first PV of a unit waits until O is read out);
// a last wave at most half full runs as split clusters
// (kSplit: two CTAs per 256-row unit, each over half the key tiles, merged
// through distributed shared memory).  Q/K/V/O are addressed through 4-D maps
// (head_dim, heads, rows, batch), so the same kernels serve [streams][rows][d]
// tensors (heads = 1) and unsplit [batch][rows][heads * d] projections.
#include <math.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace ipuc {
namespace {

using namespace sm100;

constexpr int TQ = 128;       // query rows per tile
constexpr int TK = 128;       // keys per tile
constexpr int DP = 128;       // padded head dim
constexpr int TILE_BYTES = TQ * DP * 2;   // 32 KB (two 16 KB swizzled halves)
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr int SMEM_BYTES = 6 * TILE_BYTES + 1024 + 256;
constexpr int NUM_THREADS = 576;  // 2 + 16 warps
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units
// The split merge's receive area (2*TQ padded O rows + m and l) must fit in
// the Q/K/V tiles it reuses.
static_assert((2 * TQ * (DP + 4) + 4 * TQ) * 4 <= 6 * TILE_BYTES, "split merge area");

struct AttnParams {
  void *out;
  int64_t matrices, sq, sk, d;
  float scale_log2;  // softmax scale * log2(e)
  int32_t out_f32;
  int32_t key_tiles;
  int32_t heads;      // streams per batch entry: Q/K/V/O are [batch][rows][heads * d] (1: [streams][rows][d])
  int32_t q_units;    // query units per stream: 512-row (pair, split) or 256-row blocks
  int64_t unit_base;  // first unit of this launch (split: first 256-row half-unit)
  int64_t num_units;  // pair launch: units [unit_base, unit_base + num_units), looped over by persistent pairs
  uint32_t *err;
};

// kPair: the kernel runs as 2-CTA clusters issuing cta_group::2 MMAs
// (M = 256 query rows over the pair).  Each CTA then loads only its half of
// every K tile (64 keys) and of every V tile (64 head-dim columns), halving
// per-CTA shared-memory fill and B-operand reads; the leader (rank 0) issues
// all MMAs and both CTAs' softmax warps run as in the single-CTA kernel.
// kSplit: the tail of a pair launch.  Each 2-CTA cluster owns one 256-row
// unit; CTA r runs key tiles [r*ceil(n/2), ...) of it, and CTA 1 hands its
// unnormalised O, running max and row sum to CTA 0 through distributed shared
// memory for the merge (the two-block case of the merge stage's rescale,
// device/attention_stages_f16.S:803-849).  Used when the pair units leave a
// last wave less than half full, so the split halves that wave's length.
template <bool kPair, bool kSplit>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    flash_attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int K_BYTES = kPair ? TILE_BYTES / 2 : TILE_BYTES;   // per-CTA K tile (64 or 128 keys)
  constexpr int K_HALF = K_BYTES / 2;                             // one 64-column head-dim half
  constexpr int V_BYTES = kPair ? TILE_BYTES / 2 : TILE_BYTES;   // per-CTA V tile (64 or 128 D columns)
  constexpr int TX_MULT = kPair ? 2 : 1;                          // leader counts both CTAs' bytes
  // Shared memory: Q buffers (two in the persistent pair kernel, so the next
  // unit's Q lands while this one runs), then the K and V stage rings.
  uint8_t *sQ0 = smem;
  uint8_t *sQ1 = smem + (kPair ? 2 * TILE_BYTES : 0);
  uint8_t *sK = smem + (kPair ? 4 : 2) * TILE_BYTES;  // 2 stages of K_BYTES
  uint8_t *sV = sK + 2 * K_BYTES;                      // 2 stages of V_BYTES
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 6 * TILE_BYTES);
  uint64_t *q_full = bars + 0;   // [2] per Q buffer
  uint64_t *k_full = bars + 2;   // [2]
  uint64_t *v_full = bars + 4;   // [2]
  uint64_t *k_empty = bars + 6;  // [2] K stage free (its QK^T products done)
  uint64_t *s_full = bars + 8;   // [2] per Q tile
  uint64_t *p_ready = bars + 10; // [2] per Q tile
  uint64_t *o_final = bars + 12; // a unit's last PV products done
  uint64_t *v_empty = bars + 13; // [2] V stage free (its PV products done)
  uint64_t *q_empty = bars + 15; // [2] Q buffer free (its unit's QK^T products done)
  uint64_t *o_empty = bars + 17; // [2] per Q tile: the unit's O read out, the next unit may overwrite it
  uint64_t *merge_ready = bars + 19;  // split, CTA 1: CTA 0's tiles are free to receive
  uint64_t *merge_full = bars + 20;   // split, CTA 0: CTA 1's partial has landed
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 21);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  __shared__ float xmax[2][2][TQ], xsum[2][2][TQ];  // [tile][column half][row]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = (kPair || kSplit) ? cluster_ctarank() : 0u;
  const uint32_t prank = kPair ? rank : 0u;  // half of K/V this CTA loads (pair only)
  const bool leader = prank == 0;
  // Units this CTA runs: the persistent pair kernel loops over pair units
  // (512 query rows each); the single and split kernels run one unit per CTA.
  // (unit indices fit 32 bits: streams < 2^24, units per stream < 2^22)
  int32_t u_first, u_step, u_end;
  if (kPair) {
    u_first = (int32_t)p.unit_base + (int32_t)(blockIdx.x >> 1);
    u_step = (int32_t)(gridDim.x >> 1);
    u_end = (int32_t)(p.unit_base + p.num_units);
  } else {
    u_first = (int32_t)p.unit_base + (int32_t)(kSplit ? (blockIdx.x >> 1) : blockIdx.x);
    u_step = 1;
    u_end = u_first + 1;
  }
  struct Unit {
    int64_t stream;
    int32_t q0, s_head, s_batch;
    int j_begin, n_tiles;
  };
  // Key tiles [j_begin, j_begin + n_tiles) of the stream; loop counters below
  // are local (they set stage and phase), key coordinates add j_begin.
  auto decode = [&](int32_t u) {
    Unit w;
    if (kPair) {
      w.stream = u / p.q_units;
      w.q0 = (int32_t)(u % p.q_units) * (4 * TQ) + (int32_t)rank * (2 * TQ);
    } else if (kSplit) {
      const int32_t pu = u >> 1;
      w.stream = pu / p.q_units;
      w.q0 = (int32_t)(pu % p.q_units) * (4 * TQ) + (int32_t)(u & 1) * (2 * TQ);
    } else {
      w.stream = u / p.q_units;
      w.q0 = (int32_t)(u % p.q_units) * (2 * TQ);
    }
    w.s_head = (int32_t)(w.stream % p.heads);
    w.s_batch = (int32_t)(w.stream / p.heads);
    const int split_half = (p.key_tiles + 1) / 2;
    w.j_begin = kSplit ? (int)rank * split_half : 0;
    w.n_tiles = kSplit ? min(p.key_tiles - w.j_begin, split_half) : p.key_tiles;
    return w;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], kPair ? 16 : 8);  // lane 0 of each softmax warp of the tile
      mbar_init(&o_empty[i], kPair ? 16 : 8);
    }
    mbar_init(o_final, 1);
    mbar_init(merge_ready, 1);
    mbar_init(merge_full, 16 * 32);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    if (kPair) {
      tmem_alloc_pair(tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (kPair || kSplit) cluster_sync();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S_t at t*128, O_t at 256 + t*128.

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      uint32_t jg = 0;  // key tiles loaded so far (ring stage and phase)
      int local = 0;
      for (int32_t u = u_first; u < u_end && ok; u += u_step, ++local) {
        const Unit w = decode(u);
        auto load = [&](void *dst, const CUtensorMap *map, uint64_t *bar, int32_t x, int32_t y) {
          // 4-D maps (head_dim, heads, rows, batch): a stream is (batch, head).
          if (kPair) tma_load_4d_pair(dst, map, bar, x, w.s_head, y, w.s_batch);
          else tma_load_4d(dst, map, bar, x, w.s_head, y, w.s_batch);
        };
        const int qb = local & 1;
        uint8_t *sQ = qb ? sQ1 : sQ0;
        // The Q buffer's previous unit (two back) has finished its QK^T products.
        if (kPair && local >= 2 && !mbar_wait_bounded(&q_empty[qb], ((local >> 1) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        if (leader) mbar_arrive_expect_tx(&q_full[qb], TX_MULT * 2 * TILE_BYTES);
        for (int t = 0; t < 2; ++t)
          for (int h = 0; h < 2; ++h) load(sQ + t * TILE_BYTES + h * HALF_BYTES, &tmQ, &q_full[qb], h * 64, w.q0 + t * TQ);
        for (int j = 0; j < w.n_tiles && ok; ++j, ++jg) {
          const int st = jg & 1;
          if (!mbar_wait_bounded(&k_empty[st], ((jg >> 1) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&k_full[st], TX_MULT * K_BYTES);
          for (int h = 0; h < 2; ++h)
            load(sK + st * K_BYTES + h * K_HALF, &tmK, &k_full[st], h * 64,
                 (w.j_begin + j) * TK + (int32_t)prank * (TK / 2));
          if (!mbar_wait_bounded(&v_empty[st], ((jg >> 1) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&v_full[st], TX_MULT * V_BYTES);
          if (kPair) {
            load(sV + st * V_BYTES, &tmV, &v_full[st], (int32_t)prank * 64, (w.j_begin + j) * TK);
          } else {
            for (int h = 0; h < 2; ++h)
              load(sV + st * V_BYTES + h * HALF_BYTES, &tmV, &v_full[st], h * 64, (w.j_begin + j) * TK);
          }
        }
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_ATTENTION | ERR_SITE_PRODUCER);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc_s = make_idesc(kPair ? 2 * TQ : TQ, TK, 0, false, false);  // K-major Q and K
      constexpr uint32_t idesc_o = make_idesc(kPair ? 2 * TQ : TQ, DP, 0, false, true);   // V MN-major (D contiguous)
      auto commit = [&](uint64_t *bar) {
        if (kPair) mma_commit_pair(bar, 0x3);
        else mma_commit(bar);
      };
      bool ok = true;
      // Descriptors are built once; each k-step adds a compile-time offset (in
      // 16-byte units) so the single issuing thread spends about one integer
      // add per MMA and keeps the tensor pipe fed.
      const uint64_t k_desc = make_smem_desc(smem_u32(sK), 16, 1024, kSwizzle128B);
      const uint64_t v_desc = make_smem_desc(smem_u32(sV), HALF_BYTES, 1024, kSwizzle128B);
      uint32_t jg = 0;
      int local = 0;
      for (int32_t u = u_first; u < u_end && ok; u += u_step, ++local) {
        const Unit w = decode(u);
        const int qb = local & 1;
        const uint64_t q_desc = make_smem_desc(smem_u32(qb ? sQ1 : sQ0), 16, 1024, kSwizzle128B);
        auto issue_s = [&](int t, int stage) {
          const uint64_t qd = q_desc + (uint64_t)(t * (TILE_BYTES >> 4));
          const uint64_t kd = k_desc + (uint64_t)(stage * (K_BYTES >> 4));
          const uint32_t d = tmem + t * 128;
#pragma unroll
          for (int k = 0; k < DP / 16; ++k) {
            const uint64_t adesc = qd + (uint64_t)(((k >> 2) * HALF_BYTES + (k & 3) * 32) >> 4);
            const uint64_t bdesc = kd + (uint64_t)(((k >> 2) * K_HALF + (k & 3) * 32) >> 4);
            if (kPair) mma_f16_ss_pair(d, adesc, bdesc, idesc_s, k > 0 ? 1u : 0u);
            else mma_f16_ss(d, adesc, bdesc, idesc_s, k > 0 ? 1u : 0u);
          }
          commit(&s_full[t]);
        };
        // Issue order per key tile j (stage st):
        //   [P_0(j)] PV_0(j), (release K stage of tile j after its last use)
        //            S_0(j+1)
        //   [P_1(j)] PV_1(j), release V stage st, [V(j+1) landed], S_1(j+1)
        // The bookkeeping between S_1(j+1) and PV_0(j+1) -- when the tensor
        // pipe may run dry -- is one commit and the P_0 wait.  A unit's first
        // S products follow the previous unit's last PV products in the same
        // pipe, so its S tiles (holding the last P) are free by then.
        ok = mbar_wait_bounded(&q_full[qb], (local >> 1) & 1, abort_flag);
        if (ok) ok = mbar_wait_bounded(&k_full[jg & 1], (jg >> 1) & 1, abort_flag);
        if (ok) {
          issue_s(0, jg & 1);
          issue_s(1, jg & 1);
        }
        if (ok) ok = mbar_wait_bounded(&v_full[jg & 1], (jg >> 1) & 1, abort_flag);
        for (int j = 0; j < w.n_tiles && ok; ++j, ++jg) {
          const int st = jg & 1;
          const bool more = j + 1 < w.n_tiles;
          const uint64_t vd = v_desc + (uint64_t)(st * (V_BYTES >> 4));
          for (int t = 0; t < 2 && ok; ++t) {
            if (!mbar_wait_bounded(&p_ready[t], jg & 1, abort_flag)) { ok = false; break; }
            // The previous unit's epilogue has read O_t out before the first
            // PV of this unit overwrites it.
            if (kPair && j == 0 && local > 0 && !mbar_wait_bounded(&o_empty[t], (local - 1) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem + 256 + t * 128, a = tmem + t * 128;
            const uint32_t acc0 = j > 0 ? 1u : 0u;
#pragma unroll
            for (int k = 0; k < TK / 16; ++k) {
              // A = P_t (f16, 8 TMEM columns per 16 keys); B = V rows [16k, 16k+16)
              const uint64_t bdesc = vd + (uint64_t)((k * 2048) >> 4);
              if (kPair) mma_f16_ts_pair(d, a + k * 8, bdesc, idesc_o, k > 0 ? 1u : acc0);
              else mma_f16_ts(d, a + k * 8, bdesc, idesc_o, k > 0 ? 1u : acc0);
            }
            if (t == 0) {
              // K stage st was last read by S_1(j), complete before P_1(j) could
              // have been produced; release it now that PV_0(j) is queued.
              commit(&k_empty[st]);
              if (more && !mbar_wait_bounded(&k_full[st ^ 1], ((jg + 1) >> 1) & 1, abort_flag)) { ok = false; break; }
            } else {
              commit(&v_empty[st]);
              if (more && !mbar_wait_bounded(&v_full[st ^ 1], ((jg + 1) >> 1) & 1, abort_flag)) { ok = false; break; }
            }
            if (more) issue_s(t, st ^ 1);
          }
        }
        if (ok) {
          commit(o_final);
          if (kPair) commit(&q_empty[qb]);
        }
      }
      if (!ok) {
        record_device_error(p.err, ERR_KERNEL_ATTENTION | ERR_SITE_MMA);
        *abort_flag = 1;
      }
    }
  } else {
    // Softmax: 16 warps.  Q tile t = (warp-2)/8; within a tile, column half
    // h = ((warp-2)%8)/4 of the 128-key S tile, TMEM lane quarter warp%4.  The
    // two warps sharing a lane quarter (h = 0, 1) own the same 32 query rows
    // and exchange their partial row maxima through shared memory behind a
    // 64-thread named barrier, so each thread exponentiates 64 scores.
    const int sw = warp - 2;
    const int t = sw >> 3;
    const int h = (sw >> 2) & 1;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t bar_id = 1 + t * 4 + quarter;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = tmem + lane_off + t * 128;
    const uint32_t o_col = tmem + lane_off + 256 + t * 128 + h * 64;
    const float c = p.scale_log2;
    bool ok = true;
    uint32_t jg = 0;
    int local = 0;
    for (int32_t u = u_first; u < u_end && ok; u += u_step, ++local) {
      const int split_half = (p.key_tiles + 1) / 2;
      const int j_begin = kSplit ? (int)rank * split_half : 0;
      const int n_tiles = kSplit ? min(p.key_tiles - j_begin, split_half) : p.key_tiles;
      float m = -INFINITY, l = 0.0f;
      for (int j = 0; j < n_tiles; ++j, ++jg) {
        if (!mbar_wait_bounded(&s_full[t], jg & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const int64_t rem_keys = p.sk - (int64_t)(j_begin + j) * TK - h * 64;
        const int valid = rem_keys < 64 ? (rem_keys > 0 ? (int)rem_keys : 0) : 64;
        // This warp's 64 scores stay in registers (P overwrites S columns of the
        // partner's half only after the barrier below).
        uint32_t a[32], b[32];
        tmem_ld_32x32b_x32(s_col + h * 64, a);
        tmem_ld_32x32b_x32(s_col + h * 64 + 32, b);
        tmem_wait_ld(a);
        tmem_regs_fence(b);
        float mx = -INFINITY;
        if (valid == 64) {
          float mx1 = -INFINITY;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            mx = max3(mx, __uint_as_float(a[i]), __uint_as_float(a[i + 1]));
            mx1 = max3(mx1, __uint_as_float(a[i + 2]), __uint_as_float(a[i + 3]));
            mx = max3(mx, __uint_as_float(b[i]), __uint_as_float(b[i + 1]));
            mx1 = max3(mx1, __uint_as_float(b[i + 2]), __uint_as_float(b[i + 3]));
          }
          mx = fmaxf(mx, mx1);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i >= valid) a[i] = __float_as_uint(-INFINITY);
            if (i + 32 >= valid) b[i] = __float_as_uint(-INFINITY);
            mx = fmaxf(mx, fmaxf(__uint_as_float(a[i]), __uint_as_float(b[i])));
          }
        }
        xmax[t][h][row] = mx;
        named_barrier_sync(bar_id, 64);
        mx = fmaxf(mx, xmax[t][h ^ 1][row]);
        const float m_new = fmaxf(m, mx);
        bool rescale = false;
        float alpha = 1.0f;
        if (j == 0) {
          m = m_new;
        } else if ((m_new - m) * c > RESCALE_THRESHOLD) {
          alpha = ex2_approx((m - m_new) * c);
          rescale = true;
          m = m_new;
          l *= alpha;
        }
        // P = 2^(s*c - m*c) in packed f16 written to S columns [h*32, h*32+32):
        // packed f32x2 arithmetic, one pair in three exponentiated on the FMA
        // pipe (exp2_poly2) to unload the MUFU unit (16 ex2 per clock per SM;
        // a third on the polynomial balances it against the FMA pipe).  Masked
        // keys hold -inf -> 0.
        const float mc = m * c;
        const uint64_t c2 = f2_pack(c, c), nmc2 = f2_pack(-mc, -mc);
        uint64_t sum2 = f2_pack(0.0f, 0.0f);
        uint32_t packed[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float x0 = __uint_as_float(i < 16 ? a[2 * i] : b[2 * i - 32]);
          const float x1 = __uint_as_float(i < 16 ? a[2 * i + 1] : b[2 * i - 31]);
          const uint64_t tt = f2_fma(f2_pack(x0, x1), c2, nmc2);
          uint64_t pp;
          if ((i % 3) == 2) {
            pp = exp2_poly2(tt);
          } else {
            float t0, t1;
            f2_unpack(tt, t0, t1);
            pp = f2_pack(ex2_approx(t0), ex2_approx(t1));
          }
          sum2 = f2_add(sum2, pp);
          float p0, p1;
          f2_unpack(pp, p0, p1);
          __half2 h2 = __floats2half2_rn(p0, p1);
          packed[i] = *reinterpret_cast<uint32_t *>(&h2);
        }
        tmem_st_32x32b_x32(s_col + h * 32, packed);
        float s0, s1;
        f2_unpack(sum2, s0, s1);
        l += s0 + s1;
        if (__any_sync(0xffffffffu, rescale)) {
          // O_t is stable: PV_t(j-1) was issued before S_t(j), whose completion
          // we observed.  Each warp rescales its 64 columns of O.
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(o_col + ch * 32, o);
            tmem_wait_ld(o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_32x32b_x32(o_col + ch * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (kPair) mbar_arrive_leader(&p_ready[t]);
          else mbar_arrive(&p_ready[t]);
        }
      }
      if (!ok) break;
      // Epilogue: combine the two partial row sums, then O_t / l -> out for this
      // warp's 64 columns.
      xsum[t][h][row] = l;
      named_barrier_sync(bar_id, 64);
      l += xsum[t][h ^ 1][row];
      if (!mbar_wait_bounded(o_final, local & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const Unit w = decode(u);
      const int64_t grow = (int64_t)w.q0 + t * TQ + row;
      const bool row_ok = grow < p.sq;
      const int64_t base = ((w.s_batch * p.sq + grow) * p.heads + w.s_head) * p.d;
      // Split merge area in CTA 0: its Q/K/V tiles, dead once its MMAs are
      // complete.  Rows are padded to RECV_LD floats so that one warp's
      // float4 reads of 32 rows spread over all banks.
      constexpr int RECV_LD = DP + 4;
      float *recv_o = reinterpret_cast<float *>(smem);
      float *recv_m = recv_o + 2 * TQ * RECV_LD, *recv_l = recv_m + 2 * TQ;
      const int r2 = t * TQ + row;
      float a_own = 1.0f, a_peer = 0.0f;
      bool store = true;
      if (kSplit && rank == 1) {
        // Ship this CTA's unnormalised O (64 columns per thread), m and l.
        store = false;
        if (!mbar_wait_cluster_bounded(merge_ready, 0, abort_flag)) {
          ok = false;
        } else {
          const uint32_t dst = map_shared_rank(smem_u32(recv_o + (size_t)r2 * RECV_LD + h * 64), 0);
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(o_col + ch * 32, r);
            tmem_wait_ld(r);
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              st_cluster_v4(dst + (uint32_t)(ch * 32 + i) * 4u, __uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                            __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
          }
          if (h == 0) {
            st_cluster_f32(map_shared_rank(smem_u32(recv_m + r2), 0), m);
            st_cluster_f32(map_shared_rank(smem_u32(recv_l + r2), 0), l);
          }
          mbar_arrive_cluster(map_shared_rank(smem_u32(merge_full), 0));
        }
      } else if (kSplit) {
        // CTA 0: release the tiles to CTA 1, wait for its partial, rescale
        // both halves to the larger running max.
        if (warp == 2 && lane == 0) mbar_arrive_cluster(map_shared_rank(smem_u32(merge_ready), 1));
        if (!mbar_wait_cluster_bounded(merge_full, 0, abort_flag)) {
          ok = false;
          store = false;
        } else {
          const float m_peer = recv_m[r2], l_peer = recv_l[r2];
          const float mf = fmaxf(m, m_peer);
          a_own = ex2_approx((m - mf) * c);
          a_peer = ex2_approx((m_peer - mf) * c);
          l = l * a_own + l_peer * a_peer;
        }
      }
      const float inv = 1.0f / l;
      const float *peer = recv_o + (size_t)r2 * RECV_LD + h * 64;
#pragma unroll
      for (int ch = 0; ch < 2 && store; ++ch) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(o_col + ch * 32, r);
        tmem_wait_ld(r);
        if (kPair && ch == 1) {
          // O_t is read out: the next unit's first PV may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_leader(&o_empty[t]);
        }
        if (kSplit) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 q4 = *reinterpret_cast<const float4 *>(peer + ch * 32 + i);
            r[i] = __float_as_uint(__uint_as_float(r[i]) * a_own + q4.x * a_peer);
            r[i + 1] = __float_as_uint(__uint_as_float(r[i + 1]) * a_own + q4.y * a_peer);
            r[i + 2] = __float_as_uint(__uint_as_float(r[i + 2]) * a_own + q4.z * a_peer);
            r[i + 3] = __float_as_uint(__uint_as_float(r[i + 3]) * a_own + q4.w * a_peer);
          }
        }
        const int col0 = h * 64 + ch * 32;
        if (!row_ok || col0 >= p.d) continue;
        if (p.out_f32) {
          float *o = static_cast<float *>(p.out) + base + col0;
          for (int i = 0; i < 32 && col0 + i < p.d; i += 4)
            *reinterpret_cast<float4 *>(o + i) =
                make_float4(__uint_as_float(r[i]) * inv, __uint_as_float(r[i + 1]) * inv,
                            __uint_as_float(r[i + 2]) * inv, __uint_as_float(r[i + 3]) * inv);
        } else {
          uint16_t *o = static_cast<uint16_t *>(p.out) + base + col0;
          for (int i = 0; i < 32 && col0 + i < p.d; i += 8) {
            uint4 v;
            v.x = pack_h2(__uint_as_float(r[i]) * inv, __uint_as_float(r[i + 1]) * inv);
            v.y = pack_h2(__uint_as_float(r[i + 2]) * inv, __uint_as_float(r[i + 3]) * inv);
            v.z = pack_h2(__uint_as_float(r[i + 4]) * inv, __uint_as_float(r[i + 5]) * inv);
            v.w = pack_h2(__uint_as_float(r[i + 6]) * inv, __uint_as_float(r[i + 7]) * inv);
            *reinterpret_cast<uint4 *>(o + i) = v;
          }
        }
      }
      if (kPair && !store) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_leader(&o_empty[t]);
      }
    }
    if (!ok) {
      record_device_error(p.err, ERR_KERNEL_ATTENTION | ERR_SITE_EPILOGUE);
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (kPair || kSplit) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if (kPair) tmem_dealloc_pair(tmem, 512);
    else tmem_dealloc(tmem, 512);
  }
}

}  // namespace
}  // namespace ipuc

using namespace ipuc;

namespace ipuc {
namespace {
// Streams = batch * heads; Q [batch][query_rows][heads * head_dim], K and V
// [batch][key_rows][heads * head_dim], out [batch][query_rows][heads * head_dim]
// (heads = 1: [streams][rows][head_dim]).
ipuc_status attention_launch(void *out, ipuc_precision out_precision, const void *q, const void *k, const void *v,
                             int64_t batch, int64_t heads, int64_t query_rows, int64_t key_rows, int64_t head_dim,
                             float scale, cudaStream_t stream) {
  IPUC_CHECK_ARG(out_precision == IPUC_F16 || out_precision == IPUC_F32, "flash_attention: bad output precision");
  IPUC_CHECK_ARG(batch >= 0 && heads >= 1 && query_rows >= 0 && key_rows >= 0, "flash_attention: negative extent");
  const int64_t matrices = batch * heads;
  if (matrices == 0 || query_rows == 0) return IPUC_OK;
  IPUC_CHECK_ARG(key_rows > 0, "flash_attention: key rows must be positive");
  IPUC_CHECK_ARG(head_dim > 0 && head_dim % 8 == 0, "flash_attention: head_dim must be a positive multiple of 8");
  if (head_dim > 128) return fail(IPUC_ERR_UNSUPPORTED, "flash_attention: head_dim above 128 is not supported");
  IPUC_CHECK_ARG(out && q && k && v, "flash_attention: null pointer");
  IPUC_CHECK_ALIGN(aligned(out, 16) && aligned(q, 16) && aligned(k, 16) && aligned(v, 16),
                   "flash_attention: pointers must be 16-byte aligned");
  IPUC_CHECK_ARG(matrices < (1ll << 24) && heads < (1ll << 16) && query_rows < (1ll << 31) && key_rows < (1ll << 31),
                 "flash_attention: extent too large");
  // CTA pairs when every pair gets a full 512-row query block.
  const bool pair = query_rows >= 4 * TQ;
  CUtensorMap tq, tk, tv, tk_full;
  // 4-D maps (head_dim, heads, rows, batch): one stream's rows sit head_dim
  // apart within a row of heads * head_dim, so split-heads costs no copy.
  const int64_t ld = heads * head_dim;
  const auto f16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  ipuc_status st = make_map_4d_rows(&tq, f16, 2, q, head_dim, heads, query_rows, batch, head_dim, ld,
                                    query_rows * ld, 64, TQ);
  if (st != IPUC_OK) return st;
  st = make_map_4d_rows(&tk, f16, 2, k, head_dim, heads, key_rows, batch, head_dim, ld, key_rows * ld, 64,
                        pair ? TK / 2 : TK);
  if (st != IPUC_OK) return st;
  st = make_map_4d_rows(&tv, f16, 2, v, head_dim, heads, key_rows, batch, head_dim, ld, key_rows * ld, 64, TK);
  if (st != IPUC_OK) return st;
  AttnParams p;
  p.out = out;
  p.matrices = matrices;
  p.sq = query_rows;
  p.sk = key_rows;
  p.d = head_dim;
  const float s = scale > 0.0f ? scale : 1.0f / sqrtf((float)head_dim);
  p.scale_log2 = s * 1.4426950408889634f;
  p.out_f32 = out_precision == IPUC_F32;
  p.key_tiles = (int32_t)((key_rows + TK - 1) / TK);
  p.heads = (int32_t)heads;
  p.unit_base = 0;
  p.num_units = 0;
  p.err = device_error_word();
  auto launch = [&](auto kernel, int64_t ctas, bool cluster, const CUtensorMap &kmap) -> ipuc_status {
    IPUC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cluster ? 1 : 0;
    IPUC_CUDA(cudaLaunchKernelEx(&cfg, kernel, tq, kmap, tv, p));
    return check_launch("flash_attention_kernel");
  };
  if (!pair) {
    p.q_units = (int32_t)((query_rows + 2 * TQ - 1) / (2 * TQ));
    return launch(flash_attention_kernel<false, false>, matrices * p.q_units, false, tk);
  }
  // Pair units of 512 query rows.  When they leave a last wave at most half
  // full, that tail runs as split clusters (two CTAs per 256-row unit, each
  // over half the keys), which halves the tail wave's length.
  p.q_units = (int32_t)((query_rows + 4 * TQ - 1) / (4 * TQ));
  const int64_t units = matrices * p.q_units, slots = sm_count() / 2;
  const int64_t tail = units % slots, full = units - tail;
  const bool split = tail > 0 && 4 * tail <= 2 * slots && p.key_tiles >= 2;
  const int64_t paired = split ? full : units;
  if (paired > 0) {
    // persistent pairs: each loops over pair units (the next unit's Q and the
    // previous unit's O store overlap this unit's products)
    p.num_units = paired;
    st = launch(flash_attention_kernel<true, false>, 2 * (paired < slots ? paired : slots), true, tk);
    if (st != IPUC_OK) return st;
  }
  if (!split) return IPUC_OK;
  st = make_map_4d_rows(&tk_full, f16, 2, k, head_dim, heads, key_rows, batch, head_dim, ld, key_rows * ld, 64, TK);
  if (st != IPUC_OK) return st;
  p.unit_base = 2 * full;  // 256-row half-units
  return launch(flash_attention_kernel<false, true>, 4 * tail, true, tk_full);
}
}  // namespace
}  // namespace ipuc

extern "C" ipuc_status ipuc_flash_attention_f16(void *out, ipuc_precision out_precision, const void *q, const void *k,
                                                const void *v, int64_t matrices, int64_t query_rows, int64_t key_rows,
                                                int64_t head_dim, float scale, ipuc_stream stream) {
  return ipuc::attention_launch(out, out_precision, q, k, v, matrices, 1, query_rows, key_rows, head_dim, scale,
                                stream);
}

extern "C" ipuc_status ipuc_flash_attention_heads_f16(void *out, ipuc_precision out_precision, const void *q,
                                                      const void *k, const void *v, int64_t batch, int64_t heads,
                                                      int64_t query_rows, int64_t key_rows, int64_t head_dim,
                                                      float scale, ipuc_stream stream) {
  return ipuc::attention_launch(out, out_precision, q, k, v, batch, heads, query_rows, key_rows, head_dim, scale,
                                stream);
}

