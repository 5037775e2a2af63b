// Bit-exact f16 element-order conversions: the rearrange_* and unpack_amp_*
// tile kernels of the reference (device/rearrange_f16.cpp:36-155,
// device/rearrange_amp_left_f16.S, device/rearrange_block_major_f16.S,
// device/rearrange_transposed_right_f16.S, device/unpack_amp_f16.cpp:40-81),
// the general order conversion the reference leaves unimplemented
// (crates/ipu-codegen/src/kernel.rs:1365-1370) and SplitHeads
// (crates/ipu-tests/src/diagnostic.rs:685-709).
//
// Every packed order of crates/ipu-codegen/src/storage.rs stores each 16x16
// micro-block of a matrix as 256 contiguous elements, with an order-specific
// permutation inside the block (derivation per order in block_base /
// block_offset below).  The general kernel therefore moves one micro-block per
// warp: each lane reads one 16-byte chunk of the source block, the warp
// transposes through a 16x16 shared-memory tile, and each lane writes one
// 16-byte chunk of the destination block.  Global traffic is one read and one
// write of each byte in full 32-byte sectors (HBM-bound, no tensor cores).
// Row-major -> BlockMajor{64,16} over whole 64x64 tiles (the config-5 weight
// layout) has a dedicated TMA + ldmatrix/stmatrix kernel
// (rm_to_block_major64_kernel) that moves whole contiguous 8 KB tiles.
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace ipuc {
namespace {

struct Side {
  void *ptr;
  int32_t order;
  int64_t rows, cols;  // physical extents of one matrix
  int64_t ld;          // row-major leading dimension (elements)
  int64_t mstride;     // elements between matrices
  int64_t rb, cb;      // block-major row/column block
  int32_t vec;         // 16-byte vector accesses allowed on the row-major side
};

// Inverse of the AMP-Output pair swizzle of storage.rs:333-340 (as in
// amp_matrix_coordinates, storage.rs:689-694): physical column -> logical.
__device__ __forceinline__ int unswz(int pc) {
  int pp = pc >> 1, lp = (pp & 1) * 4 + (pp >> 1);
  return lp * 2 + (pc & 1);
}

// Element index of the first element of micro-block (br, bc) within a matrix.
//   AMP-Left            idx = (c/16)*R*16 + r*16 + c%16                 (storage.rs:316-325)
//   AMP-TransposedLeft  idx = (r/16)*C*16 + c*16 + r%16                 (storage.rs:327-329)
//   AMP-TransposedRight idx = ((r/16)*(C/16) + c/16)*256 + (r%16)*16 + c%16  (storage.rs:326,353-371)
//   AMP-Output          idx = (c/16)*R*16 + r*16 + swz(c%16)           (storage.rs:330-340)
//   AMP-TransposedOut.  idx = (r/16)*C*16 + c*16 + swz(r%16)           (storage.rs:341-343)
//   BlockMajor{rb,cb}   idx = panel*16*cb + (c%cb)*16 + r%16, panel =
//                       (r/rb)*(C/cb)*(rb/16) + (c/cb)*(rb/16) + (r%rb)/16   (storage.rs:372-426)
//   BlockMajor^T        the same with (r, c, R, C) -> (c, r, C, R)
__device__ __forceinline__ int64_t block_base(const Side &s, int64_t br, int64_t bc) {
  const int64_t R = s.rows, C = s.cols;
  switch (s.order) {
    case IPUC_ORDER_AMP_LEFT:
    case IPUC_ORDER_AMP_OUTPUT:
      return bc * R * 16 + br * 256;
    case IPUC_ORDER_AMP_TRANSPOSED_LEFT:
    case IPUC_ORDER_AMP_TRANSPOSED_OUTPUT:
      return br * C * 16 + bc * 256;
    case IPUC_ORDER_AMP_TRANSPOSED_RIGHT:
      return (br * (C / 16) + bc) * 256;
    case IPUC_ORDER_BLOCK_MAJOR: {
      const int64_t r0 = br * 16, c0 = bc * 16, rg = s.rb / 16;
      const int64_t panel = (r0 / s.rb) * (C / s.cb) * rg + (c0 / s.cb) * rg + (r0 % s.rb) / 16;
      return panel * 16 * s.cb + (c0 % s.cb) * 16;
    }
    case IPUC_ORDER_BLOCK_MAJOR_TRANSPOSED: {
      const int64_t r0 = bc * 16, c0 = br * 16, rg = s.rb / 16;  // transposed view
      const int64_t panel = (r0 / s.rb) * (R / s.cb) * rg + (c0 / s.cb) * rg + (r0 % s.rb) / 16;
      return panel * 16 * s.cb + (c0 % s.cb) * 16;
    }
  }
  return 0;
}

// Whether the block stores its elements rows-outer (offset = rr*16 + f(cc)).
__device__ __forceinline__ bool rows_outer(int32_t order) {
  return order == IPUC_ORDER_AMP_LEFT || order == IPUC_ORDER_AMP_TRANSPOSED_RIGHT ||
         order == IPUC_ORDER_AMP_OUTPUT || order == IPUC_ORDER_BLOCK_MAJOR_TRANSPOSED;
}
__device__ __forceinline__ bool swizzled(int32_t order) {
  return order == IPUC_ORDER_AMP_OUTPUT || order == IPUC_ORDER_AMP_TRANSPOSED_OUTPUT;
}

// offset within the 256-element block -> (rr, cc)
__device__ __forceinline__ void offset_to_rc(int32_t order, int o, int &rr, int &cc) {
  const int outer = o >> 4, inner0 = o & 15;
  const int inner = swizzled(order) ? unswz(inner0) : inner0;
  if (rows_outer(order)) { rr = outer; cc = inner; } else { cc = outer; rr = inner; }
}

template <bool kFromRow, bool kToRow>
__global__ void __launch_bounds__(256) convert_blocks_kernel(Side src, Side dst, int64_t logical_rows,
                                                             int64_t logical_cols, int64_t matrices) {
  __shared__ uint16_t tile[8][16][17];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bR = (dst.rows + 15) / 16, bC = (dst.cols + 15) / 16;
  const int64_t total = matrices * bR * bC;
  const int64_t vr = min(logical_rows, src.rows), vc = min(logical_cols, src.cols);
  const uint16_t *sp = static_cast<const uint16_t *>(src.ptr);
  uint16_t *dp = static_cast<uint16_t *>(dst.ptr);
  for (int64_t blk = (int64_t)blockIdx.x * 8 + warp; blk < total; blk += (int64_t)gridDim.x * 8) {
    const int64_t m = blk / (bR * bC);
    const int64_t rem = blk % (bR * bC);
    const int64_t br = rem / bC, bc = rem % bC;
    const int64_t r0 = br * 16, c0 = bc * 16;
    // ---- gather the source block into tile[warp][rr][cc] ----
    uint16_t vals[8];
    int rrs[8], ccs[8];
    if (kFromRow) {
      const int rr = lane >> 1, cb0 = (lane & 1) * 8;
      const int64_t r = r0 + rr;
      const uint16_t *row = sp + m * src.mstride + r * src.ld + c0 + cb0;
      const bool full = (r < vr) && (c0 + cb0 + 8 <= vc);
      if (full && src.vec) {
        uint4 v = *reinterpret_cast<const uint4 *>(row);
        const uint16_t *pv = reinterpret_cast<const uint16_t *>(&v);
#pragma unroll
        for (int i = 0; i < 8; ++i) vals[i] = pv[i];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) vals[i] = (r < vr && c0 + cb0 + i < vc) ? row[i] : (uint16_t)0;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) { rrs[i] = rr; ccs[i] = cb0 + i; }
    } else {
      const int64_t base = m * src.mstride + block_base(src, br, bc);
      bool all = true;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        offset_to_rc(src.order, lane * 8 + i, rrs[i], ccs[i]);
        all = all && (r0 + rrs[i] < vr) && (c0 + ccs[i] < vc);
      }
      if (all) {
        uint4 v = *reinterpret_cast<const uint4 *>(sp + base + lane * 8);
        const uint16_t *pv = reinterpret_cast<const uint16_t *>(&v);
#pragma unroll
        for (int i = 0; i < 8; ++i) vals[i] = pv[i];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const bool ok = (r0 + rrs[i] < vr) && (c0 + ccs[i] < vc);
          vals[i] = ok ? sp[base + lane * 8 + i] : (uint16_t)0;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) tile[warp][rrs[i]][ccs[i]] = vals[i];
    __syncwarp();
    // ---- scatter the destination block ----
    if (kToRow) {
      const int rr = lane >> 1, cb0 = (lane & 1) * 8;
      const int64_t r = r0 + rr;
      uint16_t *row = dp + m * dst.mstride + r * dst.ld + c0 + cb0;
      if (r < dst.rows) {
        if (dst.vec && c0 + cb0 + 8 <= dst.cols) {
          uint4 v;
          uint16_t *pv = reinterpret_cast<uint16_t *>(&v);
#pragma unroll
          for (int i = 0; i < 8; ++i) pv[i] = tile[warp][rr][cb0 + i];
          *reinterpret_cast<uint4 *>(row) = v;
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (c0 + cb0 + i < dst.cols) row[i] = tile[warp][rr][cb0 + i];
        }
      }
    } else {
      const int64_t base = m * dst.mstride + block_base(dst, br, bc);
      uint16_t out[8];
      bool all = true;
      bool ok[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        int rr, cc;
        offset_to_rc(dst.order, lane * 8 + i, rr, cc);
        ok[i] = (r0 + rr < dst.rows) && (c0 + cc < dst.cols);
        all = all && ok[i];
        out[i] = tile[warp][rr][cc];
      }
      if (all) {
        uint4 v;
        uint16_t *pv = reinterpret_cast<uint16_t *>(&v);
#pragma unroll
        for (int i = 0; i < 8; ++i) pv[i] = out[i];
        *reinterpret_cast<uint4 *>(dp + base + lane * 8) = v;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (ok[i]) dp[base + lane * 8 + i] = out[i];
      }
    }
    __syncwarp();
  }
}

// Same conversion with 32-bit index arithmetic inside a matrix (used when a
// matrix holds fewer than 2^31 elements): every CTA of 8 warps owns 8
// consecutive micro-blocks of one 16-row band, so the work index is divided
// once per CTA, and each lane's in-block permutation (which depends only on the
// order and the lane) is computed once per thread, not once per block.
__device__ __forceinline__ int32_t block_base32(const Side &s, int32_t br, int32_t bc) {
  const int32_t R = (int32_t)s.rows, C = (int32_t)s.cols;
  switch (s.order) {
    case IPUC_ORDER_AMP_LEFT:
    case IPUC_ORDER_AMP_OUTPUT:
      return bc * R * 16 + br * 256;
    case IPUC_ORDER_AMP_TRANSPOSED_LEFT:
    case IPUC_ORDER_AMP_TRANSPOSED_OUTPUT:
      return br * C * 16 + bc * 256;
    case IPUC_ORDER_AMP_TRANSPOSED_RIGHT:
      return (br * (C >> 4) + bc) * 256;
    case IPUC_ORDER_BLOCK_MAJOR: {
      const int32_t rb = (int32_t)s.rb, cb = (int32_t)s.cb, r0 = br * 16, c0 = bc * 16, rg = rb >> 4;
      const int32_t panel = (r0 / rb) * (C / cb) * rg + (c0 / cb) * rg + (r0 % rb) / 16;
      return panel * 16 * cb + (c0 % cb) * 16;
    }
    case IPUC_ORDER_BLOCK_MAJOR_TRANSPOSED: {
      const int32_t rb = (int32_t)s.rb, cb = (int32_t)s.cb, r0 = bc * 16, c0 = br * 16, rg = rb >> 4;
      const int32_t panel = (r0 / rb) * (R / cb) * rg + (c0 / cb) * rg + (r0 % rb) / 16;
      return panel * 16 * cb + (c0 % cb) * 16;
    }
  }
  return 0;
}

constexpr int kBlocksPerWarp = 4;  // loads of 4 micro-blocks in flight per warp

template <bool kFromRow, bool kToRow>
__device__ __forceinline__ void lane_rc(const Side &s, bool row_major, int lane, int i, int &rr, int &cc) {
  if (row_major) { rr = lane >> 1; cc = (lane & 1) * 8 + i; }
  else offset_to_rc(s.order, lane * 8 + i, rr, cc);
}

// kMode: 0 = general in-block permutation through shared memory;
//        1 = source and destination place every lane's 8 elements at the same
//            in-block coordinates (rows-outer orders and row-major, or two
//            columns-outer orders): the 16-byte chunk passes straight through;
//        2 = one side rows-outer, the other columns-outer: a 16x16 transpose
//            through a padded tile written with 8-byte stores.
template <bool kFromRow, bool kToRow, int kMode>
__global__ void __launch_bounds__(256, 4) convert_blocks32_kernel(Side src, Side dst, int32_t logical_rows,
                                                                  int32_t logical_cols, int32_t matrices) {
  __shared__ __align__(16) uint16_t tile[8][16 * 20];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kSpan = 8 * kBlocksPerWarp;  // micro-blocks per CTA work item
  const int32_t bR = (int32_t)((dst.rows + 15) / 16), bC = (int32_t)((dst.cols + 15) / 16);
  const int32_t groups = (bC + kSpan - 1) / kSpan;
  const uint32_t total = (uint32_t)matrices * (uint32_t)bR * (uint32_t)groups;
  const int32_t vr = min(logical_rows, (int32_t)src.rows), vc = min(logical_cols, (int32_t)src.cols);
  const int32_t drows = (int32_t)dst.rows, dcols = (int32_t)dst.cols;
  const uint16_t *sp = static_cast<const uint16_t *>(src.ptr);
  uint16_t *dp = static_cast<uint16_t *>(dst.ptr);
  // Per-lane shared-memory slots (rr*17 + cc) of the 8 elements this lane
  // moves, two 16-bit slots per register, and the extreme in-block row and
  // column (for the whole-chunk bounds test).
  uint32_t sslot[4], dslot[4];
  int smax_r = 0, smax_c = 0, dmax_r = 0, dmax_c = 0;
  int srow0 = 0, scol0 = 0, drow0 = 0, dcol0 = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int rr, cc;
    lane_rc<kFromRow, kToRow>(src, kFromRow, lane, i, rr, cc);
    if (i == 0) { srow0 = rr; scol0 = cc; }
    smax_r = max(smax_r, rr); smax_c = max(smax_c, cc);
    const uint32_t sv = (uint32_t)(rr * 17 + cc);
    sslot[i >> 1] = (i & 1) ? (sslot[i >> 1] | (sv << 16)) : sv;
    lane_rc<kFromRow, kToRow>(dst, kToRow, lane, i, rr, cc);
    if (i == 0) { drow0 = rr; dcol0 = cc; }
    dmax_r = max(dmax_r, rr); dmax_c = max(dmax_c, cc);
    const uint32_t dv = (uint32_t)(rr * 17 + cc);
    dslot[i >> 1] = (i & 1) ? (dslot[i >> 1] | (dv << 16)) : dv;
  }
  uint16_t *t = tile[warp];
  for (uint32_t w = blockIdx.x; w < total; w += gridDim.x) {
    const uint32_t per_m = (uint32_t)bR * (uint32_t)groups;
    const int32_t m = (int32_t)(w / per_m);
    const uint32_t rem = w - (uint32_t)m * per_m;
    const int32_t br = (int32_t)(rem / (uint32_t)groups);
    const int32_t bc0 = (int32_t)(rem - (uint32_t)br * (uint32_t)groups) * kSpan + warp;
    const int32_t r0 = br * 16;
    const uint16_t *sbase = sp + (int64_t)m * src.mstride;
    uint16_t *dbase = dp + (int64_t)m * dst.mstride;
    uint4 v[kBlocksPerWarp];
    // Issue all loads first so kBlocksPerWarp 16-byte reads per lane are in flight.
#pragma unroll
    for (int u = 0; u < kBlocksPerWarp; ++u) {
      const int32_t bc = bc0 + 8 * u, c0 = bc * 16;
      if (bc >= bC) continue;  // warp-uniform
      const int32_t soff = kFromRow ? (r0 + srow0) * (int32_t)src.ld + c0 + scol0 : block_base32(src, br, bc) + lane * 8;
      if ((r0 + smax_r < vr) && (c0 + smax_c < vc) && (kFromRow ? src.vec != 0 : true)) {
        v[u] = *reinterpret_cast<const uint4 *>(sbase + soff);
      } else {
        uint16_t *pv = reinterpret_cast<uint16_t *>(&v[u]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          int rr, cc;
          lane_rc<kFromRow, kToRow>(src, kFromRow, lane, i, rr, cc);
          pv[i] = (r0 + rr < vr && c0 + cc < vc) ? sbase[soff + i] : (uint16_t)0;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kBlocksPerWarp; ++u) {
      const int32_t bc = bc0 + 8 * u, c0 = bc * 16;
      if (bc >= bC) continue;
      uint4 o;
      if (kMode == 1) {
        o = v[u];
      } else if (kMode == 2) {
        // Lane l holds element i of line l/2 at position 8(l%2)+i; it writes
        // the line (row stride 20 halves keeps the column reads conflict-free)
        // and reads back line positions as columns.
        uint2 *w2 = reinterpret_cast<uint2 *>(t + (lane >> 1) * 20 + (lane & 1) * 8);
        w2[0] = make_uint2(v[u].x, v[u].y);
        w2[1] = make_uint2(v[u].z, v[u].w);
        __syncwarp();
        uint32_t *po = reinterpret_cast<uint32_t *>(&o);
        const uint16_t *col = t + ((lane & 1) * 8) * 20 + (lane >> 1);
#pragma unroll
        for (int j = 0; j < 4; ++j) po[j] = (uint32_t)col[(2 * j) * 20] | ((uint32_t)col[(2 * j + 1) * 20] << 16);
        __syncwarp();
      } else {
        const uint32_t *pv = reinterpret_cast<const uint32_t *>(&v[u]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          t[sslot[j] & 0xffffu] = (uint16_t)(pv[j] & 0xffffu);
          t[sslot[j] >> 16] = (uint16_t)(pv[j] >> 16);
        }
        __syncwarp();
        uint32_t *po = reinterpret_cast<uint32_t *>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) po[j] = (uint32_t)t[dslot[j] & 0xffffu] | ((uint32_t)t[dslot[j] >> 16] << 16);
        __syncwarp();
      }
      const int32_t doff = kToRow ? (r0 + drow0) * (int32_t)dst.ld + c0 + dcol0 : block_base32(dst, br, bc) + lane * 8;
      if ((r0 + dmax_r < drows) && (c0 + dmax_c < dcols) && (kToRow ? dst.vec != 0 : true)) {
        *reinterpret_cast<uint4 *>(dbase + doff) = o;
      } else {
        const uint16_t *ph = reinterpret_cast<const uint16_t *>(&o);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          int rr, cc;
          lane_rc<kFromRow, kToRow>(dst, kToRow, lane, i, rr, cc);
          if (r0 + rr < drows && c0 + cc < dcols) dbase[doff + i] = ph[i];
        }
      }
    }
  }
}

// Host-side geometry checks for a packed side (the divisibility rules of
// storage.rs: AmpBlock / BlockMajorBlock errors).
ipuc_status check_side(const Side &s, const char *which) {
  std::string w(which);
  switch (s.order) {
    case IPUC_ORDER_ROW_MAJOR:
      IPUC_CHECK_ARG(s.ld >= s.cols, w + ": leading dimension smaller than columns");
      return IPUC_OK;
    case IPUC_ORDER_AMP_LEFT:
    case IPUC_ORDER_AMP_OUTPUT:
      IPUC_CHECK_ARG(s.cols % 16 == 0, w + ": AMP-Left/Output need physical columns % 16 == 0");
      return IPUC_OK;
    case IPUC_ORDER_AMP_TRANSPOSED_LEFT:
    case IPUC_ORDER_AMP_TRANSPOSED_OUTPUT:
      IPUC_CHECK_ARG(s.rows % 16 == 0, w + ": transposed AMP orders need physical rows % 16 == 0");
      return IPUC_OK;
    case IPUC_ORDER_AMP_TRANSPOSED_RIGHT:
      IPUC_CHECK_ARG(s.rows % 16 == 0 && s.cols % 16 == 0,
                     w + ": AMP-TransposedRight needs rows % 16 == 0 and columns % 16 == 0");
      return IPUC_OK;
    case IPUC_ORDER_BLOCK_MAJOR:
      IPUC_CHECK_ARG(s.rb > 0 && s.cb > 0 && s.rb % 16 == 0 && s.rows % s.rb == 0 && s.cols % s.cb == 0,
                     w + ": block-major needs row_block % 16 == 0, rows % row_block == 0, columns % column_block == 0");
      if (s.cb % 16 != 0) return fail(IPUC_ERR_UNSUPPORTED, w + ": block-major column_block must be a multiple of 16");
      return IPUC_OK;
    case IPUC_ORDER_BLOCK_MAJOR_TRANSPOSED:
      IPUC_CHECK_ARG(s.rb > 0 && s.cb > 0 && s.rb % 16 == 0 && s.cols % s.rb == 0 && s.rows % s.cb == 0,
                     w + ": transposed block-major needs row_block % 16 == 0, columns % row_block == 0, rows % column_block == 0");
      if (s.cb % 16 != 0) return fail(IPUC_ERR_UNSUPPORTED, w + ": block-major column_block must be a multiple of 16");
      return IPUC_OK;
  }
  return fail(IPUC_ERR_INVALID_ARGUMENT, w + ": unknown element order");
}

// ---- AMP-Output -> row-major (unpack_amp_f16.cpp:40-81, source order 0) -------------
// AMP-Output keeps 16-column panels with rows contiguous (storage.rs:330-340); inside
// a row's 16 elements the 2-element pairs are permuted (logical pair lp sits at
// physical pair (lp % 4) * 2 + lp / 4).  A CTA moves a tile of 32 rows x 16 panels
// through shared memory so that both sides stay contiguous: each panel's 32 row
// segments (1 KB) are read in order, then each row's 16 segments (512 B) are
// written in order, the pair permutation applied in registers on the way out.
// Elements outside the logical extent are written as 0.
constexpr int UNP_ROWS = 32, UNP_PANELS = 16, UNP_PITCH = UNP_PANELS * 2 + 1;  // uint4 per tile row (+1 pad)

__global__ void __launch_bounds__(256) unpack_amp_output_kernel(const uint16_t *__restrict__ src,
                                                                uint16_t *__restrict__ dst, int64_t matrices,
                                                                int64_t rows, int64_t cols, int64_t logical_rows,
                                                                int64_t logical_cols) {
  __shared__ uint4 tile[UNP_ROWS * UNP_PITCH];
  const int64_t panels = cols / 16, per_matrix = rows * cols;
  const int64_t row_tiles = (rows + UNP_ROWS - 1) / UNP_ROWS, panel_tiles = (panels + UNP_PANELS - 1) / UNP_PANELS;
  const int64_t tiles = matrices * row_tiles * panel_tiles;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t pt = t % panel_tiles, rest = t / panel_tiles;
    const int64_t rt = rest % row_tiles, m = rest / row_tiles;
    const int64_t r0 = rt * UNP_ROWS, p0 = pt * UNP_PANELS;
    const uint4 *s4 = reinterpret_cast<const uint4 *>(src + m * per_matrix);
    __syncthreads();  // the previous tile's reads of `tile` are done
    // Load: chunk q = (panel, row, half) with row and half fastest: a panel's rows are contiguous.
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = threadIdx.x + 256 * j;
      const int pl = q >> 6, r = (q >> 1) & 31, hf = q & 1;
      if (p0 + pl < panels && r0 + r < rows)
        tile[r * UNP_PITCH + pl * 2 + hf] = s4[((p0 + pl) * rows + r0 + r) * 2 + hf];
    }
    __syncthreads();
    // Store: segment s = (row, panel) with panel fastest: a row's segments are contiguous.
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int sg = threadIdx.x + 256 * j;
      const int r = sg >> 4, pl = sg & 15;
      const int64_t row = r0 + r, p = p0 + pl;
      if (p >= panels || row >= rows) continue;
      const uint4 a = tile[r * UNP_PITCH + pl * 2], b = tile[r * UNP_PITCH + pl * 2 + 1];
      // logical pairs 0..7 <- physical pairs 0, 2, 4, 6, 1, 3, 5, 7
      uint32_t w[8] = {a.x, a.z, b.x, b.z, a.y, a.w, b.y, b.w};
      const int64_t c0 = p * 16;
      if (row >= logical_rows) {
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = 0u;
      } else if (c0 + 16 > logical_cols) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int64_t c = c0 + 2 * i;
          if (c >= logical_cols) w[i] = 0u;
          else if (c + 1 >= logical_cols) w[i] &= 0xffffu;
        }
      }
      uint4 *d4 = reinterpret_cast<uint4 *>(dst + m * per_matrix + row * cols + c0);
      d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
      d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  }
}

// ---- Row-major -> BlockMajor{64,16}: TMA + ldmatrix.trans / stmatrix ------------
// BlockMajor{64,16} (storage.rs:372-426) stores each 64-row band contiguously:
// for every 16-column block, its four 16x16 row groups, each column-major.  A
// 64x64 row-major tile therefore becomes 8 KB of contiguous output.  A TMA load
// (128-byte swizzle: the 16-byte chunk j of tile row r sits at chunk j ^ (r % 8),
// so the 8 row addresses of each ldmatrix hit distinct banks) brings the tile in;
// ldmatrix.trans turns each 8x8 sub-matrix so that a lane holds one column's
// two rows, which is exactly the fragment stmatrix writes as one output row
// (the output's "rows" being the micro-block's columns); one bulk copy stores
// the tile.  About a quarter of an instruction per element, against one or more
// for lane-level transposes, so the kernel runs at HBM speed.
constexpr int BM64_TILE_BYTES = 64 * 64 * 2;  // 8 KB
constexpr int BM64_STAGES = 6;                // input tiles in flight per CTA (3 CTAs per SM)
constexpr int BM64_OUT = 3;                   // output tiles (bulk stores draining)
constexpr int BM64_SMEM = (BM64_STAGES + BM64_OUT) * BM64_TILE_BYTES + 1024 + 256;

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t &a, uint32_t &b, uint32_t &c, uint32_t &d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void stmatrix_x4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ void bulk_store(void *gdst, uint32_t ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(128, 3)
    rm_to_block_major64_kernel(const __grid_constant__ CUtensorMap src_map, uint16_t *__restrict__ dst,
                               int64_t tiles, int32_t band_tiles, int32_t bands, int64_t cols, uint32_t *err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *in = smem;
  uint8_t *out = smem + BM64_STAGES * BM64_TILE_BYTES;
  uint64_t *full = reinterpret_cast<uint64_t *>(out + BM64_OUT * BM64_TILE_BYTES);
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < BM64_STAGES; ++s) sm100::mbar_init(&full[s], 1);
    abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::tma_prefetch_desc(&src_map);
  }
  __syncthreads();
  // Tile t = (matrix * bands + band) * band_tiles + ct: 64 rows x 64 columns.
  auto issue = [&](int64_t t, int s) {
    const int64_t mb = t / band_tiles;
    const int32_t ct = (int32_t)(t - mb * band_tiles);
    const int32_t band = (int32_t)(mb % bands), m = (int32_t)(mb / bands);
    sm100::mbar_arrive_expect_tx(&full[s], BM64_TILE_BYTES);
    sm100::tma_load_3d(in + s * BM64_TILE_BYTES, &src_map, &full[s], ct * 64, band * 64, m);
  };
  if (threadIdx.x == 0)
    for (int s = 0; s < BM64_STAGES; ++s) {
      const int64_t t = blockIdx.x + (int64_t)s * gridDim.x;
      if (t < tiles) issue(t, s);
    }
  // ldmatrix row addresses (lane -> sub-matrix i = lane / 8, row lane % 8) and
  // stmatrix row addresses for this warp's row group g = warp.
  const int i = lane >> 3, j = lane & 7, g = warp;
  const int in_row = g * 16 + (i & 1) * 8 + j;  // in_row % 8 == j
  const uint32_t out_row_off = (uint32_t)((((i >> 1) * 8 + j) * 16 + (i & 1) * 8) * 2);
  uint32_t it = 0;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
    const int s = (int)(it % BM64_STAGES);
    const bool ok = sm100::mbar_wait_bounded(&full[s], (it / BM64_STAGES) & 1u, &abort_flag);
    const uint32_t src_tile = sm100::smem_u32(in + s * BM64_TILE_BYTES);
    const uint32_t ob = sm100::smem_u32(out + (it % BM64_OUT) * BM64_TILE_BYTES);
#pragma unroll
    for (int b = 0; b < 4 && ok; ++b) {
      // Micro-block (row group g, column block b): sub-matrix i covers rows
      // (i & 1) * 8 and columns (i >> 1) * 8 of it.
      const int chunk = b * 2 + (i >> 1);
      uint32_t r0, r1, r2, r3;
      ldmatrix_x4_trans(src_tile + (uint32_t)(in_row * 128 + ((chunk ^ j) << 4)), r0, r1, r2, r3);
      stmatrix_x4(ob + (uint32_t)((b * 4 + g) * 256 * 2) + out_row_off, r0, r1, r2, r3);
    }
    sm100::fence_proxy_async_smem();  // the bulk copy (async proxy) reads what stmatrix wrote
    // Tile consumed (stage s reusable, output tile complete); a timed-out wait
    // anywhere in the CTA ends every thread's loop here together.
    if (__syncthreads_or(!ok)) {
      if (threadIdx.x == 0) record_device_error(err, ERR_KERNEL_LAYOUT | ERR_SITE_PRODUCER);
      break;
    }
    if (threadIdx.x == 0) {
      const int64_t mb = t / band_tiles;
      const int64_t ct = t - mb * band_tiles;
      // Band mb (matrix-major) starts at mb * 64 * cols; column tile ct adds 4 blocks of 1024.
      bulk_store(dst + mb * 64 * cols + ct * 4096, ob, BM64_TILE_BYTES);
      bulk_wait_read_1();  // the store issued one tile ago has read its buffer
      const int64_t next = t + (int64_t)BM64_STAGES * gridDim.x;
      if (next < tiles) issue(next, s);
    }
  }
  if (threadIdx.x == 0) bulk_wait_all();
}

ipuc_status launch_convert(Side src, Side dst, int64_t logical_rows, int64_t logical_cols, int64_t matrices,
                           cudaStream_t stream) {
  ipuc_status st = check_side(src, "source");
  if (st != IPUC_OK) return st;
  st = check_side(dst, "destination");
  if (st != IPUC_OK) return st;
  IPUC_CHECK_ALIGN(aligned(src.ptr, 16) && aligned(dst.ptr, 16), "rearrange: pointers must be 16-byte aligned");
  if (src.order != IPUC_ORDER_ROW_MAJOR) IPUC_CHECK_ALIGN(src.mstride % 8 == 0, "rearrange: packed matrix size must be a multiple of 8 elements");
  if (dst.order != IPUC_ORDER_ROW_MAJOR) IPUC_CHECK_ALIGN(dst.mstride % 8 == 0, "rearrange: packed matrix size must be a multiple of 8 elements");
  src.vec = (src.ld % 8 == 0 && src.mstride % 8 == 0) ? 1 : 0;
  dst.vec = (dst.ld % 8 == 0 && dst.mstride % 8 == 0) ? 1 : 0;
  const int64_t blocks = matrices * ((dst.rows + 15) / 16) * ((dst.cols + 15) / 16);
  if (blocks == 0) return IPUC_OK;
  // Row-major -> BlockMajor{64,16} over whole 64x64 tiles (no padding): TMA path.
  if (src.order == IPUC_ORDER_ROW_MAJOR && dst.order == IPUC_ORDER_BLOCK_MAJOR && dst.rb == 64 && dst.cb == 16 &&
      src.rows == dst.rows && src.cols == dst.cols && logical_rows == dst.rows && logical_cols == dst.cols &&
      src.ld == src.cols && src.mstride == src.rows * src.cols && dst.mstride == dst.rows * dst.cols &&
      dst.rows % 64 == 0 && dst.cols % 64 == 0 && matrices < (1ll << 31)) {
    CUtensorMap map;
    ipuc_status ms = make_map_3d(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, src.ptr, (uint64_t)src.cols,
                                 (uint64_t)src.rows, (uint64_t)matrices, (uint64_t)src.cols,
                                 (uint64_t)(src.rows * src.cols), 64, 64);
    if (ms != IPUC_OK) return ms;
    const int32_t band_tiles = (int32_t)(dst.cols / 64), bands = (int32_t)(dst.rows / 64);
    const int64_t tiles = matrices * bands * band_tiles;
    const int64_t cap = (int64_t)sm_count() * 3;
    const unsigned grid = (unsigned)(tiles < cap ? tiles : cap);
    IPUC_CUDA(cudaFuncSetAttribute(rm_to_block_major64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BM64_SMEM));
    rm_to_block_major64_kernel<<<grid, 128, BM64_SMEM, stream>>>(map, static_cast<uint16_t *>(dst.ptr), tiles,
                                                                band_tiles, bands, dst.cols, device_error_word());
    return check_launch("rm_to_block_major64_kernel");
  }
  const bool fr = src.order == IPUC_ORDER_ROW_MAJOR, tr = dst.order == IPUC_ORDER_ROW_MAJOR;
  const int64_t lim = (int64_t)1 << 30;
  const int64_t work32 = matrices * ((dst.rows + 15) / 16) * (((dst.cols + 15) / 16 + 8 * kBlocksPerWarp - 1) / (8 * kBlocksPerWarp));
  if (src.mstride < lim && dst.mstride < lim && src.rows * src.ld < lim && dst.rows * dst.ld < lim &&
      dst.rows * dst.cols + 4096 < lim && src.rows * src.cols + 4096 < lim && work32 < lim && matrices < lim) {
    const int64_t cap = (int64_t)sm_count() * 8;
    const unsigned grid = (unsigned)(work32 < cap ? work32 : cap);
    const int32_t lr = (int32_t)(logical_rows < lim ? logical_rows : lim);
    const int32_t lc = (int32_t)(logical_cols < lim ? logical_cols : lim);
    // In-block lane layout of each side: 0 rows-outer, 1 columns-outer, 2 swizzled.
    auto kind = [](int32_t o) {
      switch (o) {
        case IPUC_ORDER_ROW_MAJOR: case IPUC_ORDER_AMP_LEFT: case IPUC_ORDER_AMP_TRANSPOSED_RIGHT:
        case IPUC_ORDER_BLOCK_MAJOR_TRANSPOSED: return 0;
        case IPUC_ORDER_AMP_TRANSPOSED_LEFT: case IPUC_ORDER_BLOCK_MAJOR: return 1;
        default: return 2;
      }
    };
    const int ks = kind(src.order), kd = kind(dst.order);
    const int mode = (ks == 2 || kd == 2) ? 0 : (ks == kd ? 1 : 2);
#define IPUC_CONVERT32(FR, TR, MODE) \
  convert_blocks32_kernel<FR, TR, MODE><<<grid, 256, 0, stream>>>(src, dst, lr, lc, (int32_t)matrices)
#define IPUC_CONVERT32_MODES(FR, TR)          \
  do {                                        \
    if (mode == 1) IPUC_CONVERT32(FR, TR, 1); \
    else if (mode == 2) IPUC_CONVERT32(FR, TR, 2); \
    else IPUC_CONVERT32(FR, TR, 0);           \
  } while (0)
    if (fr && tr) IPUC_CONVERT32_MODES(true, true);
    else if (fr) IPUC_CONVERT32_MODES(true, false);
    else if (tr) IPUC_CONVERT32_MODES(false, true);
    else IPUC_CONVERT32_MODES(false, false);
#undef IPUC_CONVERT32_MODES
#undef IPUC_CONVERT32
    return check_launch("convert_blocks32_kernel");
  }
  const int64_t want = (blocks + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  if (fr && tr) convert_blocks_kernel<true, true><<<grid, 256, 0, stream>>>(src, dst, logical_rows, logical_cols, matrices);
  else if (fr) convert_blocks_kernel<true, false><<<grid, 256, 0, stream>>>(src, dst, logical_rows, logical_cols, matrices);
  else if (tr) convert_blocks_kernel<false, true><<<grid, 256, 0, stream>>>(src, dst, logical_rows, logical_cols, matrices);
  else convert_blocks_kernel<false, false><<<grid, 256, 0, stream>>>(src, dst, logical_rows, logical_cols, matrices);
  return check_launch("convert_blocks_kernel");
}

// SplitHeads [b, r, h*c] -> [b*h, r, c]: one 8-element chunk per thread.
template <bool kVec>
__global__ void split_heads_kernel(uint16_t *__restrict__ out, const uint16_t *__restrict__ in, int64_t batch,
                                   int64_t rows, int64_t heads, int64_t channels) {
  const int64_t total = batch * heads * rows * channels;
  const int64_t step = (int64_t)gridDim.x * blockDim.x * 8;
  for (int64_t o = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; o < total; o += step) {
    if (kVec) {
      const int64_t c = o % channels, t = o / channels, r = t % rows, bh = t / rows;
      const int64_t b = bh / heads, h = bh % heads;
      const int64_t s = (b * rows + r) * heads * channels + h * channels + c;
      *reinterpret_cast<uint4 *>(out + o) = *reinterpret_cast<const uint4 *>(in + s);
    } else {
      for (int64_t e = o; e < o + 8 && e < total; ++e) {
        const int64_t c = e % channels, t = e / channels, r = t % rows, bh = t / rows;
        const int64_t b = bh / heads, h = bh % heads;
        out[e] = in[(b * rows + r) * heads * channels + h * channels + c];
      }
    }
  }
}

// MergeHeads [b*h, r, c] -> [b, r, h*c]: the inverse permutation.
template <bool kVec>
__global__ void merge_heads_kernel(uint16_t *__restrict__ out, const uint16_t *__restrict__ in, int64_t batch,
                                   int64_t rows, int64_t heads, int64_t channels) {
  const int64_t total = batch * heads * rows * channels;
  const int64_t width = heads * channels;
  const int64_t step = (int64_t)gridDim.x * blockDim.x * 8;
  for (int64_t o = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; o < total; o += step) {
    if (kVec) {
      const int64_t wc = o % width, t = o / width, r = t % rows, b = t / rows;
      const int64_t h = wc / channels, c = wc % channels;
      *reinterpret_cast<uint4 *>(out + o) = *reinterpret_cast<const uint4 *>(in + ((b * heads + h) * rows + r) * channels + c);
    } else {
      for (int64_t e = o; e < o + 8 && e < total; ++e) {
        const int64_t wc = e % width, t = e / width, r = t % rows, b = t / rows;
        out[e] = in[((b * heads + wc / channels) * rows + r) * channels + wc % channels];
      }
    }
  }
}

}  // namespace
}  // namespace ipuc

using namespace ipuc;

extern "C" ipuc_status ipuc_merge_heads_f16(void *out, const void *in, int64_t batch, int64_t rows, int64_t heads,
                                            int64_t channels, ipuc_stream stream) {
  IPUC_CHECK_ARG(batch >= 0 && rows >= 0 && heads > 0 && channels > 0, "merge_heads: bad extents");
  const int64_t total = batch * rows * heads * channels;
  if (total == 0) return IPUC_OK;
  const bool vec = channels % 8 == 0 && aligned(out, 16) && aligned(in, 16);
  const int64_t chunks = (total + 7) / 8;
  const int64_t want = (chunks + 255) / 256, cap = (int64_t)sm_count() * 16;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  if (vec)
    merge_heads_kernel<true><<<grid, 256, 0, stream>>>((uint16_t *)out, (const uint16_t *)in, batch, rows, heads, channels);
  else
    merge_heads_kernel<false><<<grid, 256, 0, stream>>>((uint16_t *)out, (const uint16_t *)in, batch, rows, heads, channels);
  return check_launch("merge_heads_kernel");
}

extern "C" ipuc_status ipuc_rearrange_f16(void *dst, const void *src, int64_t matrices, int64_t logical_rows,
                                          int64_t physical_rows, int32_t target_order, int64_t logical_columns,
                                          int64_t physical_columns, int64_t row_block, int64_t column_block,
                                          ipuc_stream stream) {
  IPUC_CHECK_ARG(matrices >= 0 && logical_rows >= 0 && logical_columns >= 0, "rearrange: negative extent");
  IPUC_CHECK_ARG(logical_rows <= physical_rows && logical_columns <= physical_columns,
                 "rearrange: logical extent exceeds physical extent");
  IPUC_CHECK_ARG(logical_columns % 2 == 0, "rearrange: logical columns must be even (rearrange_f16.cpp:34)");
  IPUC_CHECK_ARG(physical_columns % 16 == 0, "rearrange: physical columns must be a multiple of 16");
  int32_t order;
  switch (target_order) {
    case 0: order = IPUC_ORDER_AMP_LEFT; break;
    case 1:
      order = IPUC_ORDER_AMP_TRANSPOSED_RIGHT;
      if (column_block != 16) return fail(IPUC_ERR_UNSUPPORTED, "rearrange: AMP-TransposedRight supports 16-row panels");
      break;
    case 2: order = IPUC_ORDER_BLOCK_MAJOR; break;
    default: return fail(IPUC_ERR_INVALID_ARGUMENT, "rearrange: target_order must be 0, 1 or 2");
  }
  if (matrices == 0 || physical_rows == 0) return IPUC_OK;
  Side s{const_cast<void *>(src), IPUC_ORDER_ROW_MAJOR, logical_rows, logical_columns, logical_columns,
         logical_rows * logical_columns, 0, 0, 0};
  Side d{dst, order, physical_rows, physical_columns, physical_columns, physical_rows * physical_columns,
         row_block, column_block, 0};
  return launch_convert(s, d, logical_rows, logical_columns, matrices, stream);
}

extern "C" ipuc_status ipuc_unpack_f16(void *dst, const void *src, int32_t source_order, int64_t matrices,
                                       int64_t logical_rows, int64_t physical_rows, int64_t logical_columns,
                                       int64_t physical_columns, ipuc_stream stream) {
  IPUC_CHECK_ARG(matrices >= 0 && logical_rows >= 0 && logical_columns >= 0, "unpack: negative extent");
  IPUC_CHECK_ARG(logical_rows <= physical_rows && logical_columns <= physical_columns,
                 "unpack: logical extent exceeds physical extent");
  IPUC_CHECK_ARG(physical_columns % 2 == 0, "unpack: physical columns must be even (unpack_amp_f16.cpp:31)");
  int32_t order;
  if (source_order == 0) order = IPUC_ORDER_AMP_OUTPUT;
  else if (source_order == 1) order = IPUC_ORDER_AMP_TRANSPOSED_LEFT;
  else return fail(IPUC_ERR_INVALID_ARGUMENT, "unpack: source_order must be 0 (AMP-Output) or 1 (AMP-TransposedLeft)");
  if (matrices == 0 || physical_rows == 0) return IPUC_OK;
  const int64_t me = physical_rows * physical_columns;
  if (source_order == 0 && physical_columns % 16 == 0 && aligned(src, 16) && aligned(dst, 16) && src != dst) {
    const int64_t panels = physical_columns / 16;
    const int64_t tiles = matrices * ((physical_rows + UNP_ROWS - 1) / UNP_ROWS) *
                          ((panels + UNP_PANELS - 1) / UNP_PANELS);
    // 4 CTAs per SM: measured 0.89 of the copy peak on 4096 x 49152, against
    // 0.82 with 8 per SM and 0.88 with 16.
    const int64_t cap = (int64_t)sm_count() * 4, want = tiles;
    unpack_amp_output_kernel<<<(unsigned)(want < cap ? want : cap), 256, 0, stream>>>(
        static_cast<const uint16_t *>(src), static_cast<uint16_t *>(dst), matrices, physical_rows, physical_columns,
        logical_rows, logical_columns);
    return check_launch("unpack_amp_output_kernel");
  }
  Side s{const_cast<void *>(src), order, physical_rows, physical_columns, physical_columns, me, 0, 0, 0};
  Side d{dst, IPUC_ORDER_ROW_MAJOR, physical_rows, physical_columns, physical_columns, me, 0, 0, 0};
  return launch_convert(s, d, logical_rows, logical_columns, matrices, stream);
}

extern "C" ipuc_status ipuc_convert_order_f16(void *dst, ipuc_order to, const void *src, ipuc_order from,
                                              int64_t matrices, int64_t rows, int64_t columns, int64_t row_block,
                                              int64_t column_block, ipuc_stream stream) {
  IPUC_CHECK_ARG(matrices >= 0 && rows >= 0 && columns >= 0, "convert_order: negative extent");
  if (matrices == 0 || rows == 0 || columns == 0) return IPUC_OK;
  const int64_t me = rows * columns;
  Side s{const_cast<void *>(src), (int32_t)from, rows, columns, columns, me, row_block, column_block, 0};
  Side d{dst, (int32_t)to, rows, columns, columns, me, row_block, column_block, 0};
  return launch_convert(s, d, rows, columns, matrices, stream);
}

extern "C" ipuc_status ipuc_split_heads_f16(void *out, const void *in, int64_t batch, int64_t rows, int64_t heads,
                                            int64_t channels, ipuc_stream stream) {
  IPUC_CHECK_ARG(batch >= 0 && rows >= 0 && heads > 0 && channels > 0, "split_heads: bad extents");
  const int64_t total = batch * rows * heads * channels;
  if (total == 0) return IPUC_OK;
  const bool vec = channels % 8 == 0 && aligned(out, 16) && aligned(in, 16);
  const int64_t chunks = (total + 7) / 8;
  const int64_t want = (chunks + 255) / 256, cap = (int64_t)sm_count() * 16;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  if (vec)
    split_heads_kernel<true><<<grid, 256, 0, stream>>>((uint16_t *)out, (const uint16_t *)in, batch, rows, heads, channels);
  else
    split_heads_kernel<false><<<grid, 256, 0, stream>>>((uint16_t *)out, (const uint16_t *)in, batch, rows, heads, channels);
  return check_launch("split_heads_kernel");
}
