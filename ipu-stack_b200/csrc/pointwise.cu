// Pointwise and reduction kernels: tanh-GELU (device/gelu_f16.S), split-K
// reduce_add (device/reduce_add_f16.S), Add and Cast (the reference's
// Required-but-unimplemented kernels, crates/ipu-codegen/src/kernel.rs:
// 1275-1318).  All are HBM-bound: 16-byte vector loads and stores, grid
// sized to a multiple of the SM count, grid-stride loops.
#include "common.cuh"

namespace ipuc {
namespace {

unsigned grid_for(int64_t chunks, int threads) {
  const int64_t want = (chunks + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 8;
  int64_t g = want < cap ? want : cap;
  return (unsigned)(g < 1 ? 1 : g);
}

__global__ void __launch_bounds__(256) gelu_f16_kernel(uint4 *__restrict__ out, const uint4 *__restrict__ in,
                                                       int64_t chunks, const uint16_t *__restrict__ tail_in,
                                                       uint16_t *__restrict__ tail_out, int tail) {
  // Eight 16-byte chunks per thread and iteration (stride apart), all loaded
  // before any is computed, so that enough bytes are in flight per SM for the
  // kernel to stay HBM-bound (with 16 CTAs per SM: 0.94 of the copy peak on
  // config 3's 134M elements, against 0.78 with four chunks and 8 CTAs).
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  auto apply = [](uint4 &v) {
    __half2 *w = reinterpret_cast<__half2 *>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(w[j]);
      w[j] = __floats2half2_rn(gelu_f32(f.x), gelu_f32(f.y));
    }
  };
  constexpr int U = 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += U * stride) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i + u * stride < chunks) v[u] = in[i + u * stride];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i + u * stride < chunks) {
        apply(v[u]);
        out[i + u * stride] = v[u];
      }
  }
  if (blockIdx.x == 0 && (int)threadIdx.x < tail) tail_out[threadIdx.x] = f2h(gelu_f32(h2f(tail_in[threadIdx.x])));
}

// out = initial + sum_p remote[p]; T = float or uint16_t (f16).  8 elements/thread.
template <typename T>
__global__ void __launch_bounds__(256) reduce_sum_kernel(uint4 *__restrict__ out, const T *__restrict__ initial,
                                                         const T *__restrict__ remote, uint32_t partials,
                                                         int64_t n) {
  const int64_t chunks = n / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += stride) {
    float acc[8];
    if constexpr (sizeof(T) == 4) {
      const float4 *p0 = reinterpret_cast<const float4 *>(initial + i * 8);
      float4 a = p0[0], b = p0[1];
      acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w;
      acc[4] = b.x; acc[5] = b.y; acc[6] = b.z; acc[7] = b.w;
      for (uint32_t p = 0; p < partials; ++p) {
        const float4 *pp = reinterpret_cast<const float4 *>(remote + (int64_t)p * n + i * 8);
        float4 c = __ldcs(pp), d = __ldcs(pp + 1);
        acc[0] += c.x; acc[1] += c.y; acc[2] += c.z; acc[3] += c.w;
        acc[4] += d.x; acc[5] += d.y; acc[6] += d.z; acc[7] += d.w;
      }
    } else {
      uint4 a = *reinterpret_cast<const uint4 *>(initial + i * 8);
      const uint16_t *pa = reinterpret_cast<const uint16_t *>(&a);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = h2f(pa[j]);
      for (uint32_t p = 0; p < partials; ++p) {
        uint4 c = __ldcs(reinterpret_cast<const uint4 *>(remote + (int64_t)p * n + i * 8));
        const uint16_t *pc = reinterpret_cast<const uint16_t *>(&c);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += h2f(pc[j]);
      }
    }
    uint4 o;
    o.x = pack_h2(acc[0], acc[1]);
    o.y = pack_h2(acc[2], acc[3]);
    o.z = pack_h2(acc[4], acc[5]);
    o.w = pack_h2(acc[6], acc[7]);
    out[i] = o;
  }
}

__global__ void __launch_bounds__(256) add_f16_kernel(uint16_t *__restrict__ out, const uint16_t *__restrict__ l,
                                                      const uint16_t *__restrict__ r, int64_t n, int64_t lp,
                                                      int64_t rp, bool vec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 8;
  for (int64_t o = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; o < n; o += stride) {
    if (vec && o + 8 <= n) {
      const int64_t li = lp ? o % lp : o, ri = rp ? o % rp : o;
      uint4 a = *reinterpret_cast<const uint4 *>(l + li), b = *reinterpret_cast<const uint4 *>(r + ri);
      const uint32_t *pa = reinterpret_cast<const uint32_t *>(&a), *pb = reinterpret_cast<const uint32_t *>(&b);
      uint4 c;
      uint32_t *pc = reinterpret_cast<uint32_t *>(&c);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        pc[j] = pack_h2(h2f(pa[j] & 0xffffu) + h2f(pb[j] & 0xffffu), h2f(pa[j] >> 16) + h2f(pb[j] >> 16));
      *reinterpret_cast<uint4 *>(out + o) = c;
    } else {
      for (int64_t e = o; e < o + 8 && e < n; ++e)
        out[e] = f2h(h2f(l[lp ? e % lp : e]) + h2f(r[rp ? e % rp : e]));
    }
  }
}

// f16 <-> f32 in 8-element chunks: one 16-byte f16 access and two 16-byte f32
// accesses per chunk (16-byte aligned pointers; the tail goes through
// cast_kernel).
template <bool kToF32>
__global__ void __launch_bounds__(256) cast_vec_kernel(void *__restrict__ out, const void *__restrict__ in,
                                                       int64_t chunks) {
  // Four chunks per thread and iteration, all loaded before any is stored.
  constexpr int U = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunks; i += U * stride) {
    if constexpr (kToF32) {
      uint4 h[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i + u * stride < chunks) h[u] = reinterpret_cast<const uint4 *>(in)[i + u * stride];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (i + u * stride >= chunks) break;
        const __half2 *h2 = reinterpret_cast<const __half2 *>(&h[u]);
        const float2 a = __half22float2(h2[0]), b = __half22float2(h2[1]), c = __half22float2(h2[2]),
                     d = __half22float2(h2[3]);
        float4 *o = reinterpret_cast<float4 *>(out) + 2 * (i + u * stride);
        o[0] = make_float4(a.x, a.y, b.x, b.y);
        o[1] = make_float4(c.x, c.y, d.x, d.y);
      }
    } else {
      float4 f[U][2];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i + u * stride < chunks) {
          const float4 *src = reinterpret_cast<const float4 *>(in) + 2 * (i + u * stride);
          f[u][0] = src[0];
          f[u][1] = src[1];
        }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (i + u * stride >= chunks) break;
        uint4 h;
        __half2 *h2 = reinterpret_cast<__half2 *>(&h);
        h2[0] = __floats2half2_rn(f[u][0].x, f[u][0].y);
        h2[1] = __floats2half2_rn(f[u][0].z, f[u][0].w);
        h2[2] = __floats2half2_rn(f[u][1].x, f[u][1].y);
        h2[3] = __floats2half2_rn(f[u][1].z, f[u][1].w);
        reinterpret_cast<uint4 *>(out)[i + u * stride] = h;
      }
    }
  }
}

__global__ void cast_kernel(void *__restrict__ out, int to, const void *__restrict__ in, int from, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = from == IPUC_F16 ? h2f(static_cast<const uint16_t *>(in)[i]) : static_cast<const float *>(in)[i];
    if (to == IPUC_F16) static_cast<uint16_t *>(out)[i] = f2h(v);
    else static_cast<float *>(out)[i] = v;
  }
}

}  // namespace
}  // namespace ipuc

using namespace ipuc;

extern "C" ipuc_status ipuc_gelu_f16(void *out, const void *in, uint64_t element_count, ipuc_stream stream) {
  IPUC_CHECK_ARG(element_count % 2 == 0, "gelu: element count must be even (kernel.rs:1400-1413)");
  if (element_count == 0) return IPUC_OK;
  IPUC_CHECK_ARG(out && in, "gelu: null pointer");
  IPUC_CHECK_ALIGN(aligned(out, 16) && aligned(in, 16), "gelu: pointers must be 16-byte aligned");
  const int64_t chunks = (int64_t)(element_count / 8);
  const int tail = (int)(element_count % 8);
  const int64_t want = chunks > 0 ? (chunks + 255) / 256 : 1, cap = (int64_t)sm_count() * 16;
  gelu_f16_kernel<<<(unsigned)(want < cap ? want : cap), 256, 0, stream>>>(
      (uint4 *)out, (const uint4 *)in, chunks, (const uint16_t *)in + chunks * 8, (uint16_t *)out + chunks * 8, tail);
  return check_launch("gelu_f16_kernel");
}

extern "C" ipuc_status ipuc_reduce_sum(void *out, const void *initial, const void *remote, uint32_t num_partials,
                                       uint64_t element_count, ipuc_precision in_precision, ipuc_stream stream) {
  IPUC_CHECK_ARG(num_partials >= 1, "reduce_sum: needs at least two partials (kernel.rs:1414-1423)");
  IPUC_CHECK_ARG(element_count % 8 == 0, "reduce_sum: element count must be a multiple of 8 (kernel.rs:1414-1423)");
  IPUC_CHECK_ARG(in_precision == IPUC_F16 || in_precision == IPUC_F32, "reduce_sum: bad precision");
  if (element_count == 0) return IPUC_OK;
  IPUC_CHECK_ARG(out && initial && remote, "reduce_sum: null pointer");
  IPUC_CHECK_ALIGN(aligned(out, 16) && aligned(initial, 16) && aligned(remote, 16),
                   "reduce_sum: pointers must be 16-byte aligned");
  const int64_t n = (int64_t)element_count;
  const unsigned grid = grid_for(n / 8, 256);
  if (in_precision == IPUC_F32)
    reduce_sum_kernel<float><<<grid, 256, 0, stream>>>((uint4 *)out, (const float *)initial, (const float *)remote,
                                                       num_partials, n);
  else
    reduce_sum_kernel<uint16_t><<<grid, 256, 0, stream>>>((uint4 *)out, (const uint16_t *)initial,
                                                          (const uint16_t *)remote, num_partials, n);
  return check_launch("reduce_sum_kernel");
}

extern "C" ipuc_status ipuc_add_f16(void *out, const void *left, const void *right, uint64_t element_count,
                                    uint64_t left_broadcast_stride, uint64_t right_broadcast_stride,
                                    ipuc_stream stream) {
  if (element_count == 0) return IPUC_OK;
  IPUC_CHECK_ARG(out && left && right, "add: null pointer");
  IPUC_CHECK_ARG(left_broadcast_stride <= element_count && right_broadcast_stride <= element_count,
                 "add: broadcast stride exceeds element count");
  const bool vec = aligned(out, 16) && aligned(left, 16) && aligned(right, 16) && left_broadcast_stride % 8 == 0 &&
                   right_broadcast_stride % 8 == 0;
  const int64_t n = (int64_t)element_count;
  add_f16_kernel<<<grid_for((n + 7) / 8, 256), 256, 0, stream>>>((uint16_t *)out, (const uint16_t *)left,
                                                                 (const uint16_t *)right, n,
                                                                 (int64_t)left_broadcast_stride,
                                                                 (int64_t)right_broadcast_stride, vec);
  return check_launch("add_f16_kernel");
}

// f16 -> f32 over whole 4096-element tiles (8 KB in, 16 KB out): each
// thread converts 16 elements into a shared staging tile and one thread
// writes the tile out as a single 16 KB bulk copy (cp.async.bulk), two
// staging tiles in rotation.  The output is twice the input, and long
// contiguous bulk writes keep the DRAM write stream efficient.
constexpr int CAST_TILE = 4096;
__global__ void __launch_bounds__(256) cast_f16_f32_bulk_kernel(float *__restrict__ out,
                                                                const uint16_t *__restrict__ in, int64_t tiles) {
  __shared__ __align__(128) float stage[2][CAST_TILE];
  int buf = 0;
  // The next tile's 32 input bytes per thread are loaded before this tile is
  // converted, so every thread keeps a load in flight across the staging steps.
  auto load = [&](int64_t t, uint4 &a, uint4 &b) {
    const uint4 *src = reinterpret_cast<const uint4 *>(in + t * CAST_TILE) + 2 * threadIdx.x;
    a = __ldcs(src);
    b = __ldcs(src + 1);
  };
  uint4 n0 = make_uint4(0u, 0u, 0u, 0u), n1 = n0;
  if (blockIdx.x < tiles) load(blockIdx.x, n0, n1);
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, buf ^= 1) {
    const uint4 x0 = n0, x1 = n1;
    if (t + gridDim.x < tiles) load(t + gridDim.x, n0, n1);
    if (threadIdx.x == 0) {
      // the staging tile written two tiles ago has been read out by its copy
      asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    }
    __syncthreads();
    float4 *dst = reinterpret_cast<float4 *>(stage[buf]) + 4 * threadIdx.x;
    const __half2 *h0 = reinterpret_cast<const __half2 *>(&x0), *h1 = reinterpret_cast<const __half2 *>(&x1);
    float2 f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[i] = __half22float2(h0[i]);
      f[4 + i] = __half22float2(h1[i]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_float4(f[2 * i].x, f[2 * i].y, f[2 * i + 1].x, f[2 * i + 1].y);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t sa = (uint32_t)__cvta_generic_to_shared(stage[buf]);
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(out + t * CAST_TILE), "r"(sa),
                   "r"((uint32_t)(CAST_TILE * 4))
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
  if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

extern "C" ipuc_status ipuc_cast(void *out, ipuc_precision to, const void *in, ipuc_precision from,
                                 uint64_t element_count, ipuc_stream stream) {
  IPUC_CHECK_ARG((to == IPUC_F16 || to == IPUC_F32) && (from == IPUC_F16 || from == IPUC_F32), "cast: bad precision");
  if (element_count == 0) return IPUC_OK;
  IPUC_CHECK_ARG(out && in, "cast: null pointer");
  const int64_t n = (int64_t)element_count;
  if (to != from && aligned(out, 16) && aligned(in, 16) && n >= 8) {
    const int64_t tiles = to == IPUC_F32 ? n / CAST_TILE : 0;
    if (tiles > 0) {
      // 4 CTAs per SM with the load prefetch: 0.88 of the copy peak on 33.6M
      // elements, against 0.84 with 6 per SM and no prefetch.
      const int64_t cap = (int64_t)sm_count() * 4;
      cast_f16_f32_bulk_kernel<<<(unsigned)(tiles < cap ? tiles : cap), 256, 0, stream>>>(
          static_cast<float *>(out), static_cast<const uint16_t *>(in), tiles);
      const ipuc_status st = check_launch("cast_f16_f32_bulk_kernel");
      if (st != IPUC_OK) return st;
      if (tiles * CAST_TILE == n) return IPUC_OK;
      out = static_cast<float *>(out) + tiles * CAST_TILE;
      in = static_cast<const uint16_t *>(in) + tiles * CAST_TILE;
    }
    const int64_t rest = n - tiles * CAST_TILE;
    const int64_t chunks = rest / 8, done = chunks * 8;
    if (chunks == 0) {
      cast_kernel<<<1, 256, 0, stream>>>(out, to, in, from, rest);
      return check_launch("cast_kernel");
    }
    if (to == IPUC_F32)
      cast_vec_kernel<true><<<grid_for(chunks, 256), 256, 0, stream>>>(out, in, chunks);
    else
      cast_vec_kernel<false><<<grid_for(chunks, 256), 256, 0, stream>>>(out, in, chunks);
    if (done < rest) {
      const size_t ob = to == IPUC_F16 ? 2 : 4, ib = from == IPUC_F16 ? 2 : 4;
      cast_kernel<<<1, 256, 0, stream>>>(static_cast<uint8_t *>(out) + done * ob, to,
                                         static_cast<const uint8_t *>(in) + done * ib, from, rest - done);
    }
    return check_launch("cast_vec_kernel");
  }
  cast_kernel<<<grid_for(n, 256), 256, 0, stream>>>(out, to, in, from, n);
  return check_launch("cast_kernel");
}
