// Peer-memory all-reduce of f16 values over NVLink: the sharded session's
// sum across ranks after a row-split GEMM (the transformer block's out-proj
// and MLP-down), done by this library's own kernel on buffers every rank maps
// through CUDA IPC, in place of ncclAllReduce.  The arithmetic is the
// reference's cross-tile partial sum (ipu_stack_reduce_sum_f16,
// device/reduce_add_f16.S:31-72: out = p0 + sum_i p_i over remote partials),
// with the partials on other GPUs instead of other tiles, summed in f32 in
// rank order and rounded to f16 once, so every rank gets the same bits.
//
// Two-shot schedule, one launch of kBlocks CTAs per rank (all co-resident):
//   1. CTA b tells CTA b of every peer that this rank's input is complete
//      (stream order: the producing GEMM finished before this launch) and waits
//      for the same word from every peer.
//   2. Rank r sums slice r of all ranks' inputs (CTA b takes chunk b of the
//      slice) with 16-byte peer loads and stores the f16 sum into slice r of
//      every rank's output (its own included) with 16-byte peer stores.
//   3. CTA b signals completion to every peer's CTA b and waits for theirs; a
//      rank's launch ends only when every peer has pushed its slices, and every
//      peer has finished reading this rank's input.
// Flags are per (phase, sender, CTA) words holding a per-CTA call counter kept
// in the receiver's own signal area, so repeated calls (and graph replays)
// need no reset.  Waits are bounded by the global timer: on expiry the CTA
// records the device error word and returns (no trap); the counters of the
// ranks are then out of step and the signal area must be re-created.
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace ipuc {
namespace {

constexpr int kBlocks = 128;
constexpr int kThreads = 512;
constexpr int kMaxWorld = 8;
constexpr uint32_t ERR_KERNEL_PEER_REDUCE = 6u << 16;
// Signal area (uint32 words): flag[phase][sender][block], then epoch[block].
constexpr uint64_t kFlagWords = 2ull * kMaxWorld * kBlocks;
constexpr uint64_t kSignalWords = kFlagWords + kBlocks;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

struct PeerPtrs {
  const uint4 *in[kMaxWorld];
  uint4 *out[kMaxWorld];
  uint32_t *sig[kMaxWorld];
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// CTA-wide cross-rank barrier for `phase`: returns false if a peer's word did
// not arrive within the limit (error word recorded).
__device__ bool peer_barrier(const PeerPtrs &a, int rank, int world, int phase, uint32_t epoch, uint32_t *err) {
  __shared__ int s_ok;
  const int b = blockIdx.x;
  // Every thread's own stores into peers' memory (and local ones peers will
  // read) complete at system scope before the CTA's signal can be seen.
  fence_sys();
  __syncthreads();
  if (threadIdx.x == 0) {
    s_ok = 1;
    for (int q = 0; q < world; ++q)
      st_release_sys(a.sig[q] + ((uint64_t)phase * kMaxWorld + rank) * kBlocks + b, epoch);
  }
  __syncthreads();
  if (threadIdx.x < world) {
    const uint32_t *w = a.sig[rank] + ((uint64_t)phase * kMaxWorld + threadIdx.x) * kBlocks + b;
    const uint64_t t0 = sm100::global_timer_ns();
    uint32_t spins = 0;
    while ((int32_t)(ld_acquire_sys(w) - epoch) < 0) {
      if ((++spins & 255u) == 0 && sm100::global_timer_ns() - t0 > kWaitLimitNs) {
        record_device_error(err, ERR_KERNEL_PEER_REDUCE | (uint32_t)(phase + 1));
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  fence_sys();
  return s_ok != 0;
}

__device__ __forceinline__ void add_h8(float (&acc)[8], const uint4 &v) {
  const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}

__device__ __forceinline__ uint4 pack_h8(const float (&acc)[8]) {
  uint4 r;
  r.x = pack_h2(acc[0], acc[1]);
  r.y = pack_h2(acc[2], acc[3]);
  r.z = pack_h2(acc[4], acc[5]);
  r.w = pack_h2(acc[6], acc[7]);
  return r;
}

template <int W>
__global__ void __launch_bounds__(kThreads, 1)
    peer_all_reduce_kernel(PeerPtrs a, int rank, uint64_t slice_vecs, uint32_t *err) {
  const int b = blockIdx.x;
  uint32_t *epoch_word = a.sig[rank] + kFlagWords + b;
  const uint32_t epoch = *epoch_word + 1;
  if (!peer_barrier(a, rank, W, 0, epoch, err)) return;

  const uint64_t chunk = (slice_vecs + kBlocks - 1) / kBlocks;
  const uint64_t base = (uint64_t)rank * slice_vecs;
  const uint64_t lo = base + (uint64_t)b * chunk;
  const uint64_t hi = base + min(slice_vecs, (uint64_t)(b + 1) * chunk);
  // vectors per thread per pass: W * U = 16 loads of 16 bytes in flight per thread
  constexpr int U = W <= 2 ? 8 : W <= 4 ? 4 : 2;
  for (uint64_t i0 = lo + threadIdx.x; i0 < hi; i0 += (uint64_t)kThreads * U) {
    uint4 v[U][W];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t i = i0 + (uint64_t)u * kThreads;
      if (i < hi) {
#pragma unroll
        for (int q = 0; q < W; ++q) v[u][q] = a.in[q][i];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t i = i0 + (uint64_t)u * kThreads;
      if (i < hi) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < W; ++q) add_h8(acc, v[u][q]);
        const uint4 r = pack_h8(acc);
#pragma unroll
        for (int q = 0; q < W; ++q) a.out[q][i] = r;
      }
    }
  }

  if (!peer_barrier(a, rank, W, 1, epoch, err)) return;
  if (threadIdx.x == 0) *epoch_word = epoch;
}

}  // namespace
}  // namespace ipuc

using namespace ipuc;

extern "C" uint64_t ipuc_peer_signal_bytes(void) { return kSignalWords * sizeof(uint32_t); }

namespace {
// cuMemGetAddressRange through the runtime's driver entry point (the library
// links only the runtime): the base of the allocation holding `p`.
using AddressRangeFn = int (*)(unsigned long long *, size_t *, unsigned long long);
ipuc_status allocation_base(const void *p, uintptr_t *base) {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(f);
  });
  if (!fn) return fail(IPUC_ERR_CUDA, "ipc: cuMemGetAddressRange is unavailable");
  unsigned long long b = 0;
  size_t bytes = 0;
  if (fn(&b, &bytes, (unsigned long long)(uintptr_t)p) != 0)
    return fail(IPUC_ERR_INVALID_ARGUMENT, "ipc: pointer is not device memory of this process");
  *base = (uintptr_t)b;
  return IPUC_OK;
}
}  // namespace

extern "C" ipuc_status ipuc_ipc_handle(const void *device_ptr, void *handle_out, uint64_t size, uint64_t *offset) {
  IPUC_CHECK_ARG(device_ptr && handle_out && offset, "ipc_handle: null pointer");
  IPUC_CHECK_ARG(size >= sizeof(cudaIpcMemHandle_t), "ipc_handle: needs a 64-byte buffer");
  uintptr_t base = 0;
  if (ipuc_status st = allocation_base(device_ptr, &base)) return st;
  cudaIpcMemHandle_t h;
  IPUC_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base)));
  memcpy(handle_out, &h, sizeof(h));
  *offset = (uint64_t)((uintptr_t)device_ptr - base);
  return IPUC_OK;
}

extern "C" ipuc_status ipuc_ipc_open(const void *handle, uint64_t offset, void **device_ptr) {
  IPUC_CHECK_ARG(handle && device_ptr, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  IPUC_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *device_ptr = static_cast<char *>(base) + offset;
  return IPUC_OK;
}

extern "C" ipuc_status ipuc_ipc_close(void *device_ptr) {
  IPUC_CHECK_ARG(device_ptr, "ipc_close: null pointer");
  uintptr_t base = 0;
  if (ipuc_status st = allocation_base(device_ptr, &base)) return st;
  IPUC_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void *>(base)));
  return IPUC_OK;
}

extern "C" ipuc_status ipuc_peer_all_reduce_f16(void *const *inputs, void *const *outputs, void *const *signals,
                                                int32_t rank, int32_t world, uint64_t element_count,
                                                ipuc_stream stream) {
  IPUC_CHECK_ARG(inputs && outputs && signals, "peer_all_reduce: null pointer table");
  IPUC_CHECK_ARG(world >= 2 && world <= kMaxWorld, "peer_all_reduce: world must lie in [2, 8]");
  IPUC_CHECK_ARG(rank >= 0 && rank < world, "peer_all_reduce: rank must lie in [0, world)");
  IPUC_CHECK_ARG(element_count % (8ull * (uint64_t)world) == 0,
                 "peer_all_reduce: element count must be a multiple of 8 * world");
  if (element_count == 0) return IPUC_OK;
  PeerPtrs a = {};
  for (int q = 0; q < world; ++q) {
    IPUC_CHECK_ARG(inputs[q] && outputs[q] && signals[q], "peer_all_reduce: null buffer");
    IPUC_CHECK_ALIGN(aligned(inputs[q], 16) && aligned(outputs[q], 16) && aligned(signals[q], 16),
                     "peer_all_reduce: buffers must be 16-byte aligned");
    a.in[q] = static_cast<const uint4 *>(inputs[q]);
    a.out[q] = static_cast<uint4 *>(outputs[q]);
    a.sig[q] = static_cast<uint32_t *>(signals[q]);
  }
  uint32_t *err = device_error_word();
  const uint64_t slice_vecs = element_count / 8 / (uint64_t)world;
  const cudaStream_t s = stream;
  switch (world) {
    case 2: peer_all_reduce_kernel<2><<<kBlocks, kThreads, 0, s>>>(a, rank, slice_vecs, err); break;
    case 3: peer_all_reduce_kernel<3><<<kBlocks, kThreads, 0, s>>>(a, rank, slice_vecs, err); break;
    case 4: peer_all_reduce_kernel<4><<<kBlocks, kThreads, 0, s>>>(a, rank, slice_vecs, err); break;
    case 5: peer_all_reduce_kernel<5><<<kBlocks, kThreads, 0, s>>>(a, rank, slice_vecs, err); break;
    case 6: peer_all_reduce_kernel<6><<<kBlocks, kThreads, 0, s>>>(a, rank, slice_vecs, err); break;
    case 7: peer_all_reduce_kernel<7><<<kBlocks, kThreads, 0, s>>>(a, rank, slice_vecs, err); break;
    default: peer_all_reduce_kernel<8><<<kBlocks, kThreads, 0, s>>>(a, rank, slice_vecs, err); break;
  }
  return check_launch("peer_all_reduce_kernel");
}

