// Library-level entry points: version, status strings, thread-local error text,
// device error word, and FillZero.
#include <mutex>
#include <string>

#include "common.cuh"
#include "sm100.cuh"

namespace ipuc {

static thread_local std::string t_last_error;

void set_error(const std::string &msg) { t_last_error = msg; }

ipuc_status fail(ipuc_status st, const std::string &msg) {
  t_last_error = msg;
  return st;
}

ipuc_status cuda_fail(cudaError_t err, const char *what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")";
  return IPUC_ERR_CUDA;
}

static __device__ uint32_t s_device_error;

static constexpr int kMaxDevices = 64;

uint32_t *device_error_word() {
  static std::mutex mu;
  static uint32_t *words[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!words[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, s_device_error) != cudaSuccess) return nullptr;
    words[dev] = static_cast<uint32_t *>(p);
  }
  return words[dev];
}

int sm_count() {
  static int counts[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (!counts[dev]) {
    int c = 0;
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = c > 0 ? c : 148;
  }
  return counts[dev];
}

}  // namespace ipuc

using namespace ipuc;

extern "C" const char *ipuc_version(void) { return "ipuc-b200 0.1 (sm_100a)"; }

extern "C" const char *ipuc_status_string(ipuc_status status) {
  switch (status) {
    case IPUC_OK: return "IPUC_OK";
    case IPUC_ERR_INVALID_ARGUMENT: return "IPUC_ERR_INVALID_ARGUMENT";
    case IPUC_ERR_UNSUPPORTED: return "IPUC_ERR_UNSUPPORTED";
    case IPUC_ERR_ALIGNMENT: return "IPUC_ERR_ALIGNMENT";
    case IPUC_ERR_CUDA: return "IPUC_ERR_CUDA";
    case IPUC_ERR_NCCL: return "IPUC_ERR_NCCL";
    case IPUC_ERR_DEVICE_TIMEOUT: return "IPUC_ERR_DEVICE_TIMEOUT";
  }
  return "IPUC_ERR_UNKNOWN";
}

extern "C" const char *ipuc_last_error_string(void) { return t_last_error.c_str(); }

extern "C" ipuc_status ipuc_device_status(ipuc_stream stream) {
  IPUC_CUDA(cudaStreamSynchronize(stream));
  uint32_t *word = device_error_word();
  if (!word) return fail(IPUC_ERR_CUDA, "device error word unavailable");
  uint32_t value = 0;
  IPUC_CUDA(cudaMemcpy(&value, word, sizeof(value), cudaMemcpyDeviceToHost));
  if (value) {
    const uint32_t zero = 0;
    IPUC_CUDA(cudaMemcpy(word, &zero, sizeof(zero), cudaMemcpyHostToDevice));
    char buf[128];
    snprintf(buf, sizeof(buf), "device wait timed out: kernel %u site %u", value >> 16, value & 0xffffu);
    return fail(IPUC_ERR_DEVICE_TIMEOUT, buf);
  }
  return IPUC_OK;
}

// FillZero (device/static_runtime.S:269-316): the stream-ordered memset.
extern "C" ipuc_status ipuc_fill_zero(void *out, uint64_t bytes, ipuc_stream stream) {
  IPUC_CHECK_ARG(bytes % 8 == 0, "fill_zero: byte count must be a multiple of 8");
  if (bytes == 0) return IPUC_OK;
  IPUC_CHECK_ARG(out != nullptr, "fill_zero: null output");
  IPUC_CUDA(cudaMemsetAsync(out, 0, bytes, stream));
  return IPUC_OK;
}

// Self-test of the bounded-wait failure path: one thread waits on an mbarrier
// that nothing ever arrives on, gives up after `limit_ns`, records the device
// error word and returns — the same path every tensor-core kernel takes when a
// pipeline partner never signals.  No trap, no fault; the context stays usable.
namespace {
__global__ void bounded_wait_selftest_kernel(uint32_t *err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    ipuc::sm100::mbar_init(&bar, 1);
    ipuc::sm100::fence_barrier_init();
    if (!ipuc::sm100::mbar_wait_bounded(&bar, 0, nullptr, limit_ns))
      ipuc::record_device_error(err, ipuc::ERR_KERNEL_SELFTEST | ipuc::ERR_SITE_PRODUCER);
  }
}
}  // namespace

extern "C" ipuc_status ipuc_selftest_bounded_wait(uint64_t limit_ns, ipuc_stream stream) {
  IPUC_CHECK_ARG(limit_ns > 0 && limit_ns <= 10000000000ull, "selftest: limit must be in (0, 10 s]");
  uint32_t *word = device_error_word();
  if (!word) return fail(IPUC_ERR_CUDA, "device error word unavailable");
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(word, limit_ns);
  return check_launch("bounded_wait_selftest_kernel");
}
