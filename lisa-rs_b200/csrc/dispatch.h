// dispatch.h — host-side helpers shared by the C-ABI translation units
// (runtime.cu, noalloc.cu, batch.cu): the one decode dispatch routine, the
// per-device kernel attribute setup, and the test-only wait settings.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "decode.cuh"

namespace lisa {

// Split-KV decode of `rows` query rows over one cache window (a context's
// layer, a multi-GPU window, or a caller-owned cache): encodes the tensor maps
// and launches the split kernel plus its combine. part_o / part_ml hold
// chunk_cap chunks per (row, kv head); err is the device error word; sched the
// four chunk counters (zero at launch, reset by the combine). Exactly one of
// `gated` (final gated bf16 output), win_o / win_ml (window partials) and
// `xchg` (window partials published to every rank of an exchange) is used.
// Returns a LISA_* status.
int run_decode(uint16_t* kc, uint16_t* vc, uint32_t window_rows, uint32_t kv_lo, uint32_t base, int rows,
               int in_dtype, const void* q_gate, const void* k, const void* v, const uint16_t* qn,
               const uint16_t* kn, float eps, float* part_o, float* part_ml, uint32_t chunk_cap, int* err,
               uint32_t* sched, uint16_t* gated, float* win_o, float* win_ml, int num_sms, cudaStream_t stream,
               const XchgDev* xchg = nullptr);

// Number of SMs of the current device (queried once per device).
int current_device_sms();

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) is a per-device setting of
// a kernel: this sets it once for every device a kernel is launched on. One
// instance per kernel (a function-local static at the launch site).
class SmemAttr {
 public:
  template <typename Kernel>
  cudaError_t ensure(Kernel kernel, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const uint64_t bit = uint64_t(1) << dev;
    if (done_.load(std::memory_order_acquire) & bit) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mu_);
    if (done_.load(std::memory_order_relaxed) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done_.fetch_or(bit, std::memory_order_release);
    return e;
  }

 private:
  std::atomic<uint64_t> done_{0};
  std::mutex mu_;
};

// Test hook (lisa_attn_debug_wait_fault): the bounded-wait limit given to the
// decode kernels, and whether their producer withholds every load so that the
// consumers' first wait runs out. Process-wide; zero means the defaults.
struct WaitFault {
  uint64_t limit_ns;
  int withhold;
};
WaitFault current_wait_fault();

}  // namespace lisa
