// noalloc.cu — lisa_attn_decode_noalloc: the split-KV decode / verify of one
// layer over a caller-owned KV cache, for callers that cannot allocate device
// memory at call time (for example a host engine whose memory pool is handed
// out once at start-up, or code running where cudaMalloc is not allowed).
//
// Its scratch (the per-chunk partials of the split-KV kernel and the device
// error word) lives in one file-scope __device__ array of fixed size, so the
// call itself allocates nothing. Every GPU that loads this library holds the
// array until the process exits. All calls on a device share it and it keeps
// the last call's contents, so calls that overlap on the GPU (different
// streams, or different host threads) race and must be serialised by the
// caller.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/lisa_attn.h"
#include "common.cuh"
#include "decode.cuh"
#include "dispatch.h"

using namespace lisa;

namespace {

constexpr uint32_t NOALLOC_MAX_POS = LISA_ATTN_NOALLOC_MAX_POSITIONS;
constexpr uint32_t NOALLOC_CHUNKS = (NOALLOC_MAX_POS + DEC_CHUNK - 1) / DEC_CHUNK;
constexpr int NOALLOC_ROWS = 3;
constexpr size_t NOALLOC_PO = (size_t)NOALLOC_ROWS * KVH * NOALLOC_CHUNKS * 2048;  // floats
constexpr size_t NOALLOC_PM = (size_t)NOALLOC_ROWS * KVH * NOALLOC_CHUNKS * 16;    // floats
constexpr size_t NOALLOC_FLOATS = NOALLOC_PO + NOALLOC_PM + 64;  // + error word, chunk counters

// The fixed scratch. In host code `g_noalloc_scratch` is only a stand-in
// symbol, not a device address; the device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_FLOATS];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
float* g_scratch_ptr[MAX_DEVICES] = {};

// Device address of the scratch on the current device (looked up once per
// device, with that device current).
int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return LISA_ECUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    float* p = nullptr;
    if (cudaGetSymbolAddress((void**)&p, g_noalloc_scratch) != cudaSuccess || !p) return LISA_ECUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return LISA_OK;
}

}  // namespace

#pragma GCC visibility push(default)
extern "C" int lisa_attn_decode_noalloc(void* k_cache, void* v_cache, uint32_t capacity, uint32_t base, int rows,
                                        int in_dtype, const void* q_gate, const void* k, const void* v,
                                        const uint16_t* q_norm_w, const uint16_t* k_norm_w, float eps,
                                        uint16_t* gated_out, void* stream) {
  if (!k_cache || !v_cache || !q_gate || !k || !v || !q_norm_w || !k_norm_w || !gated_out) return LISA_EINVAL;
  if (rows != 1 && rows != 3) return LISA_EINVAL;
  if (in_dtype != LISA_DTYPE_F32 && in_dtype != LISA_DTYPE_BF16) return LISA_EINVAL;
  if (capacity == 0 || capacity > (1u << 31)) return LISA_EINVAL;  // as lisa_attn_create
  if (((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15)) return LISA_EINVAL;
  if ((uint64_t)base + rows > capacity) return LISA_ENOSPC;
  if ((uint64_t)base + rows > NOALLOC_MAX_POS) return LISA_E2BIG;  // beyond the fixed scratch

  float* scratch = nullptr;
  int s = scratch_for_current_device(&scratch);
  if (s != LISA_OK) return s;
  int* err = reinterpret_cast<int*>(scratch + NOALLOC_PO + NOALLOC_PM);
  uint32_t* sched = reinterpret_cast<uint32_t*>(scratch + NOALLOC_PO + NOALLOC_PM + 16);
  // Partials are fully written before they are read; the error word (read
  // back by lisa_attn_noalloc_check_device_error) and the chunk counters must
  // start at zero.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(err, 0, 128, st) != cudaSuccess) return LISA_ECUDA;
  return run_decode(static_cast<uint16_t*>(k_cache), static_cast<uint16_t*>(v_cache), capacity, 0, base, rows,
                    in_dtype, q_gate, k, v, q_norm_w, k_norm_w, eps, scratch, scratch + NOALLOC_PO, NOALLOC_CHUNKS,
                    err, sched, gated_out, nullptr, nullptr, current_device_sms(), st);
}

// Reads the error word the last lisa_attn_decode_noalloc call on the current
// device left in the fixed scratch: synchronises the device, returns LISA_OK
// or LISA_ETIMEOUT (a bounded wait of that call gave up and its output is not
// valid) and clears the word. Allocates nothing.
extern "C" int lisa_attn_noalloc_check_device_error(void) {
  float* scratch = nullptr;
  int s = scratch_for_current_device(&scratch);
  if (s != LISA_OK) return s;
  if (cudaDeviceSynchronize() != cudaSuccess) return LISA_ECUDA;
  int h = 0;
  int* err = reinterpret_cast<int*>(scratch + NOALLOC_PO + NOALLOC_PM);
  if (cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return LISA_ECUDA;
  if (h && cudaMemset(err, 0, sizeof(int)) != cudaSuccess) return LISA_ECUDA;
  return h ? LISA_ETIMEOUT : LISA_OK;
}
#pragma GCC visibility pop
