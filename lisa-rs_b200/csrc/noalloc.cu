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
#include "prefill.cuh"

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
  if (capacity == 0 || ((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15)) return LISA_EINVAL;
  if (((uintptr_t)q_gate & 15) || ((uintptr_t)q_norm_w & 15)) return LISA_EINVAL;
  if ((uint64_t)base + rows > capacity) return LISA_ENOSPC;
  if ((uint64_t)base + rows > NOALLOC_MAX_POS) return LISA_E2BIG;  // beyond the fixed scratch

  float* scratch = nullptr;
  int s = scratch_for_current_device(&scratch);
  if (s != LISA_OK) return s;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);

  DecodeParams p = {};
  p.q_gate = q_gate;
  p.k_in = k;
  p.v_in = v;
  p.in_bf16 = in_dtype == LISA_DTYPE_BF16;
  p.q_norm_w = q_norm_w;
  p.k_norm_w = k_norm_w;
  p.eps = eps;
  p.k_cache = static_cast<uint16_t*>(k_cache);
  p.v_cache = static_cast<uint16_t*>(v_cache);
  p.window_rows = capacity;
  p.kv_lo = 0;
  p.base = base;
  p.extent = base + (uint32_t)rows;
  p.nchunks = (p.extent + DEC_CHUNK - 1) / DEC_CHUNK;
  p.chunk_cap = NOALLOC_CHUNKS;
  p.part_o = scratch;
  p.part_ml = scratch + NOALLOC_PO;
  p.err = reinterpret_cast<int*>(scratch + NOALLOC_PO + NOALLOC_PM);
  p.sched = reinterpret_cast<uint32_t*>(scratch + NOALLOC_PO + NOALLOC_PM + 16);
  p.gated_out = gated_out;
  // Partials are fully written before they are read; the error word and the
  // chunk counters must start at zero.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(p.err, 0, 128, st) != cudaSuccess) return LISA_ECUDA;
  CUtensorMap tk, tv;
  if (lisa_encode_group_map(&tk, k_cache, p.extent, capacity, KVH, DEC_TILE, 4) != LISA_OK ||
      lisa_encode_group_map(&tv, v_cache, p.extent, capacity, KVH, DEC_TILE, 4) != LISA_OK)
    return LISA_ECUDA;
  return launch_decode(p, rows, tk, tv, sms, st) == cudaSuccess ? LISA_OK : LISA_ECUDA;
}
#pragma GCC visibility pop
