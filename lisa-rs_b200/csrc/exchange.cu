// exchange.cu — multi-GPU split-KV decode of one long sequence with the
// window partials exchanged through peer memory (CUDA IPC over NVLink /
// NVSwitch) instead of a collective library call.
//
// Each rank holds one contiguous window of the sequence's KV positions. Per
// step, on every rank, on one stream:
//   decode_split_kernel    streams the window (appending the new rows when the
//                          window owns them), chunk partials to the workspace
//   decode_combine_kernel  folds the chunks into one window partial per
//                          (row, head) and stores it straight into every
//                          rank's receive region (peer stores), each value in
//                          one 8-byte word with the step number beside it
//   merge_exchange_kernel  waits (bounded) until the words it needs from every
//                          rank carry this step, merges the partials by
//                          log-sum-exp in rank order and applies the gate
// Tagging every word with its step (the low-latency protocol of collective
// libraries) needs neither a flag nor a memory fence: an aligned 8-byte store
// is seen whole or not at all. A first version that published one flag per
// block after the data saw stale data on 4 GPUs once the fences were removed.
// Receive regions are double-buffered by step parity: a rank can only publish
// step e+2 after finishing step e+1, which needed every rank's step-e+1
// partials, which each rank published after finishing its step-e merge; so
// the parity-e data a slow rank is still reading is never overwritten.
// Words hold the step number, so the region is never cleared. The step
// counter lives on the device (advanced by the merge kernel), so a step can be
// captured in a CUDA graph and replayed.
//
// Reference: lisa-rs drives one GPU and has no multi-device code; the merge is
// the log-sum-exp combine of sdpa_decode_final (attention.metal:611-641) taken
// across GPUs.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/lisa_attn.h"
#include "common.cuh"
#include "decode.cuh"
#include "dispatch.h"

using namespace lisa;

struct lisa_attn_xchg {
  int device = 0;
  int world = 1;
  int rank = 0;
  int max_rows = 3;
  uint32_t window_rows = 0;
  uint8_t* region = nullptr;     // receive region (tagged words), exported by IPC
  size_t region_bytes = 0;
  uint32_t* state = nullptr;     // local only: step counter, merge CTAs done, error word
  XchgDev* dev = nullptr;        // device copy of the peer table
  void* workspace = nullptr;     // window workspace (chunk partials, error word, chunk counters)
  size_t workspace_bytes = 0;
  void* peer_base[XCHG_MAX_WORLD] = {};  // IPC mappings of the other ranks' regions
  bool opened = false;
};

namespace {


struct DevGuard {
  int prev = -1;
  explicit DevGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DevGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

void release(lisa_attn_xchg* x) {
  for (int i = 0; i < XCHG_MAX_WORLD; ++i)
    if (x->peer_base[i]) cudaIpcCloseMemHandle(x->peer_base[i]);
  cudaFree(x->region);
  cudaFree(x->state);
  cudaFree(x->dev);
  cudaFree(x->workspace);
  delete x;
}

}  // namespace

#pragma GCC visibility push(default)
extern "C" {

int lisa_attn_xchg_create(int device, int world, int rank, int max_rows, uint32_t window_rows,
                          lisa_attn_xchg** out) {
  if (!out || world < 1 || world > XCHG_MAX_WORLD || rank < 0 || rank >= world || max_rows < 1 || max_rows > 3 ||
      window_rows == 0 || window_rows > (1u << 31))
    return LISA_EINVAL;
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return LISA_EINVAL;
  DevGuard guard(device);
  lisa_attn_xchg* x = new lisa_attn_xchg();
  x->device = device;
  x->world = world;
  x->rank = rank;
  x->max_rows = max_rows;
  x->window_rows = window_rows;
  x->region_bytes = xchg_recv_words(world, max_rows) * sizeof(uint64_t);
  x->workspace_bytes = lisa_attn_window_workspace_bytes(window_rows, max_rows);
  bool ok = cudaMalloc(&x->region, x->region_bytes) == cudaSuccess &&
            cudaMalloc(&x->state, 256) == cudaSuccess && cudaMalloc(&x->dev, sizeof(XchgDev)) == cudaSuccess &&
            cudaMalloc(&x->workspace, x->workspace_bytes) == cudaSuccess;
  ok = ok && cudaMemset(x->region, 0, x->region_bytes) == cudaSuccess &&
       cudaMemset(x->state, 0, 256) == cudaSuccess && cudaMemset(x->workspace, 0, 256) == cudaSuccess &&
       cudaDeviceSynchronize() == cudaSuccess;
  if (!ok) {
    release(x);
    return LISA_ECUDA;
  }
  *out = x;
  return LISA_OK;
}

int lisa_attn_xchg_handle(lisa_attn_xchg* x, void* handle_out) {
  if (!x || !handle_out) return LISA_EINVAL;
  DevGuard guard(x->device);
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, x->region) != cudaSuccess) return LISA_ECUDA;
  static_assert(sizeof(h) == LISA_ATTN_XCHG_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  return LISA_OK;
}

int lisa_attn_xchg_open(lisa_attn_xchg* x, const void* handles) {
  if (!x || !handles || x->opened) return LISA_EINVAL;
  DevGuard guard(x->device);
  XchgDev d = {};
  d.world = x->world;
  d.rank = x->rank;
  d.max_rows = x->max_rows;
  d.state = x->state;
  for (int i = 0; i < x->world; ++i) {
    uint8_t* base = nullptr;
    if (i == x->rank) {
      base = x->region;
    } else {
      cudaIpcMemHandle_t h;
      memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)i * sizeof(h), sizeof(h));
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return LISA_ECUDA;
      x->peer_base[i] = p;
      base = static_cast<uint8_t*>(p);
    }
    d.recv[i] = reinterpret_cast<uint64_t*>(base);
  }
  if (cudaMemcpy(x->dev, &d, sizeof(d), cudaMemcpyHostToDevice) != cudaSuccess) return LISA_ECUDA;
  x->opened = true;
  return LISA_OK;
}

int lisa_attn_xchg_decode(lisa_attn_xchg* x, void* k_cache, void* v_cache, uint32_t kv_lo, uint32_t base, int rows,
                          int in_dtype, const void* q_gate, const void* k, const void* v, const uint16_t* q_norm_w,
                          const uint16_t* k_norm_w, float eps, uint16_t* gated_out, void* stream) {
  if (!x || !x->opened) return LISA_ESTATE;
  if (!k_cache || !v_cache || !q_gate || !k || !v || !q_norm_w || !k_norm_w || !gated_out) return LISA_EINVAL;
  if (rows < 1 || rows > x->max_rows || rows == 2) return LISA_EINVAL;
  if (in_dtype != LISA_DTYPE_F32 && in_dtype != LISA_DTYPE_BF16) return LISA_EINVAL;
  if (((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15)) return LISA_EINVAL;
  if ((uint64_t)base + rows > (uint64_t)1 << 31) return LISA_ENOSPC;
  DevGuard guard(x->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint32_t chunks = (x->window_rows + DEC_CHUNK - 1) / DEC_CHUNK;
  const size_t po = (size_t)x->max_rows * KVH * chunks * 2048 * sizeof(float);
  uint8_t* ws = static_cast<uint8_t*>(x->workspace);
  // error word and chunk counters at the head of the workspace; the word stays
  // set until lisa_attn_xchg_check_device_error clears it
  const WaitFault wf = current_wait_fault();
  int s = run_decode(static_cast<uint16_t*>(k_cache), static_cast<uint16_t*>(v_cache), x->window_rows, kv_lo, base,
                     rows, in_dtype, q_gate, k, v, q_norm_w, k_norm_w, eps, reinterpret_cast<float*>(ws + 256),
                     reinterpret_cast<float*>(ws + 256 + ((po + 255) & ~size_t(255))), chunks,
                     reinterpret_cast<int*>(ws), reinterpret_cast<uint32_t*>(ws + 64), nullptr, nullptr, nullptr,
                     current_device_sms(), st, x->dev);
  if (s != LISA_OK) return s;
  const cudaError_t e = launch_merge_exchange(x->dev, rows, in_dtype == LISA_DTYPE_BF16, q_gate, gated_out,
                                              wf.limit_ns ? wf.limit_ns : WAIT_LIMIT_NS, st);
  return e == cudaSuccess ? LISA_OK : LISA_ECUDA;
}

int lisa_attn_xchg_check_device_error(lisa_attn_xchg* x, void* stream) {
  if (!x) return LISA_EINVAL;
  DevGuard guard(x->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int h[2] = {0, 0};
  if (cudaMemcpyAsync(&h[0], x->workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(&h[1], x->state + 2, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return LISA_ECUDA;
  if ((h[0] || h[1]) && (cudaMemsetAsync(x->workspace, 0, sizeof(int), st) != cudaSuccess ||
                         cudaMemsetAsync(x->state + 2, 0, sizeof(int), st) != cudaSuccess ||
                         cudaStreamSynchronize(st) != cudaSuccess))
    return LISA_ECUDA;
  return (h[0] || h[1]) ? LISA_ETIMEOUT : LISA_OK;
}

int lisa_attn_xchg_destroy(lisa_attn_xchg* x) {
  if (!x) return LISA_EINVAL;
  DevGuard guard(x->device);
  cudaDeviceSynchronize();
  release(x);
  return LISA_OK;
}

}  // extern "C"
#pragma GCC visibility pop
