// runtime.cu — the C ABI of include/lisa_attn.h: context (KV cache + scratch
// ownership), argument checks, the KV position contract, tensor-map encoding
// and kernel dispatch. Host code only; the kernels live in decode.cu and
// prefill.cu.
//
// Reference counterparts: QwenRunner/MtpRunner in lisa-rs src/model/runner.rs
// (KV allocation 384-390, reset 423-444, restore 476-503, encode_attention
// 1426-1592, encode_prefill_attention 1962-2062, commit_verified_prefix
// 911-944, MTP checkpoint/trim/set_position 2376-2545).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "../../include/lisa_attn.h"
#include "decode.cuh"
#include "prefill.cuh"
#include "common.cuh"
#include "dispatch.h"
#include "ctx.h"

using namespace lisa;


namespace {

constexpr int MAX_DECODE_ROWS = 3;

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

// Tensor map over a bf16 [planes][window_rows][256] array seen as 64-dim
// groups: dims {64, rows, 4 groups, planes} (strides 512 B, 128 B,
// window_rows * 512 B); boxes {64, box_rows, box_groups, 1} with 128-byte
// swizzle land in shared memory as [group][row][64 dims], one 128-byte row per
// (group, row); positions >= rows read as zero.
int lisa_encode_group_map(CUtensorMap* map, const void* base, uint32_t rows, uint32_t window_rows, uint32_t planes,
                          uint32_t box_rows, uint32_t box_groups) {
  auto enc = get_encode();
  if (!enc) return LISA_ECUDA;
  cuuint64_t dims[4] = {64, rows, 4, planes};
  cuuint64_t strides[3] = {512, 128, (cuuint64_t)window_rows * 512};
  cuuint32_t box[4] = {64, box_rows, box_groups, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LISA_OK : LISA_ECUDA;
}

// Tensor map over a bf16 [rows][heads][head_elems] array (row stride
// row_elems) seen as 64-element groups: dims {64, rows, groups, heads} with
// strides {row_elems * 2, 128, head_elems * 2} bytes; boxes {64, box_rows, 4,
// 1} (one head, four groups) with 128-byte swizzle, [group][row][64] in
// shared memory. Rows >= `rows` read as zero and are not written.
int lisa_encode_rows_map(CUtensorMap* map, const void* base, uint32_t rows, uint32_t row_elems, uint32_t groups,
                         uint32_t heads, uint32_t head_elems, uint32_t box_rows) {
  auto enc = get_encode();
  if (!enc) return LISA_ECUDA;
  cuuint64_t dims[4] = {64, rows, groups, heads};
  cuuint64_t strides[3] = {(cuuint64_t)row_elems * 2, 128, (cuuint64_t)head_elems * 2};
  cuuint32_t box[4] = {64, box_rows, 4, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LISA_OK : LISA_ECUDA;
}

namespace lisa {

namespace {
std::atomic<uint64_t> g_fault_limit_ns{0};
std::atomic<int> g_fault_withhold{0};
}  // namespace


WaitFault current_wait_fault() {
  return WaitFault{g_fault_limit_ns.load(std::memory_order_relaxed), g_fault_withhold.load(std::memory_order_relaxed)};
}

int current_device_sms() {
  static std::mutex mu;
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms[dev] = 148;
  return sms[dev];
}

int run_decode(uint16_t* kc, uint16_t* vc, uint32_t window_rows, uint32_t kv_lo, uint32_t base, int rows,
               int in_dtype, const void* q_gate, const void* k, const void* v, const uint16_t* qn,
               const uint16_t* kn, float eps, float* part_o, float* part_ml, uint32_t chunk_cap, int* err,
               uint32_t* sched, uint16_t* gated, float* win_o, float* win_ml, int num_sms, cudaStream_t stream,
               const XchgDev* xchg) {
  DecodeParams p = {};
  p.q_gate = q_gate;
  p.k_in = k;
  p.v_in = v;
  p.in_bf16 = in_dtype == LISA_DTYPE_BF16;
  p.q_norm_w = qn;
  p.k_norm_w = kn;
  p.eps = eps;
  p.k_cache = kc;
  p.v_cache = vc;
  p.window_rows = window_rows;
  p.kv_lo = kv_lo;
  p.base = base;
  const int64_t want = (int64_t)base + rows - (int64_t)kv_lo;
  p.extent = (uint32_t)std::max<int64_t>(1, std::min<int64_t>(want, window_rows));
  p.nchunks = (p.extent + DEC_CHUNK - 1) / DEC_CHUNK;
  p.chunk_cap = chunk_cap;
  p.part_o = part_o;
  p.part_ml = part_ml;
  p.err = err;
  const WaitFault wf = current_wait_fault();
  p.wait_ns = wf.limit_ns ? wf.limit_ns : WAIT_LIMIT_NS;
  p.withhold = wf.withhold;
  p.sched = sched;
  p.gated_out = gated;
  p.win_o = win_o;
  p.win_ml = win_ml;
  p.xchg = xchg;
  if (p.nchunks > chunk_cap) return LISA_EINVAL;
  // the kernel bulk-copies q rows and the q gains: 16-byte alignment required
  if (((uintptr_t)q_gate & 15) || ((uintptr_t)qn & 15)) return LISA_EINVAL;
  CUtensorMap tk, tv;
  int s = lisa_encode_group_map(&tk, kc, p.extent, window_rows, KVH, DEC_TILE, 4);
  if (s == LISA_OK) s = lisa_encode_group_map(&tv, vc, p.extent, window_rows, KVH, DEC_TILE, 4);
  if (s != LISA_OK) return s;
  return launch_decode(p, rows, tk, tv, num_sms, stream) == cudaSuccess ? LISA_OK : LISA_ECUDA;
}

}  // namespace lisa

namespace {

int cuda_status(cudaError_t e) { return e == cudaSuccess ? LISA_OK : LISA_ECUDA; }

size_t layer_elems(const lisa_attn_ctx* c) { return (size_t)KVH * c->capacity * HD; }

bool bad_dtype(int d) { return d != LISA_DTYPE_F32 && d != LISA_DTYPE_BF16; }

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

int check_layer_args(lisa_attn_ctx* c, int layer, int in_dtype, const void* q_gate, const void* k, const void* v,
                     const uint16_t* qn, const uint16_t* kn, const void* out) {
  if (!c || layer < 0 || layer >= c->n_layers || bad_dtype(in_dtype)) return LISA_EINVAL;
  if (!q_gate || !k || !v || !qn || !kn || !out) return LISA_EINVAL;
  return LISA_OK;
}

}  // namespace

#pragma GCC visibility push(default)
extern "C" {

int lisa_attn_create(int device, int n_layers, uint32_t capacity, lisa_attn_ctx** out) {
  if (!out || n_layers <= 0 || capacity == 0 || capacity > (1u << 31)) return LISA_EINVAL;
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return LISA_EINVAL;
  DeviceGuard guard(device);
  lisa_attn_ctx* c = new lisa_attn_ctx();
  c->device = device;
  c->n_layers = n_layers;
  c->capacity = capacity;
  c->chunk_cap = (capacity + DEC_CHUNK - 1) / DEC_CHUNK;
  c->num_sms = current_device_sms();
  const size_t cache_bytes = (size_t)n_layers * layer_elems(c) * sizeof(uint16_t);
  const size_t po = (size_t)MAX_DECODE_ROWS * KVH * c->chunk_cap * 2048 * sizeof(float);
  const size_t pm = (size_t)MAX_DECODE_ROWS * KVH * c->chunk_cap * 16 * sizeof(float);
  c->prefill_ws_bytes = prefill_workspace_bytes();
  bool ok = cudaMalloc(&c->k, cache_bytes) == cudaSuccess && cudaMalloc(&c->v, cache_bytes) == cudaSuccess &&
            cudaMalloc(&c->part_o, po) == cudaSuccess && cudaMalloc(&c->part_ml, pm) == cudaSuccess &&
            cudaMalloc(&c->prefill_ws, c->prefill_ws_bytes) == cudaSuccess &&
            cudaMalloc(&c->err, sizeof(int)) == cudaSuccess && cudaMalloc(&c->sched, 64) == cudaSuccess;
  ok = ok && cudaMemset(c->k, 0, cache_bytes) == cudaSuccess && cudaMemset(c->v, 0, cache_bytes) == cudaSuccess &&
       cudaMemset(c->prefill_ws, 0, c->prefill_ws_bytes) == cudaSuccess &&
       cudaMemset(c->err, 0, sizeof(int)) == cudaSuccess && cudaMemset(c->sched, 0, 64) == cudaSuccess &&
       cudaDeviceSynchronize() == cudaSuccess;
  // Tensor maps of every layer's K and V over the whole capacity (64-position
  // boxes of all four dim groups), kept on the device for the batched decode,
  // whose sequences each bring their own maps.
  ok = ok && cudaMalloc(&c->tmaps, (size_t)n_layers * 2 * sizeof(CUtensorMap)) == cudaSuccess;
  if (ok) {
    CUtensorMap* h = new CUtensorMap[(size_t)n_layers * 2];
    for (int l = 0; ok && l < n_layers; ++l) {
      const size_t off = (size_t)l * layer_elems(c);
      ok = lisa_encode_group_map(&h[2 * l], c->k + off, capacity, capacity, KVH, DEC_TILE, 4) == LISA_OK &&
           lisa_encode_group_map(&h[2 * l + 1], c->v + off, capacity, capacity, KVH, DEC_TILE, 4) == LISA_OK;
    }
    ok = ok && cudaMemcpy(c->tmaps, h, (size_t)n_layers * 2 * sizeof(CUtensorMap), cudaMemcpyHostToDevice) ==
                   cudaSuccess;
    delete[] h;
  }
  if (!ok) {
    lisa_attn_destroy(c);
    return LISA_ECUDA;
  }
  *out = c;
  return LISA_OK;
}

int lisa_attn_destroy(lisa_attn_ctx* c) {
  if (!c) return LISA_EINVAL;
  DeviceGuard guard(c->device);
  cudaFree(c->k);
  cudaFree(c->v);
  cudaFree(c->part_o);
  cudaFree(c->part_ml);
  cudaFree(c->prefill_ws);
  cudaFree(c->err);
  cudaFree(c->sched);
  cudaFree(c->tmaps);
  delete c;
  return LISA_OK;
}

int lisa_attn_kv_cache(lisa_attn_ctx* c, int layer, void** k_cache, void** v_cache) {
  if (!c || layer < 0 || layer >= c->n_layers || !k_cache || !v_cache) return LISA_EINVAL;
  *k_cache = c->k + (size_t)layer * layer_elems(c);
  *v_cache = c->v + (size_t)layer * layer_elems(c);
  return LISA_OK;
}

uint32_t lisa_attn_capacity(const lisa_attn_ctx* c) { return c ? c->capacity : 0; }
int lisa_attn_n_layers(const lisa_attn_ctx* c) { return c ? c->n_layers : 0; }

int lisa_attn_decode(lisa_attn_ctx* c, int layer, uint32_t base, int rows, int in_dtype, const void* q_gate,
                     const void* k, const void* v, const uint16_t* qn, const uint16_t* kn, float eps,
                     uint16_t* gated_out, void* stream) {
  int s = check_layer_args(c, layer, in_dtype, q_gate, k, v, qn, kn, gated_out);
  if (s != LISA_OK) return s;
  if (rows != 1 && rows != 3) return LISA_EINVAL;  // encode_attention serves batch 1 and 3
  if ((uint64_t)base + rows > c->capacity) return LISA_ENOSPC;
  DeviceGuard guard(c->device);
  const size_t off = (size_t)layer * layer_elems(c);
  return run_decode(c->k + off, c->v + off, c->capacity, 0, base, rows, in_dtype, q_gate, k, v, qn, kn, eps,
                    c->part_o, c->part_ml, c->chunk_cap, c->err, c->sched, gated_out, nullptr, nullptr, c->num_sms,
                    (cudaStream_t)stream);
}

int lisa_attn_prefill_chunk(lisa_attn_ctx* c, int layer, uint32_t base, int rows, int in_dtype,
                            const void* q_gate, const void* k, const void* v, const uint16_t* qn,
                            const uint16_t* kn, float eps, uint16_t* gated_out, void* stream) {
  int s = check_layer_args(c, layer, in_dtype, q_gate, k, v, qn, kn, gated_out);
  if (s != LISA_OK) return s;
  if (rows < 1 || rows > PF_MAX_ROWS) return LISA_EINVAL;
  // vector loads of the inputs and TMA on q_gate / gated_out: 16-byte alignment
  if (((uintptr_t)q_gate | (uintptr_t)k | (uintptr_t)v | (uintptr_t)gated_out) & 15) return LISA_EINVAL;
  if ((uint64_t)base + rows > c->capacity) return LISA_ENOSPC;
  DeviceGuard guard(c->device);
  const size_t off = (size_t)layer * layer_elems(c);
  PrefillParams p = {};
  p.q_gate = q_gate;
  p.k_in = k;
  p.v_in = v;
  p.in_bf16 = in_dtype == LISA_DTYPE_BF16;
  p.q_norm_w = qn;
  p.k_norm_w = kn;
  p.eps = eps;
  p.k_cache = c->k + off;
  p.v_cache = c->v + off;
  p.capacity = c->capacity;
  p.base = base;
  p.rows = rows;
  p.q_ws = reinterpret_cast<uint16_t*>(c->prefill_ws);
  p.gated_out = gated_out;
  p.err = c->err;
  return cuda_status(launch_prefill(p, c->num_sms, (cudaStream_t)stream));
}

uint32_t lisa_attn_position(const lisa_attn_ctx* c) { return c ? c->position : 0; }

int lisa_attn_advance(lisa_attn_ctx* c, int rows, int is_verify) {
  if (!c || rows < 1 || rows > PF_MAX_ROWS || (is_verify && rows != 3)) return LISA_EINVAL;
  if ((uint64_t)c->position + rows > c->capacity) return LISA_ENOSPC;
  if (is_verify) {
    c->verify_pending = true;
    c->verify_base = c->position;
  } else {
    c->verify_pending = false;
  }
  c->position += rows;
  return LISA_OK;
}

int lisa_attn_commit_verified_prefix(lisa_attn_ctx* c, int rows) {
  if (!c) return LISA_EINVAL;
  if (!c->verify_pending) return LISA_ESTATE;  // "no pending block-3 verification"
  c->verify_pending = false;                   // take() consumes it even on a bad row count
  if (rows < 1 || rows > 3) return LISA_EINVAL;
  c->position = c->verify_base + (uint32_t)rows;
  return LISA_OK;
}

int lisa_attn_trim_state(lisa_attn_ctx* c, uint32_t count) {
  if (!c) return LISA_EINVAL;
  if (count > c->position) return LISA_ESTATE;
  c->position -= count;
  return LISA_OK;
}

int lisa_attn_set_position(lisa_attn_ctx* c, uint32_t position) {
  if (!c) return LISA_EINVAL;
  if (position > c->position) return LISA_ESTATE;
  c->position = position;
  return LISA_OK;
}

int lisa_attn_restore_position(lisa_attn_ctx* c, uint32_t position) {
  if (!c) return LISA_EINVAL;
  if (position > c->capacity) return LISA_ENOSPC;
  c->position = position;
  c->verify_pending = false;
  return LISA_OK;
}

int lisa_attn_reset_state(lisa_attn_ctx* c, void* stream) {
  if (!c) return LISA_EINVAL;
  DeviceGuard guard(c->device);
  const size_t bytes = (size_t)c->n_layers * layer_elems(c) * sizeof(uint16_t);
  cudaError_t e = cudaMemsetAsync(c->k, 0, bytes, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(c->v, 0, bytes, (cudaStream_t)stream);
  if (e != cudaSuccess) return LISA_ECUDA;
  c->position = 0;
  c->verify_pending = false;
  return LISA_OK;
}

size_t lisa_attn_snapshot_bytes(const lisa_attn_ctx* c) {
  return c ? 2 * (size_t)c->n_layers * layer_elems(c) * sizeof(uint16_t) : 0;
}

int lisa_attn_kv_snapshot(lisa_attn_ctx* c, void* dst, size_t dst_bytes, uint32_t* position_out, void* stream) {
  if (!c || !dst) return LISA_EINVAL;
  const size_t half = lisa_attn_snapshot_bytes(c) / 2;
  if (dst_bytes < 2 * half) return LISA_EINVAL;
  DeviceGuard guard(c->device);
  cudaError_t e = cudaMemcpyAsync(dst, c->k, half, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync((uint8_t*)dst + half, c->v, half, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
  if (e != cudaSuccess) return LISA_ECUDA;
  if (position_out) *position_out = c->position;
  return LISA_OK;
}

int lisa_attn_kv_restore(lisa_attn_ctx* c, const void* src, size_t src_bytes, uint32_t position, void* stream) {
  if (!c || !src) return LISA_EINVAL;
  if (position > c->capacity) return LISA_ENOSPC;  // runner.rs:2404-2409
  const size_t half = lisa_attn_snapshot_bytes(c) / 2;
  if (src_bytes < 2 * half) return LISA_EINVAL;
  DeviceGuard guard(c->device);
  cudaError_t e = cudaMemcpyAsync(c->k, src, half, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(c->v, (const uint8_t*)src + half, half, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
  if (e != cudaSuccess) return LISA_ECUDA;
  c->position = position;
  c->verify_pending = false;
  return LISA_OK;
}

int lisa_attn_check_device_error(lisa_attn_ctx* c) {
  if (!c) return LISA_EINVAL;
  DeviceGuard guard(c->device);
  if (cudaDeviceSynchronize() != cudaSuccess) return LISA_ECUDA;
  int h = 0;
  if (cudaMemcpy(&h, c->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return LISA_ECUDA;
  if (h) {
    cudaMemset(c->err, 0, sizeof(int));
    // a prefill launch that gave up may have left a split-merge ticket taken
    cudaMemset(static_cast<uint8_t*>(c->prefill_ws) + prefill_ticket_offset(), 0, prefill_ticket_bytes());
    cudaDeviceSynchronize();
  }
  return h ? LISA_ETIMEOUT : LISA_OK;
}

// Window workspace layout: [0, 256) the device error word (offset 0) and the
// four chunk counters (offset 64); then the chunk partials O and (max, sum),
// each 256-byte aligned.
size_t lisa_attn_window_workspace_bytes(uint32_t window_rows, int rows) {
  if (window_rows == 0 || rows < 1 || rows > MAX_DECODE_ROWS) return 0;
  const size_t chunks = (window_rows + DEC_CHUNK - 1) / DEC_CHUNK;
  const size_t po = (size_t)rows * KVH * chunks * 2048 * sizeof(float);
  const size_t pm = (size_t)rows * KVH * chunks * 16 * sizeof(float);
  return 256 + ((po + 255) & ~size_t(255)) + ((pm + 255) & ~size_t(255));
}

int lisa_attn_decode_window(void* k_cache, void* v_cache, uint32_t window_rows, uint32_t kv_lo, uint32_t base,
                            int rows, int in_dtype, const void* q_gate, const void* k, const void* v,
                            const uint16_t* qn, const uint16_t* kn, float eps, float* part_o, float* part_ml,
                            void* workspace, size_t workspace_bytes, void* stream) {
  if (!k_cache || !v_cache || window_rows == 0 || rows < 1 || rows > MAX_DECODE_ROWS || bad_dtype(in_dtype))
    return LISA_EINVAL;
  if (!q_gate || !k || !v || !qn || !kn || !part_o || !part_ml || !workspace) return LISA_EINVAL;
  if (((uintptr_t)workspace & 255) || ((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15)) return LISA_EINVAL;
  if (window_rows > (1u << 31)) return LISA_EINVAL;  // row stride limit of the tensor maps
  const size_t need = lisa_attn_window_workspace_bytes(window_rows, rows);
  if (workspace_bytes < need) return LISA_EINVAL;
  if ((uint64_t)base + rows > (uint64_t)1 << 31) return LISA_ENOSPC;
  const uint32_t chunks = (window_rows + DEC_CHUNK - 1) / DEC_CHUNK;
  const size_t po = (size_t)rows * KVH * chunks * 2048 * sizeof(float);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  int* err = reinterpret_cast<int*>(ws);
  uint32_t* sched = reinterpret_cast<uint32_t*>(ws + 64);
  float* wo = reinterpret_cast<float*>(ws + 256);
  float* wm = reinterpret_cast<float*>(ws + 256 + ((po + 255) & ~size_t(255)));
  // The error word (read back by lisa_attn_window_check_device_error) and the
  // chunk counters start at zero on every call.
  if (cudaMemsetAsync(ws, 0, 128, (cudaStream_t)stream) != cudaSuccess) return LISA_ECUDA;
  return run_decode((uint16_t*)k_cache, (uint16_t*)v_cache, window_rows, kv_lo, base, rows, in_dtype, q_gate, k, v,
                    qn, kn, eps, wo, wm, chunks, err, sched, nullptr, part_o, part_ml, current_device_sms(),
                    (cudaStream_t)stream);
}

int lisa_attn_window_check_device_error(void* workspace, void* stream) {
  if (!workspace || ((uintptr_t)workspace & 255)) return LISA_EINVAL;
  int h = 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return LISA_ECUDA;
  if (h && cudaMemsetAsync(workspace, 0, sizeof(int), st) != cudaSuccess) return LISA_ECUDA;
  return h ? LISA_ETIMEOUT : LISA_OK;
}

int lisa_attn_debug_wait_fault(uint32_t wait_limit_us, int withhold_loads) {
  if (withhold_loads && wait_limit_us == 0) return LISA_EINVAL;  // a withheld load needs a short limit
  if (wait_limit_us > 10u * 1000u * 1000u) return LISA_EINVAL;
  g_fault_limit_ns.store((uint64_t)wait_limit_us * 1000u, std::memory_order_relaxed);
  g_fault_withhold.store(withhold_loads ? 1 : 0, std::memory_order_relaxed);
  return LISA_OK;
}

int lisa_attn_merge_windows(int n_parts, int rows, const float* part_o, const float* part_ml, int in_dtype,
                            const void* q_gate, uint16_t* gated_out, void* stream) {
  if (n_parts < 1 || rows < 1 || rows > MAX_DECODE_ROWS || !part_o || !part_ml || !q_gate || !gated_out ||
      bad_dtype(in_dtype))
    return LISA_EINVAL;
  return cuda_status(launch_merge_windows(n_parts, rows, part_o, part_ml, in_dtype == LISA_DTYPE_BF16, q_gate,
                                          gated_out, (cudaStream_t)stream));
}

const char* lisa_attn_build_info(void) {
  return "lisa_attn sm_100a: split-KV decode (mma.sync + TMA ring, 448-position chunks), tcgen05 cta_group::2 prefill";
}

}  // extern "C"
#pragma GCC visibility pop
