// gdn.cu — the Gated DeltaNet recurrence of the hybrid decoder's linear-
// attention layers (48 of its 64 layers): for every value head h and value
// column c a 128-long state row s (over the key dims) evolves per token t as
//   s <- s * decay[t][h]
//   delta = (v[t][h][c] - s . k[t][kh]) * beta[t][h]
//   s <- s + delta * k[t][kh]
//   y[t][h][c] = bf16(s . q[t][kh])
// with kh = h / repeat (value heads share key heads), all in f32.
//
// Reference: gdn_recurrence (src/kernels/shaders/gdn.metal:245-330), the same
// layouts: state [value_heads][128 value cols][128 key dims], q/k [M][key_dim],
// v inside the fused conv output [M][2 key_dim + value_dim] at offset
// 2 key_dim, beta / decay [M][value_heads], y [M][value_dim], optional
// per-token state snapshots (state_slots, slot_stride > 0) for rollback.
//
// B200 layout: one warp per (value head, value column) state row; lane l
// holds key dims l, l+32, l+64, l+96 (the reference's split), so both dot
// products are 4 FMAs per lane plus one warp reduction, and every state
// read / write is a coalesced 128-byte access per dim quarter. Eight warps
// (eight value columns of one head) share a CTA, so the token's k and q rows
// are read once from L2 and then hit L1. The state stays in registers for the
// whole call: a multi-token call (prefill chunk) streams the state once,
// however many tokens it covers. The reduction order is fixed, so a call over
// n tokens and n one-token calls give identical bits (the invariant the
// reference tests, tests/gdn_recurrence_state.rs:70-175).
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lisa_attn.h"
#include "common.cuh"

namespace lisa {

namespace {
constexpr int GDN_D = 128;
constexpr int GDN_WARPS = 8;

struct GdnParams {
  int steps, value_heads, repeat;
  const float* conv_out;
  const float* q;
  const float* k;
  const float* beta;
  const float* decay;
  float* state;
  float* y;
  float* slots;
  size_t slot_stride;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}
}  // namespace

__global__ void __launch_bounds__(32 * GDN_WARPS) gdn_recurrence_kernel(const GdnParams p) {
  pdl_wait_primary();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * GDN_WARPS + (threadIdx.x >> 5);  // value head * 128 + value column
  if (row >= p.value_heads * GDN_D) return;
  const int vh = row / GDN_D;
  const int key_heads = p.value_heads / p.repeat;
  const int key_dim = key_heads * GDN_D, value_dim = p.value_heads * GDN_D;
  const int conv_dim = 2 * key_dim + value_dim;
  const int kbase = (vh / p.repeat) * GDN_D + lane;
  float* st = p.state + (size_t)row * GDN_D + lane;
  float s0 = st[0], s1 = st[32], s2 = st[64], s3 = st[96];
  for (int t = 0; t < p.steps; ++t) {
    const float d = __ldg(p.decay + (size_t)t * p.value_heads + vh);
    const float bv = __ldg(p.beta + (size_t)t * p.value_heads + vh);
    const float* kt = p.k + (size_t)t * key_dim + kbase;
    const float* qt = p.q + (size_t)t * key_dim + kbase;
    const float k0 = __ldg(kt), k1 = __ldg(kt + 32), k2 = __ldg(kt + 64), k3 = __ldg(kt + 96);
    const float q0 = __ldg(qt), q1 = __ldg(qt + 32), q2 = __ldg(qt + 64), q3 = __ldg(qt + 96);
    const float v = __ldg(p.conv_out + (size_t)t * conv_dim + 2 * key_dim + row);
    s0 *= d;
    s1 *= d;
    s2 *= d;
    s3 *= d;
    const float kv_mem = warp_sum(s0 * k0 + s1 * k1 + s2 * k2 + s3 * k3);
    const float delta = (v - kv_mem) * bv;
    s0 += delta * k0;
    s1 += delta * k1;
    s2 += delta * k2;
    s3 += delta * k3;
    const float out = warp_sum(s0 * q0 + s1 * q1 + s2 * q2 + s3 * q3);
    if (lane == 0) p.y[(size_t)t * value_dim + row] = round_bf16(out);
    if (p.slot_stride) {
      float* sl = p.slots + (size_t)t * p.slot_stride + (size_t)row * GDN_D + lane;
      sl[0] = s0;
      sl[32] = s1;
      sl[64] = s2;
      sl[96] = s3;
    }
  }
  st[0] = s0;
  st[32] = s1;
  st[64] = s2;
  st[96] = s3;
}

}  // namespace lisa

using namespace lisa;

#pragma GCC visibility push(default)
extern "C" int lisa_attn_gdn_recurrence(int steps, int value_heads, int repeat, const float* conv_out,
                                        const float* q_norm, const float* k_norm, const float* beta,
                                        const float* decay, float* ssm_state, float* y, float* state_slots,
                                        size_t slot_stride, void* stream) {
  if (steps < 1 || value_heads < 1 || repeat < 1 || value_heads % repeat) return LISA_EINVAL;
  if (!conv_out || !q_norm || !k_norm || !beta || !decay || !ssm_state || !y) return LISA_EINVAL;
  if (slot_stride && (!state_slots || slot_stride < (size_t)value_heads * GDN_D * GDN_D)) return LISA_EINVAL;
  GdnParams p = {steps, value_heads, repeat, conv_out, q_norm, k_norm, beta, decay, ssm_state, y, state_slots,
                 slot_stride};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((value_heads * GDN_D + GDN_WARPS - 1) / GDN_WARPS);
  cfg.blockDim = dim3(32 * GDN_WARPS);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gdn_recurrence_kernel, p) == cudaSuccess ? LISA_OK : LISA_ECUDA;
}
#pragma GCC visibility pop
