// qmv.cu — affine-u4 matrix-vector products (QMV) for the decode (M=1) and
// MTP-verify (M=3) shapes: the q/k/v projections that feed the attention
// layer and the o_proj that reads its gated output.
//
// Reference: q4_qmv_fast_impl and its fused2/3/4 entry points
// (src/kernels/shaders/qmv.metal:1-133), dispatched by encode_qmv_fused
// (src/model/runner.rs:1134-1192). Weights are MLX affine 4-bit with group
// size 64: row n of a projection is K/8 uint32 words, element k in bits
// 4*(k%8) of word k/8; w[n][k] = q * scale[n][k/64] + bias[n][k/64] with bf16
// scales and biases; x is bf16, accumulation and output f32:
//   out[m][n] = sum_k x[m][k] * (q[n][k] * scale[n][k/64] + bias[n][k/64]).
//
// B200 layout. The kernel is bound by streaming the packed weights from HBM
// (K/2 + K/16 bytes per row). One launch covers up to four projections of the
// same x (q, k, v fused). A CTA of 8 warps owns 32 consecutive rows of one
// projection (16 for x with several rows); warp w takes 4 rows (2), and lane l takes the 32-element chunks
// c = l, l + 32, ... of K: one 16-byte load of packed weights per (row, chunk)
// (32 nibbles), its group's scale and bias, so the warp reads each row with
// fully coalesced 512-byte requests, four rows in flight at once. x is staged
// in shared memory as f32, one 32-element chunk per 36-float slot, so a
// quarter warp's 16-byte reads of 8 consecutive chunks hit 8 disjoint bank
// quads; the per-chunk sums of x (for the bias term) sit after it.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lisa_attn.h"
#include "common.cuh"
#include "dispatch.h"

namespace lisa {

namespace {

constexpr int QMV_WARPS = 8;  // rows per warp: 4 for one x row, 2 for 2..4 rows (register budget)
constexpr int QMV_MAX_M = LISA_ATTN_QMV_MAX_ROWS;
constexpr int QMV_MAX_PROJ = LISA_ATTN_QMV_MAX_PROJ;
constexpr int QMV_SLOT = 36;  // floats per staged 32-element chunk of x

struct QmvProj {
  const uint32_t* packed;   // [N][K/8]
  const uint16_t* scales;   // [N][K/64] bf16
  const uint16_t* biases;   // [N][K/64] bf16
  float* out;               // [M][N]
  int n;
  int cta0;                 // first CTA of this projection
};

struct QmvParams {
  int m, k, n_proj;
  const uint16_t* x;        // [M][K] bf16
  QmvProj proj[QMV_MAX_PROJ];
};

}  // namespace

template <int M, int RPW = (M == 1 ? 4 : 2)>
__global__ void __launch_bounds__(32 * QMV_WARPS, 2) qmv_u4_kernel(const __grid_constant__ QmvParams p) {
  extern __shared__ float qmv_smem[];
  const int K = p.k;
  const int chunks = K / 32;
  // xs[m][c][i] = x[m][32 c + i] (slot stride QMV_SLOT floats); xsum[m][c]
  float* xs = qmv_smem;
  float* xsum = qmv_smem + (size_t)M * chunks * QMV_SLOT;
  pdl_wait_primary();
  pdl_launch_dependents();
  for (int e = threadIdx.x; e < M * K; e += blockDim.x) {
    const int m = e / K, k = e % K;
    xs[((size_t)m * chunks + (k >> 5)) * QMV_SLOT + (k & 31)] = bf16_bits_to_f32(p.x[e]);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < M * chunks; e += blockDim.x) {
    const float* sl = xs + (size_t)e * QMV_SLOT;
    float s = 0.f;
    for (int i = 0; i < 32; ++i) s += sl[i];
    xsum[e] = s;
  }
  __syncthreads();

  int pi = 0;
  while (pi + 1 < p.n_proj && (int)blockIdx.x >= p.proj[pi + 1].cta0) ++pi;
  const QmvProj& pr = p.proj[pi];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = ((int)blockIdx.x - pr.cta0) * (RPW * QMV_WARPS) + warp * RPW;
  if (row0 >= pr.n) return;
  const int groups = K / 64;
  const int words = K / 8;

  float acc[RPW][M];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.f;

  for (int c = lane; c < chunks; c += 32) {
    uint4 w[RPW];
    float sc[RPW], bi[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int row = min(row0 + r, pr.n - 1);  // rows past N repeat the last one, never stored
      w[r] = __ldcs(reinterpret_cast<const uint4*>(pr.packed + (size_t)row * words) + c);
      sc[r] = bf16_bits_to_f32(__ldg(pr.scales + (size_t)row * groups + (c >> 1)));
      bi[r] = bf16_bits_to_f32(__ldg(pr.biases + (size_t)row * groups + (c >> 1)));
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float4* xm = reinterpret_cast<const float4*>(xs + ((size_t)m * chunks + c) * QMV_SLOT);
      float dot[RPW] = {};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 a = xm[2 * j], b4 = xm[2 * j + 1];
        const float xv[8] = {a.x, a.y, a.z, a.w, b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          const uint32_t word = (&w[r].x)[j];
#pragma unroll
          for (int b = 0; b < 8; ++b) dot[r] = fmaf(xv[b], (float)((word >> (4 * b)) & 0xfu), dot[r]);
        }
      }
      const float s = xsum[m * chunks + c];
#pragma unroll
      for (int r = 0; r < RPW; ++r) acc[r][m] += fmaf(sc[r], dot[r], bi[r] * s);
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      acc[r][m] = v;
    }
  if (lane < RPW * M) {
    const int r = lane / M, m = lane % M;
    float v = 0.f;
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr)
#pragma unroll
      for (int mm = 0; mm < M; ++mm)
        if (rr == r && mm == m) v = acc[rr][mm];
    if (row0 + r < pr.n) pr.out[(size_t)m * pr.n + row0 + r] = v;
  }
}

}  // namespace lisa

using namespace lisa;

#pragma GCC visibility push(default)
extern "C" int lisa_attn_qmv_u4(int n_proj, const lisa_attn_q4_proj* projs, int rows, int k, const uint16_t* x,
                                void* stream) {
  if (n_proj < 1 || n_proj > QMV_MAX_PROJ || !projs || !x) return LISA_EINVAL;
  if (rows < 1 || rows > QMV_MAX_M || k < 64 || k % 64 != 0 || k > LISA_ATTN_QMV_MAX_K) return LISA_EINVAL;
  QmvParams p = {};
  p.m = rows;
  p.k = k;
  p.n_proj = n_proj;
  p.x = x;
  int ctas = 0;
  for (int i = 0; i < n_proj; ++i) {
    const lisa_attn_q4_proj& q = projs[i];
    if (!q.packed || !q.scales || !q.biases || !q.out || q.n < 1) return LISA_EINVAL;
    if ((uintptr_t)q.packed & 15) return LISA_EINVAL;  // 16-byte loads of packed words
    p.proj[i] = QmvProj{static_cast<const uint32_t*>(q.packed), q.scales, q.biases, q.out, q.n, ctas};
    const int rows_per_cta = (rows == 1 ? 4 : 2) * QMV_WARPS;
    ctas += (q.n + rows_per_cta - 1) / rows_per_cta;
  }
  const size_t smem = ((size_t)rows * (k / 32) * QMV_SLOT + (size_t)rows * (k / 32)) * sizeof(float);
  // the attribute is set once per device, for the largest request
  constexpr int kMaxSmem = (QMV_MAX_M * (LISA_ATTN_QMV_MAX_K / 32) * QMV_SLOT + QMV_MAX_M * (LISA_ATTN_QMV_MAX_K / 32)) *
                           (int)sizeof(float);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(32 * QMV_WARPS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static SmemAttr a1, a2, a3, a4;
  cudaError_t e;
  switch (rows) {
    case 1: e = a1.ensure(qmv_u4_kernel<1>, kMaxSmem); if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, qmv_u4_kernel<1>, p); break;
    case 2: e = a2.ensure(qmv_u4_kernel<2>, kMaxSmem); if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, qmv_u4_kernel<2>, p); break;
    case 3: e = a3.ensure(qmv_u4_kernel<3>, kMaxSmem); if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, qmv_u4_kernel<3>, p); break;
    default: e = a4.ensure(qmv_u4_kernel<4>, kMaxSmem); if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, qmv_u4_kernel<4>, p); break;
  }
  return e == cudaSuccess ? LISA_OK : LISA_ECUDA;
}
#pragma GCC visibility pop
