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
// same x (q, k, v fused). One persistent CTA per SM: a producer warp moves
// blocks of 32 (or 16) consecutive rows (packed words, scales, biases: three
// bulk copies) through a ring of shared-memory stages, and one consumer warp
// per two rows of a block: lane l dequantises the 32-element chunks l, l + 32, ... (a
// nibble dropped into the mantissa of 2^23, minus 2^23: no int -> float
// conversion) and dots them with x in packed f32x2 FMAs, each x chunk read
// from shared memory once for both rows (x, not the weights, is most of the
// shared-memory traffic: 32 f32 per 16 bytes of packed weights). x is staged in shared
// memory as f32, one 32-element chunk per 36-float slot, so a quarter warp's
// 16-byte reads of 8 consecutive chunks hit 8 disjoint bank quads; the
// per-chunk sums of x (for the bias term) sit after it.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "../../include/lisa_attn.h"
#include "common.cuh"
#include "dispatch.h"

namespace lisa {

namespace {

// Rows per stage (BR): 32 for M <= 2 when x and two such stages fit in shared
// memory (K <= 6144 at M = 1), else 16; the verify shapes always take 16, as
// their larger accumulators would spill with 16 consumer warps. Measured at
// M = 1, K = 5120 (q/k/v fused): 14.7 us with 32 rows and 2 rows per warp,
// 16.0 with 16 and 2, 15.3 with 32 and 4, 16.6 with 16 and 4, 17.5 with one
// row per warp.
constexpr int QMV_RPW = 2;  // rows per consumer warp: each x chunk read from shared memory serves both
__host__ __device__ constexpr int qmv_cw(int br) { return br / QMV_RPW; }  // consumer warps
constexpr int QMV_STAGES = 4;  // weight blocks in flight per SM (fewer when x is large)
constexpr int QMV_MAX_M = LISA_ATTN_QMV_MAX_ROWS;
constexpr int QMV_MAX_PROJ = LISA_ATTN_QMV_MAX_PROJ;
constexpr int QMV_SLOT = 36;  // floats per staged 32-element chunk of x

struct QmvProj {
  const uint32_t* packed;   // [N][K/8]
  const uint16_t* scales;   // [N][K/64] bf16
  const uint16_t* biases;   // [N][K/64] bf16
  float* out;               // [M][N]
  int n;
  int grp0;                 // first row block of this projection in the launch's list
};

struct QmvParams {
  int m, k, n_proj, groups;  // groups: blocks of rows (one stage each) over all projections
  int stages;                // ring depth (2..QMV_STAGES, as shared memory allows)
  const uint16_t* x;         // [M][K] bf16
  QmvProj proj[QMV_MAX_PROJ];
};

}  // namespace

// Persistent, one CTA per SM: a producer warp streams blocks of QMV_BR
// consecutive weight rows of the projections (packed words, scales and biases
// by bulk copies) through a ring of up to QMV_STAGES shared-memory stages
// (mbarrier full / empty), and QMV_BR / 2 consumer warps dequantise and dot them
// against x (staged once per CTA as f32). The ring keeps the stages' weights
// in flight per SM whatever the registers.
template <int M, int QMV_BR>
__global__ void __launch_bounds__(32 * (qmv_cw(QMV_BR) + 1), 1) qmv_u4_kernel(const __grid_constant__ QmvParams p) {
  constexpr int QMV_CW = qmv_cw(QMV_BR);
  extern __shared__ __align__(16) uint8_t qmv_smem_raw[];
  const int K = p.k;
  const int chunks = K / 32, groups_k = K / 64;
  const size_t row_bytes = (size_t)K / 2;
  // [x: M][chunks][QMV_SLOT] f32 | xsum [M][chunks] | stages | barriers
  float* xs = reinterpret_cast<float*>(qmv_smem_raw);
  float* xsum = xs + (size_t)M * chunks * QMV_SLOT;
  const size_t x_bytes = (((size_t)M * chunks * (QMV_SLOT + 1)) * sizeof(float) + 127) & ~size_t(127);
  const size_t sg_bytes = ((size_t)QMV_BR * groups_k * 2 + 15) & ~size_t(15);  // bf16 scales (then biases) of a block
  const size_t stage_bytes = (QMV_BR * row_bytes + 2 * sg_bytes + 127) & ~size_t(127);
  uint8_t* stages = qmv_smem_raw + x_bytes;
  const int n_st = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + n_st * stage_bytes);
  uint64_t* empty = full + n_st;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_blocks = p.groups;  // blocks of QMV_BR rows over all projections

  if (threadIdx.x == 0) {
    for (int s = 0; s < n_st; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], QMV_CW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == QMV_CW) {
    // ---------------- producer ----------------
    // The weights are never written by a kernel: streaming starts before the
    // wait on the previous kernel (which may produce x).
    int it = 0;
    for (int blk = blockIdx.x; blk < n_blocks; blk += gridDim.x, ++it) {
      const int s = it % n_st;
      if (it >= n_st && !mbar_wait(&empty[s], ((it / n_st) - 1) & 1, nullptr, 0)) break;
      int pi = 0;
      while (pi + 1 < p.n_proj && blk >= p.proj[pi + 1].grp0) ++pi;
      const QmvProj& pr = p.proj[pi];
      const int row0 = (blk - pr.grp0) * QMV_BR;
      const int nrows = min(QMV_BR, pr.n - row0);
      uint8_t* st = stages + (size_t)s * stage_bytes;
      // packed rows, scales and biases of the block are each contiguous:
      // three bulk copies (sizes rounded down to 16 bytes; a short tail of the
      // scales / biases is copied by the lanes)
      const uint32_t pk_bytes = (uint32_t)(nrows * row_bytes);
      const uint32_t g_bytes = (uint32_t)(nrows * groups_k * 2);
      const uint32_t g_bulk = g_bytes & ~15u;
      const uint8_t* sc_src = reinterpret_cast<const uint8_t*>(pr.scales + (size_t)row0 * groups_k);
      const uint8_t* bi_src = reinterpret_cast<const uint8_t*>(pr.biases + (size_t)row0 * groups_k);
      uint8_t* sc_dst = st + QMV_BR * row_bytes;
      uint8_t* bi_dst = sc_dst + sg_bytes;
      for (uint32_t b = g_bulk + 2 * lane; b < g_bytes; b += 64) {
        *reinterpret_cast<uint16_t*>(sc_dst + b) = *reinterpret_cast<const uint16_t*>(sc_src + b);
        *reinterpret_cast<uint16_t*>(bi_dst + b) = *reinterpret_cast<const uint16_t*>(bi_src + b);
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], pk_bytes + 2 * g_bulk);  // also publishes the lanes' tail stores
        bulk_load(st, reinterpret_cast<const uint8_t*>(pr.packed) + (size_t)row0 * row_bytes, pk_bytes, &full[s]);
        if (g_bulk) {
          bulk_load(sc_dst, sc_src, g_bulk, &full[s]);
          bulk_load(bi_dst, bi_src, g_bulk, &full[s]);
        }
      }
    }
    return;
  }

  pdl_wait_primary();
  pdl_launch_dependents();
  // x arrives as 16-byte vectors of 8 bf16 (a run of 8 never crosses a row)
  for (int e8 = threadIdx.x; e8 < M * K / 8; e8 += 32 * QMV_CW) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.x) + e8);
    const int m = (8 * e8) / K, k = 8 * e8 - m * K;
    float4* dst = reinterpret_cast<float4*>(xs + ((size_t)m * chunks + (k >> 5)) * QMV_SLOT + (k & 31));
    const float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y), c2 = unpack_bf16x2(v.z), d = unpack_bf16x2(v.w);
    dst[0] = make_float4(a.x, a.y, b.x, b.y);
    dst[1] = make_float4(c2.x, c2.y, d.x, d.y);
  }
  named_bar_sync(1, 32 * QMV_CW);
  for (int e = threadIdx.x; e < M * chunks; e += 32 * QMV_CW) {
    const float* sl = xs + (size_t)e * QMV_SLOT;
    float sum = 0.f;
#pragma unroll 8
    for (int i = 0; i < 32; ++i) sum += sl[i];
    xsum[e] = sum;
  }
  named_bar_sync(1, 32 * QMV_CW);

  // Consumer warp w takes rows QMV_RPW * w .. of each stage; lane l the
  // 32-element chunks l, l + 32, ... of K, each x chunk read once for all of
  // the warp's rows.
  int it = 0;
  for (int blk = blockIdx.x; blk < n_blocks; blk += gridDim.x, ++it) {
    const int s = it % n_st;
    if (!mbar_wait(&full[s], (it / n_st) & 1, nullptr, 0)) break;
    int pi = 0;
    while (pi + 1 < p.n_proj && blk >= p.proj[pi + 1].grp0) ++pi;
    const QmvProj& pr = p.proj[pi];
    const int lr0 = warp * QMV_RPW;  // first local row of this warp
    const int row0 = (blk - pr.grp0) * QMV_BR + lr0;
    const uint8_t* st = stages + (size_t)s * stage_bytes;
    if (row0 < pr.n) {
      const uint16_t* scr = reinterpret_cast<const uint16_t*>(st + QMV_BR * row_bytes) + (size_t)lr0 * groups_k;
      const uint16_t* bir =
          reinterpret_cast<const uint16_t*>(st + QMV_BR * row_bytes + sg_bytes) + (size_t)lr0 * groups_k;
      float acc[QMV_RPW][M];
#pragma unroll
      for (int j = 0; j < QMV_RPW; ++j)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[j][m] = 0.f;
      for (int c = lane; c < chunks; c += 32) {
        // nibble 2i is the low half of byte i, nibble 2i+1 the high half; a
        // nibble placed in the low mantissa bits of 2^23 is 2^23 + q, and
        // 2^23 + q - 2^23 = q exactly (no int -> float conversion)
        float2 qv[QMV_RPW][16];
#pragma unroll
        for (int j = 0; j < QMV_RPW; ++j) {
          const uint4 w4 = reinterpret_cast<const uint4*>(st + (size_t)(lr0 + j) * row_bytes)[c];
#pragma unroll
          for (int wq = 0; wq < 4; ++wq) {
            const uint32_t word = (&w4.x)[wq];
            const uint32_t lo = word & 0x0F0F0F0Fu, hi = (word >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t sel = (uint32_t)i | 0x7540u;  // byte i of the nibbles, then 00 00 4B
              qv[j][4 * wq + i] = fadd2(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, sel)),
                                                    __uint_as_float(__byte_perm(hi, 0x4B000000u, sel))),
                                        make_float2(-8388608.0f, -8388608.0f));
            }
          }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float4* xm = reinterpret_cast<const float4*>(xs + ((size_t)m * chunks + c) * QMV_SLOT);
          float2 dot[QMV_RPW];
#pragma unroll
          for (int j = 0; j < QMV_RPW; ++j) dot[j] = make_float2(0.f, 0.f);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 x4 = xm[q];
#pragma unroll
            for (int j = 0; j < QMV_RPW; ++j) {
              dot[j] = ffma2(make_float2(x4.x, x4.y), qv[j][2 * q], dot[j]);
              dot[j] = ffma2(make_float2(x4.z, x4.w), qv[j][2 * q + 1], dot[j]);
            }
          }
          const float xsc = xsum[m * chunks + c];
#pragma unroll
          for (int j = 0; j < QMV_RPW; ++j) {
            const float scale = bf16_bits_to_f32(scr[j * groups_k + (c >> 1)]);
            const float bias = bf16_bits_to_f32(bir[j * groups_k + (c >> 1)]);
            acc[j][m] += fmaf(scale, dot[j].x + dot[j].y, bias * xsc);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
      for (int j = 0; j < QMV_RPW; ++j) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
          float v = acc[j][m];
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
          if (lane == 0 && row0 + j < pr.n) pr.out[(size_t)m * pr.n + row0 + j] = v;
        }
      }
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
}

}  // namespace lisa

using namespace lisa;

namespace {

constexpr size_t kSmemMax = 227 * 1024;

size_t qmv_x_bytes(int m, int k) { return ((size_t)m * (k / 32) * (QMV_SLOT + 1) * sizeof(float) + 127) & ~size_t(127); }
size_t qmv_stage_bytes(int br, int k) {
  const size_t sg = ((size_t)br * (k / 64) * 2 + 15) & ~size_t(15);
  return ((size_t)br * k / 2 + 2 * sg + 127) & ~size_t(127);
}
int qmv_stages(int br, int m, int k) {
  const size_t room = kSmemMax - qmv_x_bytes(m, k) - 2 * QMV_STAGES * sizeof(uint64_t);
  return (int)std::max<size_t>(2, std::min<size_t>(QMV_STAGES, room / qmv_stage_bytes(br, k)));
}
size_t qmv_smem_bytes(int br, int m, int k) {
  const int st = qmv_stages(br, m, k);
  return qmv_x_bytes(m, k) + st * qmv_stage_bytes(br, k) + 2 * st * sizeof(uint64_t);
}
int qmv_rows_per_stage(int m, int k) { return m <= 2 && qmv_smem_bytes(32, m, k) <= kSmemMax ? 32 : 16; }

template <int M, int BR>
cudaError_t launch_m(cudaLaunchConfig_t& cfg, const QmvParams& p) {
  static SmemAttr attr_once;  // per kernel and device, for the largest request
  const cudaError_t e = attr_once.ensure(qmv_u4_kernel<M, BR>, (int)kSmemMax);
  return e == cudaSuccess ? cudaLaunchKernelEx(&cfg, qmv_u4_kernel<M, BR>, p) : e;
}

}  // namespace

#pragma GCC visibility push(default)
extern "C" int lisa_attn_qmv_u4(int n_proj, const lisa_attn_q4_proj* projs, int rows, int k, const uint16_t* x,
                                void* stream) {
  if (n_proj < 1 || n_proj > QMV_MAX_PROJ || !projs || !x || ((uintptr_t)x & 15)) return LISA_EINVAL;
  if (rows < 1 || rows > QMV_MAX_M || k < 64 || k % 64 != 0 || k > LISA_ATTN_QMV_MAX_K) return LISA_EINVAL;
  QmvParams p = {};
  p.m = rows;
  p.k = k;
  p.n_proj = n_proj;
  p.x = x;
  const int br = qmv_rows_per_stage(rows, k);
  int blocks = 0;  // blocks of br rows over all projections
  for (int i = 0; i < n_proj; ++i) {
    const lisa_attn_q4_proj& q = projs[i];
    if (!q.packed || !q.scales || !q.biases || !q.out || q.n < 1) return LISA_EINVAL;
    if ((uintptr_t)q.packed & 15) return LISA_EINVAL;  // bulk copies of packed rows
    p.proj[i] = QmvProj{static_cast<const uint32_t*>(q.packed), q.scales, q.biases, q.out, q.n, blocks};
    blocks += (q.n + br - 1) / br;
  }
  p.groups = blocks;
  p.stages = qmv_stages(br, rows, k);
  if (qmv_smem_bytes(br, rows, k) > kSmemMax) return LISA_EINVAL;  // x and two weight stages must fit
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(current_device_sms(), blocks));
  cfg.blockDim = dim3(32 * (qmv_cw(br) + 1));
  cfg.dynamicSmemBytes = qmv_smem_bytes(br, rows, k);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (rows) {
    case 1: e = br == 32 ? launch_m<1, 32>(cfg, p) : launch_m<1, 16>(cfg, p); break;
    case 2: e = br == 32 ? launch_m<2, 32>(cfg, p) : launch_m<2, 16>(cfg, p); break;
    case 3: e = launch_m<3, 16>(cfg, p); break;
    default: e = launch_m<4, 16>(cfg, p); break;
  }
  return e == cudaSuccess ? LISA_OK : LISA_ECUDA;
}
#pragma GCC visibility pop
