// batch.cu — one decode step (M=1) of one attention layer for many independent
// sequences in three launches, instead of two launches per sequence.
//
// lisa-rs decodes one sequence at a time: encode_attention (runner.rs:
// 1426-1592) issues q norm/RoPE, the KV append, sdpa_decode_partial +
// sdpa_decode_final and the gate for batch 1. Serving many sequences with
// that launch pair per sequence and layer is bound by per-launch fixed cost,
// not by HBM. Here, per layer:
//   batch_prologue_kernel   one CTA per sequence: q RMSNorm + RoPE of the 24
//                           heads into a bf16 query workspace, k norm + RoPE
//                           and the K/V append into the sequence's own cache
//                           (attention.metal:118-197)
//   batch_split_kernel      persistent, 148 CTAs (37 per kv head): work units
//                           (sequence, kv head, 448-position chunk) of every
//                           sequence taken from one counter per kv head; a
//                           producer warp streams each unit's K/V stages with
//                           the sequence's own tensor maps (kept on the device
//                           by its context) and, with the unit's first stage,
//                           the sequence's 6 normalised query heads; 4 compute
//                           warps run the same mma.sync flash-decoding step as
//                           decode_split_kernel (attention.metal:550-604)
//   batch_combine_kernel    one CTA per (sequence, kv head): log-sum-exp merge
//                           of the sequence's chunk partials in a fixed order
//                           and the sigmoid gate (attention.metal:520-531,
//                           611-641)
// The per-sequence parameters travel in the kernel parameter block (up to
// LISA_ATTN_BATCH_MAX_SEQS sequences), so a step can be captured in a graph.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "../../include/lisa_attn.h"
#include "common.cuh"
#include "ctx.h"
#include "decode.cuh"
#include "dispatch.h"

namespace lisa {

namespace {

constexpr int BAT_MAX_SEQS = LISA_ATTN_BATCH_MAX_SEQS;
constexpr int BAT_STAGES = 3;
constexpr int BAT_Q_OFF = DEC_STAGE_BYTES;                  // Q of the unit: [8 heads][256] bf16 (6 used)
constexpr int BAT_STAGE_BYTES = DEC_STAGE_BYTES + 4096;     // K 32 KB, V 32 KB, Q 4 KB
constexpr int BAT_Q_BYTES = GQA * HD * 2;                   // 3 KB copied per unit
constexpr int BAT_XCH_OFF = BAT_STAGES * BAT_STAGE_BYTES;
constexpr int BAT_BAR_OFF = BAT_XCH_OFF + 4096;
constexpr int BAT_SMEM_BYTES = BAT_BAR_OFF + 256 + 1024;
constexpr int BAT_THREADS = 32 * 5;  // 4 compute warps + 1 producer warp
constexpr int BCMB_PHASES = 4;

struct BatchSeq {
  const CUtensorMap* tm;  // device: the layer's K map, V map at tm + 1
  uint16_t* k_cache;      // [4][capacity][256]
  uint16_t* v_cache;
  uint32_t capacity;
  uint32_t base;   // position of the new row; the sequence attends positions 0..base
  uint32_t unit0;  // first work unit of the sequence (per kv head)
  uint32_t pad;
};

struct BatchParams {
  int n_seqs;
  uint32_t total_units;  // per kv head
  uint32_t unit_cap;     // unit stride of the partial buffers
  int in_bf16;
  const void* q_gate;  // [n][24][512]
  const void* k_in;    // [n][4][256]
  const void* v_in;
  const uint16_t* q_norm_w;
  const uint16_t* k_norm_w;
  float eps;
  uint16_t* q_ws;   // [n][24][256] normalised, roped query (bf16)
  float* part_o;    // [4][unit_cap][256][8]
  float* part_ml;   // [4][unit_cap][2][8]
  int* err;
  uint32_t* sched;  // [4] unit counters: zero at launch, reset by the combine
  uint64_t wait_ns;
  int withhold;
  uint16_t* gated_out;  // [n][6144]
  float inv_freq[32];
  BatchSeq seq[BAT_MAX_SEQS];
};

struct UnitInfo {
  int unit;       // -1: no more work
  uint32_t row0;  // position of the stage's first row
  uint32_t lim;   // the sequence attends positions [0, lim)
  uint32_t flags; // bit 0: first stage of the unit (new query), bit 1: last stage
};

// 4-D tiled TMA load through a tensor map that lives in global memory.
__device__ __forceinline__ void tma_load_4d_gmap(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 int c2, int c3, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(pol)
      : "memory");
}

}  // namespace

// One CTA (8 warps) per sequence. Items 0..23 are the query heads, 24..27 the
// kv heads; warp w takes items w, w+8, w+16, w+24. Lane l holds dims
// 8l..8l+7; the RoPE partner of dims 0..31 (lanes 0..3) is dims 32..63
// (lanes 4..7).
__global__ void __launch_bounds__(256) batch_prologue_kernel(const __grid_constant__ BatchParams p) {
  __shared__ float s_cs[2 * ROT_PAIRS];
  pdl_wait_primary();  // the previous step may still read q_ws and the caches
  pdl_launch_dependents();
  const int s = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const BatchSeq& sq = p.seq[s];
  const uint32_t pos = sq.base;
  if (warp == 0) {
    float c, sn;
    rope_cs(pos, p.inv_freq[lane], c, sn);
    s_cs[2 * lane] = c;
    s_cs[2 * lane + 1] = sn;
  }
  __syncthreads();
  for (int hh = warp; hh < QH + KVH; hh += 8) {
    const bool is_q = hh < QH;
    const size_t in = is_q ? (size_t)s * QROW + (size_t)hh * 512 + lane * 8
                           : (size_t)s * KROW + (size_t)(hh - QH) * HD + lane * 8;
    float x[8], ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] = load_in_bf16(is_q ? p.q_gate : p.k_in, in + i, p.in_bf16);
      ss += x[i] * x[i];
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = 1.0f / sqrtf(ss / 256.0f + p.eps);
    const uint16_t* wn = is_q ? p.q_norm_w : p.k_norm_w;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float n = x[i] * inv * bf16_bits_to_f32(wn[lane * 8 + i]);
      const float partner = __shfl_xor_sync(0xffffffffu, n, 4);
      o[i] = n;
      if (lane < 8) {
        const int j = (lane & 3) * 8 + i;
        const float c = s_cs[2 * j], sn = s_cs[2 * j + 1];
        o[i] = lane < 4 ? n * c - partner * sn : n * c + partner * sn;
      }
    }
    const uint4 packed = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                                    pack_bf16x2(o[6], o[7]));
    if (is_q) {
      *reinterpret_cast<uint4*>(p.q_ws + ((size_t)s * QH + hh) * HD + lane * 8) = packed;
    } else {
      const size_t go = ((size_t)(hh - QH) * sq.capacity + pos) * HD + lane * 8;
      *reinterpret_cast<uint4*>(sq.k_cache + go) = packed;
      float vv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) vv[i] = load_in_bf16(p.v_in, in + i, p.in_bf16);
      *reinterpret_cast<uint4*>(sq.v_cache + go) = make_uint4(pack_bf16x2(vv[0], vv[1]), pack_bf16x2(vv[2], vv[3]),
                                                             pack_bf16x2(vv[4], vv[5]), pack_bf16x2(vv[6], vv[7]));
    }
  }
}

struct BatchXch {
  float red[2][4][8];
  float lsum[2][4][8];
  uint2 pb[2][4][32];
};

__global__ void __launch_bounds__(BAT_THREADS, 1) batch_split_kernel(const __grid_constant__ BatchParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  BatchXch& X = *reinterpret_cast<BatchXch*>(smem + BAT_XCH_OFF);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAT_BAR_OFF);
  uint64_t* empty = full + BAT_STAGES;
  UnitInfo* info = reinterpret_cast<UnitInfo*>(empty + BAT_STAGES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int kvh = blockIdx.x & 3;

  if (threadIdx.x == 0) {
    for (int s = 0; s < BAT_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_mbar_init();
  }
  // query heads 6, 7 of every stage's Q slot are the zero padding of the
  // 8-wide MMA N dimension; the unit's copy only writes heads 0..5
  for (int i = threadIdx.x; i < BAT_STAGES * 64; i += BAT_THREADS) {
    const int st = i / 64, c = i % 64;
    *reinterpret_cast<uint4*>(smem + st * BAT_STAGE_BYTES + BAT_Q_OFF + BAT_Q_BYTES + c * 16) =
        make_uint4(0u, 0u, 0u, 0u);
  }
  fence_proxy_async_smem();
  __syncthreads();
  // the prologue has written q_ws and the new K/V rows
  pdl_wait_primary();
  pdl_launch_dependents();

  if (warp == 4) {
    // ---------------- producer ----------------
    if (lane == 0 && !p.withhold) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t i = 0;
      bool done = false;
      while (!done) {
        const uint32_t u = atomicAdd(&p.sched[kvh], 1u);
        done = u >= p.total_units;
        int s = 0;
        uint32_t nt = 1, chunk = 0, ctx = 0;
        if (!done) {
          // the sequence holding unit u: last s with unit0 <= u
          int lo = 0, hi = p.n_seqs - 1;
          while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.seq[mid].unit0 <= u) lo = mid;
            else hi = mid - 1;
          }
          s = lo;
          chunk = u - p.seq[s].unit0;
          ctx = p.seq[s].base + 1;
          const uint32_t n = min((uint32_t)DEC_CHUNK, ctx - chunk * DEC_CHUNK);
          nt = (n + DEC_TILE - 1) / DEC_TILE;
        }
        for (uint32_t t = 0; t < nt; ++t, ++i) {
          const uint32_t slot = i % BAT_STAGES;
          if (i >= BAT_STAGES &&
              !mbar_wait(&empty[slot], ((i / BAT_STAGES) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY, p.wait_ns)) {
            done = true;
            break;
          }
          if (done) {
            info[slot].unit = -1;
            mbar_arrive(&full[slot]);
            break;
          }
          const uint32_t row0 = chunk * DEC_CHUNK + t * DEC_TILE;
          info[slot] = UnitInfo{(int)u, row0, ctx, (t == 0 ? 1u : 0u) | (t + 1 == nt ? 2u : 0u)};
          uint8_t* stage = smem + slot * BAT_STAGE_BYTES;
          mbar_arrive_expect_tx(&full[slot], DEC_STAGE_BYTES + (t == 0 ? BAT_Q_BYTES : 0));
          if (t == 0)
            bulk_load(stage + BAT_Q_OFF, p.q_ws + ((size_t)s * QH + kvh * GQA) * HD, BAT_Q_BYTES, &full[slot]);
          const CUtensorMap* tm = p.seq[s].tm;
          tma_load_4d_gmap(stage, tm, &full[slot], 0, (int)row0, 0, kvh, pol);
          tma_load_4d_gmap(stage + DEC_STAGE_BYTES / 2, tm + 1, &full[slot], 0, (int)row0, 0, kvh, pol);
        }
      }
    }
    return;
  }

  // ---------------- compute warps: w = warp ----------------
  const int w = warp;
  uint32_t bq0[16], bq1[16];
  float o[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  for (uint32_t it = 0;; ++it) {
    const int s = it % BAT_STAGES, par = it & 1;
    uint8_t* stage = smem + s * BAT_STAGE_BYTES;
    if (!mbar_wait(&full[s], (it / BAT_STAGES) & 1, p.err, ERR_TIMEOUT_FULL, p.wait_ns)) return;
    const UnitInfo inf = info[s];
    if (inf.unit < 0) break;
    const uint32_t sK = smem_u32(stage), sV = sK + DEC_STAGE_BYTES / 2;
    if (inf.flags & 1u) {
      // a new unit: its sequence's query heads as B fragments
      const uint32_t qaddr = smem_u32(stage + BAT_Q_OFF) + (lane & 7) * (HD * 2) + (lane >> 3) * 16;
#pragma unroll
      for (int kp = 0; kp < 8; ++kp)
        ldmatrix_x4(qaddr + kp * 64, bq0[2 * kp], bq1[2 * kp], bq0[2 * kp + 1], bq1[2 * kp + 1]);
    }
    // S^T[16 tok x 8 heads] = K[16w.., :] . Q^T
    float sc[4] = {0.f, 0.f, 0.f, 0.f}, sd[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int mi = lane >> 3, rr = lane & 7;
      const uint32_t tok = 16 * w + rr + (mi & 1) * 8;
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        const uint32_t chunk = kk * 2 + (mi >> 1);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(sK + (chunk >> 3) * (DEC_TILE * 128) + swz128(tok, chunk & 7), a0, a1, a2, a3);
        if (kk & 1)
          mma_bf16_16816(sd, a0, a1, a2, a3, bq0[kk], bq1[kk]);
        else
          mma_bf16_16816(sc, a0, a1, a2, a3, bq0[kk], bq1[kk]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[e] += sd[e];
    }
    const uint32_t t0 = inf.row0 + 16 * w + g;
    const bool v0 = t0 < inf.lim, v1 = t0 + 8 < inf.lim;
    sc[0] = v0 ? sc[0] * SCALE : -INFINITY;
    sc[1] = v0 ? sc[1] * SCALE : -INFINITY;
    sc[2] = v1 ? sc[2] * SCALE : -INFINITY;
    sc[3] = v1 ? sc[3] * SCALE : -INFINITY;
    float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    if (g == 0) *reinterpret_cast<float2*>(&X.red[par][w][2 * q]) = make_float2(mx0, mx1);
    named_bar_sync(1, 128);
#pragma unroll
    for (int ww = 0; ww < 4; ++ww) {
      const float2 r2 = *reinterpret_cast<const float2*>(&X.red[par][ww][2 * q]);
      mx0 = fmaxf(mx0, r2.x);
      mx1 = fmaxf(mx1, r2.y);
    }
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float al0 = n0 == -INFINITY ? 1.f : fast_exp2(LOG2E * (m0 - n0));
    const float al1 = n1 == -INFINITY ? 1.f : fast_exp2(LOG2E * (m1 - n1));
    const float p0 = n0 == -INFINITY ? 0.f : fast_exp2(LOG2E * (sc[0] - n0));
    const float p1 = n1 == -INFINITY ? 0.f : fast_exp2(LOG2E * (sc[1] - n1));
    const float p2 = n0 == -INFINITY ? 0.f : fast_exp2(LOG2E * (sc[2] - n0));
    const float p3 = n1 == -INFINITY ? 0.f : fast_exp2(LOG2E * (sc[3] - n1));
    m0 = n0;
    m1 = n1;
    const uint32_t x0 = pack_bf16x2(p0, p1), x1 = pack_bf16x2(p2, p3);
    float ls0 = bf16_bits_to_f32(x0 & 0xffffu) + bf16_bits_to_f32(x1 & 0xffffu);
    float ls1 = bf16_bits_to_f32(x0 >> 16) + bf16_bits_to_f32(x1 >> 16);
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      ls0 += __shfl_xor_sync(0xffffffffu, ls0, off);
      ls1 += __shfl_xor_sync(0xffffffffu, ls1, off);
    }
    if (g == 0) *reinterpret_cast<float2*>(&X.lsum[par][w][2 * q]) = make_float2(ls0, ls1);
    X.pb[par][w][lane] = make_uint2(movmatrix_trans(x0), movmatrix_trans(x1));
    named_bar_sync(1, 128);
    {
      float t0s = 0.f, t1s = 0.f;
#pragma unroll
      for (int ww = 0; ww < 4; ++ww) {
        const float2 r2 = *reinterpret_cast<const float2*>(&X.lsum[par][ww][2 * q]);
        t0s += r2.x;
        t1s += r2.y;
      }
      l0 = l0 * al0 + t0s;
      l1 = l1 * al1 + t1s;
    }
    if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        o[i][0] *= al0;
        o[i][1] *= al1;
        o[i][2] *= al0;
        o[i][3] *= al1;
      }
    }
    {
      const int mi = lane >> 3, rr = lane & 7;
      const uint32_t vbase = sV + w * (DEC_TILE * 128);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint2 b = X.pb[par][kk][lane];
        const uint32_t tok = 16 * kk + rr + (mi >> 1) * 8;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4_trans(vbase + swz128(tok, 2 * i + (mi & 1)), a0, a1, a2, a3);
          mma_bf16_16816(o[i], a0, a1, a2, a3, b.x, b.y);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (inf.flags & 2u) {
      const size_t unit = (size_t)kvh * p.unit_cap + (uint32_t)inf.unit;
      if (w == 0 && g == 0) {
        float* ml = p.part_ml + unit * 16;
        *reinterpret_cast<float2*>(ml + 2 * q) = make_float2(m0, m1);
        *reinterpret_cast<float2*>(ml + 8 + 2 * q) = make_float2(l0, l1);
      }
      float* po = p.part_o + unit * 2048;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int d = 64 * w + 16 * i + g;
        *reinterpret_cast<float2*>(po + d * 8 + 2 * q) = make_float2(o[i][0], o[i][1]);
        *reinterpret_cast<float2*>(po + (d + 8) * 8 + 2 * q) = make_float2(o[i][2], o[i][3]);
        o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      }
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
    }
  }
}

// One CTA per (sequence, kv head), 4 phases x 256 dims: phase ph folds the
// sequence's chunks ph, ph+4, ... for all 6 heads of the kv head at one dim;
// the phases are then merged in a fixed tree (2,3 into 0,1; 1 into 0), so the
// result depends only on the sequence's own context. Applies the gate.
__global__ void __launch_bounds__(256 * BCMB_PHASES) batch_combine_kernel(const __grid_constant__ BatchParams p) {
  pdl_wait_primary();
  pdl_launch_dependents();
  if (blockIdx.x == 0 && threadIdx.x < KVH) p.sched[threadIdx.x] = 0;  // ready for the next launch
  __shared__ float s_st[2][GQA * 3][256];
  const int s = blockIdx.x >> 2, kvh = blockIdx.x & 3;
  const int ph = threadIdx.x >> 8, d = threadIdx.x & 255;
  const BatchSeq& sq = p.seq[s];
  const uint32_t nch = (sq.base + 1 + DEC_CHUNK - 1) / DEC_CHUNK;
  const size_t u0 = (size_t)kvh * p.unit_cap + sq.unit0;
  float mm[GQA], aa[GQA], dd[GQA];
#pragma unroll
  for (int h = 0; h < GQA; ++h) {
    mm[h] = -INFINITY;
    aa[h] = 0.f;
    dd[h] = 0.f;
  }
  constexpr int U = 2;
  for (uint32_t c0 = ph; c0 < nch; c0 += U * BCMB_PHASES) {
    float4 ml[U][4], ov[U][2];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t c = c0 + u * BCMB_PHASES;
      if (c < nch) {
        const float4* m4 = reinterpret_cast<const float4*>(p.part_ml + (u0 + c) * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) ml[u][i] = m4[i];
        const float4* o4 = reinterpret_cast<const float4*>(p.part_o + (u0 + c) * 2048 + d * 8);
        ov[u][0] = o4[0];
        ov[u][1] = o4[1];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (c0 + u * BCMB_PHASES < nch) {
        const float cm[8] = {ml[u][0].x, ml[u][0].y, ml[u][0].z, ml[u][0].w,
                             ml[u][1].x, ml[u][1].y, ml[u][1].z, ml[u][1].w};
        const float cl[8] = {ml[u][2].x, ml[u][2].y, ml[u][2].z, ml[u][2].w,
                             ml[u][3].x, ml[u][3].y, ml[u][3].z, ml[u][3].w};
        const float co[8] = {ov[u][0].x, ov[u][0].y, ov[u][0].z, ov[u][0].w,
                             ov[u][1].x, ov[u][1].y, ov[u][1].z, ov[u][1].w};
#pragma unroll
        for (int h = 0; h < GQA; ++h) {
          const float nm = fmaxf(mm[h], cm[h]);
          if (nm == -INFINITY) continue;
          const float wo = fast_exp2(LOG2E * (mm[h] - nm)), wn = fast_exp2(LOG2E * (cm[h] - nm));
          aa[h] = aa[h] * wo + co[h] * wn;
          dd[h] = dd[h] * wo + cl[h] * wn;
          mm[h] = nm;
        }
      }
    }
  }
  // fixed merge tree over the phases
#pragma unroll
  for (int level = 0; level < 2; ++level) {
    const int half = level == 0 ? 2 : 1;
    if (ph >= half && ph < 2 * half) {
#pragma unroll
      for (int h = 0; h < GQA; ++h) {
        s_st[ph - half][3 * h][d] = mm[h];
        s_st[ph - half][3 * h + 1][d] = aa[h];
        s_st[ph - half][3 * h + 2][d] = dd[h];
      }
    }
    __syncthreads();
    if (ph < half) {
#pragma unroll
      for (int h = 0; h < GQA; ++h) {
        const float cm = s_st[ph][3 * h][d], ca = s_st[ph][3 * h + 1][d], cd = s_st[ph][3 * h + 2][d];
        const float nm = fmaxf(mm[h], cm);
        if (nm == -INFINITY) continue;
        const float wo = fast_exp2(LOG2E * (mm[h] - nm)), wn = fast_exp2(LOG2E * (cm - nm));
        aa[h] = aa[h] * wo + ca * wn;
        dd[h] = dd[h] * wo + cd * wn;
        mm[h] = nm;
      }
    }
    __syncthreads();
  }
  if (ph != 0) return;
#pragma unroll
  for (int hl = 0; hl < GQA; ++hl) {
    const int h = kvh * GQA + hl;
    const float o = aa[hl] / dd[hl];
    const float gv = load_in_bf16(p.q_gate, (size_t)s * QROW + (size_t)h * 512 + 256 + d, p.in_bf16);
    const float sg = 1.0f / (1.0f + exp2f(-LOG2E * gv));
    p.gated_out[(size_t)s * OROW + h * HD + d] = f32_to_bf16_bits(o * sg);
  }
}

}  // namespace lisa

using namespace lisa;

struct lisa_attn_batch {
  int device = 0;
  int max_seqs = 0;
  uint32_t unit_cap = 0;
  uint16_t* q_ws = nullptr;
  float* part_o = nullptr;
  float* part_ml = nullptr;
  int* err = nullptr;  // [0] error word, [16..19] unit counters
};

namespace {

struct BGuard {
  int prev = -1;
  explicit BGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~BGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

void batch_free(lisa_attn_batch* b) {
  cudaFree(b->q_ws);
  cudaFree(b->part_o);
  cudaFree(b->part_ml);
  cudaFree(b->err);
  delete b;
}

cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t st, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace

#pragma GCC visibility push(default)
extern "C" {

int lisa_attn_batch_create(int device, int max_seqs, uint64_t max_total_positions, lisa_attn_batch** out) {
  if (!out || max_seqs < 1 || max_seqs > BAT_MAX_SEQS || max_total_positions == 0 ||
      max_total_positions > ((uint64_t)1 << 36))
    return LISA_EINVAL;
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return LISA_EINVAL;
  BGuard guard(device);
  lisa_attn_batch* b = new lisa_attn_batch();
  b->device = device;
  b->max_seqs = max_seqs;
  // every sequence adds at most one partly filled chunk
  const uint64_t units = (max_total_positions + DEC_CHUNK - 1) / DEC_CHUNK + (uint64_t)max_seqs;
  if (units > (1u << 30)) {
    delete b;
    return LISA_EINVAL;
  }
  b->unit_cap = (uint32_t)units;
  bool ok = cudaMalloc(&b->q_ws, (size_t)max_seqs * QH * HD * 2) == cudaSuccess &&
            cudaMalloc(&b->part_o, (size_t)KVH * units * 2048 * sizeof(float)) == cudaSuccess &&
            cudaMalloc(&b->part_ml, (size_t)KVH * units * 16 * sizeof(float)) == cudaSuccess &&
            cudaMalloc(&b->err, 256) == cudaSuccess;
  ok = ok && cudaMemset(b->err, 0, 256) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  if (!ok) {
    batch_free(b);
    return LISA_ECUDA;
  }
  *out = b;
  return LISA_OK;
}

int lisa_attn_batch_destroy(lisa_attn_batch* b) {
  if (!b) return LISA_EINVAL;
  BGuard guard(b->device);
  batch_free(b);
  return LISA_OK;
}

int lisa_attn_decode_batch(lisa_attn_batch* b, int n_seqs, lisa_attn_ctx* const* ctxs, int layer,
                           const uint32_t* bases, int in_dtype, const void* q_gate, const void* k, const void* v,
                           const uint16_t* q_norm_w, const uint16_t* k_norm_w, float eps, uint16_t* gated_out,
                           void* stream) {
  if (!b || !ctxs || !bases || n_seqs < 1 || n_seqs > b->max_seqs) return LISA_EINVAL;
  if (!q_gate || !k || !v || !q_norm_w || !k_norm_w || !gated_out) return LISA_EINVAL;
  if (in_dtype != LISA_DTYPE_F32 && in_dtype != LISA_DTYPE_BF16) return LISA_EINVAL;
  BatchParams p = {};
  uint64_t units = 0;
  for (int i = 0; i < n_seqs; ++i) {
    const lisa_attn_ctx* c = ctxs[i];
    if (!c || c->device != b->device || layer < 0 || layer >= c->n_layers) return LISA_EINVAL;
    if ((uint64_t)bases[i] + 1 > c->capacity) return LISA_ENOSPC;
    const size_t off = (size_t)layer * KVH * c->capacity * HD;
    p.seq[i] = BatchSeq{c->tmaps + 2 * layer, c->k + off, c->v + off, c->capacity, bases[i], (uint32_t)units, 0};
    units += ((uint64_t)bases[i] + 1 + DEC_CHUNK - 1) / DEC_CHUNK;
  }
  if (units > b->unit_cap) return LISA_E2BIG;
  BGuard guard(b->device);
  p.n_seqs = n_seqs;
  p.total_units = (uint32_t)units;
  p.unit_cap = b->unit_cap;
  p.in_bf16 = in_dtype == LISA_DTYPE_BF16;
  p.q_gate = q_gate;
  p.k_in = k;
  p.v_in = v;
  p.q_norm_w = q_norm_w;
  p.k_norm_w = k_norm_w;
  p.eps = eps;
  p.q_ws = b->q_ws;
  p.part_o = b->part_o;
  p.part_ml = b->part_ml;
  p.err = b->err;
  p.sched = reinterpret_cast<uint32_t*>(b->err + 16);
  const WaitFault wf = current_wait_fault();
  p.wait_ns = wf.limit_ns ? wf.limit_ns : WAIT_LIMIT_NS;
  p.withhold = wf.withhold;
  p.gated_out = gated_out;
  host_inv_freq(p.inv_freq);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  static SmemAttr attr_once;
  if (attr_once.ensure(batch_split_kernel, BAT_SMEM_BYTES) != cudaSuccess) return LISA_ECUDA;
  cudaLaunchAttribute a1[1], a2[1], a3[1];
  cudaLaunchConfig_t c1 = pdl_config(dim3(n_seqs), dim3(256), 0, st, a1);
  if (cudaLaunchKernelEx(&c1, batch_prologue_kernel, p) != cudaSuccess) return LISA_ECUDA;
  const int per_head = std::max(1, current_device_sms() / KVH);
  cudaLaunchConfig_t c2 = pdl_config(dim3(per_head * KVH), dim3(BAT_THREADS), BAT_SMEM_BYTES, st, a2);
  if (cudaLaunchKernelEx(&c2, batch_split_kernel, p) != cudaSuccess) return LISA_ECUDA;
  cudaLaunchConfig_t c3 = pdl_config(dim3(n_seqs * KVH), dim3(256 * BCMB_PHASES), 0, st, a3);
  if (cudaLaunchKernelEx(&c3, batch_combine_kernel, p) != cudaSuccess) return LISA_ECUDA;
  return LISA_OK;
}

int lisa_attn_batch_check_device_error(lisa_attn_batch* b, void* stream) {
  if (!b) return LISA_EINVAL;
  BGuard guard(b->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int h = 0;
  if (cudaMemcpyAsync(&h, b->err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return LISA_ECUDA;
  if (h && (cudaMemsetAsync(b->err, 0, sizeof(int), st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess))
    return LISA_ECUDA;
  return h ? LISA_ETIMEOUT : LISA_OK;
}

}  // extern "C"
#pragma GCC visibility pop
