// decode.cu — split-KV flash-decoding for the M=1 decode and M=3 MTP-verify
// shapes of the lisa-rs full-attention layer, written for sm_100a.
//
// Replaces, in one kernel plus one combine:
//   q_norm_gate_rope_decode/_block3   attention.metal:118-155, 245-281
//   kv_cache_store_decode/_block3     attention.metal:158-197, 283-319
//   sdpa_decode_partial               attention.metal:550-604
//   sdpa_decode_final                 attention.metal:611-641
//   gate_out_bf16                     attention.metal:520-531
//
// Work decomposition. The KV cache of one layer is [4 kv heads][pos][256] bf16.
// A work unit is (kv head, 128-token chunk). A persistent CTA owns one kv head
// (blockIdx & 3) and a strided set of chunks; it streams each chunk's K and V
// through a 3-stage ring of 16-token tiles with TMA (SWIZZLE_128B boxes, one
// mbarrier per stage), so the 6 query heads that share the kv head (x rows)
// read each KV byte from HBM once. One warp per query row:
//   S^T[16 tok x 8 heads] = K_tile[16 x 256] . Q^T      (mma.m16n8k16, Q in regs)
//   online softmax per head column (warp shuffles), P rounded to bf16
//   P^T to B-fragment layout with movmatrix.trans
//   O^T[256 x 8 heads]   += V_tile^T[256 x 16] . P^T    (mma.m16n8k16)
// Heads 6,7 of the 8-wide N dimension are zero padding. The new K/V rows of
// this call are normalised/roped by the CTA whose chunk holds them, written to
// the cache and substituted into the staged tile, so the append needs no launch
// of its own. Each (row, kv head, chunk) leaves an unnormalised partial
// (max, sum, O); the combine kernel merges a row's chunks in a fixed order and
// applies the sigmoid gate.
#include "common.cuh"
#include "decode.cuh"

#include <algorithm>

namespace lisa {

namespace {

struct TileCursor {
  uint32_t chunk;   // chunk index
  uint32_t tile;    // tile within chunk
  uint32_t ntiles;  // tiles in this chunk
};

__device__ __forceinline__ uint32_t chunk_tiles(uint32_t chunk, uint32_t extent) {
  const uint32_t lo = chunk * DEC_CHUNK;
  const uint32_t n = min((uint32_t)DEC_CHUNK, extent - lo);
  return (n + DEC_TILE - 1) / DEC_TILE;
}

__device__ __forceinline__ void cursor_next(TileCursor& c, uint32_t stride, uint32_t extent, uint32_t nchunks) {
  if (++c.tile == c.ntiles) {
    c.tile = 0;
    c.chunk += stride;
    c.ntiles = c.chunk < nchunks ? chunk_tiles(c.chunk, extent) : 0;
  }
}

// Issues the TMA loads of one 16-token tile (K and V, 4 boxes of 64 dims each).
__device__ __forceinline__ void issue_tile(uint8_t* stage, uint64_t* full, const CUtensorMap* tk,
                                           const CUtensorMap* tv, uint32_t row0, int kvh) {
  mbar_arrive_expect_tx(full, DEC_STAGE_BYTES);
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    tma_load_3d(stage + st * 2048, tk, full, st * 64, (int)row0, kvh);
    tma_load_3d(stage + 8192 + st * 2048, tv, full, st * 64, (int)row0, kvh);
  }
}

// Normalises + ropes one new K row (position pos) and rounds one V row, 8 dims
// per lane (lane l holds dims 8l..8l+7). attention.metal:158-197.
__device__ __forceinline__ void new_kv_row(const DecodeParams& p, int r, int kvh, uint32_t pos, int lane,
                                           uint4& kout, uint4& vout) {
  const size_t in = (size_t)r * KROW + kvh * HD + lane * 8;
  float x[8], ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    x[i] = load_in_bf16(p.k_in, in + i, p.in_bf16);
    ss += x[i] * x[i];
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = 1.0f / sqrtf(ss / 256.0f + p.eps);
  float n[8], o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) n[i] = x[i] * inv * bf16_bits_to_f32(p.k_norm_w[lane * 8 + i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float partner = __shfl_xor_sync(0xffffffffu, n[i], 4);
    o[i] = n[i];
    if (lane < 8) {
      const int j = (lane & 3) * 8 + i;  // pair index 0..31
      float c, s;
      rope_cs(pos, j, c, s);
      o[i] = lane < 4 ? n[i] * c - partner * s : n[i] * c + partner * s;
    }
  }
  kout = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                    pack_bf16x2(o[6], o[7]));
  float vv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) vv[i] = load_in_bf16(p.v_in, in + i, p.in_bf16);
  vout = make_uint4(pack_bf16x2(vv[0], vv[1]), pack_bf16x2(vv[2], vv[3]), pack_bf16x2(vv[4], vv[5]),
                    pack_bf16x2(vv[6], vv[7]));
}

}  // namespace

// One CTA = one kv head x a strided set of chunks; ROWS warps, warp m serves
// query row m (6 heads). Thread 0 is also the TMA producer.
template <int ROWS>
__global__ void __launch_bounds__(32 * ROWS, DEC_CTAS_PER_SM)
    decode_split_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                        const DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + DEC_STAGES * DEC_STAGE_BYTES);
  uint64_t* empty = full + DEC_STAGES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int kvh = blockIdx.x & 3;
  const uint32_t stride = gridDim.x >> 2;
  const uint32_t first_chunk = blockIdx.x >> 2;
  const int m = warp;  // query row of this warp

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    for (int s = 0; s < DEC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], ROWS);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // Producer cursor (thread 0 only) runs DEC_STAGES-1 tiles ahead.
  TileCursor pc{first_chunk, 0, first_chunk < p.nchunks ? chunk_tiles(first_chunk, p.extent) : 0};
  uint32_t issued = 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < DEC_STAGES - 1 && pc.ntiles; ++s) {
      issue_tile(smem + (issued % DEC_STAGES) * DEC_STAGE_BYTES, &full[issued % DEC_STAGES], &tk, &tv,
                 pc.chunk * DEC_CHUNK + pc.tile * DEC_TILE, kvh);
      ++issued;
      cursor_next(pc, stride, p.extent, p.nchunks);
    }
  }

  // ---- query prologue: q RMSNorm + RoPE straight into B fragments ----------
  // b0[kk] = Q[head g][16kk + 2q, +1], b1[kk] = Q[head g][16kk + 8 + 2q, +1].
  uint32_t bq0[16], bq1[16];
  {
    const uint32_t pos = p.base + m;
    float x[64];
    float ss = 0.f;
    const int h = kvh * GQA + g;
    const size_t qb = (size_t)m * QROW + (size_t)h * 512;
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = 16 * kk + 2 * q + (e & 1) + (e >> 1) * 8;
        const float v = g < GQA ? load_in_bf16(p.q_gate, qb + d, p.in_bf16) : 0.f;
        x[kk * 4 + e] = v;
        ss += v * v;
      }
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    const float inv = 1.0f / sqrtf(ss / 256.0f + p.eps);
#pragma unroll
    for (int kk = 0; kk < 16; ++kk)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = 16 * kk + 2 * q + (e & 1) + (e >> 1) * 8;
        x[kk * 4 + e] = x[kk * 4 + e] * inv * bf16_bits_to_f32(p.q_norm_w[d]);
      }
    // pairs (d, d+32) for d < 32 live in (kk, kk+2) of the same lane
#pragma unroll
    for (int kk = 0; kk < 2; ++kk)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = 16 * kk + 2 * q + (e & 1) + (e >> 1) * 8;
        float c, s;
        rope_cs(pos, d, c, s);
        const float a = x[kk * 4 + e], b = x[(kk + 2) * 4 + e];
        x[kk * 4 + e] = a * c - b * s;
        x[(kk + 2) * 4 + e] = b * c + a * s;
      }
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      bq0[kk] = g < GQA ? pack_bf16x2(x[kk * 4 + 0], x[kk * 4 + 1]) : 0u;
      bq1[kk] = g < GQA ? pack_bf16x2(x[kk * 4 + 2], x[kk * 4 + 3]) : 0u;
    }
  }

  // Row m attends local rows [0, lim).
  const int64_t lim64 = (int64_t)p.base + m + 1 - (int64_t)p.kv_lo;
  const uint32_t lim = lim64 <= 0 ? 0u : (uint32_t)(lim64 < (int64_t)p.extent ? lim64 : (int64_t)p.extent);

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  TileCursor cc{first_chunk, 0, first_chunk < p.nchunks ? chunk_tiles(first_chunk, p.extent) : 0};
  uint32_t it = 0;
  while (cc.ntiles) {
    const int s = it % DEC_STAGES;
    uint8_t* stage = smem + s * DEC_STAGE_BYTES;
    // producer: refill the stage consumed in the previous iteration
    if (threadIdx.x == 0 && pc.ntiles) {
      const uint32_t slot = issued % DEC_STAGES;
      if (issued >= DEC_STAGES &&
          !mbar_wait(&empty[slot], ((issued / DEC_STAGES) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) {
        pc.ntiles = 0;
      } else {
        issue_tile(smem + slot * DEC_STAGE_BYTES, &full[slot], &tk, &tv, pc.chunk * DEC_CHUNK + pc.tile * DEC_TILE,
                   kvh);
        ++issued;
        cursor_next(pc, stride, p.extent, p.nchunks);
      }
    }
    if (!mbar_wait(&full[s], (it / DEC_STAGES) & 1, p.err, ERR_TIMEOUT_FULL)) return;

    const uint32_t row0 = cc.chunk * DEC_CHUNK + cc.tile * DEC_TILE;
    const uint32_t sK = smem_u32(stage), sV = sK + 8192;

    // Substitute this call's new K/V rows (they are appended here).
    {
      bool wrote = false;
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int64_t lp = (int64_t)p.base + r - (int64_t)p.kv_lo;
        if (lp >= (int64_t)row0 && lp < (int64_t)row0 + DEC_TILE && lp < (int64_t)p.extent) {
          uint4 kr, vr;
          new_kv_row(p, r, kvh, p.base + r, lane, kr, vr);
          const uint32_t trow = (uint32_t)lp - row0;
          const uint32_t off = (lane >> 3) * 2048 + swz128(trow, lane & 7);
          *reinterpret_cast<uint4*>(stage + off) = kr;
          *reinterpret_cast<uint4*>(stage + 8192 + off) = vr;
          if (m == 0) {
            const size_t go = ((size_t)kvh * p.window_rows + (size_t)lp) * HD + lane * 8;
            *reinterpret_cast<uint4*>(p.k_cache + go) = kr;
            *reinterpret_cast<uint4*>(p.v_cache + go) = vr;
          }
          wrote = true;
        }
      }
      if (wrote) {
        fence_proxy_async_smem();
        __syncwarp();
      }
    }

    // S^T = K . Q^T
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int mi = lane >> 3, rr = lane & 7;
      const uint32_t tok = rr + (mi & 1) * 8;
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        const uint32_t chunk = kk * 2 + (mi >> 1);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(sK + (chunk >> 3) * 2048 + swz128(tok, chunk & 7), a0, a1, a2, a3);
        mma_bf16_16816(sc, a0, a1, a2, a3, bq0[kk], bq1[kk]);
      }
    }
    // scale + causal mask: c0,c1 -> token row0+g, c2,c3 -> token row0+g+8
    const bool v0 = row0 + g < lim, v1 = row0 + g + 8 < lim;
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
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float al0 = n0 == -INFINITY ? 1.f : exp2f(LOG2E * (m0 - n0));
    const float al1 = n1 == -INFINITY ? 1.f : exp2f(LOG2E * (m1 - n1));
    const float p0 = n0 == -INFINITY ? 0.f : exp2f(LOG2E * (sc[0] - n0));
    const float p1 = n1 == -INFINITY ? 0.f : exp2f(LOG2E * (sc[1] - n1));
    const float p2 = n0 == -INFINITY ? 0.f : exp2f(LOG2E * (sc[2] - n0));
    const float p3 = n1 == -INFINITY ? 0.f : exp2f(LOG2E * (sc[3] - n1));
    m0 = n0;
    m1 = n1;
    const uint32_t x0 = pack_bf16x2(p0, p1), x1 = pack_bf16x2(p2, p3);
    // the denominator sums the same bf16 weights the PV product uses
    l0 = l0 * al0 + (bf16_bits_to_f32(x0 & 0xffffu) + bf16_bits_to_f32(x1 & 0xffffu));
    l1 = l1 * al1 + (bf16_bits_to_f32(x0 >> 16) + bf16_bits_to_f32(x1 >> 16));
    if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        o[i][0] *= al0;
        o[i][1] *= al1;
        o[i][2] *= al0;
        o[i][3] *= al1;
      }
    }
    const uint32_t b0 = movmatrix_trans(x0), b1 = movmatrix_trans(x1);
    // O^T += V^T . P^T
    {
      const int mi = lane >> 3, rr = lane & 7;
      const uint32_t tok = rr + (mi >> 1) * 8;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t chunk = 2 * i + (mi & 1);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(sV + (chunk >> 3) * 2048 + swz128(tok, chunk & 7), a0, a1, a2, a3);
        mma_bf16_16816(o[i], a0, a1, a2, a3, b0, b1);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    if (cc.tile + 1 == cc.ntiles) {
      // chunk done: write its partial
      float t0 = l0, t1 = l1;
#pragma unroll
      for (int off = 4; off <= 16; off <<= 1) {
        t0 += __shfl_xor_sync(0xffffffffu, t0, off);
        t1 += __shfl_xor_sync(0xffffffffu, t1, off);
      }
      const size_t unit = ((size_t)m * KVH + kvh) * p.chunk_cap + cc.chunk;
      if (g == 0) {
        float* ml = p.part_ml + unit * 16;
        *reinterpret_cast<float2*>(ml + 2 * q) = make_float2(m0, m1);
        *reinterpret_cast<float2*>(ml + 8 + 2 * q) = make_float2(t0, t1);
      }
      float* po = p.part_o + unit * 2048;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int d = 16 * i + g;
        *reinterpret_cast<float2*>(po + d * 8 + 2 * q) = make_float2(o[i][0], o[i][1]);
        *reinterpret_cast<float2*>(po + (d + 8) * 8 + 2 * q) = make_float2(o[i][2], o[i][3]);
        o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      }
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
    }
    cursor_next(cc, stride, p.extent, p.nchunks);
    ++it;
  }
}

// Merges one row's chunk partials for one kv head and 8 dims, in a fixed
// order that depends only on the row's own context (8 interleaved phases,
// summed phase 0..7), then either applies the gate (gated_out) or writes the
// window partial (win_o / win_ml). Grid: rows * 4 * 32 CTAs of 256 threads.
// Thread: slot = tid & 31 -> (dim = db*8 + slot/4, heads 2*(slot&3), +1),
// phase = tid >> 5 takes chunks c = phase, phase + 8, ...
__global__ void __launch_bounds__(256) decode_combine_kernel(const DecodeParams p) {
  pdl_wait_primary();
  __shared__ float2 s_acc[CMB_PHASES][32];
  __shared__ float2 s_den[CMB_PHASES][32];
  __shared__ float2 s_max[CMB_PHASES][32];
  const int db = blockIdx.x & 31;
  const int kvh = (blockIdx.x >> 5) & 3;
  const int m = blockIdx.x >> 7;
  const int slot = threadIdx.x & 31, phase = threadIdx.x >> 5;
  const int dim = db * CMB_DIMS_PER_CTA + (slot >> 2);
  const int hp = slot & 3;

  const int64_t lim64 = (int64_t)p.base + m + 1 - (int64_t)p.kv_lo;
  const uint32_t lim = lim64 <= 0 ? 0u : (uint32_t)(lim64 < (int64_t)p.extent ? lim64 : (int64_t)p.extent);
  const uint32_t nch = (lim + DEC_CHUNK - 1) / DEC_CHUNK;
  const size_t unit0 = ((size_t)m * KVH + kvh) * p.chunk_cap;

  // global max per head (exact in any order)
  float2 mx = make_float2(-INFINITY, -INFINITY);
  for (uint32_t c = phase; c < nch; c += CMB_PHASES) {
    const float2 v = *reinterpret_cast<const float2*>(p.part_ml + (unit0 + c) * 16 + 2 * hp);
    mx.x = fmaxf(mx.x, v.x);
    mx.y = fmaxf(mx.y, v.y);
  }
  s_max[phase][slot] = mx;
  __syncthreads();
  float2 gm = make_float2(-INFINITY, -INFINITY);
#pragma unroll
  for (int ph = 0; ph < CMB_PHASES; ++ph) {
    gm.x = fmaxf(gm.x, s_max[ph][slot].x);
    gm.y = fmaxf(gm.y, s_max[ph][slot].y);
  }
  float2 acc = make_float2(0.f, 0.f), den = make_float2(0.f, 0.f);
  for (uint32_t c = phase; c < nch; c += CMB_PHASES) {
    const float* ml = p.part_ml + (unit0 + c) * 16;
    const float2 cm = *reinterpret_cast<const float2*>(ml + 2 * hp);
    const float2 cl = *reinterpret_cast<const float2*>(ml + 8 + 2 * hp);
    const float2 ov = *reinterpret_cast<const float2*>(p.part_o + (unit0 + c) * 2048 + dim * 8 + 2 * hp);
    const float w0 = exp2f(LOG2E * (cm.x - gm.x)), w1 = exp2f(LOG2E * (cm.y - gm.y));
    acc.x += w0 * ov.x;
    acc.y += w1 * ov.y;
    den.x += w0 * cl.x;
    den.y += w1 * cl.y;
  }
  s_acc[phase][slot] = acc;
  s_den[phase][slot] = den;
  __syncthreads();
  if (phase != 0) return;
  acc = s_acc[0][slot];
  den = s_den[0][slot];
#pragma unroll
  for (int ph = 1; ph < CMB_PHASES; ++ph) {
    acc.x += s_acc[ph][slot].x;
    acc.y += s_acc[ph][slot].y;
    den.x += s_den[ph][slot].x;
    den.y += s_den[ph][slot].y;
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int hl = 2 * hp + e;
    if (hl >= GQA) continue;
    const int h = kvh * GQA + hl;
    const float a = e ? acc.y : acc.x, dn = e ? den.y : den.x, gmax = e ? gm.y : gm.x;
    const float o = nch ? a / dn : 0.f;
    if (p.gated_out) {
      // gate_out_bf16 (attention.metal:520-531); gate = bf16-rounded raw gate
      const float gv = load_in_bf16(p.q_gate, (size_t)m * QROW + (size_t)h * 512 + 256 + dim, p.in_bf16);
      const float sg = 1.0f / (1.0f + exp2f(-LOG2E * gv));
      p.gated_out[(size_t)m * OROW + h * HD + dim] = f32_to_bf16_bits(o * sg);
    } else {
      p.win_o[((size_t)m * QH + h) * HD + dim] = o;
      if (dim == 0) {
        p.win_ml[((size_t)m * QH + h) * 2 + 0] = nch ? gmax : -INFINITY;
        p.win_ml[((size_t)m * QH + h) * 2 + 1] = nch ? dn : 0.f;
      }
    }
  }
}

// LSE merge of window partials + gate. Grid rows*24, 256 threads (one per dim).
__global__ void __launch_bounds__(256) merge_windows_kernel(int n_parts, int rows, const float* part_o,
                                                            const float* part_ml, int in_bf16,
                                                            const void* q_gate, uint16_t* gated_out) {
  const int mh = blockIdx.x;  // m * 24 + h
  const int m = mh / QH, h = mh % QH, d = threadIdx.x;
  float gmax = -INFINITY;
  for (int g = 0; g < n_parts; ++g) gmax = fmaxf(gmax, part_ml[((size_t)g * rows * QH + mh) * 2]);
  float acc = 0.f, den = 0.f;
  for (int g = 0; g < n_parts; ++g) {
    const float mg = part_ml[((size_t)g * rows * QH + mh) * 2];
    const float lg = part_ml[((size_t)g * rows * QH + mh) * 2 + 1];
    if (lg == 0.f) continue;
    const float w = exp2f(LOG2E * (mg - gmax)) * lg;
    acc += w * part_o[((size_t)g * rows * QH + mh) * HD + d];
    den += w;
  }
  const float o = den > 0.f ? acc / den : 0.f;
  const float gv = load_in_bf16(q_gate, (size_t)m * QROW + (size_t)h * 512 + 256 + d, in_bf16);
  const float sg = 1.0f / (1.0f + exp2f(-LOG2E * gv));
  gated_out[(size_t)m * OROW + h * HD + d] = f32_to_bf16_bits(o * sg);
}

template <int ROWS>
static cudaError_t launch_split(const DecodeParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int num_sms,
                                cudaStream_t stream) {
  static bool configured = false;  // per process; the attribute is per function
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         DEC_SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const uint32_t per_head = std::min<uint32_t>(p.nchunks, (uint32_t)(num_sms * DEC_CTAS_PER_SM / KVH));
  decode_split_kernel<ROWS><<<per_head * KVH, 32 * ROWS, DEC_SMEM_BYTES, stream>>>(tk, tv, p);
  return cudaGetLastError();
}

cudaError_t launch_decode(const DecodeParams& p, int rows, const CUtensorMap& tk, const CUtensorMap& tv,
                          int num_sms, cudaStream_t stream) {
  cudaError_t e;
  switch (rows) {
    case 1: e = launch_split<1>(p, tk, tv, num_sms, stream); break;
    case 2: e = launch_split<2>(p, tk, tv, num_sms, stream); break;
    case 3: e = launch_split<3>(p, tk, tv, num_sms, stream); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows * KVH * (HD / CMB_DIMS_PER_CTA));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_combine_kernel, p);
}

cudaError_t launch_merge_windows(int n_parts, int rows, const float* part_o, const float* part_ml, int in_bf16,
                                 const void* q_gate, uint16_t* gated_out, cudaStream_t stream) {
  merge_windows_kernel<<<rows * QH, HD, 0, stream>>>(n_parts, rows, part_o, part_ml, in_bf16, q_gate, gated_out);
  return cudaGetLastError();
}

}  // namespace lisa
