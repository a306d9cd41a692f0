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
// A work unit is (kv head, 448-position chunk). 148 persistent CTAs, 37 per kv
// head (blockIdx & 3), take chunks from a per-head atomic counter; a
// producer warp streams each chunk's K and V through a 3-stage ring of
// 64-position stages (one 32 KB TMA box for K and one for V per stage,
// 128-byte swizzle, one mbarrier per stage, evict-first L2 hint), so the 6
// query heads that share the kv head (x rows) read each KV byte from HBM once.
// Four compute warps per query row, warp w taking positions 16w..16w+15 of a
// stage for Q.K^T and head dims 64w..64w+63 for P.V:
//   S^T[16 tok x 8 heads] = K_tile[16 x 256] . Q^T      (mma.m16n8k16, Q in regs)
//   stage max per head exchanged through shared memory, P rounded to bf16
//   P^T to B-fragment layout with movmatrix.trans
//   O^T[64 dims x 8 heads] += V_tile^T[64 x 64] . P^T   (mma.m16n8k16)
// Heads 6,7 of the 8-wide N dimension are zero padding. The new K/V rows of
// this call are normalised/roped by the CTA whose chunk holds them, written to
// the cache and substituted into the staged tile, so the append needs no launch
// of its own. Each (row, kv head, chunk) leaves an unnormalised partial
// (max, sum, O); the combine kernel merges a row's chunks in a fixed order and
// applies the sigmoid gate.
#include "common.cuh"
#include "decode.cuh"
#include "dispatch.h"

#include <algorithm>
#include <cmath>

namespace lisa {

namespace {

__device__ __forceinline__ uint32_t chunk_tiles(uint32_t chunk, uint32_t extent) {
  const uint32_t lo = chunk * DEC_CHUNK;
  const uint32_t n = min((uint32_t)DEC_CHUNK, extent - lo);
  return (n + DEC_TILE - 1) / DEC_TILE;
}

// Issues the TMA loads of one 64-token stage: K and V, one box each of all
// four 64-dim groups (32 KB, landing as [group][token][64 dims] with
// 128-byte swizzled rows). A TMA operation costs a fixed latency whatever its
// size, so two large boxes stream faster than eight small ones.
// The KV stream is read once: it is loaded with an evict-first L2 policy so
// it does not push the chunk partials (read back by the combine) out of L2.
__device__ __forceinline__ void issue_tile(uint8_t* stage, uint64_t* full, const CUtensorMap* tk,
                                           const CUtensorMap* tv, uint32_t row0, int kvh, uint64_t pol) {
  mbar_arrive_expect_tx(full, DEC_STAGE_BYTES);
  tma_load_4d_hint(stage, tk, full, 0, (int)row0, 0, kvh, pol);
  tma_load_4d_hint(stage + DEC_STAGE_BYTES / 2, tv, full, 0, (int)row0, 0, kvh, pol);
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
      const float c = p.rope_c[r][j], s = p.rope_s[r][j];
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

// Per query row, in shared memory: stage maxima and sums per (warp, head) and
// the warps' P^T fragments, double-buffered by stage parity.
struct RowXch {
  float red[2][4][8];
  float lsum[2][4][8];
  uint2 pb[2][4][32];
};

// CTA = one kv head x a strided set of chunks. ROWS query rows x 4 compute
// warps + 1 TMA producer warp. Compute warp (m, w): row m, tokens 16w..16w+15
// of each 64-token stage for Q.K^T, head dims 64w..64w+63 for P.V.
template <int ROWS>
__global__ void __launch_bounds__(32 * (4 * ROWS + 1), 1)
    decode_split_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                        const DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  RowXch* xch = reinterpret_cast<RowXch*>(smem + DEC_STAGES * DEC_STAGE_BYTES);
  // query rows in bf16 at DEC_QS_OFF: [ROWS][8 heads][256]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + DEC_STAGES * DEC_STAGE_BYTES + 3 * DEC_XCH_BYTES);
  uint64_t* empty = full + DEC_STAGES;
  uint64_t* qbar = empty + DEC_STAGES;                               // raw q + gains landed
  int* slot_code = reinterpret_cast<int*>(qbar + 1);                 // chunk << 8 | tile, or -1 = end

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int kvh = blockIdx.x & 3;
  constexpr int NCOMPUTE = 4 * ROWS;

#ifdef LISA_DECODE_TRACE
  if (threadIdx.x == 0) p.trace[16 + blockIdx.x * 4 + 0] = global_timer_ns();
#endif
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    for (int s = 0; s < DEC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCOMPUTE);
    }
    mbar_init(qbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Everything above overlaps the previous kernel on the stream; nothing
  // global is read before it has completed.
  pdl_wait_primary();
  pdl_launch_dependents();

  if (warp == NCOMPUTE) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && !p.withhold) {
      // The query rows go first, so they are not queued behind the KV ring.
      const uint32_t hb = p.in_bf16 ? 512u : 1024u;  // bytes of one head's 256 query values
      mbar_arrive_expect_tx(qbar, ROWS * GQA * hb + 512);
      for (int r = 0; r < ROWS; ++r)
        for (int hl = 0; hl < GQA; ++hl) {
          const size_t el = (size_t)r * QROW + (size_t)(kvh * GQA + hl) * 512;
          const uint8_t* src = reinterpret_cast<const uint8_t*>(p.q_gate) + el * (p.in_bf16 ? 2 : 4);
          bulk_load(smem + DEC_QS_OFF + r * DEC_QROW_BYTES + hl * hb, src, hb, qbar);
        }
      bulk_load(smem + DEC_WN_OFF, p.q_norm_w, 512, qbar);
      // Chunks of this kv head are taken dynamically (one atomic per chunk);
      // a chunk's numerics do not depend on which CTA runs it.
      uint32_t i = 0;
      bool done = false;
      const uint64_t pol = l2_policy_evict_first();
      while (!done) {
        const uint32_t chunk = atomicAdd(&p.sched[kvh], 1u);
        done = chunk >= p.nchunks;
        const uint32_t nt = done ? 1 : chunk_tiles(chunk, p.extent);
        for (uint32_t t = 0; t < nt; ++t, ++i) {
          const uint32_t slot = i % DEC_STAGES;
          if (i >= DEC_STAGES && !mbar_wait(&empty[slot], ((i / DEC_STAGES) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY, p.wait_ns)) {
            done = true;
            break;
          }
          slot_code[slot] = done ? -1 : (int)((chunk << 8) | t);
          if (done) {
            mbar_arrive(&full[slot]);  // end marker, no data
            break;
          }
          issue_tile(smem + slot * DEC_STAGE_BYTES, &full[slot], &tk, &tv, chunk * DEC_CHUNK + t * DEC_TILE, kvh,
                     pol);
        }
      }
    }
    return;
  }

  const int m = warp >> 2, w = warp & 3;
  RowXch& X = xch[m];

  // ---- query prologue: q RMSNorm + RoPE (attention.metal:118-155) ----------
  // The raw query of row m (6 heads) is in shared memory. Warp w normalises
  // heads w and w+4 (heads 6, 7 are zero padding), 8 dims per lane, and writes
  // bf16 rows [8][256] over the raw data; then every warp loads its B
  // fragments b0[kk] = Q[head g][16kk + 2q, +1], b1[kk] = Q[head g][16kk+8+2q, +1].
  uint32_t bq0[16], bq1[16];
  {
    uint8_t* qrow = smem + DEC_QS_OFF + m * DEC_QROW_BYTES;
    const uint16_t* wn = reinterpret_cast<const uint16_t*>(smem + DEC_WN_OFF);
    if (!mbar_wait(qbar, 0, p.err, ERR_TIMEOUT_FULL, p.wait_ns)) return;
    uint4 packed[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int hl = w + 4 * u;
      packed[u] = make_uint4(0u, 0u, 0u, 0u);
      if (hl < GQA) {
        float x[8], ss = 0.f;
        if (p.in_bf16) {
          const uint4 raw = *reinterpret_cast<const uint4*>(qrow + hl * 512 + lane * 16);
          const uint32_t wds[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            x[2 * i] = bf16_bits_to_f32(wds[i] & 0xffffu);
            x[2 * i + 1] = bf16_bits_to_f32(wds[i] >> 16);
          }
        } else {
          const float4 a = *reinterpret_cast<const float4*>(qrow + hl * 1024 + lane * 32);
          const float4 b = *reinterpret_cast<const float4*>(qrow + hl * 1024 + lane * 32 + 16);
          x[0] = round_bf16(a.x); x[1] = round_bf16(a.y); x[2] = round_bf16(a.z); x[3] = round_bf16(a.w);
          x[4] = round_bf16(b.x); x[5] = round_bf16(b.y); x[6] = round_bf16(b.z); x[7] = round_bf16(b.w);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const float inv = 1.0f / sqrtf(ss / 256.0f + p.eps);
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float n = x[i] * inv * bf16_bits_to_f32(wn[lane * 8 + i]);
          const float partner = __shfl_xor_sync(0xffffffffu, n, 4);
          o[i] = n;
          if (lane < 8) {
            const int j = (lane & 3) * 8 + i;  // pair index 0..31
            const float c = p.rope_c[m][j], sn = p.rope_s[m][j];
            o[i] = lane < 4 ? n * c - partner * sn : n * c + partner * sn;
          }
        }
        packed[u] = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                               pack_bf16x2(o[6], o[7]));
      }
    }
    named_bar_sync(1 + m, 128);  // every raw value of row m has been read
    uint16_t* qs = reinterpret_cast<uint16_t*>(qrow);
#pragma unroll
    for (int u = 0; u < 2; ++u) *reinterpret_cast<uint4*>(qs + (w + 4 * u) * HD + lane * 8) = packed[u];
    named_bar_sync(1 + m, 128);
    const uint32_t qaddr = smem_u32(qs) + (lane & 7) * (HD * 2) + (lane >> 3) * 16;
#pragma unroll
    for (int kp = 0; kp < 8; ++kp) ldmatrix_x4(qaddr + kp * 64, bq0[2 * kp], bq1[2 * kp], bq0[2 * kp + 1], bq1[2 * kp + 1]);
  }

  // Row m attends local rows [0, lim).
  const int64_t lim64 = (int64_t)p.base + m + 1 - (int64_t)p.kv_lo;
  const uint32_t lim = lim64 <= 0 ? 0u : (uint32_t)(lim64 < (int64_t)p.extent ? lim64 : (int64_t)p.extent);

  float o[4][4];  // O^T for dims 64w + 16i + {g, g+8}, heads 2q, 2q+1
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads 2q, 2q+1

#ifdef LISA_DECODE_TRACE
  if (threadIdx.x == 0) p.trace[16 + blockIdx.x * 4 + 1] = global_timer_ns();
  unsigned long long tr[8] = {};
  long long tlast = clock64();
#define DEC_TRACE(k)            \
  {                             \
    const long long tn = clock64(); \
    tr[k] += tn - tlast;        \
    tlast = tn;                 \
  }
#else
#define DEC_TRACE(k)
#endif
  const int bar_row = 1 + m;  // named barrier of row m's 4 warps
  for (uint32_t it = 0;; ++it) {
    const int s = it % DEC_STAGES, par = it & 1;
    uint8_t* stage = smem + s * DEC_STAGE_BYTES;
    DEC_TRACE(0);
    if (!mbar_wait(&full[s], (it / DEC_STAGES) & 1, p.err, ERR_TIMEOUT_FULL, p.wait_ns)) return;
    DEC_TRACE(1);
#ifdef LISA_DECODE_TRACE
    if (it == 0 && threadIdx.x == 0) p.trace[16 + blockIdx.x * 4 + 3] = global_timer_ns();
#endif
    const int code = slot_code[s];
    if (code < 0) break;
    const uint32_t cur_chunk = (uint32_t)code >> 8, cur_tile = (uint32_t)code & 0xffu;
    const uint32_t row0 = cur_chunk * DEC_CHUNK + cur_tile * DEC_TILE;
    const uint32_t sK = smem_u32(stage), sV = sK + DEC_STAGE_BYTES / 2;

    // This call's new K/V rows are appended here: warp (0, 0) normalises and
    // ropes them, writes the cache and substitutes them in the staged tile.
    bool has_new = false;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int64_t lp = (int64_t)p.base + r - (int64_t)p.kv_lo;
      has_new |= lp >= (int64_t)row0 && lp < (int64_t)row0 + DEC_TILE && lp < (int64_t)p.extent;
    }
    if (has_new) {
      if (warp == 0) {
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          const int64_t lp = (int64_t)p.base + r - (int64_t)p.kv_lo;
          if (lp >= (int64_t)row0 && lp < (int64_t)row0 + DEC_TILE && lp < (int64_t)p.extent) {
            uint4 kr, vr;
            new_kv_row(p, r, kvh, p.base + r, lane, kr, vr);
            const uint32_t off = (lane >> 3) * (DEC_TILE * 128) + swz128((uint32_t)lp - row0, lane & 7);
            *reinterpret_cast<uint4*>(stage + off) = kr;
            *reinterpret_cast<uint4*>(stage + DEC_STAGE_BYTES / 2 + off) = vr;
            const size_t go = ((size_t)kvh * p.window_rows + (size_t)lp) * HD + lane * 8;
            *reinterpret_cast<uint4*>(p.k_cache + go) = kr;
            *reinterpret_cast<uint4*>(p.v_cache + go) = vr;
          }
        }
        fence_proxy_async_smem();
      }
      named_bar_sync(5, 32 * NCOMPUTE);
    }

    // S^T[16 tok x 8 heads] = K[16w.., :] . Q^T, two independent mma chains
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
    // scale + causal mask: c0,c1 -> token row0+16w+g, c2,c3 -> +8
    const uint32_t t0 = row0 + 16 * w + g;
    const bool v0 = t0 < lim, v1 = t0 + 8 < lim;
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
    DEC_TRACE(2);
    if (g == 0) *reinterpret_cast<float2*>(&X.red[par][w][2 * q]) = make_float2(mx0, mx1);
    named_bar_sync(bar_row, 128);
    DEC_TRACE(3);
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
    // the denominator sums the same bf16 weights the PV product uses
    float ls0 = bf16_bits_to_f32(x0 & 0xffffu) + bf16_bits_to_f32(x1 & 0xffffu);
    float ls1 = bf16_bits_to_f32(x0 >> 16) + bf16_bits_to_f32(x1 >> 16);
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      ls0 += __shfl_xor_sync(0xffffffffu, ls0, off);
      ls1 += __shfl_xor_sync(0xffffffffu, ls1, off);
    }
    if (g == 0) *reinterpret_cast<float2*>(&X.lsum[par][w][2 * q]) = make_float2(ls0, ls1);
    X.pb[par][w][lane] = make_uint2(movmatrix_trans(x0), movmatrix_trans(x1));
    DEC_TRACE(4);
    named_bar_sync(bar_row, 128);
    DEC_TRACE(5);
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
    // O^T[64w.., heads] += V^T . P^T over the stage's 64 tokens
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
    DEC_TRACE(6);

    if (cur_tile + 1 == chunk_tiles(cur_chunk, p.extent)) {
      // chunk done: write its partial
      const size_t unit = ((size_t)m * KVH + kvh) * p.chunk_cap + cur_chunk;
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
    DEC_TRACE(7);
  }
#ifdef LISA_DECODE_TRACE
  if (lane == 0)
    for (int k = 0; k < 8; ++k) atomicAdd(&p.trace[k], tr[k]);
  if (lane == 0 && warp == 0) atomicAdd(&p.trace[8], 1ull);
  if (threadIdx.x == 0) p.trace[16 + blockIdx.x * 4 + 2] = global_timer_ns();
#endif
}

// Merges one row's chunk partials for one kv head and 8 dims. Thread
// (phase, slot): slot = tid & 31 -> (dim = db*8 + slot/4, heads 2*(slot&3), +1);
// phase = tid >> 5 folds chunks c = phase, phase + 32, ... with an online
// log-sum-exp merge; the 32 phase states are then merged in phase order. The
// order depends only on the row's own context, so verify rows stay
// bit-identical to single-row decode. Applies the gate (gated_out) or writes
// the window partial (win_o / win_ml). Grid rows * 4 * 32 CTAs of 1024 threads.
struct Lse2 {
  float m0, m1, a0, a1, d0, d1;  // max, weighted O, weighted sum for 2 heads
};

__device__ __forceinline__ void lse_fold(float& m, float& a, float& d, float cm, float ca, float cd) {
  const float nm = fmaxf(m, cm);
  if (nm == -INFINITY) return;
  const float wo = fast_exp2(LOG2E * (m - nm)), wn = fast_exp2(LOG2E * (cm - nm));
  a = a * wo + ca * wn;
  d = d * wo + cd * wn;
  m = nm;
}

__global__ void __launch_bounds__(CMB_THREADS) decode_combine_kernel(const DecodeParams p) {
  pdl_wait_primary();
#ifdef LISA_DECODE_TRACE
  if (threadIdx.x == 0) atomicMin(&p.trace[10], (unsigned long long)global_timer_ns());
#endif
  pdl_launch_dependents();
  if (blockIdx.x == 0 && threadIdx.x < KVH) p.sched[threadIdx.x] = 0;  // ready for the next launch
  __shared__ Lse2 s_state[CMB_PHASES][32];
  const int db = blockIdx.x & 31;
  const int kvh = (blockIdx.x >> 5) & 3;
  const int m = blockIdx.x >> 7;
  const int slot = threadIdx.x & 31, phase = threadIdx.x >> 5;
  const int dim = db * CMB_DIMS_PER_CTA + (slot >> 2);
  const int hp = slot & 3;

  const int64_t lim64 = (int64_t)p.base + m + 1 - (int64_t)p.kv_lo;
  const uint32_t lim = lim64 <= 0 ? 0u : (uint32_t)(lim64 < (int64_t)p.extent ? lim64 : (int64_t)p.extent);
  const uint32_t nch = (lim + DEC_CHUNK - 1) / DEC_CHUNK;
  // the gate of this thread's two heads, loaded now so that its latency
  // overlaps the partials' (phase 0 applies it at the end)
  float sig[2] = {0.f, 0.f};
  if (phase == 0 && p.gated_out) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int hl = 2 * hp + e;
      if (hl < GQA) {
        // gate_out_bf16 (attention.metal:520-531); gate = bf16-rounded raw gate
        const float gv = load_in_bf16(p.q_gate, (size_t)m * QROW + (size_t)(kvh * GQA + hl) * 512 + 256 + dim,
                                      p.in_bf16);
        sig[e] = 1.0f / (1.0f + exp2f(-LOG2E * gv));
      }
    }
  }
  const size_t unit0 = ((size_t)m * KVH + kvh) * p.chunk_cap;

  Lse2 st = {-INFINITY, -INFINITY, 0.f, 0.f, 0.f, 0.f};
  constexpr int U = 4;  // chunks whose loads are in flight together
  for (uint32_t c0 = phase; c0 < nch; c0 += U * CMB_PHASES) {
    float2 cm[U], cl[U], ov[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t c = c0 + u * CMB_PHASES;
      if (c < nch) {
        const float* ml = p.part_ml + (unit0 + c) * 16;
        cm[u] = *reinterpret_cast<const float2*>(ml + 2 * hp);
        cl[u] = *reinterpret_cast<const float2*>(ml + 8 + 2 * hp);
        ov[u] = *reinterpret_cast<const float2*>(p.part_o + (unit0 + c) * 2048 + dim * 8 + 2 * hp);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (c0 + u * CMB_PHASES < nch) {
        lse_fold(st.m0, st.a0, st.d0, cm[u].x, ov[u].x, cl[u].x);
        lse_fold(st.m1, st.a1, st.d1, cm[u].y, ov[u].y, cl[u].y);
      }
    }
  }
  s_state[phase][slot] = st;
  __syncthreads();
  // fixed binary tree over the 32 phase states
#pragma unroll
  for (int half = CMB_PHASES / 2; half >= 1; half >>= 1) {
    if (phase < half) {
      const Lse2 o = s_state[phase + half][slot];
      lse_fold(st.m0, st.a0, st.d0, o.m0, o.a0, o.d0);
      lse_fold(st.m1, st.a1, st.d1, o.m1, o.a1, o.d1);
      s_state[phase][slot] = st;
    }
    __syncthreads();
  }
#ifdef LISA_DECODE_TRACE
  if (threadIdx.x == 0) atomicMax(&p.trace[11], (unsigned long long)global_timer_ns());
#endif
  if (phase != 0) return;
  if (p.xchg) {
    // Exchange mode: this CTA's slice of the window partial (row m, kv head,
    // 8 dims, 6 heads) goes to every rank's receive region (peer stores over
    // NVLink). Every value travels with the step number in one aligned 8-byte
    // store (value bits low, step high), so a reader that sees the step in a
    // word has that word's value: no flag and no fence.
    const XchgDev& x = *p.xchg;
    const uint32_t epoch = x.state[0] + 1;
    const size_t xs = (size_t)(epoch & 1) * x.world + x.rank;  // parity, source rank
    const uint64_t tag = (uint64_t)epoch << 32;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int hl = 2 * hp + e;
      if (hl >= GQA) continue;
      const int h = kvh * GQA + hl;
      const float a = e ? st.a1 : st.a0, dn = e ? st.d1 : st.d0, gmax = e ? st.m1 : st.m0;
      const float o = nch ? a / dn : 0.f;
      const size_t rec = ((xs * x.max_rows + m) * QH + h) * XCHG_REC;
      for (int dst = 0; dst < x.world; ++dst) {
        uint64_t* r = x.recv[dst] + rec;
        st_relaxed_sys_u64(r + dim, tag | __float_as_uint(o));
        if (dim == 0) {
          st_relaxed_sys_u64(r + HD, tag | __float_as_uint(nch ? gmax : -INFINITY));
          st_relaxed_sys_u64(r + HD + 1, tag | __float_as_uint(nch ? dn : 0.f));
        }
      }
    }
    return;
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int hl = 2 * hp + e;
    if (hl >= GQA) continue;
    const int h = kvh * GQA + hl;
    const float a = e ? st.a1 : st.a0, dn = e ? st.d1 : st.d0, gmax = e ? st.m1 : st.m0;
    const float o = nch ? a / dn : 0.f;
    if (p.gated_out) {
      p.gated_out[(size_t)m * OROW + h * HD + dim] = f32_to_bf16_bits(o * sig[e]);
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

// Exchange merge: grid rows * 24 CTAs (row m, head h) of 256 threads (one per
// dim). Thread d waits (bounded) until its dim and the (max, sum) words of
// every rank's record carry this step; then the
// world partials are merged by log-sum-exp in rank order (the same order on
// every rank, so every rank produces identical bits) and gated. The last CTA
// to finish advances the step counter.
__global__ void __launch_bounds__(256) merge_exchange_kernel(const XchgDev* xp, int rows, int in_bf16,
                                                             const void* q_gate, uint16_t* gated_out,
                                                             uint64_t wait_ns) {
  pdl_wait_primary();
  // the next kernel may set up now; it reads nothing before this one completes
  pdl_launch_dependents();
  const XchgDev& x = *xp;
  const int mh = blockIdx.x;
  const int m = mh / QH, h = mh % QH, d = threadIdx.x, kvh = h / GQA;
  const uint32_t epoch = x.state[0] + 1;
  const uint64_t* base = x.recv[x.rank] + (size_t)(epoch & 1) * x.world * x.max_rows * QH * XCHG_REC;
  // the value of word w of source g's record, once it carries this step
  const uint64_t t0 = global_timer_ns();
  bool fail = false;
  auto take = [&](int g, int w) -> float {
    const uint64_t* a = base + (((size_t)g * x.max_rows + m) * QH + h) * XCHG_REC + w;
    uint64_t v = ld_relaxed_sys_u64(a);
    while ((uint32_t)(v >> 32) != epoch && !fail) {
      if (global_timer_ns() - t0 > wait_ns) {
        atomicExch(reinterpret_cast<int*>(x.state + 2), ERR_TIMEOUT_XCHG);
        fail = true;
        break;
      }
      __nanosleep(32);
      v = ld_relaxed_sys_u64(a);
    }
    return __uint_as_float((uint32_t)v);
  };
  float mg[XCHG_MAX_WORLD], lgv[XCHG_MAX_WORLD], og[XCHG_MAX_WORLD];
  float gmax = -INFINITY;
  for (int g = 0; g < x.world; ++g) {
    mg[g] = take(g, HD);
    lgv[g] = take(g, HD + 1);
    og[g] = take(g, d);
    gmax = fmaxf(gmax, mg[g]);
  }
  if (!fail) {
    float acc = 0.f, den = 0.f;
    for (int g = 0; g < x.world; ++g) {
      if (lgv[g] == 0.f) continue;
      const float w = exp2f(LOG2E * (mg[g] - gmax)) * lgv[g];
      acc += w * og[g];
      den += w;
    }
    const float o = den > 0.f ? acc / den : 0.f;
    const float gv = load_in_bf16(q_gate, (size_t)m * QROW + (size_t)h * 512 + 256 + d, in_bf16);
    const float sg = 1.0f / (1.0f + exp2f(-LOG2E * gv));
    gated_out[(size_t)m * OROW + h * HD + d] = f32_to_bf16_bits(o * sg);
  }
  // every CTA has read the step counter before the last one advances it
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(x.state + 1, 1u) == gridDim.x - 1) {
      x.state[1] = 0;
      x.state[0] = epoch;
    }
  }
}

template <int ROWS>
static cudaError_t launch_split(const DecodeParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int num_sms,
                                cudaStream_t stream) {
  static SmemAttr attr_once;  // the attribute is per kernel and per device
  cudaError_t e = attr_once.ensure(decode_split_kernel<ROWS>, DEC_SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const uint32_t per_head = std::min<uint32_t>(p.nchunks, (uint32_t)(num_sms / KVH));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(per_head * KVH);
  cfg.blockDim = dim3(32 * (4 * ROWS + 1));
  cfg.dynamicSmemBytes = DEC_SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_split_kernel<ROWS>, tk, tv, p);
}

#ifdef LISA_DECODE_TRACE
unsigned long long* g_decode_trace = nullptr;  // debug builds: set by a trace harness
#endif

cudaError_t launch_decode(const DecodeParams& p_in, int rows, const CUtensorMap& tk, const CUtensorMap& tv,
                          int num_sms, cudaStream_t stream) {
  DecodeParams p = p_in;
#ifdef LISA_DECODE_TRACE
  p.trace = g_decode_trace;
#endif
  // inverse frequencies once per process; cos/sin of the f32 angle in double,
  // for the rows of this call only (host time is part of every layer call)
  static const struct InvFreqTable {
    float v[32];
    InvFreqTable() { host_inv_freq(v); }
  } inv;
  for (int r = 0; r < rows && r < 3; ++r)
    for (int j = 0; j < 32; ++j) {
      const float angle = (float)(p.base + (uint32_t)r) * inv.v[j];
      double sd, cd;
      ::sincos((double)angle, &sd, &cd);
      p.rope_c[r][j] = (float)cd;
      p.rope_s[r][j] = (float)sd;
    }
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
  cfg.blockDim = dim3(CMB_THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_combine_kernel, p);
}

cudaError_t launch_merge_exchange(const XchgDev* x, int rows, int in_bf16, const void* q_gate, uint16_t* gated_out,
                                  uint64_t wait_ns, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows * QH);
  cfg.blockDim = dim3(HD);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, merge_exchange_kernel, x, rows, in_bf16, q_gate, gated_out, wait_ns);
}

cudaError_t launch_merge_windows(int n_parts, int rows, const float* part_o, const float* part_ml, int in_bf16,
                                 const void* q_gate, uint16_t* gated_out, cudaStream_t stream) {
  merge_windows_kernel<<<rows * QH, HD, 0, stream>>>(n_parts, rows, part_o, part_ml, in_bf16, q_gate, gated_out);
  return cudaGetLastError();
}

}  // namespace lisa
