// prefill.cu — chunked prefill of the lisa-rs full-attention layer on the
// sm_100a 5th-generation tensor core (tcgen05.mma, TMEM accumulators, TMA).
//
// Replaces encode_prefill_attention's attention part (runner.rs:1976-2060):
//   q_norm_gate_rope_prefill   attention.metal:364-401  -> prefill_prologue_kernel
//   kv_cache_store_prefill     attention.metal:403-440  -> prefill_prologue_kernel
//   sdpa_decode_prefill        attention.metal:442-480  -> prefill_attn_kernel
//   gate_out_bf16              attention.metal:520-531  -> prefill_attn_kernel epilogue
// The reference scans every key serially per (row, head) on scalar lanes;
// here a cluster of two CTAs runs a flash-attention loop over 128-key tiles
// of the causal prefix for 256 query rows of one head, as M=256
// tcgen05.mma.cta_group::2 tiles issued by rank 0. Each CTA holds 128 rows
// (its own Q tile in shared memory, its own TMEM: columns [0,256) O,
// [256,384) and [384,512) two S/P tiles) and loads half of every K tile (64
// keys) and half of every V tile (128 dims) with one 32 KB TMA box each:
//   warp 0       Q load, K half-tiles through a 2-slot ring, then the gate tile
//   warp 2       V half-tiles through a 2-slot ring
//   warp 1       allocates TMEM; on rank 0 one thread issues
//                S_j = Q.K_j^T  (A, B from smem; M256 N128 K256)
//                O  += P_j.V_j  (A = P from TMEM, B = V read MN-major; M256 N256 K128)
//                in the order S_0, S_1, PV_0, S_2, PV_1, ... without waits
//                between groups (the next group's inputs are tested before
//                the current group's last MMA)
//   warps 4..11  softmax: thread = query row = TMEM lane; warps 4+w and 8+w
//                share lanes 32w.. and split the columns, exchange their
//                maxima through shared memory, keep an online max that is only
//                moved (and O rescaled in TMEM) when it grows by more than 2^8,
//                and write bf16 P over the S tile it came from; epilogue
//                O/l * sigmoid(gate) staged in shared memory and written by
//                one TMA store.
// Key tiles past the pair's last query row are skipped (causal tile skipping).
// For chunks deep into the context the host planner (plan_segments) splits
// every (pair, head) unit into two key ranges run by separate clusters, so
// that the grid fills the SMs that 48 units leave idle; the two ranges merge
// through a global partial (ticket + flag per CTA rank).
#include <algorithm>
#include <atomic>

#include "../../include/lisa_attn.h"
#include "common.cuh"
#include "prefill.cuh"
#include "dispatch.h"
#include "tcgen05.cuh"

namespace lisa {

namespace {

constexpr int PF_BM = 128;        // query rows per CTA (TMEM lanes)
constexpr int PF_BN = 128;        // keys per tile
constexpr int PF_Q_BYTES = PF_BM * HD * 2;          // 64 KB: this CTA's 128 query rows
constexpr int PF_KH_BYTES = (PF_BN / 2) * HD * 2;   // 32 KB: this CTA's 64 keys of a K tile
constexpr int PF_VH_BYTES = PF_BN * (HD / 2) * 2;   // 32 KB: this CTA's 128 dims of a V tile
constexpr int PF_OFF_K = PF_Q_BYTES;                // 2 K slots
constexpr int PF_OFF_V = PF_OFF_K + 2 * PF_KH_BYTES;  // 2 V slots
constexpr int PF_OFF_BAR = PF_OFF_V + 2 * PF_VH_BYTES;
constexpr int PF_SMEM_BYTES = PF_OFF_BAR + 4096 + 1024;  // barriers, TMEM slot, max/sum exchange
constexpr int PF_THREADS = 384;  // warp 0 Q/K loads, 1 MMA, 2 V loads, 4..11 softmax
constexpr uint32_t PF_TMEM_COLS = 512;
constexpr uint32_t PF_TMEM_O = 0;    // O accumulator: columns [0, 256)
constexpr uint32_t PF_TMEM_S = 256;  // S / P tiles: columns [256, 384), [384, 512)
constexpr float PF_RESCALE_LOG2 = 8.0f;
constexpr float kLog2Scale = SCALE * LOG2E;  // raw score -> exp2 argument
constexpr uint16_t PF_PAIR = 3;  // multicast mask: both CTAs of the pair

// mbarrier slots. *FULL, Q and PFULL are waited on by the pair's MMA issuer
// (rank 0) and complete with both CTAs' loads / arrivals; SFULL and PVDONE
// are signalled to both CTAs by the MMA commits.
enum {
  B_Q = 0,
  B_KFULL = 1,   // [2]
  B_VFULL = 3,   // [2]
  B_SFULL = 5,   // [2] S tile in TMEM; also: the K slot it read is free
  B_PFULL = 7,   // [2] P tile in TMEM (8 softmax warps x 2 CTAs)
  B_PVDONE = 9,  // [2] P.V finished (O updated); also: its P tile and V slot are free
  B_G = 11,      // this CTA's gate tile in the K ring (bf16 inputs)
  B_COUNT = 12
};

}  // namespace

// Eight consecutive inputs rounded to bf16, vectorised (idx multiple of 8).
__device__ __forceinline__ void load8_in(const void* src, size_t idx, int is_bf16, float (&out)[8]) {
  if (is_bf16) {
    const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + idx);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      out[2 * i] = bf16_bits_to_f32(u[i] & 0xffffu);
      out[2 * i + 1] = bf16_bits_to_f32(u[i] >> 16);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx + 4);
    out[0] = round_bf16(a.x); out[1] = round_bf16(a.y); out[2] = round_bf16(a.z); out[3] = round_bf16(a.w);
    out[4] = round_bf16(b.x); out[5] = round_bf16(b.y); out[6] = round_bf16(b.z); out[7] = round_bf16(b.w);
  }
}

// Eight consecutive inputs as packed bf16 pairs (f32 inputs rounded to
// nearest-even, as the reference rounds its inputs), idx a multiple of 8.
__device__ __forceinline__ uint4 load8_bf16(const void* src, size_t idx, int is_bf16) {
  if (is_bf16) return *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(src) + idx);
  const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx);
  const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx + 4);
  return make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
}

// One 256-thread CTA per prompt row; warp w handles items w, w+8, w+16, w+24
// (items 0..23 are the query heads, 24..27 the KV heads). Lane l holds dims
// 8l..8l+7; the RoPE partner of dims 0..31 (lanes 0..3) is dims 32..63
// (lanes 4..7). Warp 0 first computes the row's 32 RoPE (cos, sin) pairs (one
// double-precision sincos per lane) into shared memory, then every warp issues
// its loads; the one CTA barrier falls inside the load latency. At most 64
// registers: all 512 CTAs of a chunk fit in one wave.
__global__ void __launch_bounds__(256, 4) prefill_prologue_kernel(const PrefillParams p) {
  __shared__ float s_cs[2 * ROT_PAIRS];  // pair j: cos at [2j], sin at [2j + 1]
  pdl_wait_primary();       // the previous chunk may still read q_ws
  pdl_launch_dependents();  // let the attention kernel set up meanwhile
  const int r = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t pos = p.base + r;
#ifdef LISA_PREFILL_TRACE
  if (threadIdx.x == 0) atomicMin(&p.trace[32], (unsigned long long)global_timer_ns());
  if (threadIdx.x == 0 && r < 512) p.trace[3072 + r] = global_timer_ns();
#endif
  if (warp == 0) {
    float c, sn;
    rope_cs(pos, p.inv_freq[lane], c, sn);
    s_cs[2 * lane] = c;
    s_cs[2 * lane + 1] = sn;
  }
  constexpr int NI = 4;  // items per warp
  uint4 xr[NI], vr = make_uint4(0, 0, 0, 0);  // 8 inputs as bf16 pairs; vr: the V row of the KV item
  const uint4 qw4 = *reinterpret_cast<const uint4*>(p.q_norm_w + lane * 8);
  const uint4 kw4 = *reinterpret_cast<const uint4*>(p.k_norm_w + lane * 8);
#pragma unroll
  for (int t = 0; t < NI; ++t) {
    const int hh = warp + 8 * t;
    if (hh >= QH + KVH) continue;
    const bool is_q = hh < QH;
    const size_t in = is_q ? (size_t)r * QROW + (size_t)hh * 512 + lane * 8
                           : (size_t)r * KROW + (size_t)(hh - QH) * HD + lane * 8;
    xr[t] = load8_bf16(is_q ? p.q_gate : p.k_in, in, p.in_bf16);
    if (!is_q) vr = load8_bf16(p.v_in, in, p.in_bf16);
  }
  __syncthreads();  // RoPE table ready
  // Per-lane factors shared by every item of the row (the same position):
  // element i of lane l becomes n_i * rc_i + partner_i * rs_i, with (rc, rs)
  // = (cos, -sin) on lanes 0..3, (cos, +sin) on lanes 4..7 and (1, 0) on the
  // other lanes; and the query gains as f32.
  float rc[8], rs[8], gq[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 cs = *reinterpret_cast<const float2*>(&s_cs[2 * ((lane & 3) * 8 + i)]);
    rc[i] = lane < 8 ? cs.x : 1.0f;
    rs[i] = lane < 4 ? -cs.y : lane < 8 ? cs.y : 0.0f;
    const float2 g2 = unpack_bf16x2((&qw4.x)[i >> 1]);
    gq[i] = (i & 1) ? g2.y : g2.x;
  }
#pragma unroll
  for (int t = 0; t < NI; ++t) {
    const int hh = warp + 8 * t;
    if (hh >= QH + KVH) continue;  // uniform per warp
    const bool is_q = hh < QH;
    float x8[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2((&xr[t].x)[i]);
      x8[2 * i] = f.x;
      x8[2 * i + 1] = f.y;
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(x8[i], x8[i], ss);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(ss / 256.0f + p.eps);  // the shader's rsqrt (attention.metal:364-401)
    float n[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float g = gq[i];
      if (!is_q) {
        const float2 g2 = unpack_bf16x2((&kw4.x)[i >> 1]);
        g = (i & 1) ? g2.y : g2.x;
      }
      n[i] = x8[i] * inv * g;
    }
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float partner = __shfl_xor_sync(0xffffffffu, n[i], 4);
      o[i] = fmaf(partner, rs[i], n[i] * rc[i]);  // lanes >= 8: n * 1 + partner * 0
    }
    const uint4 packed = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                                    pack_bf16x2(o[6], o[7]));
    if (is_q) {
      // q_ws [head][row][256]
      *reinterpret_cast<uint4*>(p.q_ws + ((size_t)hh * PF_MAX_ROWS + r) * HD + lane * 8) = packed;
    } else {
      const size_t out = ((size_t)(hh - QH) * p.capacity + pos) * HD + lane * 8;
      *reinterpret_cast<uint4*>(p.k_cache + out) = packed;
      *reinterpret_cast<uint4*>(p.v_cache + out) = vr;
    }
  }
#ifdef LISA_PREFILL_TRACE
  __syncthreads();
  if (threadIdx.x == 0) atomicMax(&p.trace[33], (unsigned long long)global_timer_ns());
  if (threadIdx.x == 0 && r < 512) p.trace[3584 + r] = global_timer_ns();
#endif
}

// Grid: clusters of 2 CTAs, one per key-range segment of p.seg_*: a (query
// row pair, head) unit whole, or one of the two consecutive key ranges of a
// split unit. Cluster rank 0 holds query rows [256 qp, 256 qp + 128), rank 1
// the next 128. The two segments of a split unit merge through p.part: per
// CTA rank, the first to finish stores its unnormalised O, running max and
// sum, the second folds them into its own and writes the gated output.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PF_THREADS, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tg,
                        const __grid_constant__ CUtensorMap to, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PF_OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  float* xmax = reinterpret_cast<float*>(smem + PF_OFF_BAR + 1024);  // [2 parity][2 half][128 rows]
  float* xsum = xmax + 2 * 2 * PF_BM;                                  // [2 half][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cl = (int)(blockIdx.x >> 1);
  const uint32_t su = p.seg_unit[cl];
  const int h = (int)(su & 0xffu), qp = (int)((su >> 8) & 0xfu), kvh = h / GQA;
  const bool split = (su >> 12) & 1u;
  const int r0 = qp * 2 * PF_BM + (int)rank * PF_BM;
  // key tiles [t_lo, t_lo + n_tiles); loop indices below are relative to t_lo
  const uint32_t t_lo = p.seg_lo[cl];
  const int n_tiles = (int)(p.seg_hi[cl] - t_lo);
  const int slot = (qp * QH + h) * 2 + (int)rank;  // split partial / ticket slot

#ifdef LISA_PREFILL_TRACE
  if (threadIdx.x == 0) p.trace[64 + blockIdx.x * 8 + 0] = global_timer_ns();
#endif
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    tma_prefetch_desc(&to);
    for (int b = 0; b < B_COUNT; ++b) mbar_init(&bars[b], (b == B_PFULL || b == B_PFULL + 1) ? 16 : 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, PF_TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // shared::cluster address of rank 0's barrier `i`
  const uint32_t lead_bars = cluster_map(smem_u32(bars), 0);
  auto lead_bar = [&](int i) -> uint32_t { return lead_bars + 8u * (uint32_t)i; };
  // Setup above overlaps the prologue kernel; its q_ws / KV writes are read
  // only after it has completed. The K/V producers first issue the loads of
  // the first two key tiles when they hold only positions below `base`
  // (written by earlier calls), then wait too.
  const int n_early = min(min(2, n_tiles), max(0, (int)(p.base / PF_BN) - (int)t_lo));
  if (!((warp == 0 || warp == 2) && lane == 0)) pdl_wait_primary();
  pdl_launch_dependents();
#ifdef LISA_PREFILL_TRACE
  if (threadIdx.x == 0) p.trace[64 + blockIdx.x * 8 + 1] = global_timer_ns();
  unsigned long long tr[8] = {};
  long long tl = clock64();
#define PT(k)                        \
  {                                  \
    const long long tn = clock64();  \
    tr[k] += tn - tl;                \
    tl = tn;                         \
  }
#define PT_FLUSH(role)                                                             \
  if (lane == 0)                                                                   \
    for (int k = 0; k < 8; ++k) atomicAdd(&p.trace[(role) * 8 + k], tr[k]);
// per-tile event clocks of the first CTA (rank 0 of the heaviest pair)
#define PE(ev, j) \
  if (blockIdx.x == 0 && (j) < 64) p.trace[2048 + (ev) * 64 + (j)] = clock64();
#else
#define PT(k)
#define PT_FLUSH(role)
#define PE(ev, j)
#endif

  if (warp == 0 && lane == 0) {
    // ---------------- Q and K loads ----------------
    // Each CTA loads its own 128 query rows and its half (64 keys) of every
    // K tile; completion is counted on rank 0's barriers, whose expected
    // byte count rank 0 sets for both.
    auto load_k = [&](int j) {
      const int s = j & 1;
      if (rank == 0) mbar_arrive_expect_tx(&bars[B_KFULL + s], 2 * PF_KH_BYTES);
      tma_load_4d_pair(smem + PF_OFF_K + s * PF_KH_BYTES, &tk, lead_bar(B_KFULL + s), 0,
                       ((int)t_lo + j) * PF_BN + (int)rank * (PF_BN / 2), 0, kvh);
    };
    for (int j = 0; j < n_early; ++j) load_k(j);
    pdl_wait_primary();
    if (rank == 0) mbar_arrive_expect_tx(&bars[B_Q], 2 * PF_Q_BYTES);
    tma_load_4d_pair(smem, &tq, lead_bar(B_Q), 0, r0, 0, h);
    for (int j = n_early; j < n_tiles; ++j) {
      // slot j & 1 is free once S_{j-2}, which read it, has completed
      if (j >= 2 && !mbar_wait(&bars[B_SFULL + (j & 1)], ((j >> 1) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) break;
      load_k(j);
    }
    if (p.in_bf16) {
      // once the last two S MMAs have read the K ring, it takes this CTA's
      // gate tile: rows r0.., gate dims 256..511 of head h
      bool free = true;
      for (int j = max(0, n_tiles - 2); free && j < n_tiles; ++j)
        free = mbar_wait(&bars[B_SFULL + (j & 1)], (j >> 1) & 1, p.err, ERR_TIMEOUT_EMPTY);
      if (free) {
        mbar_arrive_expect_tx(&bars[B_G], PF_BM * HD * 2);
        tma_load_4d(smem + PF_OFF_K, &tg, &bars[B_G], 0, r0, 4, h);
      }
    }
  } else if (warp == 2 && lane == 0) {
    // ---------------- V loads: this CTA's 128 dims of every V tile ----------------
    auto load_v = [&](int j) {
      const int s = j & 1;
      if (rank == 0) mbar_arrive_expect_tx(&bars[B_VFULL + s], 2 * PF_VH_BYTES);
      tma_load_4d_pair(smem + PF_OFF_V + s * PF_VH_BYTES, &tv, lead_bar(B_VFULL + s), 0,
                       ((int)t_lo + j) * PF_BN, 2 * (int)rank, kvh);
    };
    for (int j = 0; j < n_early; ++j) load_v(j);
    pdl_wait_primary();
    for (int j = n_early; j < n_tiles; ++j) {
      // slot j & 1 is free once P_{j-2}.V_{j-2}, which read it, has completed
      if (j >= 2 && !mbar_wait(&bars[B_PVDONE + (j & 1)], ((j >> 1) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) break;
      load_v(j);
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------- MMA issuer (rank 0 only, M = 256 over the pair) ----------------
    // The tensor pipe keeps almost no queue: every cycle this thread spends
    // between two MMAs is a cycle the pipe idles. So the group sequence
    // S_0, S_1, PV_0, S_2, PV_1, ... is issued without waits between groups:
    // the inputs of the next group are tested (non-blocking) before the last
    // MMA of the current group, and descriptors are base + constant offsets.
    constexpr uint32_t IDESC_S = umma_idesc_bf16(2 * PF_BM, PF_BN, false);
    constexpr uint32_t IDESC_O = umma_idesc_bf16(2 * PF_BM, HD, true);
    // S_j = Q . K_j^T: 16 k-steps of 16 dims; Q rows and K keys are stored as
    // [64-dim group][row][64 dims]. O += P_j . V_j: 8 k-steps of 16 keys; P
    // (bf16 pairs) lives over the S tile, key k at column k/2; V is stored
    // [64-dim group][key][64 dims] and read MN-major (this CTA holds 2 of the
    // 4 groups).
    const uint64_t dQ = umma_desc_sw128(smem_u32(smem), 16, 1024);
    const uint64_t dK = umma_desc_sw128(smem_u32(smem + PF_OFF_K), 16, 1024);
    const uint64_t dV = umma_desc_sw128(smem_u32(smem + PF_OFF_V), PF_BN * 128, 1024);
    auto s_mma = [&](int j, int kk) {
      const uint32_t g = kk >> 2, sub = kk & 3, s = j & 1;
      umma_pair_bf16(tmem + PF_TMEM_S + s * PF_BN, dQ + ((g * (PF_BM * 128) + sub * 32) >> 4),
                     dK + ((s * PF_KH_BYTES + g * ((PF_BN / 2) * 128) + sub * 32) >> 4), IDESC_S, kk ? 1u : 0u);
    };
    auto pv_mma = [&](int j, int kk) {
      const uint32_t b = j & 1;
      umma_pair_bf16_ts(tmem + PF_TMEM_O, tmem + PF_TMEM_S + b * PF_BN + kk * 8,
                        dV + ((b * PF_VH_BYTES + kk * 2048) >> 4), IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
    };
    auto k_ready = [&](int j) { return mbar_test_wait(&bars[B_KFULL + (j & 1)], (j >> 1) & 1); };
    auto pv_ready = [&](int j) {
      return mbar_test_wait(&bars[B_PFULL + (j & 1)], (j >> 1) & 1) &&
             mbar_test_wait(&bars[B_VFULL + (j & 1)], (j >> 1) & 1);
    };
    bool ok = mbar_wait(&bars[B_Q], 0, p.err, ERR_TIMEOUT_FULL) &&
              mbar_wait(&bars[B_KFULL], 0, p.err, ERR_TIMEOUT_FULL);
    if (ok) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) s_mma(0, kk);
      umma_pair_commit(&bars[B_SFULL], PF_PAIR);
    }
    bool next_ready = false;  // inputs of the next group already seen complete
    for (int j = 0; ok && j < n_tiles; ++j) {
      const int b = j & 1;
      if (j + 1 < n_tiles) {
        // S_{j+1}
        if (!next_ready && !mbar_wait(&bars[B_KFULL + ((j + 1) & 1)], ((j + 1) >> 1) & 1, p.err, ERR_TIMEOUT_FULL))
          break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 15; ++kk) s_mma(j + 1, kk);
        next_ready = pv_ready(j);
        s_mma(j + 1, 15);
        umma_pair_commit(&bars[B_SFULL + ((j + 1) & 1)], PF_PAIR);
      } else {
        next_ready = false;
      }
      // P_j . V_j
      if (!next_ready && !(mbar_wait(&bars[B_PFULL + b], (j >> 1) & 1, p.err, ERR_TIMEOUT_MMA) &&
                           mbar_wait(&bars[B_VFULL + b], (j >> 1) & 1, p.err, ERR_TIMEOUT_FULL)))
        break;
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 7; ++kk) pv_mma(j, kk);
      next_ready = j + 2 < n_tiles && k_ready(j + 2);
      pv_mma(j, 7);
      umma_pair_commit(&bars[B_PVDONE + b], PF_PAIR);
    }
    PT_FLUSH(0);
  }
#if defined(LISA_PREFILL_TRACE) || defined(LISA_PREFILL_OBSERVE)
  else if (warp == 3 && lane == 0 && blockIdx.x == 0) {
    // observer: completion clocks of S_j (event 8) and P_j.V_j (event 9)
    for (int j = 0; j < n_tiles && j < 64; ++j) {
      mbar_wait(&bars[B_SFULL + (j & 1)], (j >> 1) & 1, nullptr, 0);
      p.trace[2048 + 8 * 64 + j] = clock64();
      if (j >= 1) {
        mbar_wait(&bars[B_PVDONE + ((j - 1) & 1)], ((j - 1) >> 1) & 1, nullptr, 0);
        p.trace[2048 + 9 * 64 + j - 1] = clock64();
      }
    }
  }
#endif
  else if (warp >= 4) {
    // ---------------- softmax / correction / epilogue (warps 4..11) ----------------
    // Warp 4+w and warp 8+w share TMEM lanes 32w..32w+31 (one query row per
    // thread); each reads and exponentiates one half (64 keys) of a tile, and
    // the two halves exchange their maxima once per tile.
    const int wi = (warp - 4) & 3;
    const int half = (warp - 4) >> 2;
    const int row = wi * 32 + lane;  // row within the CTA's tile == TMEM lane
    const uint32_t lane_addr = tmem + ((uint32_t)(wi * 32) << 16);
    const uint32_t pos_row = p.base + (uint32_t)(r0 + row);
    bool ok = true;
    float mr = -INFINITY, l = 0.f;  // running max of the raw scores, this half's sum
    for (int j = 0; j < n_tiles; ++j) {
      const int b = j & 1;
      PT(7);
      if (!mbar_wait(&bars[B_SFULL + b], (j >> 1) & 1, p.err, ERR_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
      PT(0);
      if (lane == 0 && warp == 4) { PE(4, j); }
      if (lane == 0 && j == 10) { PE(14, warp - 4); }
      tc_fence_after();
      uint32_t sa[32], sb[32];
      const uint32_t scol = PF_TMEM_S + b * PF_BN + half * 64;
      tmem_ld32(lane_addr + scol, sa);
      tmem_ld32(lane_addr + scol + 32, sb);
      tmem_wait_ld();
      float x[64];  // raw scores Q.K (unscaled)
#pragma unroll
      for (int c = 0; c < 64; ++c) x[c] = __uint_as_float(c < 32 ? sa[c] : sb[c - 32]);
      const uint32_t key0 = (t_lo + (uint32_t)j) * PF_BN + half * 64;
      if (key0 + 63 > pos_row) {  // diagonal tile: keys past this row's position
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (key0 + c > pos_row) x[c] = -INFINITY;
      }
      float t8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        t8[i] = fmaxf(fmax3(fmax3(x[8 * i], x[8 * i + 1], x[8 * i + 2]), x[8 * i + 3], x[8 * i + 4]),
                      fmax3(x[8 * i + 5], x[8 * i + 6], x[8 * i + 7]));
      const float hmax = fmax3(fmax3(t8[0], t8[1], t8[2]), fmax3(t8[3], t8[4], t8[5]), fmaxf(t8[6], t8[7]));
      xmax[(b * 2 + half) * PF_BM + row] = hmax;
      // both halves have read this S tile (P overwrites its first 64 columns)
      // and published their maxima
      named_bar_sync(2 + wi, 64);
      const float mnew = fmax3(mr, hmax, xmax[(b * 2 + (half ^ 1)) * PF_BM + row]);
      // the running max moves only when it grows by more than 2^8 (in exp2 units)
      const bool need = (mnew - mr) * kLog2Scale > PF_RESCALE_LOG2;  // also true for the first finite max
      float alpha = 1.f;
      if (need) {
        alpha = fast_exp2((mr - mnew) * kLog2Scale);
        mr = mnew;
      }
      // P = exp2(x * scale*log2e - m), rounded to bf16 and written over the S
      // tile 16 keys at a time so the TMEM stores overlap the exponentials.
      // 1 of every 8 key pairs is exponentiated on the FMA pipe, the rest on
      // the SFU (measured on config 2: 1/8 and 2/8 are equal, 3/8 is 2 % and
      // 4/8 6 % slower). The denominator sums the
      // f32 values, as the reference's f32 softmax does.
      const float2 cc = make_float2(kLog2Scale, kLog2Scale);
      const float2 nm = make_float2(-mr * kLog2Scale, -mr * kLog2Scale);
      float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t pk[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float2 e = ffma2(make_float2(x[16 * q + 2 * c], x[16 * q + 2 * c + 1]), cc, nm);
          const float2 pe = c < 1 ? exp2_poly2(e) : make_float2(fast_exp2(e.x), fast_exp2(e.y));
          pk[c] = pack_bf16x2(pe.x, pe.y);
          if (c & 1) acc1 = fadd2(acc1, pe);
          else acc0 = fadd2(acc0, pe);
        }
        tmem_st8(lane_addr + PF_TMEM_S + b * PF_BN + half * 32 + q * 8, pk);
      }
      const float2 acc = fadd2(acc0, acc1);
      l = l * alpha + (acc.x + acc.y);
      PT(1);
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O must hold exactly tiles < j before it is rescaled
        if (!mbar_wait(&bars[B_PVDONE + (b ^ 1)], ((j - 1) >> 1) & 1, p.err, ERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < HD / 64; ++c) {
          const uint32_t col = PF_TMEM_O + half * (HD / 2) + c * 32;
          uint32_t ov[32];
          tmem_ld32(lane_addr + col, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st32(lane_addr + col, ov);
        }
      }
      PT(2);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_relaxed(lead_bar(B_PFULL + b));
      if (lane == 0 && warp == 4) { PE(5, j); }
      if (lane == 0 && warp == 8) { PE(6, j); }
      if (lane == 0 && j == 10) { PE(13, warp - 4); }
      PT(4);
    }
#ifdef LISA_PREFILL_TRACE
    if (threadIdx.x == 128) p.trace[64 + blockIdx.x * 8 + 3] = global_timer_ns();
#endif
    // Gate values of this row and half. bf16 inputs: the K producer has
    // brought this CTA's gate tile into the K ring ([group][row][64],
    // 128-byte swizzle) once the last S was computed. f32 inputs: loaded
    // here, rounded to bf16 as the reference does.
    const int r = r0 + row;
    uint32_t gpk[64];
    if (!p.in_bf16 && ok && r < p.rows) {
      const size_t gbase = (size_t)r * QROW + (size_t)h * 512 + 256 + half * 128;
#pragma unroll
      for (int g8 = 0; g8 < 16; ++g8) {
        float gv[8];
        load8_in(p.q_gate, gbase + g8 * 8, 0, gv);
#pragma unroll
        for (int i = 0; i < 4; ++i) gpk[g8 * 4 + i] = pack_bf16x2(gv[2 * i], gv[2 * i + 1]);
      }
    }
    const int last = n_tiles - 1;
    ok = ok && mbar_wait(&bars[B_PVDONE + (last & 1)], (last >> 1) & 1, p.err, ERR_TIMEOUT_MMA);
#ifdef LISA_PREFILL_TRACE
    if (threadIdx.x == 128) p.trace[64 + blockIdx.x * 8 + 2] = global_timer_ns();
#endif
    // Sum the two halves' denominators (half 0 + half 1).
    xsum[half * PF_BM + row] = l;
    named_bar_sync(2 + wi, 64);
    float l_row = xsum[row] + xsum[PF_BM + row];
    if (p.in_bf16) ok = ok && mbar_wait(&bars[B_G], 0, p.err, ERR_TIMEOUT_FULL);
#ifdef LISA_PREFILL_TRACE
    if (threadIdx.x == 128) p.trace[64 + blockIdx.x * 8 + 5] = global_timer_ns();
#endif
    // Split unit: the first segment to get here stores its partial and
    // leaves; the second merges it. Both scale by 2^(m_seg - max(m_a, m_b)),
    // a formula symmetric in the two segments, so the result does not depend
    // on which finished first.
    float a_own = 1.f, a_oth = 0.f;
    const float4* oth = nullptr;
    if (split) {
      uint32_t* ticket = p.tickets + slot;
      uint32_t* ready = p.tickets + 2 * PF_MAX_UNITS + slot;
      float4* po = reinterpret_cast<float4*>(p.part + (size_t)slot * (PF_BM * HD));
      float* pml = p.part + (size_t)2 * PF_MAX_UNITS * PF_BM * HD + (size_t)slot * 2 * PF_BM;
      int* tk_sh = reinterpret_cast<int*>(smem + PF_OFF_BAR + 512);
      if (threadIdx.x == 128) *tk_sh = (int)atomicAdd(ticket, 1u);
      named_bar_sync(6, 256);
      const bool first = *tk_sh == 0;
      if (first) {
        if (ok) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < HD / 64; ++c) {
            const int col = half * (HD / 2) + c * 32;
            uint32_t ov[32];
            tmem_ld32(lane_addr + PF_TMEM_O + col, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i)  // layout [dim/4][row][4]: a warp stores 512 contiguous bytes
              __stcg(po + (col / 4 + i) * PF_BM + row,
                     make_float4(__uint_as_float(ov[4 * i]), __uint_as_float(ov[4 * i + 1]),
                                 __uint_as_float(ov[4 * i + 2]), __uint_as_float(ov[4 * i + 3])));
          }
          if (half == 0) {
            __stcg(pml + row, mr);
            __stcg(pml + PF_BM + row, l_row);
          }
        }
        __threadfence();
        named_bar_sync(6, 256);
        if (threadIdx.x == 128) st_release_gpu(ready, 1u);
        ok = false;  // no output from this segment
      } else {
        if (threadIdx.x == 128) {
          // the first segment has passed its ticket: its store is in flight
          const uint64_t t0 = global_timer_ns();
          bool got = true;
          while (ld_acquire_gpu(ready) == 0u) {
            if (global_timer_ns() - t0 > WAIT_LIMIT_NS) {
              atomicExch(p.err, ERR_TIMEOUT_MERGE);
              got = false;
              break;
            }
          }
          *tk_sh = got ? 1 : -1;
          // ready for the next launch (stream-ordered after this one)
          *ticket = 0u;
          *ready = 0u;
        }
        named_bar_sync(6, 256);
        ok = ok && *tk_sh == 1;
        const float m_oth = __ldcg(pml + row);
        const float m = fmaxf(mr, m_oth);
        a_own = fast_exp2((mr - m) * kLog2Scale);
        a_oth = fast_exp2((m_oth - m) * kLog2Scale);
        l_row = __fadd_rn(__fmul_rn(l_row, a_own), __fmul_rn(__ldcg(pml + PF_BM + row), a_oth));
        oth = po;
      }
    }
    // gated rows staged in the (now idle) V ring as [group][row][64] with the
    // 128-byte swizzle, then written by one TMA store (rows >= p.rows clipped)
#ifdef LISA_PREFILL_TRACE
    if (threadIdx.x == 128) p.trace[64 + blockIdx.x * 8 + 6] = global_timer_ns();
#endif
    // no contraction into an FMA: keeps the merge symmetric in its two terms
    auto mix = [&](float own, float other) { return __fadd_rn(__fmul_rn(own, a_own), __fmul_rn(other, a_oth)); };
    uint8_t* stage = smem + PF_OFF_V;
    const uint8_t* gtile = smem + PF_OFF_K;
    if (ok) {
      tc_fence_after();
      const float inv_l = 1.0f / l_row;
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        const int col = half * (HD / 2) + c * 32;  // first of this pass's 32 dims
        const int grp = col >> 6, ch0 = (col & 63) >> 3;
        uint32_t ov[32];
        tmem_ld32(lane_addr + PF_TMEM_O + col, ov);
        float4 ot[8];
        if (oth) {
#pragma unroll
          for (int i = 0; i < 8; ++i) ot[i] = __ldcg(oth + (col / 4 + i) * PF_BM + row);
        }
        uint32_t gw[16];
        if (p.in_bf16) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 g4 = *reinterpret_cast<const uint4*>(gtile + grp * (PF_BM * 128) + row * 128 +
                                                             (((ch0 + i) ^ (row & 7)) << 4));
            gw[4 * i] = g4.x; gw[4 * i + 1] = g4.y; gw[4 * i + 2] = g4.z; gw[4 * i + 3] = g4.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) gw[i] = gpk[c * 16 + i];
        }
        tmem_wait_ld();
        if (oth) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            ov[4 * i] = __float_as_uint(mix(__uint_as_float(ov[4 * i]), ot[i].x));
            ov[4 * i + 1] = __float_as_uint(mix(__uint_as_float(ov[4 * i + 1]), ot[i].y));
            ov[4 * i + 2] = __float_as_uint(mix(__uint_as_float(ov[4 * i + 2]), ot[i].z));
            ov[4 * i + 3] = __float_as_uint(mix(__uint_as_float(ov[4 * i + 3]), ot[i].w));
          }
        }
        uint32_t outw[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 g2 = unpack_bf16x2(gw[i]);
          outw[i] = pack_bf16x2(__uint_as_float(ov[2 * i]) * inv_l * fast_sigmoid(g2.x),
                                __uint_as_float(ov[2 * i + 1]) * inv_l * fast_sigmoid(g2.y));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
          *reinterpret_cast<uint4*>(stage + grp * (PF_BM * 128) + row * 128 + (((ch0 + i) ^ (row & 7)) << 4)) =
              make_uint4(outw[4 * i], outw[4 * i + 1], outw[4 * i + 2], outw[4 * i + 3]);
      }
    }
#ifdef LISA_PREFILL_TRACE
    if (threadIdx.x == 128) p.trace[64 + blockIdx.x * 8 + 7] = global_timer_ns();
#endif
    fence_proxy_async_smem();
    named_bar_sync(6, 256);  // the staged tile is complete
    if (ok && threadIdx.x == 128) {
      tma_store_4d(&to, stage, 0, r0, 0, h);
      bulk_commit_group();
      bulk_wait_read();  // the staging must stay until the store has read it
    }
    PT(5);
    if (warp == 4) { PT_FLUSH(1); }
#ifdef LISA_PREFILL_TRACE
    if (threadIdx.x == 128) p.trace[64 + blockIdx.x * 8 + 4] = global_timer_ns();
#endif
  }
  // Both CTAs are done with TMEM and with each other's barriers before either
  // frees its columns or exits.
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, PF_TMEM_COLS);
  }
}

namespace {
constexpr size_t PF_QWS_BYTES = (size_t)QH * PF_MAX_ROWS * HD * sizeof(uint16_t);
// partials: O per (unit, rank) then (max, sum) per row
constexpr size_t PF_PART_BYTES = (size_t)2 * PF_MAX_UNITS * (PF_BM * HD + 2 * PF_BM) * sizeof(float);
constexpr size_t PF_TICKET_BYTES = (size_t)2 * 2 * PF_MAX_UNITS * sizeof(uint32_t);

// Cost model of the segment planner, in key-tile times (about 1.45 us each
// with 96 busy SMs), fitted to a globaltimer trace of the config-2 chunks: a
// cluster's fixed cost (start, pipeline fill, epilogue), the extra cost of a
// split segment (storing or loading its partial), and the slower tiles when
// the split grid keeps every SM busy (shared L2 and TMA traffic).
constexpr float PF_PLAN_FIXED = 4.5f;
constexpr float PF_PLAN_SPLIT = 1.5f;
constexpr float PF_PLAN_BUSY = 1.1f;
// a split plan is taken only when it is predicted this much faster: on short
// segments the model is optimistic (a chunk at base 1536 predicted 4 % faster
// measured 18 % slower; at base 3584 predicted 7 %, measured 6 %)
constexpr float PF_PLAN_MIN_GAIN = 0.90f;

// Completion time of the segments when the hardware hands them, in launch
// order, to `slots` cluster slots (each to the slot that frees first).
float plan_makespan(const float* cost, int n, int slots) {
  float fin[128] = {};
  float makespan = 0.f;
  for (int i = 0; i < n; ++i) {
    int s = 0;
    for (int k = 1; k < slots && k < 128; ++k)
      if (fin[k] < fin[s]) s = k;
    fin[s] += cost[i];
    makespan = std::max(makespan, fin[s]);
  }
  return makespan;
}
}  // namespace

size_t prefill_workspace_bytes() { return PF_QWS_BYTES + PF_PART_BYTES + PF_TICKET_BYTES; }
size_t prefill_ticket_offset() { return PF_QWS_BYTES + PF_PART_BYTES; }
size_t prefill_ticket_bytes() { return PF_TICKET_BYTES; }

std::atomic<int> g_prefill_split_mode{LISA_PREFILL_SPLIT_AUTO};

// Splits the chunk's (query pair, head) units into the cluster segments of
// the attention grid. A unit covers key tiles [0, n); split in two it becomes
// [0, a) (launched with the whole units, heaviest first) and [a, n) (launched
// after all of them), which fills the SMs a one-cluster-per-unit grid leaves
// idle: 48 units on 74 cluster slots. The split point is one fraction of n
// for all units, chosen by simulating the dispatch; a is at most the first
// query row's position / 128, so every row sees a key in both ranges.
void plan_segments(PrefillParams& p, int num_sms, int mode) {
  const int n_qt = (p.rows + PF_BM - 1) / PF_BM;
  const int n_pairs = (n_qt + 1) / 2;
  const int slots = std::max(1, std::min(128, num_sms / 2));
  int n_unit = 0, un[PF_MAX_UNITS], amax[PF_MAX_UNITS], uid[PF_MAX_UNITS];
  for (int qp = n_pairs - 1; qp >= 0; --qp) {
    const uint32_t pair_end = (uint32_t)std::min(qp * 2 * PF_BM + 2 * PF_BM, p.rows);
    const uint32_t n = (p.base + pair_end + PF_BN - 1) / PF_BN;
    for (int h = 0; h < QH; ++h) {
      un[n_unit] = (int)n;
      amax[n_unit] = (int)((p.base + (uint32_t)(qp * 2 * PF_BM)) / PF_BN);
      uid[n_unit] = (qp << 8) | h;
      ++n_unit;
    }
  }
  // candidate split fractions in 1/20 steps; 0 = no split
  int best_f = 0;
  float best_t = 0.f, unsplit_t = 0.f;
  for (int f = 0; f <= 17; ++f) {
    if (f != 0 && f < 10) continue;
    float cost[PF_MAX_SEGS], shorts[PF_MAX_UNITS];
    int n = 0, n_short = 0;
    for (int u = 0; u < n_unit; ++u) {
      const int a = f ? std::min(amax[u], (un[u] * f + 10) / 20) : 0;
      if (f && a >= 2 && un[u] - a >= 2) {
        cost[n++] = a * PF_PLAN_BUSY + PF_PLAN_FIXED + PF_PLAN_SPLIT;
        shorts[n_short++] = (un[u] - a) * PF_PLAN_BUSY + PF_PLAN_FIXED + PF_PLAN_SPLIT;
      } else {
        cost[n++] = un[u] + PF_PLAN_FIXED;
      }
    }
    for (int i = 0; i < n_short; ++i) cost[n++] = shorts[i];
    const float t = plan_makespan(cost, n, slots);
    if (f == 0 || t < best_t) {
      best_t = t;
      best_f = f;
    }
    if (f == 0) unsplit_t = t;
  }
  if (best_t > PF_PLAN_MIN_GAIN * unsplit_t) best_f = 0;
  if (mode == LISA_PREFILL_SPLIT_NEVER) best_f = 0;
  if (mode == LISA_PREFILL_SPLIT_ALWAYS) best_f = 14;
  int n = 0;
  uint32_t s_lo[PF_MAX_UNITS], s_hi[PF_MAX_UNITS];
  uint16_t s_unit[PF_MAX_UNITS];
  int n_short = 0;
  for (int u = 0; u < n_unit; ++u) {
    const int a = best_f ? std::min(amax[u], (un[u] * best_f + 10) / 20) : 0;
    if (best_f && a >= 2 && un[u] - a >= 2) {
      p.seg_lo[n] = 0;
      p.seg_hi[n] = (uint32_t)a;
      p.seg_unit[n++] = (uint16_t)(uid[u] | 0x1000);
      s_lo[n_short] = (uint32_t)a;
      s_hi[n_short] = (uint32_t)un[u];
      s_unit[n_short++] = (uint16_t)(uid[u] | 0x1000);
    } else {
      p.seg_lo[n] = 0;
      p.seg_hi[n] = (uint32_t)un[u];
      p.seg_unit[n++] = (uint16_t)uid[u];
    }
  }
  for (int i = 0; i < n_short; ++i) {
    p.seg_lo[n] = s_lo[i];
    p.seg_hi[n] = s_hi[i];
    p.seg_unit[n++] = s_unit[i];
  }
  p.n_seg = n;
}

#ifdef LISA_PREFILL_TRACE
unsigned long long* g_prefill_trace = nullptr;  // debug builds: set by a trace harness
#endif

cudaError_t launch_prefill(const PrefillParams& p_in, int num_sms, cudaStream_t stream) {
  PrefillParams p = p_in;
#ifdef LISA_PREFILL_TRACE
  p.trace = g_prefill_trace;
#endif
  host_inv_freq(p.inv_freq);
  p.part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(p.q_ws) + PF_QWS_BYTES);
  p.tickets = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(p.q_ws) + PF_QWS_BYTES + PF_PART_BYTES);
  plan_segments(p, num_sms, g_prefill_split_mode.load(std::memory_order_relaxed));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.rows);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, prefill_prologue_kernel, p);
  if (e != cudaSuccess) return e;
  static SmemAttr attr_once;  // the attribute is per kernel and per device
  e = attr_once.ensure(prefill_attn_kernel, PF_SMEM_BYTES);
  if (e != cudaSuccess) return e;
  CUtensorMap tq, tk, tv, tg = {}, to;
  const uint32_t kv_rows = p.base + (uint32_t)p.rows;
  if (lisa_encode_group_map(&tq, p.q_ws, PF_MAX_ROWS, PF_MAX_ROWS, QH, PF_BM, 4) != 0 ||
      lisa_encode_group_map(&tk, p.k_cache, kv_rows, p.capacity, KVH, PF_BN / 2, 4) != 0 ||
      lisa_encode_group_map(&tv, p.v_cache, kv_rows, p.capacity, KVH, PF_BN, 2) != 0 ||
      lisa_encode_rows_map(&to, p.gated_out, (uint32_t)p.rows, OROW, 4, QH, HD, PF_BM) != 0 ||
      (p.in_bf16 && lisa_encode_rows_map(&tg, p.q_gate, (uint32_t)p.rows, QROW, 8, QH, 512, PF_BM) != 0))
    return cudaErrorInvalidValue;
  cfg.gridDim = dim3(p.n_seg * 2);
  cfg.blockDim = dim3(PF_THREADS);
  cfg.dynamicSmemBytes = PF_SMEM_BYTES;
  return cudaLaunchKernelEx(&cfg, prefill_attn_kernel, tq, tk, tv, tg, to, p);
}

}  // namespace lisa

#pragma GCC visibility push(default)
extern "C" int lisa_attn_debug_prefill_plan(uint32_t base, int rows, int num_sms, int mode, uint32_t* seg_lo,
                                            uint32_t* seg_hi, uint16_t* seg_unit, int cap) {
  if (rows < 1 || rows > lisa::PF_MAX_ROWS || num_sms < 2 || !seg_lo || !seg_hi || !seg_unit ||
      cap < lisa::PF_MAX_SEGS || base > (1u << 30) ||
      (mode != LISA_PREFILL_SPLIT_AUTO && mode != LISA_PREFILL_SPLIT_NEVER && mode != LISA_PREFILL_SPLIT_ALWAYS))
    return LISA_EINVAL;
  lisa::PrefillParams p = {};
  p.base = base;
  p.rows = rows;
  lisa::plan_segments(p, num_sms, mode);
  for (int i = 0; i < p.n_seg; ++i) {
    seg_lo[i] = p.seg_lo[i];
    seg_hi[i] = p.seg_hi[i];
    seg_unit[i] = p.seg_unit[i];
  }
  return p.n_seg;
}

extern "C" int lisa_attn_debug_prefill_split(int mode) {
  if (mode != LISA_PREFILL_SPLIT_AUTO && mode != LISA_PREFILL_SPLIT_NEVER && mode != LISA_PREFILL_SPLIT_ALWAYS)
    return LISA_EINVAL;
  return lisa::g_prefill_split_mode.exchange(mode);
}
#pragma GCC visibility pop
