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
#include <algorithm>
#include <mutex>

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
constexpr int PF_MAX_PIECES = 24;   // pieces of one cluster's tile range (kept in shared memory)

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

// The work list of one call: units (query-row pair qp, head h) heaviest first,
// unit u -> qp = n_pairs - 1 - u / 24, h = u % 24; its key tiles 0..n(qp)-1.
struct PfWork {
  int n_pairs, rows;
  uint32_t base;
  int streamk, clusters, total;
  __device__ __forceinline__ int qp_tiles(int qp) const {
    const int end = min(qp * 2 * PF_BM + 2 * PF_BM, rows);
    return (int)((base + (uint32_t)end + PF_BN - 1) / PF_BN);
  }
  __device__ __forceinline__ int unit_tiles(int u) const { return qp_tiles(n_pairs - 1 - u / QH); }
  __device__ __forceinline__ int unit_off(int u) const {
    const int g = u / QH;
    int off = 0;
    for (int k = 0; k < g; ++k) off += QH * qp_tiles(n_pairs - 1 - k);
    return off + (u % QH) * qp_tiles(n_pairs - 1 - g);
  }
  __device__ __forceinline__ int unit_at(int t) const {
    int off = 0;
    for (int g = 0; g < n_pairs; ++g) {
      const int n = qp_tiles(n_pairs - 1 - g);
      if (t < off + QH * n) return g * QH + (t - off) / n;
      off += QH * n;
    }
    return -1;
  }
  // first tile of cluster c's range (c == clusters gives the end of the list)
  __device__ __forceinline__ int range_start(int c) const {
    if (streamk) return (int)(((int64_t)c * total) / clusters);
    return c >= clusters ? total : unit_off(c);
  }
};

// One contiguous run of a unit's key tiles inside a cluster's range.
struct PfPiece {
  int unit, j0, j1;  // tiles [j0, j1) of the unit
  bool first, last;  // holds the unit's first / last tile
};

struct PfPieces {
  const PfWork& w;
  int t, t_end;
  __device__ __forceinline__ bool next(PfPiece& pc) {
    if (t >= t_end) return false;
    const int u = w.unit_at(t);
    const int off = w.unit_off(u), n = w.unit_tiles(u);
    pc.unit = u;
    pc.j0 = t - off;
    pc.j1 = min(n, t_end - off);
    pc.first = pc.j0 == 0;
    pc.last = pc.j1 == n;
    t = off + pc.j1;
    return true;
  }
};

// Persistent attention: each cluster of two CTAs runs the pieces of its tile
// range in order. Cluster rank 0 holds query rows [256 qp, 256 qp + 128) of a
// unit, rank 1 the next 128. Tiles are numbered J = 0, 1, ... across the
// cluster's pieces so that the ring barriers' phases continue from piece to
// piece; query tile, accumulator and running softmax state restart with every
// piece.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PF_THREADS, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PF_OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  volatile uint32_t* seg_ok = tmem_slot + 1;  // this CTA arrived last at a split unit
  int* n_pieces_s = reinterpret_cast<int*>(smem + PF_OFF_BAR + 112);
  PfPiece* pieces = reinterpret_cast<PfPiece*>(smem + PF_OFF_BAR + 128);  // [PF_MAX_PIECES]
  float* xmax = reinterpret_cast<float*>(smem + PF_OFF_BAR + 1024);  // [2 parity][2 half][128 rows]
  float* xsum = xmax + 2 * 2 * PF_BM;                                  // [2 half][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cl = (int)(blockIdx.x >> 1);
  const int n_qt = (p.rows + PF_BM - 1) / PF_BM;
  const PfWork work{(n_qt + 1) / 2, p.rows, p.base, p.streamk, p.clusters, p.total_tiles};
  const int t_begin = work.range_start(cl), t_end = work.range_start(cl + 1);

#ifdef LISA_PREFILL_TRACE
  if (threadIdx.x == 0) p.trace[64 + blockIdx.x * 8 + 0] = global_timer_ns();
#endif
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    for (int b = 0; b < B_COUNT; ++b) mbar_init(&bars[b], (b == B_PFULL || b == B_PFULL + 1) ? 16 : 1);
    fence_mbar_init();
    // the cluster's pieces, in order (the host keeps them within PF_MAX_PIECES)
    PfPieces it{work, t_begin, t_end};
    int np = 0;
    PfPiece pc;
    while (np < PF_MAX_PIECES && it.next(pc)) pieces[np++] = pc;
    *n_pieces_s = np;
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, PF_TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lead_bars = cluster_map(smem_u32(bars), 0);
  auto lead_bar = [&](int i) -> uint32_t { return lead_bars + 8u * (uint32_t)i; };
  // The setup above overlaps the prologue kernel; the K/V producers first
  // issue the loads of up to two key tiles of the first piece that hold only
  // positions below `base` (written by earlier calls), then wait too.
  const int n_pieces = *n_pieces_s;
  const PfPiece first_pc = n_pieces ? pieces[0] : PfPiece{0, 0, 0, true, true};
  const int n_early = max(0, min(min(2, first_pc.j1 - first_pc.j0), (int)(p.base / PF_BN) - first_pc.j0));
  if (!((warp == 0 || warp == 2) && lane == 0)) pdl_wait_primary();
  pdl_launch_dependents();
#ifdef LISA_PREFILL_TRACE
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
#else
#define PT(k)
#define PT_FLUSH(role)
#endif

  if (warp == 0 && lane == 0) {
    // ---------------- Q and K loads ----------------
    // Each CTA loads its own 128 query rows and its half (64 keys) of every
    // K tile; completion is counted on rank 0's barriers, whose expected
    // byte count rank 0 sets for both.
    int J = 0;
    bool ok = true;
    for (int pi = 0; ok && pi < n_pieces; ++pi) {
      const PfPiece pc = pieces[pi];
      const int qp = work.n_pairs - 1 - pc.unit / QH, h = pc.unit % QH, kvh = h / GQA;
      auto load_k = [&](int JJ, int j) {
        const int s = JJ & 1;
        if (rank == 0) mbar_arrive_expect_tx(&bars[B_KFULL + s], 2 * PF_KH_BYTES);
        tma_load_4d_pair(smem + PF_OFF_K + s * PF_KH_BYTES, &tk, lead_bar(B_KFULL + s), 0,
                         j * PF_BN + (int)rank * (PF_BN / 2), 0, kvh);
      };
      int j = pc.j0;
      if (pi == 0) {
        for (; j < pc.j0 + n_early; ++j, ++J) load_k(J, j);
        pdl_wait_primary();
      } else {
        // the query tile is overwritten once the previous piece's last S,
        // which read it, has completed
        ok = mbar_wait(&bars[B_SFULL + ((J - 1) & 1)], ((J - 1) >> 1) & 1, p.err, ERR_TIMEOUT_EMPTY);
        if (!ok) break;
      }
      if (rank == 0) mbar_arrive_expect_tx(&bars[B_Q], 2 * PF_Q_BYTES);
      tma_load_4d_pair(smem, &tq, lead_bar(B_Q), 0, qp * 2 * PF_BM + (int)rank * PF_BM, 0, h);
      for (; j < pc.j1; ++j, ++J) {
        // slot J & 1 is free once S_{J-2}, which read it, has completed
        if (J >= 2 && !mbar_wait(&bars[B_SFULL + (J & 1)], ((J >> 1) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) {
          ok = false;
          break;
        }
        load_k(J, j);
      }
    }
  } else if (warp == 2 && lane == 0) {
    // ---------------- V loads: this CTA's 128 dims of every V tile ----------------
    int J = 0;
    bool ok = true;
    for (int pi = 0; ok && pi < n_pieces; ++pi) {
      const PfPiece pc = pieces[pi];
      const int kvh = (pc.unit % QH) / GQA;
      auto load_v = [&](int JJ, int j) {
        const int s = JJ & 1;
        if (rank == 0) mbar_arrive_expect_tx(&bars[B_VFULL + s], 2 * PF_VH_BYTES);
        tma_load_4d_pair(smem + PF_OFF_V + s * PF_VH_BYTES, &tv, lead_bar(B_VFULL + s), 0, j * PF_BN,
                         2 * (int)rank, kvh);
      };
      int j = pc.j0;
      if (pi == 0) {
        for (; j < pc.j0 + n_early; ++j, ++J) load_v(J, j);
        pdl_wait_primary();
      }
      for (; j < pc.j1; ++j, ++J) {
        // slot J & 1 is free once P_{J-2}.V_{J-2}, which read it, has completed
        if (J >= 2 && !mbar_wait(&bars[B_PVDONE + (J & 1)], ((J >> 1) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) {
          ok = false;
          break;
        }
        load_v(J, j);
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------- MMA issuer (rank 0 only, M = 256 over the pair) ----------------
    // The tensor pipe keeps almost no queue: every cycle this thread spends
    // between two MMAs is a cycle the pipe idles. Inside a piece the group
    // sequence S_0, S_1, PV_0, S_2, PV_1, ... is issued without waits between
    // groups (the next group's inputs are tested before the current group's
    // last MMA); at a piece boundary the last P.V goes first, then the next
    // piece's first S once its query tile has landed.
    constexpr uint32_t IDESC_S = umma_idesc_bf16(2 * PF_BM, PF_BN, false);
    constexpr uint32_t IDESC_O = umma_idesc_bf16(2 * PF_BM, HD, true);
    const uint64_t dQ = umma_desc_sw128(smem_u32(smem), 16, 1024);
    const uint64_t dK = umma_desc_sw128(smem_u32(smem + PF_OFF_K), 16, 1024);
    const uint64_t dV = umma_desc_sw128(smem_u32(smem + PF_OFF_V), PF_BN * 128, 1024);
    auto s_mma = [&](int J, int kk) {
      const uint32_t g = kk >> 2, sub = kk & 3, s = J & 1;
      umma_pair_bf16(tmem + PF_TMEM_S + s * PF_BN, dQ + ((g * (PF_BM * 128) + sub * 32) >> 4),
                     dK + ((s * PF_KH_BYTES + g * ((PF_BN / 2) * 128) + sub * 32) >> 4), IDESC_S, kk ? 1u : 0u);
    };
    auto pv_mma = [&](int J, bool acc, int kk) {
      const uint32_t b = J & 1;
      umma_pair_bf16_ts(tmem + PF_TMEM_O, tmem + PF_TMEM_S + b * PF_BN + kk * 8,
                        dV + ((b * PF_VH_BYTES + kk * 2048) >> 4), IDESC_O, (acc || kk > 0) ? 1u : 0u);
    };
    auto k_ready = [&](int J) { return mbar_test_wait(&bars[B_KFULL + (J & 1)], (J >> 1) & 1); };
    auto pv_ready = [&](int J) {
      return mbar_test_wait(&bars[B_PFULL + (J & 1)], (J >> 1) & 1) &&
             mbar_test_wait(&bars[B_VFULL + (J & 1)], (J >> 1) & 1);
    };
    int J0 = 0;
    bool ok = true;
    for (int pi = 0; ok && pi < n_pieces; ++pi) {
      const PfPiece pc = pieces[pi];
      const int n = pc.j1 - pc.j0;
      ok = mbar_wait(&bars[B_Q], pi & 1, p.err, ERR_TIMEOUT_FULL) &&
           mbar_wait(&bars[B_KFULL + (J0 & 1)], (J0 >> 1) & 1, p.err, ERR_TIMEOUT_FULL);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) s_mma(J0, kk);
      umma_pair_commit(&bars[B_SFULL + (J0 & 1)], PF_PAIR);
      bool next_ready = false;  // inputs of the next group already seen complete
      for (int i = 0; ok && i < n; ++i) {
        const int J = J0 + i, b = J & 1;
        if (i + 1 < n) {
          if (!next_ready &&
              !mbar_wait(&bars[B_KFULL + ((J + 1) & 1)], ((J + 1) >> 1) & 1, p.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 15; ++kk) s_mma(J + 1, kk);
          next_ready = pv_ready(J);
          s_mma(J + 1, 15);
          umma_pair_commit(&bars[B_SFULL + ((J + 1) & 1)], PF_PAIR);
        } else {
          next_ready = false;
        }
        if (!next_ready && !(mbar_wait(&bars[B_PFULL + b], (J >> 1) & 1, p.err, ERR_TIMEOUT_MMA) &&
                             mbar_wait(&bars[B_VFULL + b], (J >> 1) & 1, p.err, ERR_TIMEOUT_FULL))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 7; ++kk) pv_mma(J, i > 0, kk);
        next_ready = i + 2 < n && k_ready(J + 2);
        pv_mma(J, i > 0, 7);
        umma_pair_commit(&bars[B_PVDONE + b], PF_PAIR);
      }
      J0 += n;
    }
    PT_FLUSH(0);
  } else if (warp >= 4) {
    // ---------------- softmax / correction / epilogue (warps 4..11) ----------------
    // Warp 4+w and warp 8+w share TMEM lanes 32w..32w+31 (one query row per
    // thread); each reads and exponentiates one half (64 keys) of a tile, and
    // the two halves exchange their maxima once per tile.
    const int wi = (warp - 4) & 3;
    const int half = (warp - 4) >> 2;
    const int row = wi * 32 + lane;  // row within the CTA's tile == TMEM lane
    const uint32_t lane_addr = tmem + ((uint32_t)(wi * 32) << 16);
    int J0 = 0;
    bool ok = true;
    for (int pi = 0; ok && pi < n_pieces; ++pi) {
      const PfPiece pc = pieces[pi];
      const uint32_t pos_row =
          p.base + (uint32_t)((work.n_pairs - 1 - pc.unit / QH) * 2 * PF_BM + (int)rank * PF_BM + row);
      const int n = pc.j1 - pc.j0;
      const int j0 = pc.j0;
      float mr = -INFINITY, l = 0.f;  // running max of the raw scores, this half's sum
      for (int i = 0; i < n; ++i) {
        const int J = J0 + i, b = J & 1;
        PT(7);
        if (!mbar_wait(&bars[B_SFULL + b], (J >> 1) & 1, p.err, ERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        PT(0);
        tc_fence_after();
        uint32_t sa[32], sb[32];
        const uint32_t scol = PF_TMEM_S + b * PF_BN + half * 64;
        tmem_ld32(lane_addr + scol, sa);
        tmem_ld32(lane_addr + scol + 32, sb);
        tmem_wait_ld();
        float x[64];  // raw scores Q.K (unscaled)
#pragma unroll
        for (int c = 0; c < 64; ++c) x[c] = __uint_as_float(c < 32 ? sa[c] : sb[c - 32]);
        const uint32_t key0 = (uint32_t)(j0 + i) * PF_BN + half * 64;
        if (key0 + 63 > pos_row) {  // diagonal tile: keys past this row's position
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (key0 + c > pos_row) x[c] = -INFINITY;
        }
        float t8[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          t8[q] = fmaxf(fmax3(fmax3(x[8 * q], x[8 * q + 1], x[8 * q + 2]), x[8 * q + 3], x[8 * q + 4]),
                        fmax3(x[8 * q + 5], x[8 * q + 6], x[8 * q + 7]));
        const float hmax = fmax3(fmax3(t8[0], t8[1], t8[2]), fmax3(t8[3], t8[4], t8[5]), fmaxf(t8[6], t8[7]));
        xmax[(b * 2 + half) * PF_BM + row] = hmax;
        // both halves have read this S tile (P overwrites its first 64 columns)
        // and published their maxima
        named_bar_sync(2 + wi, 64);
        const float mnew = fmax3(mr, hmax, xmax[(b * 2 + (half ^ 1)) * PF_BM + row]);
        // The running max moves only when it grows by more than 2^8 (in exp2
        // units), or first becomes finite. A row whose keys in this piece are
        // all masked so far keeps mr = -inf and gets P = 0.
        const bool need = mnew != -INFINITY && (mr == -INFINITY || (mnew - mr) * kLog2Scale > PF_RESCALE_LOG2);
        float alpha = 1.f;
        if (need) {
          alpha = fast_exp2((mr - mnew) * kLog2Scale);  // 0 when mr was -inf
          mr = mnew;
        }
        // P = exp2(x * scale*log2e - m), rounded to bf16 and written over the S
        // tile 16 keys at a time so the TMEM stores overlap the exponentials.
        // 1 of every 8 key pairs is exponentiated on the FMA pipe, the rest on
        // the SFU. The denominator sums the f32 values, as the reference's f32
        // softmax does.
        const float2 cc = make_float2(kLog2Scale, kLog2Scale);
        const float moff = mr == -INFINITY ? 0.f : -mr * kLog2Scale;
        const float2 nm = make_float2(moff, moff);
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
        if (i > 0 && __any_sync(0xffffffffu, need)) {
          // O must hold exactly tiles < J of this piece before it is rescaled
          if (!mbar_wait(&bars[B_PVDONE + (b ^ 1)], ((J - 1) >> 1) & 1, p.err, ERR_TIMEOUT_MMA)) {
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
            for (int q = 0; q < 32; ++q) ov[q] = __float_as_uint(__uint_as_float(ov[q]) * alpha);
            tmem_st32(lane_addr + col, ov);
          }
        }
        PT(2);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(lead_bar(B_PFULL + b));
        PT(4);
      }
      if (!ok) break;
      const int Jl = J0 + n - 1;
      J0 += n;
      ok = mbar_wait(&bars[B_PVDONE + (Jl & 1)], (Jl >> 1) & 1, p.err, ERR_TIMEOUT_MMA);
      if (!ok) break;
      // Row denominators: this half's plus the other half's.
      xsum[half * PF_BM + row] = l;
      named_bar_sync(2 + wi, 64);
      const float l_row = xsum[row] + xsum[PF_BM + row];
      named_bar_sync(2 + wi, 64);  // both halves have read xsum before the next piece writes it
      tc_fence_after();
      const PfPiece pe = pieces[pi];
      float den = l_row;
      if (!(pe.first && pe.last)) {
        // ---- a unit split over clusters c_first .. c_last. Every segment
        // leaves its partial (unnormalised O of this CTA's rows, max, row
        // sum); the last one to finish (counted per unit and rank) merges all
        // of them in cluster order, so the result does not depend on which
        // cluster arrives last. Nobody waits, so the clusters need not be
        // resident at the same time. ----
        const int u_off = work.unit_off(pe.unit), u_end = u_off + work.unit_tiles(pe.unit);
        int c_first = cl, c_last = cl;
        while (c_first > 0 && work.range_start(c_first) > u_off) --c_first;
        while (c_last + 1 < work.clusters && work.range_start(c_last + 1) < u_end) ++c_last;
        // a segment's slot: its cluster's first piece (which 0) or, for the
        // cluster whose range starts before the unit, its last piece (1)
        auto slot_ptr = [&](int c) -> float* {
          const int which = work.range_start(c) < u_off ? 1 : 0;
          return p.part + ((((size_t)c * 2 + which) * 2 + rank) * PF_BM + row) * PF_PART_STRIDE;
        };
        float* dst = slot_ptr(cl);
#pragma unroll 1
        for (int c = 0; c < HD / 64; ++c) {
          const int col = half * (HD / 2) + c * 32;
          uint32_t ov[32];
          tmem_ld32(lane_addr + PF_TMEM_O + col, ov);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 8; ++q)
            __stcg(reinterpret_cast<uint4*>(dst + col + 4 * q),
                   make_uint4(ov[4 * q], ov[4 * q + 1], ov[4 * q + 2], ov[4 * q + 3]));
        }
        if (half == 0) __stcg(reinterpret_cast<float2*>(dst + HD), make_float2(mr, l_row));
        __threadfence();
        named_bar_sync(6, 256);  // the whole partial of this CTA is written
        if (threadIdx.x == 128) {
          uint32_t* cnt = p.ready + pe.unit * 2 + rank;
          const uint32_t before = atomicAdd(cnt, 1u);
          const bool last = before == (uint32_t)(c_last - c_first);
          if (last) *cnt = 0u;  // every segment has arrived: ready for the next call
          __threadfence();
          *seg_ok = last ? 1u : 0u;
        }
        named_bar_sync(6, 256);
        const bool merge = *seg_ok != 0u;
        named_bar_sync(6, 256);
        if (!merge) {
          tc_fence_before();
          continue;
        }
        // O = sum_s O_s * w_s, den = sum_s l_s * w_s, w_s = 2^((m_s - m_all) c)
        float mall = -INFINITY;
        for (int c = c_first; c <= c_last; ++c) mall = fmaxf(mall, __ldcg(slot_ptr(c) + HD));
        den = 0.f;
        for (int c = c_first; c <= c_last; ++c) {
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(slot_ptr(c) + HD));
          den += ml.y * (ml.x == -INFINITY ? 0.f : fast_exp2((ml.x - mall) * kLog2Scale));
        }
#pragma unroll 1
        for (int c = 0; c < HD / 64; ++c) {
          const int col = half * (HD / 2) + c * 32;
          uint32_t ov[32];
#pragma unroll
          for (int q = 0; q < 32; ++q) ov[q] = 0u;
          for (int cc = c_first; cc <= c_last; ++cc) {
            const float* sp = slot_ptr(cc);
            const float mk = __ldcg(sp + HD);
            const float wk = mk == -INFINITY ? 0.f : fast_exp2((mk - mall) * kLog2Scale);
            const float4* s4 = reinterpret_cast<const float4*>(sp + col);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 v4 = __ldcg(s4 + q);
              ov[4 * q] = __float_as_uint(fmaf(v4.x, wk, __uint_as_float(ov[4 * q])));
              ov[4 * q + 1] = __float_as_uint(fmaf(v4.y, wk, __uint_as_float(ov[4 * q + 1])));
              ov[4 * q + 2] = __float_as_uint(fmaf(v4.z, wk, __uint_as_float(ov[4 * q + 2])));
              ov[4 * q + 3] = __float_as_uint(fmaf(v4.w, wk, __uint_as_float(ov[4 * q + 3])));
            }
          }
          tmem_st32(lane_addr + PF_TMEM_O + col, ov);
        }
        tmem_wait_st();
      }
      // ---- gated output of the unit's rows: O / den * sigmoid(gate). Every
      // lane takes part in the TMEM loads (warp-collective); rows past the
      // chunk only skip their gate loads and stores. ----
      {
        const int h = pe.unit % QH;
        const int r = (work.n_pairs - 1 - pe.unit / QH) * 2 * PF_BM + (int)rank * PF_BM + row;
        const bool valid = r < p.rows;
        const float inv_l = 1.0f / den;
        const size_t gbase = (size_t)r * QROW + (size_t)h * 512 + 256 + half * 128;
        uint16_t* out = p.gated_out + (size_t)r * OROW + (size_t)h * HD + half * (HD / 2);
        uint4 g4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          g4[q] = valid ? load8_bf16(p.q_gate, gbase + 8 * q, p.in_bf16) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          const int col = half * (HD / 2) + c * 32;
          uint32_t ov[32];
          tmem_ld32(lane_addr + PF_TMEM_O + col, ov);
          uint4 gn[4];  // the next 32 dims' gate, in flight during this pass
#pragma unroll
          for (int q = 0; q < 4; ++q)
            gn[q] = (valid && c + 1 < HD / 64) ? load8_bf16(p.q_gate, gbase + 32 * (c + 1) + 8 * q, p.in_bf16)
                                               : make_uint4(0u, 0u, 0u, 0u);
          tmem_wait_ld();
          uint32_t outw[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const uint32_t gw = (&g4[q >> 2].x)[q & 3];
            const float2 g2 = unpack_bf16x2(gw);
            outw[q] = pack_bf16x2(__uint_as_float(ov[2 * q]) * inv_l * fast_sigmoid(g2.x),
                                  __uint_as_float(ov[2 * q + 1]) * inv_l * fast_sigmoid(g2.y));
          }
          if (valid) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(out + c * 32 + 8 * q) =
                  make_uint4(outw[4 * q], outw[4 * q + 1], outw[4 * q + 2], outw[4 * q + 3]);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) g4[q] = gn[q];
        }
      }
      tc_fence_before();
    }
    PT(5);
    if (warp == 4) { PT_FLUSH(1); }
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
constexpr size_t PF_PART_BYTES = (size_t)PF_MAX_CLUSTERS * 2 * 2 * PF_BM * PF_PART_STRIDE * sizeof(float);
}  // namespace

size_t prefill_workspace_bytes() { return PF_QWS_BYTES + PF_PART_BYTES + PF_MAX_CLUSTERS * 2 * sizeof(uint32_t); }

void prefill_workspace_layout(void* ws, uint16_t** q_ws, float** part, uint32_t** ready) {
  uint8_t* b = static_cast<uint8_t*>(ws);
  *q_ws = reinterpret_cast<uint16_t*>(b);
  *part = reinterpret_cast<float*>(b + PF_QWS_BYTES);
  *ready = reinterpret_cast<uint32_t*>(b + PF_QWS_BYTES + PF_PART_BYTES);
}

namespace {
// cudaOccupancyMaxActiveClusters for the attention kernel, per device.
int max_resident_clusters(const cudaLaunchConfig_t& base_cfg) {
  static std::mutex mu;
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[dev]) {
    cudaLaunchConfig_t cfg = base_cfg;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2 * PF_MAX_CLUSTERS);
    cfg.blockDim = dim3(PF_THREADS);
    cfg.dynamicSmemBytes = PF_SMEM_BYTES;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, prefill_attn_kernel, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = 1;
    }
    cached[dev] = n;
  }
  return cached[dev];
}
}  // namespace

cudaError_t launch_prefill(const PrefillParams& p_in, int num_sms, cudaStream_t stream) {
  PrefillParams p = p_in;
  host_inv_freq(p.inv_freq);
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
  CUtensorMap tq, tk, tv;
  const uint32_t kv_rows = p.base + (uint32_t)p.rows;
  if (lisa_encode_group_map(&tq, p.q_ws, PF_MAX_ROWS, PF_MAX_ROWS, QH, PF_BM, 4) != 0 ||
      lisa_encode_group_map(&tk, p.k_cache, kv_rows, p.capacity, KVH, PF_BN / 2, 4) != 0 ||
      lisa_encode_group_map(&tv, p.v_cache, kv_rows, p.capacity, KVH, PF_BN, 2) != 0)
    return cudaErrorInvalidValue;
  // Work split: one cluster per unit, or (stream-K) every cluster slot of the
  // GPU taking an equal share of all units' key tiles when that shortens the
  // longest cluster by more than the cost of splitting (about two tiles: the
  // query reload, the partial written and merged).
  const int n_qt = (p.rows + PF_BM - 1) / PF_BM;
  const int n_pairs = (n_qt + 1) / 2;
  const int units = n_pairs * QH;
  int total = 0, longest = 0, shortest = 1 << 30;
  for (int qp = 0; qp < n_pairs; ++qp) {
    const int end = std::min(qp * 2 * PF_BM + 2 * PF_BM, p.rows);
    const int n = (int)((p.base + (uint32_t)end + PF_BN - 1) / PF_BN);
    total += QH * n;
    longest = std::max(longest, n);
    shortest = std::min(shortest, n);
  }
  // Stream-K clusters wait for one another's partials, so all of them must be
  // resident at once: at most the number of 2-CTA clusters of this kernel the
  // device can hold (queried once per device).
  const int slots = std::min(PF_MAX_CLUSTERS, std::max(1, std::min(num_sms / 2, max_resident_clusters(cfg))));
  const int share = (total + slots - 1) / slots;
  p.total_tiles = total;
  const int mode = current_prefill_split();
  const bool fits = (share + shortest - 1) / shortest + 2 <= PF_MAX_PIECES;  // pieces per cluster
  if (units < slots && fits && (mode == 2 || (mode == 0 && share + 2 < longest))) {
    p.streamk = 1;
    p.clusters = slots;
  } else {
    p.streamk = 0;
    p.clusters = units;
  }
  cfg.gridDim = dim3(p.clusters * 2);
  cfg.blockDim = dim3(PF_THREADS);
  cfg.dynamicSmemBytes = PF_SMEM_BYTES;
  return cudaLaunchKernelEx(&cfg, prefill_attn_kernel, tq, tk, tv, p);
}

}  // namespace lisa
