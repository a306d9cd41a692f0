// prefill.cu — chunked prefill of the lisa-rs full-attention layer on the
// sm_100a 5th-generation tensor core (tcgen05.mma, TMEM accumulators, TMA).
//
// Replaces encode_prefill_attention's attention part (runner.rs:1976-2060):
//   q_norm_gate_rope_prefill   attention.metal:364-401  -> prefill_prologue_kernel
//   kv_cache_store_prefill     attention.metal:403-440  -> prefill_prologue_kernel
//   sdpa_decode_prefill        attention.metal:442-480  -> prefill_attn_kernel
//   gate_out_bf16              attention.metal:520-531  -> prefill_attn_kernel epilogue
// The reference scans every key serially per (row, head) on scalar lanes; here
// a CTA owns 128 query rows of one head and runs a flash-attention loop over
// 64-key tiles of the causal prefix, with every MMA operand that is reused
// kept in tensor memory (TMEM, 512 columns):
//   columns [0,256) O accumulator, [256,384) two S tiles, [384,512) Q (bf16)
//   warp 0       TMA producer: K/V tiles through a 3-stage ring
//   warp 1       allocates TMEM, issues tcgen05.mma (one thread):
//                S_j = Q.K_j^T  (A = Q from TMEM, B = K from smem; M128 N64 K256)
//                O  += P_j.V_j  (A = P from TMEM, B = V from smem read MN-major;
//                                M128 N256 K64)
//   warps 4..11  softmax: thread = query row = TMEM lane; warps 4+w and 8+w
//                share lanes 32w.. and split the columns. They load Q into
//                TMEM, read S with tcgen05.ld, mask causally, keep an online
//                max that is only moved (and O rescaled in TMEM) when it grows
//                by more than 2^8, and write bf16 P over the S tile it came
//                from; epilogue O/l * sigmoid(gate).
// Key tiles past the last query row are skipped (causal tile skipping).
#include <algorithm>

#include "common.cuh"
#include "prefill.cuh"
#include "tcgen05.cuh"

namespace lisa {

namespace {

constexpr int PF_BM = 128;   // query rows per CTA
constexpr int PF_BN = 128;   // keys per tile
constexpr int PF_SLOT = 16384;  // ring slot: K sub-tile [128 keys][64 dims] or V sub-tile [32 keys][256 dims]
constexpr int PF_RING = 9;
constexpr int PF_Q_BYTES = PF_BM * HD * 2;  // 64 KB
constexpr int PF_OFF_RING = PF_Q_BYTES;
constexpr int PF_OFF_BAR = PF_OFF_RING + PF_RING * PF_SLOT;
constexpr int PF_SMEM_BYTES = PF_OFF_BAR + 4096 + 1024;  // barriers, TMEM slot, max/sum exchange
constexpr int PF_THREADS = 384;  // warp 0 TMA, warp 1 MMA, warps 4..11 softmax
constexpr uint32_t PF_TMEM_COLS = 512;
constexpr uint32_t PF_TMEM_O = 0;    // O accumulator: columns [0, 256)
constexpr uint32_t PF_TMEM_S = 256;  // S / P tiles: columns [256, 384), [384, 512)
constexpr float PF_RESCALE_LOG2 = 8.0f;

// mbarrier slots
enum {
  B_Q = 0,        // Q tile landed
  B_FULL = 1,     // [PF_RING] ring slot landed
  B_EMPTY = 1 + PF_RING,        // [PF_RING] MMA that read the slot finished
  B_SFULL = 1 + 2 * PF_RING,    // [2] S tile in TMEM
  B_PFULL = 3 + 2 * PF_RING,    // [2] P tile in TMEM (256 softmax threads)
  B_PVDONE = 5 + 2 * PF_RING,   // [2] PV MMA that read the P tile finished (O updated)
  B_COUNT = 7 + 2 * PF_RING
};

// Ring positions: the loads go in the order the MMAs need them,
// K0, K1, V0, K2, V1, ..., each tile as 4 slots.
__host__ __device__ constexpr int kpos(int j) { return j == 0 ? 0 : 8 * j - 4; }
__host__ __device__ constexpr int vpos(int j) { return 8 * (j + 1); }

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

// One 256-thread CTA per prompt row; warp w handles items w, w+8, w+16, w+24
// (items 0..23 are the query heads, 24..27 the KV heads). The row's 32 RoPE
// (cos, sin) pairs are computed once into shared memory while the loads are in
// flight. Lane l holds dims 8l..8l+7; the RoPE partner of dims 0..31
// (lanes 0..3) is dims 32..63 (lanes 4..7).
__global__ void __launch_bounds__(256) prefill_prologue_kernel(const PrefillParams p) {
  __shared__ float s_cos[ROT_PAIRS], s_sin[ROT_PAIRS];
  pdl_wait_primary();       // the previous chunk may still read q_ws
  pdl_launch_dependents();  // let the attention kernel set up meanwhile
  const int r = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t pos = p.base + r;
  constexpr int NI = 4;  // items per warp
  float x[NI][8], v[NI][8];  // v: the V row of KV items
#pragma unroll
  for (int t = 0; t < NI; ++t) {
    const int hh = warp + 8 * t;
    if (hh >= QH + KVH) continue;
    const bool is_q = hh < QH;
    const size_t in = is_q ? (size_t)r * QROW + (size_t)hh * 512 + lane * 8
                           : (size_t)r * KROW + (size_t)(hh - QH) * HD + lane * 8;
    load8_in(is_q ? p.q_gate : p.k_in, in, p.in_bf16, x[t]);
    if (!is_q) load8_in(p.v_in, in, p.in_bf16, v[t]);
  }
  if (threadIdx.x < ROT_PAIRS) rope_cs(pos, p.inv_freq[threadIdx.x], s_cos[threadIdx.x], s_sin[threadIdx.x]);
  __syncthreads();  // RoPE table ready
#pragma unroll
  for (int t = 0; t < NI; ++t) {
    const int hh = warp + 8 * t;
    if (hh >= QH + KVH) continue;  // uniform per warp
    const bool is_q = hh < QH;
    const uint16_t* w = is_q ? p.q_norm_w : p.k_norm_w;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += x[t][i] * x[t][i];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = 1.0f / sqrtf(ss / 256.0f + p.eps);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float n = x[t][i] * inv * bf16_bits_to_f32(w[lane * 8 + i]);
      const float partner = __shfl_xor_sync(0xffffffffu, n, 4);
      o[i] = n;
      if (lane < 8) {
        const int j = (lane & 3) * 8 + i;
        o[i] = lane < 4 ? n * s_cos[j] - partner * s_sin[j] : n * s_cos[j] + partner * s_sin[j];
      }
    }
    const uint4 packed = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                                    pack_bf16x2(o[6], o[7]));
    if (is_q) {
      // chunk-major [head][chunk = lane][row]: a warp reading 32 rows of one
      // chunk touches 512 contiguous bytes
      *reinterpret_cast<uint4*>(p.q_ws + ((size_t)hh * PF_MAX_ROWS + r) * HD + lane * 8) = packed;
    } else {
      const size_t out = ((size_t)(hh - QH) * p.capacity + pos) * HD + lane * 8;
      *reinterpret_cast<uint4*>(p.k_cache + out) = packed;
      *reinterpret_cast<uint4*>(p.v_cache + out) =
          make_uint4(pack_bf16x2(v[t][0], v[t][1]), pack_bf16x2(v[t][2], v[t][3]), pack_bf16x2(v[t][4], v[t][5]),
                     pack_bf16x2(v[t][6], v[t][7]));
    }
  }
}

// Grid: n_qtiles * 24 CTAs, heaviest (last) query tiles first.
__global__ void __launch_bounds__(PF_THREADS, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PF_OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  float* xmax = reinterpret_cast<float*>(smem + PF_OFF_BAR + 1024);  // [2 parity][2 half][128 rows]
  float* xsum = xmax + 2 * 2 * PF_BM;                                  // [2 half][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.rows + PF_BM - 1) / PF_BM;
  const int qt = n_qt - 1 - (int)(blockIdx.x / QH);
  const int h = blockIdx.x % QH, kvh = h / GQA;
  const int r0 = qt * PF_BM;
  const int r_end = min(r0 + PF_BM, p.rows);
  const uint32_t kv_end = p.base + (uint32_t)r_end;  // keys [0, kv_end)
  const int n_tiles = (int)((kv_end + PF_BN - 1) / PF_BN);

#ifdef LISA_PREFILL_TRACE
  if (threadIdx.x == 0) p.trace[64 + blockIdx.x * 8 + 0] = global_timer_ns();
#endif
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    for (int b = 0; b < B_COUNT; ++b) mbar_init(&bars[b], (b == B_PFULL || b == B_PFULL + 1) ? 256 : 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, PF_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Setup above overlaps the prologue kernel; its q_ws / KV writes are read
  // only after it has completed.
  pdl_wait_primary();
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
#else
#define PT(k)
#define PT_FLUSH(role)
#endif

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars[B_Q], PF_Q_BYTES);
      for (int st = 0; st < 4; ++st) tma_load_3d(smem + st * (PF_BM * 128), &tq, &bars[B_Q], st * 64, r0, h);
      // one ring slot: K sub-tile (keys j*128.., dims 64*part..) or V sub-tile
      // (keys j*128 + 32*part.., all 256 dims as 4 boxes)
      auto load_slot = [&](int pos, bool is_k, int j, int part) -> bool {
        const int slot = pos % PF_RING;
        if (pos >= PF_RING &&
            !mbar_wait(&bars[B_EMPTY + slot], ((pos / PF_RING) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY))
          return false;
        uint8_t* dst = smem + PF_OFF_RING + slot * PF_SLOT;
        mbar_arrive_expect_tx(&bars[B_FULL + slot], PF_SLOT);
        if (is_k) {
          tma_load_3d(dst, &tk, &bars[B_FULL + slot], part * 64, j * PF_BN, kvh);
        } else {
          for (int st = 0; st < 4; ++st)
            tma_load_3d(dst + st * 4096, &tv, &bars[B_FULL + slot], st * 64, j * PF_BN + part * 32, kvh);
        }
        return true;
      };
      bool ok = true;
      for (int i = 0; ok && i <= n_tiles; ++i) {
        if (i < n_tiles)
          for (int part = 0; ok && part < 4; ++part) ok = load_slot(kpos(i) + part, true, i, part);
        if (i >= 1)
          for (int part = 0; ok && part < 4; ++part) ok = load_slot(vpos(i - 1) + part, false, i - 1, part);
      }
    }
    return;
  }

  if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t IDESC_S = umma_idesc_bf16(PF_BM, PF_BN, false);
      constexpr uint32_t IDESC_O = umma_idesc_bf16(PF_BM, HD, true);
      const uint32_t sQ = smem_u32(smem);
      const uint32_t sRing = smem_u32(smem + PF_OFF_RING);
      bool ok = mbar_wait(&bars[B_Q], 0, p.err, ERR_TIMEOUT_FULL);
      // S_j = Q . K_j^T, 4 K slots (64 dims each) x 4 k-steps of 16
      auto issue_s = [&](int j) -> bool {
        const uint32_t d = tmem + PF_TMEM_S + (j & 1) * PF_BN;
        for (int part = 0; part < 4; ++part) {
          const int pos = kpos(j) + part, slot = pos % PF_RING;
          PT(7);
          if (!mbar_wait(&bars[B_FULL + slot], (pos / PF_RING) & 1, p.err, ERR_TIMEOUT_FULL)) return false;
          PT(0);
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t a = umma_desc_sw128(sQ + part * (PF_BM * 128) + kk * 32, 16, 1024);
            const uint64_t b = umma_desc_sw128(sRing + slot * PF_SLOT + kk * 32, 16, 1024);
            umma_bf16(d, a, b, IDESC_S, (part | kk) ? 1u : 0u);
          }
          umma_commit(&bars[B_EMPTY + slot]);
        }
        umma_commit(&bars[B_SFULL + (j & 1)]);
        PT(1);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int b = j & 1;
        if (j + 1 < n_tiles && !issue_s(j + 1)) break;
        PT(7);
        if (!mbar_wait(&bars[B_PFULL + b], (j >> 1) & 1, p.err, ERR_TIMEOUT_MMA)) break;
        PT(2);
        tc_fence_after();
        // O += P_j . V_j: 4 V slots of 32 keys x 2 k-steps; P (bf16 pairs) lives
        // over the S tile, key k at column k/2
        for (int part = 0; ok && part < 4; ++part) {
          const int pos = vpos(j) + part, slot = pos % PF_RING;
          if (!mbar_wait(&bars[B_FULL + slot], (pos / PF_RING) & 1, p.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const uint64_t bd = umma_desc_sw128(sRing + slot * PF_SLOT + kk * 2048, 4096, 1024);
            umma_bf16_ts(tmem + PF_TMEM_O, tmem + PF_TMEM_S + b * PF_BN + part * 16 + kk * 8, bd, IDESC_O,
                         (j > 0 || part > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&bars[B_EMPTY + slot]);
        }
        umma_commit(&bars[B_PVDONE + b]);
        PT(4);
      }
      PT_FLUSH(0);
    }
    __syncwarp();
    named_bar_sync(1, 288);
    tc_fence_after();
    tmem_dealloc(tmem, PF_TMEM_COLS);
    return;
  }

  if (warp < 4) return;

  // ---------------- softmax / correction / epilogue (warps 4..11) ----------------
  // Warp 4+w and warp 8+w share TMEM lanes 32w..32w+31 (one query row per
  // thread); each reads and exponentiates one half (64 keys) of a tile, and the
  // two halves exchange their maxima once per tile.
  const int wi = (warp - 4) & 3;
  const int half = (warp - 4) >> 2;
  const int row = wi * 32 + lane;  // row within the tile == TMEM lane
  const uint32_t lane_addr = tmem + ((uint32_t)(wi * 32) << 16);
  const uint32_t pos_row = p.base + (uint32_t)(r0 + row);
  bool ok = true;
  float m2 = -INFINITY, l = 0.f;  // running max (log2 domain), this half's sum
  for (int j = 0; j < n_tiles; ++j) {
    const int b = j & 1;
    PT(7);
    if (!mbar_wait(&bars[B_SFULL + b], (j >> 1) & 1, p.err, ERR_TIMEOUT_MMA)) {
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
    const uint32_t key0 = (uint32_t)j * PF_BN + half * 64;
    const bool full_half = key0 + 63 <= pos_row;
    float s2[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      const float raw = __uint_as_float(c < 32 ? sa[c] : sb[c - 32]);
      s2[c] = (full_half || key0 + c <= pos_row) ? raw * (SCALE * LOG2E) : -INFINITY;
    }
    float t[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) t[c] = fmaxf(s2[c], s2[c + 32]);
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1)
#pragma unroll
      for (int c = 0; c < w; ++c) t[c] = fmaxf(t[c], t[c + w]);
    xmax[(b * 2 + half) * PF_BM + row] = t[0];
    // both halves have read this S tile (P overwrites its first 64 columns)
    // and published their maxima
    named_bar_sync(2 + wi, 64);
    const float tmax = fmaxf(t[0], xmax[(b * 2 + (half ^ 1)) * PF_BM + row]);
    const float mnew = fmaxf(m2, tmax);
    const bool need = mnew > m2 + PF_RESCALE_LOG2;  // also true for the first finite max
    float alpha = 1.f;
    if (need) {
      alpha = fast_exp2(m2 - mnew);
      m2 = mnew;
    }
    uint32_t pk[32];
    float ps[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      pk[c] = pack_bf16x2(fast_exp2(s2[2 * c] - m2), fast_exp2(s2[2 * c + 1] - m2));
      ps[c] = bf16_bits_to_f32(pk[c] & 0xffffu) + bf16_bits_to_f32(pk[c] >> 16);
    }
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1)
#pragma unroll
      for (int c = 0; c < w; ++c) ps[c] += ps[c + w];
    l = l * alpha + ps[0];
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
      tmem_wait_st();
    }
    PT(2);
    tmem_st32(lane_addr + PF_TMEM_S + b * PF_BN + half * 32, pk);
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&bars[B_PFULL + b]);
    PT(4);
  }
#ifdef LISA_PREFILL_TRACE
  if (threadIdx.x == 128) p.trace[64 + blockIdx.x * 8 + 3] = global_timer_ns();
#endif
  // gate values of this row and half, prefetched while the last P.V runs
  const int r = r0 + row;
  uint32_t gpk[64];
  if (ok && r < p.rows) {
    const size_t gbase = (size_t)r * QROW + (size_t)h * 512 + 256 + half * 128;
#pragma unroll
    for (int g8 = 0; g8 < 16; ++g8) {
      float gv[8];
      load8_in(p.q_gate, gbase + g8 * 8, p.in_bf16, gv);
#pragma unroll
      for (int i = 0; i < 4; ++i) gpk[g8 * 4 + i] = pack_bf16x2(gv[2 * i], gv[2 * i + 1]);
    }
  }
  const int last = n_tiles - 1;
  ok = ok && mbar_wait(&bars[B_PVDONE + (last & 1)], (last >> 1) & 1, p.err, ERR_TIMEOUT_MMA);
  // Sum the two halves' denominators (half 0 + half 1).
  xsum[half * PF_BM + row] = l;
  named_bar_sync(2 + wi, 64);
  const float l_row = xsum[row] + xsum[PF_BM + row];
  if (ok) {
    tc_fence_after();
    const float inv_l = 1.0f / l_row;
#pragma unroll
    for (int c = 0; c < HD / 64; ++c) {
      const int col = half * (HD / 2) + c * 32;
      uint32_t ov[32];
      tmem_ld32(lane_addr + PF_TMEM_O + col, ov);
      tmem_wait_ld();
      if (r < p.rows) {
        uint32_t outw[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t gg = gpk[c * 16 + i];
          float y[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float gv = bf16_bits_to_f32(e ? gg >> 16 : gg & 0xffffu);
            const float sg = fast_rcp(1.0f + fast_exp2(-LOG2E * gv));
            y[e] = __uint_as_float(ov[2 * i + e]) * inv_l * sg;
          }
          outw[i] = pack_bf16x2(y[0], y[1]);
        }
        uint4* dst = reinterpret_cast<uint4*>(p.gated_out + (size_t)r * OROW + h * HD + col);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(outw[4 * i], outw[4 * i + 1], outw[4 * i + 2], outw[4 * i + 3]);
      }
    }
  }
  PT(5);
  if (warp == 4) { PT_FLUSH(1); }
#ifdef LISA_PREFILL_TRACE
  if (threadIdx.x == 128) p.trace[64 + blockIdx.x * 8 + 4] = global_timer_ns();
#endif
  tc_fence_before();
  named_bar_sync(1, 288);
}

size_t prefill_workspace_bytes() { return (size_t)QH * PF_MAX_ROWS * HD * sizeof(uint16_t); }

cudaError_t launch_prefill(const PrefillParams& p_in, int num_sms, cudaStream_t stream) {
  (void)num_sms;
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
  static bool configured = false;
  if (!configured) {
    e = cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  CUtensorMap tq, tk, tv;
  const uint32_t kv_rows = p.base + (uint32_t)p.rows;
  if (lisa_encode_kv_map(&tq, p.q_ws, PF_MAX_ROWS, PF_MAX_ROWS, PF_BM, QH) != 0 ||
      lisa_encode_kv_map(&tk, p.k_cache, kv_rows, p.capacity, PF_BN, KVH) != 0 ||
      lisa_encode_kv_map(&tv, p.v_cache, kv_rows, p.capacity, 32, KVH) != 0)
    return cudaErrorInvalidValue;
  const int n_qt = (p.rows + PF_BM - 1) / PF_BM;
  cfg.gridDim = dim3(n_qt * QH);
  cfg.blockDim = dim3(PF_THREADS);
  cfg.dynamicSmemBytes = PF_SMEM_BYTES;
  return cudaLaunchKernelEx(&cfg, prefill_attn_kernel, tq, tk, tv, p);
}

}  // namespace lisa
