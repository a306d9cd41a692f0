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
// 64-key tiles of the causal prefix:
//   warp 0      TMA producer: Q tile once, K/V tiles through a 2-stage ring
//   warp 1      allocates 512 TMEM columns, issues tcgen05.mma (one thread):
//               S_j = Q.K_j^T (M128 N64 K256) into a double-buffered TMEM S,
//               O  += P_j.V_j (M128 N256 K64, V read MN-major)
//   warps 4..7  softmax: thread = query row = TMEM lane; reads S with
//               tcgen05.ld, masks causally, keeps an online max that is only
//               moved (and O rescaled in TMEM) when it grows by more than 2^8,
//               writes bf16 P to shared memory; epilogue O/l * sigmoid(gate).
// Key tiles past the last query row are skipped (causal tile skipping).
#include <algorithm>

#include "common.cuh"
#include "prefill.cuh"
#include "tcgen05.cuh"

namespace lisa {

namespace {

constexpr int PF_BM = 128;  // query rows per CTA
constexpr int PF_BN = 64;   // keys per tile
constexpr int PF_Q_BYTES = PF_BM * HD * 2;    // 64 KB
constexpr int PF_KV_BYTES = PF_BN * HD * 2;   // 32 KB
constexpr int PF_P_BYTES = PF_BM * PF_BN * 2; // 16 KB
constexpr int PF_OFF_K = PF_Q_BYTES;
constexpr int PF_OFF_V = PF_OFF_K + 2 * PF_KV_BYTES;
constexpr int PF_OFF_P = PF_OFF_V + 2 * PF_KV_BYTES;
constexpr int PF_OFF_BAR = PF_OFF_P + PF_P_BYTES;
constexpr int PF_SMEM_BYTES = PF_OFF_BAR + 256 + 1024;
constexpr int PF_THREADS = 256;
constexpr uint32_t PF_TMEM_COLS = 512;
constexpr uint32_t PF_TMEM_O = 0;    // O accumulator: columns [0, 256)
constexpr uint32_t PF_TMEM_S = 256;  // S buffers: columns [256, 320), [320, 384)
constexpr float PF_RESCALE_LOG2 = 8.0f;

// Barrier slots inside the barrier block.
enum { B_Q = 0, B_KFULL = 1, B_VFULL = 3, B_EMPTY = 5, B_SFULL = 7, B_PFULL = 9, B_ODONE = 10, B_COUNT = 11 };

}  // namespace

// One warp per (row, head) item; items 0..27 per row are the 24 query heads
// then the 4 KV heads. Lane l holds dims 8l..8l+7; the RoPE partner of dims
// 0..31 (lanes 0..3) is dims 32..63 (lanes 4..7).
__global__ void __launch_bounds__(256) prefill_prologue_kernel(const PrefillParams p) {
  const int item = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= p.rows * (QH + KVH)) return;
  const int r = item / (QH + KVH), hh = item % (QH + KVH);
  const bool is_q = hh < QH;
  const uint32_t pos = p.base + r;
  const size_t in = is_q ? (size_t)r * QROW + (size_t)hh * 512 + lane * 8
                         : (size_t)r * KROW + (size_t)(hh - QH) * HD + lane * 8;
  const void* src = is_q ? p.q_gate : p.k_in;
  const uint16_t* w = is_q ? p.q_norm_w : p.k_norm_w;
  float x[8], ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    x[i] = load_in_bf16(src, in + i, p.in_bf16);
    ss += x[i] * x[i];
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = 1.0f / sqrtf(ss / 256.0f + p.eps);
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float n = x[i] * inv * bf16_bits_to_f32(w[lane * 8 + i]);
    const float partner = __shfl_xor_sync(0xffffffffu, n, 4);
    o[i] = n;
    if (lane < 8) {
      float c, s;
      rope_cs(pos, (lane & 3) * 8 + i, c, s);
      o[i] = lane < 4 ? n * c - partner * s : n * c + partner * s;
    }
  }
  const uint4 packed = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                                  pack_bf16x2(o[6], o[7]));
  if (is_q) {
    *reinterpret_cast<uint4*>(p.q_ws + ((size_t)hh * PF_MAX_ROWS + r) * HD + lane * 8) = packed;
  } else {
    const size_t out = ((size_t)(hh - QH) * p.capacity + pos) * HD + lane * 8;
    *reinterpret_cast<uint4*>(p.k_cache + out) = packed;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = load_in_bf16(p.v_in, in + i, p.in_bf16);
    *reinterpret_cast<uint4*>(p.v_cache + out) =
        make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
}

// Grid: n_qtiles * 24 CTAs, heaviest (last) query tiles first. 256 threads.
__global__ void __launch_bounds__(PF_THREADS, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PF_OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.rows + PF_BM - 1) / PF_BM;
  const int qt = n_qt - 1 - (int)(blockIdx.x / QH);
  const int h = blockIdx.x % QH, kvh = h / GQA;
  const int r0 = qt * PF_BM;
  const int r_end = min(r0 + PF_BM, p.rows);
  const uint32_t kv_end = p.base + (uint32_t)r_end;  // keys [0, kv_end)
  const int n_tiles = (int)((kv_end + PF_BN - 1) / PF_BN);

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    mbar_init(&bars[B_Q], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[B_KFULL + s], 1);
      mbar_init(&bars[B_VFULL + s], 1);
      mbar_init(&bars[B_EMPTY + s], 1);
      mbar_init(&bars[B_SFULL + s], 1);
    }
    mbar_init(&bars[B_PFULL], 128);
    mbar_init(&bars[B_ODONE], 1);
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

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars[B_Q], PF_Q_BYTES);
      for (int st = 0; st < 4; ++st) tma_load_3d(smem + st * (PF_BM * 128), &tq, &bars[B_Q], st * 64, r0, h);
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&bars[B_EMPTY + s], ((j >> 1) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) break;
        uint8_t* ks = smem + PF_OFF_K + s * PF_KV_BYTES;
        uint8_t* vs = smem + PF_OFF_V + s * PF_KV_BYTES;
        mbar_arrive_expect_tx(&bars[B_KFULL + s], PF_KV_BYTES);
        for (int st = 0; st < 4; ++st) tma_load_3d(ks + st * 8192, &tk, &bars[B_KFULL + s], st * 64, j * PF_BN, kvh);
        mbar_arrive_expect_tx(&bars[B_VFULL + s], PF_KV_BYTES);
        for (int st = 0; st < 4; ++st) tma_load_3d(vs + st * 8192, &tv, &bars[B_VFULL + s], st * 64, j * PF_BN, kvh);
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
      bool ok = mbar_wait(&bars[B_Q], 0, p.err, ERR_TIMEOUT_FULL);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&bars[B_KFULL + s], (j >> 1) & 1, p.err, ERR_TIMEOUT_FULL)) return false;
        tc_fence_after();
        const uint32_t sK = smem_u32(smem + PF_OFF_K + s * PF_KV_BYTES);
        const uint32_t d = tmem + PF_TMEM_S + s * PF_BN;
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
          const uint64_t a = umma_desc_sw128(sQ + (kk >> 2) * (PF_BM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t b = umma_desc_sw128(sK + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024);
          umma_bf16(d, a, b, IDESC_S, kk > 0);
        }
        umma_commit(&bars[B_SFULL + s]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int s = j & 1;
        if (j + 1 < n_tiles && !issue_s(j + 1)) break;
        if (!mbar_wait(&bars[B_PFULL], j & 1, p.err, ERR_TIMEOUT_MMA)) break;
        if (!mbar_wait(&bars[B_VFULL + s], (j >> 1) & 1, p.err, ERR_TIMEOUT_FULL)) break;
        tc_fence_after();
        const uint32_t sP = smem_u32(smem + PF_OFF_P);
        const uint32_t sV = smem_u32(smem + PF_OFF_V + s * PF_KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t a = umma_desc_sw128(sP + kk * 32, 16, 1024);
          const uint64_t b = umma_desc_sw128(sV + kk * 2048, 8192, 1024);
          umma_bf16(tmem + PF_TMEM_O, a, b, IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars[B_ODONE]);
        umma_commit(&bars[B_EMPTY + s]);
      }
    }
    __syncwarp();
    named_bar_sync(1, 160);
    tc_fence_after();
    tmem_dealloc(tmem, PF_TMEM_COLS);
    return;
  }

  if (warp < 4) return;

  // ---------------- softmax / correction / epilogue (warps 4..7) ----------------
  const int wi = warp - 4;
  const int row = wi * 32 + lane;  // row within the tile == TMEM lane
  const uint32_t lane_addr = tmem + ((uint32_t)(wi * 32) << 16);
  const uint32_t pos_row = p.base + (uint32_t)(r0 + row);
  uint8_t* sP = smem + PF_OFF_P;
  float m2 = -INFINITY, l = 0.f;
  bool ok = true;
  for (int j = 0; j < n_tiles; ++j) {
    const int b = j & 1;
    if (!mbar_wait(&bars[B_SFULL + b], (j >> 1) & 1, p.err, ERR_TIMEOUT_MMA)) {
      ok = false;
      break;
    }
    tc_fence_after();
    uint32_t sa[32], sb[32];
    tmem_ld32(lane_addr + PF_TMEM_S + b * PF_BN, sa);
    tmem_ld32(lane_addr + PF_TMEM_S + b * PF_BN + 32, sb);
    tmem_wait_ld();
    const uint32_t key0 = (uint32_t)j * PF_BN;
    float s2[64];
    float tmax = -INFINITY;
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      const float raw = __uint_as_float(c < 32 ? sa[c] : sb[c - 32]);
      s2[c] = key0 + c <= pos_row ? raw * (SCALE * LOG2E) : -INFINITY;
      tmax = fmaxf(tmax, s2[c]);
    }
    const float mnew = fmaxf(m2, tmax);
    const bool need = mnew > m2 + PF_RESCALE_LOG2;  // also true for the first finite max
    float alpha = 1.f;
    if (need) {
      alpha = exp2f(m2 - mnew);
      m2 = mnew;
    }
    uint32_t pk[32];
    float psum = 0.f;
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const float e0 = m2 == -INFINITY ? 0.f : exp2f(s2[2 * c] - m2);
      const float e1 = m2 == -INFINITY ? 0.f : exp2f(s2[2 * c + 1] - m2);
      pk[c] = pack_bf16x2(e0, e1);
      psum += bf16_bits_to_f32(pk[c] & 0xffffu) + bf16_bits_to_f32(pk[c] >> 16);
    }
    l = l * alpha + psum;
    if (j > 0) {
      if (!mbar_wait(&bars[B_ODONE], (j - 1) & 1, p.err, ERR_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t ov[32];
          tmem_ld32(lane_addr + PF_TMEM_O + c * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st32(lane_addr + PF_TMEM_O + c * 32, ov);
        }
        tmem_wait_st();
      }
    }
    // P row -> shared memory, K-major 128-byte-swizzled rows of 64 keys
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(sP + swz128((uint32_t)row, (uint32_t)c)) =
          make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(&bars[B_PFULL]);
  }
  if (ok && mbar_wait(&bars[B_ODONE], (n_tiles - 1) & 1, p.err, ERR_TIMEOUT_MMA)) {
    tc_fence_after();
    const int r = r0 + row;
    const float inv_l = 1.0f / l;
#pragma unroll 1
    for (int c = 0; c < HD / 32; ++c) {
      uint32_t ov[32];
      tmem_ld32(lane_addr + PF_TMEM_O + c * 32, ov);
      tmem_wait_ld();
      if (r < p.rows) {
        uint32_t outw[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float y[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int d = c * 32 + 2 * i + e;
            const float gv = load_in_bf16(p.q_gate, (size_t)r * QROW + (size_t)h * 512 + 256 + d, p.in_bf16);
            const float sg = 1.0f / (1.0f + exp2f(-LOG2E * gv));
            y[e] = __uint_as_float(ov[2 * i + e]) * inv_l * sg;
          }
          outw[i] = pack_bf16x2(y[0], y[1]);
        }
        uint4* dst = reinterpret_cast<uint4*>(p.gated_out + (size_t)r * OROW + h * HD + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(outw[4 * i], outw[4 * i + 1], outw[4 * i + 2], outw[4 * i + 3]);
      }
    }
  }
  tc_fence_before();
  named_bar_sync(1, 160);
}

size_t prefill_workspace_bytes() { return (size_t)QH * PF_MAX_ROWS * HD * sizeof(uint16_t); }

cudaError_t launch_prefill(const PrefillParams& p, int num_sms, cudaStream_t stream) {
  (void)num_sms;
  const int items = p.rows * (QH + KVH);
  prefill_prologue_kernel<<<(items + 7) / 8, 256, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
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
      lisa_encode_kv_map(&tv, p.v_cache, kv_rows, p.capacity, PF_BN, KVH) != 0)
    return cudaErrorInvalidValue;
  const int n_qt = (p.rows + PF_BM - 1) / PF_BM;
  prefill_attn_kernel<<<n_qt * QH, PF_THREADS, PF_SMEM_BYTES, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace lisa
