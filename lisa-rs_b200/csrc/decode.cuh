// decode.cuh — launch interface of the split-KV decode/verify kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lisa {

// Split-KV geometry. A chunk is the unit of numerics: the online softmax runs
// over the chunk's 64-token stages in order and the chunk partials are merged
// in a fixed order. Chunk boundaries depend only on the token index, so a
// verify row gives bit-identical results to the same row decoded alone.
#ifndef LISA_DEC_CHUNK
#define LISA_DEC_CHUNK 448
#endif
constexpr int DEC_CHUNK = LISA_DEC_CHUNK;  // tokens per chunk (a multiple of DEC_TILE)
constexpr int DEC_TILE = 64;    // tokens per pipeline stage (4 warps x 16)
constexpr int DEC_STAGES = 3;   // TMA ring depth per CTA
constexpr int DEC_STAGE_BYTES = 2 * DEC_TILE * 256 * 2;  // K + V stage, 64 KB
constexpr int DEC_XCH_BYTES = 2 * 4 * 8 * 4 * 2 + 2 * 4 * 32 * 8;  // per query row: max, sums, P fragments
// Per query row: the raw q of the kv head's 6 heads (f32 or bf16, 6 KB max),
// later overwritten by the normalised bf16 rows [8 heads][256] (4 KB).
constexpr int DEC_QROW_BYTES = 6 * 1024;
constexpr int DEC_QS_OFF = DEC_STAGES * DEC_STAGE_BYTES + 3 * DEC_XCH_BYTES + 256;  // after the mbarriers
constexpr int DEC_WN_OFF = DEC_QS_OFF + 3 * DEC_QROW_BYTES;                           // q_norm gains, 512 B
constexpr int DEC_SMEM_BYTES = DEC_WN_OFF + 512 + 1024;
constexpr int CMB_DIMS_PER_CTA = 8;
constexpr int CMB_PHASES = 32;
constexpr int CMB_THREADS = 32 * CMB_PHASES;
constexpr int HD_FLOATS_PLUS_ML = 256 + 2;

// Window-partial exchange between the ranks of one split-KV sequence (one
// GPU per rank, peer memory mapped by CUDA IPC). Lives in device memory.
constexpr int XCHG_MAX_WORLD = 8;
constexpr int XCHG_REC = HD_FLOATS_PLUS_ML;  // words per (row, head) record: O[256], max, sum
struct XchgDev {
  uint64_t* recv[XCHG_MAX_WORLD];   // receive region of rank i, as mapped in this process
  uint32_t* state;                  // this rank: [0] completed exchanges, [1] merge CTAs done, [2] error word
  int world, rank, max_rows;
};
// recv[parity][src rank][row][24 heads][XCHG_REC] words: value bits | step << 32
__host__ __device__ constexpr size_t xchg_recv_words(int world, int max_rows) {
  return (size_t)2 * world * max_rows * 24 * XCHG_REC;
}

struct DecodeParams {
  const void* q_gate;  // [rows][24][512]
  const void* k_in;    // [rows][4][256]
  const void* v_in;
  int in_bf16;
  const uint16_t* q_norm_w;
  const uint16_t* k_norm_w;
  float eps;
  uint16_t* k_cache;     // window base: [4][window_rows][256]
  uint16_t* v_cache;
  uint32_t window_rows;  // row stride of the window (capacity)
  uint32_t kv_lo;        // global position of window row 0
  uint32_t base;         // global position of query row 0
  uint32_t extent;       // window rows visible to this call (>= 1)
  uint32_t nchunks;      // ceil(extent / DEC_CHUNK)
  uint32_t chunk_cap;    // chunk stride of the partial buffers
  float* part_o;         // [rows][4][chunk_cap][256][8] unnormalised sums
  float* part_ml;        // [rows][4][chunk_cap][2][8]  {max, sum}
  int* err;
  uint64_t wait_ns;      // bounded-wait limit of every mbarrier wait
  int withhold;          // test hook: the producer issues nothing (waits run out)
  uint32_t* sched;       // [4] per-kv-head chunk counters: zero at launch, reset by the combine
  // RoPE tables filled by launch_decode on the host: cos/sin of rows
  // base..base+2 for the 32 rotated pairs.
  float rope_c[3][32];
  float rope_s[3][32];
  // combine outputs: gated bf16 [rows][6144] (final) or window partials
  uint16_t* gated_out;
  float* win_o;   // [rows][24][256]
  float* win_ml;  // [rows][24][2]
  const XchgDev* xchg;  // or: publish the window partials to every rank (exchange mode)
#ifdef LISA_DECODE_TRACE
  unsigned long long* trace;  // debug builds only: per-phase cycle totals
#endif
};

// Launches the split-KV kernel and its combine (programmatic dependent launch)
// for rows in {1, 2, 3}. The tensor maps cover k_cache / v_cache as
// {256, extent, 4} with SWIZZLE_128B boxes of {64, 16, 1}.
cudaError_t launch_decode(const DecodeParams& p, int rows, const CUtensorMap& tk, const CUtensorMap& tv,
                          int num_sms, cudaStream_t stream);

// Exchange mode: waits (bounded) for every rank's window partials of this
// step, merges them by log-sum-exp and applies the gate; then advances the
// exchange step counter.
cudaError_t launch_merge_exchange(const XchgDev* x, int rows, int in_bf16, const void* q_gate,
                                  uint16_t* gated_out, uint64_t wait_ns, cudaStream_t stream);

// Merges n_parts window partials and applies the gate.
cudaError_t launch_merge_windows(int n_parts, int rows, const float* part_o, const float* part_ml,
                                 int in_bf16, const void* q_gate, uint16_t* gated_out, cudaStream_t stream);

}  // namespace lisa
