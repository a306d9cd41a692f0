// decode.cuh — launch interface of the split-KV decode/verify kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lisa {

// Split-KV geometry. A chunk is the unit of numerics: the online softmax runs
// sequentially over the chunk's 16-token tiles and the chunk partials are
// merged in a fixed order. Chunk boundaries depend only on the token index, so
// a verify row gives bit-identical results to the same row decoded alone.
constexpr int DEC_CHUNK = 128;  // tokens per chunk
constexpr int DEC_TILE = 16;    // tokens per pipeline stage (one mma M-tile)
constexpr int DEC_STAGES = 3;   // TMA ring depth per CTA
constexpr int DEC_CTAS_PER_SM = 4;
constexpr int DEC_STAGE_BYTES = 2 * DEC_TILE * 256 * 2;  // K + V tile, 16 KB
constexpr int DEC_SMEM_BYTES = DEC_STAGES * DEC_STAGE_BYTES + 1024 + 256;
constexpr int CMB_DIMS_PER_CTA = 8;
constexpr int CMB_PHASES = 8;

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
  // combine outputs: gated bf16 [rows][6144] (final) or window partials
  uint16_t* gated_out;
  float* win_o;   // [rows][24][256]
  float* win_ml;  // [rows][24][2]
};

// Launches the split-KV kernel and its combine (programmatic dependent launch)
// for rows in {1, 2, 3}. The tensor maps cover k_cache / v_cache as
// {256, extent, 4} with SWIZZLE_128B boxes of {64, 16, 1}.
cudaError_t launch_decode(const DecodeParams& p, int rows, const CUtensorMap& tk, const CUtensorMap& tv,
                          int num_sms, cudaStream_t stream);

// Merges n_parts window partials and applies the gate.
cudaError_t launch_merge_windows(int n_parts, int rows, const float* part_o, const float* part_ml,
                                 int in_bf16, const void* q_gate, uint16_t* gated_out, cudaStream_t stream);

}  // namespace lisa
