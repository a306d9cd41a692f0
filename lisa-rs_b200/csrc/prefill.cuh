// prefill.cuh — launch interface of the chunked-prefill attention kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Encodes a TMA map over a bf16 [planes][window_rows][256] array (a cache
// window has 4 planes) seen as 64-dim groups: dims {64, rows, 4, planes}, boxes
// {64, box_rows, box_groups, 1} landing as [group][row][64]. Defined in runtime.cu.
int lisa_encode_group_map(CUtensorMap* map, const void* base, uint32_t rows, uint32_t window_rows, uint32_t planes,
                          uint32_t box_rows, uint32_t box_groups);
// A bf16 [rows][heads][head_elems] array (row stride row_elems) as 64-element
// groups: dims {64, rows, groups, heads}, boxes {64, box_rows, 4, 1}. Defined
// in runtime.cu.
int lisa_encode_rows_map(CUtensorMap* map, const void* base, uint32_t rows, uint32_t row_elems, uint32_t groups,
                         uint32_t heads, uint32_t head_elems, uint32_t box_rows);

namespace lisa {

constexpr int PF_MAX_ROWS = 512;
// (query row pair, head) units of a chunk: at most 2 pairs x 24 heads; each is
// one cluster, or two clusters over consecutive key ranges (split units).
constexpr int PF_MAX_UNITS = 48;
constexpr int PF_MAX_SEGS = 2 * PF_MAX_UNITS;

struct PrefillParams {
  const void* q_gate;  // [rows][24][512]
  const void* k_in;    // [rows][4][256]
  const void* v_in;
  int in_bf16;
  const uint16_t* q_norm_w;
  const uint16_t* k_norm_w;
  float eps;
  uint16_t* k_cache;  // [4][capacity][256]
  uint16_t* v_cache;
  uint32_t capacity;
  uint32_t base;      // position of row 0
  int rows;           // 1..512
  uint16_t* q_ws;     // workspace: normalised query, bf16 [24 heads][512 rows][256]
  uint16_t* gated_out;  // [rows][6144]
  int* err;
  // Key-range segments, one per cluster in launch order (filled by
  // launch_prefill): key tiles [seg_lo, seg_hi) of unit seg_unit (bits 0-7
  // head, 8-11 query pair, bit 12 set when the unit is split in two).
  int n_seg;
  uint32_t seg_lo[PF_MAX_SEGS];
  uint32_t seg_hi[PF_MAX_SEGS];
  uint16_t seg_unit[PF_MAX_SEGS];
  float* part;          // split partials, per (unit, CTA rank): O [64][128 rows][4] f32, then max / sum per row
  uint32_t* tickets;    // per (unit, CTA rank): arrival count, then the partial-ready flag
  float inv_freq[32];  // filled by launch_prefill
#if defined(LISA_PREFILL_TRACE) || defined(LISA_PREFILL_OBSERVE)
  unsigned long long* trace;  // debug builds only
#endif
};

// Bytes of device workspace launch_prefill needs.
size_t prefill_workspace_bytes();
// Byte offset and size of the split-merge tickets inside that workspace; a
// launch that gave up (device error) may leave them non-zero, and the
// context's error check clears them.
size_t prefill_ticket_offset();
size_t prefill_ticket_bytes();

// Prologue (q norm/RoPE into q_ws, K/V append) then the tcgen05 attention.
cudaError_t launch_prefill(const PrefillParams& p, int num_sms, cudaStream_t stream);

}  // namespace lisa
