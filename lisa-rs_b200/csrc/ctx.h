// ctx.h — the context object behind the opaque lisa_attn_ctx handle (shared
// by the C-ABI translation units).
#pragma once
#include <cuda.h>
#include <stdint.h>

struct lisa_attn_ctx {
  int device = 0;
  int n_layers = 0;
  uint32_t capacity = 0;
  uint16_t* k = nullptr;  // [layer][4][capacity][256]
  uint16_t* v = nullptr;
  float* part_o = nullptr;   // decode chunk partials
  float* part_ml = nullptr;
  uint32_t chunk_cap = 0;
  void* prefill_ws = nullptr;  // prefill scratch
  size_t prefill_ws_bytes = 0;
  int* err = nullptr;
  uint32_t* sched = nullptr;  // decode chunk counters [4]
  CUtensorMap* tmaps = nullptr;  // device: per layer the K and V maps over the whole capacity (batched decode)
  int num_sms = 148;
  uint32_t position = 0;
  bool verify_pending = false;
  uint32_t verify_base = 0;
};
