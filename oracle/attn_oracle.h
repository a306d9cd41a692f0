/*
 * attn_oracle.h — TEST INFRASTRUCTURE ONLY. A plain-C, f32 CPU restatement of
 * the lisa-rs full-attention hot path, used as the parity checker for the CUDA
 * path and as the timed CPU baseline. Nothing in the product links it.
 *
 * Parity pin: lisa-rs runs only on Metal, and its Rust sources cannot be built
 * here, so the oracle is pinned against the CPU expectations written in the
 * reference's own tests (tests/attn_sliced.rs:114-130, tests/attn_cache.rs:
 * 14-292), regenerated from their input formulas by tests/golden/make_golden.py.
 * See each function for the reference file:line it restates.
 */
#ifndef LISA_ATTN_ORACLE_H
#define LISA_ATTN_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

float orc_bf16_to_f32(uint16_t b);
uint16_t orc_f32_to_bf16(float f);        /* round to nearest even (Metal bfloat(float)) */
uint16_t orc_f32_to_bf16_trunc(float f);  /* truncation (src/format/dtype.rs:42-47) */
float orc_rope_inv_freq(int pair);        /* 1 / theta^(2*pair/64), theta = 1e7 */

/* q_norm_gate_rope_{decode,block3,prefill} (attention.metal:118-155, 245-281,
 * 364-401). q_gate f32 [rows][24][512]; query bf16 [rows][24][256]; gate f32
 * [rows][24][256]; row r uses position base + r. */
void orc_q_prologue(const float* q_gate, int rows, uint32_t base, const uint16_t* q_norm_w, float eps,
                    uint16_t* query, float* gate);

/* kv_cache_store_{decode,block3,prefill} (attention.metal:158-197, 283-319,
 * 403-440). k, v f32 [rows][4][256]; caches bf16 [4][capacity][256]. Rows at
 * positions >= capacity are skipped, as in the reference. */
void orc_kv_append(const float* k, const float* v, int rows, uint32_t base, const uint16_t* k_norm_w,
                   float eps, uint16_t* k_cache, uint16_t* v_cache, uint32_t capacity);

/* Serial online-softmax attention, sdpa_decode_streaming{,_block3} and
 * sdpa_decode_prefill (attention.metal:201-241, 321-358, 442-480): row r
 * attends positions 0 .. base + r. query bf16 [rows][24][256]; out f32
 * [rows][24][256]. OpenMP over (row, head). */
void orc_sdpa_serial(const uint16_t* query, const uint16_t* k_cache, const uint16_t* v_cache,
                     uint32_t capacity, uint32_t base, int rows, float* out);

/* Sliced attention, sdpa_decode_partial + sdpa_decode_final
 * (attention.metal:550-641): 64-token slices, each an online softmax, merged by
 * log-sum-exp. Unlike the reference there is no 256-slice cap (the reference
 * merges garbage past 16384 tokens). OpenMP over (row, head, slice) — the
 * reference's own work split. */
void orc_sdpa_sliced(const uint16_t* query, const uint16_t* k_cache, const uint16_t* v_cache,
                     uint32_t capacity, uint32_t base, int rows, float* out);

/* gate_out_bf16 (attention.metal:520-531): gated = bf16(o * sigmoid(g)). */
void orc_gate(const float* out, const float* gate, int n, uint16_t* gated);

/* One whole attention layer for rows at base (decode rows=1, verify rows=3,
 * prefill rows<=512): prologue, append, sliced (sliced=1) or serial attention,
 * gate. q_gate/k/v f32. Writes the caches and gated bf16 [rows][6144]. */
void orc_attention_layer(const float* q_gate, const float* k, const float* v, int rows, uint32_t base,
                         const uint16_t* q_norm_w, const uint16_t* k_norm_w, float eps,
                         uint16_t* k_cache, uint16_t* v_cache, uint32_t capacity, int sliced,
                         uint16_t* gated);

/* Legacy batch path used as the second opinion in tests/attn_cache.rs:14-192:
 * qk_norm_gate_rope + k_norm_rope + sdpa_scalar (attention.metal:33-94,
 * 485-517). q f32 [L][12288], k/v f32 [L][1024]; out f32 [L][24][256]. */
void orc_legacy_batch(const float* q, const float* k, const float* v, int L, const uint16_t* q_norm_w,
                      const uint16_t* k_norm_w, float eps, float* out);

int orc_num_threads(void);
void orc_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
