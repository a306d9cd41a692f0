/*
 * lisa_attn.h — C ABI of the B200 (sm_100a) gated-GQA full-attention path.
 *
 * The layer is the full-attention layer of the lisa-rs Qwen3.x hybrid decoder
 * (every 4th layer, src/model/mod.rs:16-22): 24 query heads, 4 KV heads,
 * head_dim 256, per-head q/k RMSNorm (eps 1e-6), partial NeoX RoPE on dims
 * 0..63 with theta 1e7, a bf16 KV-cache append, causal softmax(QK^T/16)V with
 * f32 accumulation, and a sigmoid output gate (src/kernels/shaders/
 * attention.metal:1-27).
 *
 * In lisa-rs there is no FFI for this path: it is the private methods
 * QwenRunner::encode_attention (src/model/runner.rs:1426-1592),
 * QwenRunner::encode_prefill_attention (runner.rs:1962-2062) and the KV
 * position contract (runner.rs:423-503, 911-944, 2376-2545). Each entry point
 * below names the reference code it replaces. A Rust crate binds them with a
 * plain `extern "C"` block of the same signatures (pointers as *mut/*const,
 * uint32_t as u32, void* stream as *mut c_void).
 *
 * Conventions
 *   - Every entry point returns an int status (LISA_OK or a negative code).
 *     Invalid arguments are rejected before anything is launched; no call is a
 *     silent no-op (the reference kernels silently return when out of range,
 *     attention.metal:172/294/415/450/564).
 *   - All tensor pointers are CUDA device pointers unless a name says "host".
 *     The caller owns inputs and outputs; a context owns its KV cache and its
 *     scratch memory.
 *   - Work is ordered on the `stream` argument (a cudaStream_t passed as
 *     void*; NULL = legacy default stream). A context is not thread-safe: use
 *     one context per thread or a lock, as lisa-rs serialises its runner
 *     behind a Mutex (src/serve/mod.rs:37-38).
 *   - Layouts (row-major, elements):
 *       q_gate  [rows][24][512]  per head: 256 query values then 256 gate values
 *                                (the q_proj output, runner.rs:204-209)
 *       k, v    [rows][4][256]   (k_proj / v_proj outputs)
 *       norm weights  bf16 [256]
 *       gated_out     bf16 [rows][24*256]  (the o_proj input, runner.rs:1574-1590)
 *       KV cache      bf16 [layer][4][capacity][256], K and V separately
 *                     (runner.rs:384-390, 1463-1464)
 *     q_gate and the norm weights must be 16-byte aligned, and for prefill also
 *     k, v and gated_out (LISA_EINVAL otherwise).
 *     q_gate/k/v are f32 (LISA_DTYPE_F32, the QMV/GEMM output type of the
 *     reference) or bf16 (LISA_DTYPE_BF16). The reference rounds them to bf16
 *     before use (attention.metal:40-42), so both give identical results.
 */
#ifndef LISA_ATTN_H
#define LISA_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LISA_ATTN_Q_HEADS 24
#define LISA_ATTN_KV_HEADS 4
#define LISA_ATTN_HEAD_DIM 256
#define LISA_ATTN_ROPE_DIM 64
#define LISA_ATTN_PREFILL_MAX_ROWS 512 /* PREFILL_BATCH, runner.rs:48-51 */

/* Status codes. */
#define LISA_OK 0
#define LISA_EINVAL (-22)   /* bad argument: null pointer, rows, layer, dtype */
#define LISA_ENOSPC (-28)   /* base + rows > capacity ("KV capacity exhausted") */
#define LISA_ESTATE (-71)   /* position contract violated (no pending verify, trim too far) */
#define LISA_ETIMEOUT (-62) /* a device-side bounded wait gave up (error flag set) */
#define LISA_ECUDA (-1000)  /* a CUDA runtime/driver call failed */
#define LISA_E2BIG (-7)     /* request larger than the fixed scratch of lisa_attn_decode_noalloc */

/* Input element types of q_gate / k / v. */
#define LISA_DTYPE_F32 0
#define LISA_DTYPE_BF16 1

typedef struct lisa_attn_ctx lisa_attn_ctx;

/* ---- context ------------------------------------------------------------
 * Replaces the KV-cache allocation of QwenRunner::load (runner.rs:384-390) and
 * MtpRunner::load (runner.rs:2455-2470): n_layers attention layers (16 for the
 * target, 1 for the MTP drafter), each with K and V caches of
 * [4][capacity][256] bf16, zero-filled, position 0. Also allocates the split-KV
 * scratch and a device error flag. capacity must be in 1..2^31. */
int lisa_attn_create(int device, int n_layers, uint32_t capacity, lisa_attn_ctx** out);
int lisa_attn_destroy(lisa_attn_ctx* ctx);

/* Device pointers of one layer's K and V cache ([4][capacity][256] bf16). */
int lisa_attn_kv_cache(lisa_attn_ctx* ctx, int layer, void** k_cache, void** v_cache);
uint32_t lisa_attn_capacity(const lisa_attn_ctx* ctx);
int lisa_attn_n_layers(const lisa_attn_ctx* ctx);

/* ---- per-layer dispatch ---------------------------------------------------
 * Decode (rows = 1) or MTP verify (rows = 3) of one attention layer at absolute
 * positions base .. base+rows-1. Replaces encode_attention's attention part
 * (runner.rs:1439-1590): q norm+RoPE+gate split (attention.metal:118-155,
 * 245-281), K/V append (158-197, 283-319), split-KV attention and merge
 * (550-641) and the gate (520-531). Row r attends causally over positions
 * 0 .. base+r. Rows of a verify are bit-identical to the same rows decoded one
 * at a time (the invariant tested at tests/attn_sliced.rs:186-187).
 * Errors: LISA_EINVAL (rows not 1 or 3, bad layer, null pointer, bad dtype),
 * LISA_ENOSPC (base + rows > capacity). */
int lisa_attn_decode(lisa_attn_ctx* ctx, int layer, uint32_t base, int rows, int in_dtype,
                     const void* q_gate, const void* k, const void* v,
                     const uint16_t* q_norm_w, const uint16_t* k_norm_w, float eps,
                     uint16_t* gated_out, void* stream);

/* Chunked prefill of one attention layer: rows (1..512) prompt rows at
 * positions base .. base+rows-1, causal over the whole cached prefix.
 * Replaces encode_prefill_attention's attention part (runner.rs:1976-2060):
 * attention.metal:364-480 and 520-531. Errors as lisa_attn_decode, with rows
 * allowed in 1..512. */
int lisa_attn_prefill_chunk(lisa_attn_ctx* ctx, int layer, uint32_t base, int rows, int in_dtype,
                            const void* q_gate, const void* k, const void* v,
                            const uint16_t* q_norm_w, const uint16_t* k_norm_w, float eps,
                            uint16_t* gated_out, void* stream);

/* ---- position contract ----------------------------------------------------
 * The logical KV length. Entries past it stay in the cache and are overwritten
 * by the next append; nothing is cleared (runner.rs:474-503, 2522-2545). */
uint32_t lisa_attn_position(const lisa_attn_ctx* ctx);

/* End of one forward over all layers: position += rows (runner.rs:589 for
 * rows = 1, runner.rs:2225 for a prefill chunk). rows == 3 is a block-3
 * verify: the base is remembered for lisa_attn_commit_verified_prefix
 * (runner.rs:906-907). LISA_ENOSPC if position + rows > capacity. */
int lisa_attn_advance(lisa_attn_ctx* ctx, int rows, int is_verify);

/* QwenRunner::commit_verified_prefix (runner.rs:911-944): position =
 * verify_base + rows, rows in 1..3. LISA_ESTATE if no verify is pending,
 * LISA_EINVAL for rows outside 1..3. The KV cache is not touched. */
int lisa_attn_commit_verified_prefix(lisa_attn_ctx* ctx, int rows);

/* MtpRunner::trim_state (runner.rs:2522-2531): position -= count;
 * LISA_ESTATE if count > position. */
int lisa_attn_trim_state(lisa_attn_ctx* ctx, uint32_t count);

/* MtpRunner::set_position (runner.rs:2536-2545): only moves backwards;
 * LISA_ESTATE if position > current position. */
int lisa_attn_set_position(lisa_attn_ctx* ctx, uint32_t position);

/* QwenRunner::restore_state's position part (runner.rs:476-503): any position
 * up to capacity (LISA_ENOSPC beyond it); clears a pending verify. */
int lisa_attn_restore_position(lisa_attn_ctx* ctx, uint32_t position);

/* reset_state (runner.rs:423-444, 2505-2516): zero the whole KV cache,
 * position 0, no pending verify. Stream-ordered. */
int lisa_attn_reset_state(lisa_attn_ctx* ctx, void* stream);

/* MtpCheckpoint (runner.rs:2376-2441): copy all layers' K then V caches
 * (2 * n_layers * 4 * capacity * 256 * 2 bytes, lisa_attn_snapshot_bytes) to a
 * caller-owned device buffer, or back, plus the position. Stream-ordered. */
size_t lisa_attn_snapshot_bytes(const lisa_attn_ctx* ctx);
int lisa_attn_kv_snapshot(lisa_attn_ctx* ctx, void* dst, size_t dst_bytes, uint32_t* position_out,
                          void* stream);
int lisa_attn_kv_restore(lisa_attn_ctx* ctx, const void* src, size_t src_bytes, uint32_t position,
                         void* stream);

/* Device-side error flag of the context (bounded waits that gave up).
 * Synchronises the context's device; returns LISA_OK, LISA_ETIMEOUT or
 * LISA_ECUDA, and clears the flag (and, after an error, the prefill's
 * split-merge tickets, so that later prefill calls start clean). */
int lisa_attn_check_device_error(lisa_attn_ctx* ctx);

/* ---- split-KV window entry points (multi-GPU) ------------------------------
 * No lisa-rs counterpart: lisa-rs drives one GPU. These let one long sequence's
 * KV be split along the position axis over several GPUs. A window holds cache
 * positions [kv_lo, kv_lo + window_rows) of one layer at k_cache / v_cache
 * ([4][window_rows][256] bf16, row i = position kv_lo + i). The call appends
 * the new rows that fall inside the window, attends rows 0..rows-1 over the
 * window's positions below base+r+1, and writes one partial per (row, head):
 * part_o f32 [rows][24][256] (normalised), part_ml f32 [rows][24][2] = {max
 * score, sum of exp(score - max)}. A window holding no position for a row gives
 * max = -inf, sum = 0. workspace: lisa_attn_window_workspace_bytes(window_rows,
 * rows) bytes of device memory, 256-byte aligned. */
size_t lisa_attn_window_workspace_bytes(uint32_t window_rows, int rows);
int lisa_attn_decode_window(void* k_cache, void* v_cache, uint32_t window_rows, uint32_t kv_lo,
                            uint32_t base, int rows, int in_dtype, const void* q_gate,
                            const void* k, const void* v, const uint16_t* q_norm_w,
                            const uint16_t* k_norm_w, float eps, float* part_o, float* part_ml,
                            void* workspace, size_t workspace_bytes, void* stream);

/* Device error word of the last lisa_attn_decode_window call that used this
 * workspace (each call zeroes it first). Synchronises `stream`, returns LISA_OK
 * or LISA_ETIMEOUT (a bounded device wait of that call gave up: its partials
 * are not valid) and clears the word. No lisa-rs counterpart (its kernels have
 * no failure channel). */
int lisa_attn_window_check_device_error(void* workspace, void* stream);

/* Merge n_parts window partials (stacked: part_o [n_parts][rows][24][256],
 * part_ml [n_parts][rows][24][2]) by log-sum-exp and apply the sigmoid gate
 * taken from q_gate: gated_out bf16 [rows][24*256]. */
int lisa_attn_merge_windows(int n_parts, int rows, const float* part_o, const float* part_ml,
                            int in_dtype, const void* q_gate, uint16_t* gated_out, void* stream);

/* ---- batched decode of many sequences -------------------------------------
 * One M=1 decode step of one attention layer for n_seqs independent
 * sequences, each with its own context (KV cache, capacity), in three kernel
 * launches: encode_attention (runner.rs:1426-1592) for batch 1, taken over all
 * sequences at once. Row i of q_gate [n_seqs][24][512], k, v [n_seqs][4][256]
 * and gated_out [n_seqs][6144] belongs to ctxs[i], whose new row is appended
 * at bases[i] (host array); sequence i attends positions 0..bases[i]. The
 * norm gains are shared (one model). Positions are not advanced (call
 * lisa_attn_advance per context, as after lisa_attn_decode). Results equal
 * lisa_attn_decode's for each sequence within the decode tolerance.
 * A lisa_attn_batch owns the scratch for up to max_seqs sequences
 * (<= LISA_ATTN_BATCH_MAX_SEQS) whose contexts sum to at most
 * max_total_positions (LISA_E2BIG beyond). Every context must live on the
 * batch's device (LISA_EINVAL); bases[i] + 1 > capacity gives LISA_ENOSPC.
 * Calls on one batch object must not overlap on the GPU. */
#define LISA_ATTN_BATCH_MAX_SEQS 128
typedef struct lisa_attn_batch lisa_attn_batch;
int lisa_attn_batch_create(int device, int max_seqs, uint64_t max_total_positions, lisa_attn_batch** out);
int lisa_attn_batch_destroy(lisa_attn_batch* b);
int lisa_attn_decode_batch(lisa_attn_batch* b, int n_seqs, lisa_attn_ctx* const* ctxs, int layer,
                           const uint32_t* bases, int in_dtype, const void* q_gate, const void* k, const void* v,
                           const uint16_t* q_norm_w, const uint16_t* k_norm_w, float eps, uint16_t* gated_out,
                           void* stream);
/* Synchronises `stream`; LISA_ETIMEOUT if a bounded wait of an earlier
 * lisa_attn_decode_batch call gave up (its output is not valid); clears. */
int lisa_attn_batch_check_device_error(lisa_attn_batch* b, void* stream);

/* ---- split-KV decode with a peer-memory exchange (multi-GPU) ---------------
 * No lisa-rs counterpart (lisa-rs drives one GPU). One long sequence's KV is
 * split into contiguous windows, one per rank (one process per GPU, the GPUs
 * of one node, world <= 8). Per step every rank runs lisa_attn_xchg_decode on
 * its window with the same inputs: the split kernel streams the window, the
 * combine kernel writes the window's per-(row, head) partial (normalised O,
 * max, sum) into every rank's receive region with peer stores, every value in
 * an 8-byte word tagged with the step number, and a merge kernel waits
 * (bounded) until the words it needs carry the step, merges the partials by
 * log-sum-exp in rank order and applies the
 * gate, so every rank ends with the same gated_out. The merge of
 * sdpa_decode_final (attention.metal:611-641), taken across GPUs.
 * Setup: every rank calls lisa_attn_xchg_create, exports its receive region
 * with lisa_attn_xchg_handle (LISA_ATTN_XCHG_HANDLE_BYTES bytes, a CUDA IPC
 * handle), the caller all-gathers the handles in rank order (any host
 * transport), and every rank calls lisa_attn_xchg_open with the world's
 * handles before the first step. All ranks must make the same sequence of
 * lisa_attn_xchg_decode calls (same rows), as they would of a collective.
 * The step counter is kept on the device, so a step can be captured in a CUDA
 * graph and replayed. A rank whose peer never delivers gets LISA_ETIMEOUT from
 * lisa_attn_xchg_check_device_error (the merge's wait gives up after 2 s). */
#define LISA_ATTN_XCHG_HANDLE_BYTES 64
#define LISA_ATTN_XCHG_MAX_WORLD 8
typedef struct lisa_attn_xchg lisa_attn_xchg;
/* window_rows: positions this rank's window holds; max_rows: 1 or 3. */
int lisa_attn_xchg_create(int device, int world, int rank, int max_rows, uint32_t window_rows,
                          lisa_attn_xchg** out);
int lisa_attn_xchg_handle(lisa_attn_xchg* x, void* handle_out);
int lisa_attn_xchg_open(lisa_attn_xchg* x, const void* handles);
/* k_cache / v_cache: this rank's window, [4][window_rows][256] bf16, row i =
 * position kv_lo + i. rows 1 or 3 (<= max_rows). LISA_ESTATE before open. */
int lisa_attn_xchg_decode(lisa_attn_xchg* x, void* k_cache, void* v_cache, uint32_t kv_lo, uint32_t base, int rows,
                          int in_dtype, const void* q_gate, const void* k, const void* v, const uint16_t* q_norm_w,
                          const uint16_t* k_norm_w, float eps, uint16_t* gated_out, void* stream);
/* Synchronises `stream`; LISA_ETIMEOUT if a bounded wait of an earlier step
 * (this rank's split kernel, or the merge waiting for a peer) gave up; clears. */
int lisa_attn_xchg_check_device_error(lisa_attn_xchg* x, void* stream);
int lisa_attn_xchg_destroy(lisa_attn_xchg* x);

/* ---- decode without allocation -------------------------------------------
 * No counterpart in lisa-rs. For callers that may not allocate device memory
 * while they run: an engine that hands out all of its GPU memory from a pool
 * reserved at start-up, or a caller whose allocator must not be entered on the
 * decode path. Same work and results as lisa_attn_decode, but over a KV cache
 * the caller owns (k_cache / v_cache, [4][capacity][256] bf16, row i =
 * position i) and with its scratch in a fixed array compiled into the library
 * (about 3.7 MB per GPU that loads it, held until the process exits), so the
 * call allocates nothing.
 *   - base + rows must not exceed LISA_ATTN_NOALLOC_MAX_POSITIONS; larger
 *     requests return LISA_E2BIG (use lisa_attn_decode for them).
 *   - The first call on a device looks up the array's device address; make
 *     that first call before any stream capture on that device.
 *   - All calls share the one array: calls that can overlap on the GPU (other
 *     streams, other host threads) race; the caller must serialise them.
 * Errors otherwise as lisa_attn_decode (LISA_EINVAL, LISA_ENOSPC when
 * base + rows > capacity). A device-side failure (a bounded wait that gave
 * up) is not visible in the return value, which comes back before the kernels
 * run: lisa_attn_noalloc_check_device_error reports it. */
#define LISA_ATTN_NOALLOC_MAX_POSITIONS 16384
int lisa_attn_decode_noalloc(void* k_cache, void* v_cache, uint32_t capacity, uint32_t base, int rows,
                             int in_dtype, const void* q_gate, const void* k, const void* v,
                             const uint16_t* q_norm_w, const uint16_t* k_norm_w, float eps,
                             uint16_t* gated_out, void* stream);

/* Error word of the last lisa_attn_decode_noalloc call on the current device
 * (kept in the fixed array, zeroed by every call): synchronises the device,
 * returns LISA_OK or LISA_ETIMEOUT and clears it. Allocates nothing. */
int lisa_attn_noalloc_check_device_error(void);

/* ---- test hook ------------------------------------------------------------
 * No lisa-rs counterpart. Process-wide: every later decode launch (contexts,
 * windows, no-alloc) gives its bounded mbarrier waits a limit of
 * wait_limit_us microseconds instead of the default 2 s, and with
 * withhold_loads != 0 its load warp issues no copy at all, so the compute
 * warps' first wait runs out, they record LISA_ETIMEOUT in the error word and
 * return (no copy is in flight, nothing is read or written out of bounds).
 * lisa_attn_debug_wait_fault(0, 0) restores the defaults. LISA_EINVAL for
 * withhold_loads without a limit or a limit above 10 s. */
int lisa_attn_debug_wait_fault(uint32_t wait_limit_us, int withhold_loads);

/* Test and measurement hook for the prefill attention grid; no lisa-rs
 * counterpart. A prefill chunk's (query row pair, head) units may each be split
 * into two consecutive key ranges that run as separate clusters and merge
 * their partial results (used when a cost model of the dispatch predicts at
 * least 10 % less time, i.e. for chunks deep into the context). mode:
 * LISA_PREFILL_SPLIT_AUTO (default), _NEVER, or _ALWAYS (every unit that can
 * be split, at 70 % of its keys, whatever the model says). Process-wide;
 * returns the previous mode, or LISA_EINVAL for an unknown mode. */
#define LISA_PREFILL_SPLIT_AUTO 0
#define LISA_PREFILL_SPLIT_NEVER 1
#define LISA_PREFILL_SPLIT_ALWAYS 2
int lisa_attn_debug_prefill_split(int mode);

/* Host only, no device work: the cluster segments the prefill planner gives a
 * chunk of `rows` rows at `base` on a device with num_sms SMs under `mode`, in
 * launch order: key tiles [seg_lo, seg_hi) of unit seg_unit (bits 0-7 head,
 * 8-11 query row pair, bit 12 set for a split unit). cap >= 96. Returns the
 * segment count, or LISA_EINVAL. */
int lisa_attn_debug_prefill_plan(uint32_t base, int rows, int num_sms, int mode, uint32_t* seg_lo,
                                 uint32_t* seg_hi, uint16_t* seg_unit, int cap);

/* ---- affine-u4 projections (QMV) --------------------------------------------
 * The quantised matrix-vector products around the attention layer for the
 * decode (rows = 1) and verify (rows = 3) shapes: q4_qmv_fast / fused2/3/4
 * (src/kernels/shaders/qmv.metal:1-133) as dispatched by encode_qmv_fused
 * (src/model/runner.rs:1134-1192). Weights are MLX affine 4-bit, group size
 * 64: packed [n][k/8] uint32 (element j in bits 4*(j%8) of word j/8), scales
 * and biases bf16 [n][k/64], w = q * scale + bias. x is bf16 [rows][k]; each
 * projection writes f32 out [rows][n]:
 *   out[m][r] = sum_j x[m][j] * (q[r][j] * scale[r][j/64] + bias[r][j/64]).
 * One launch serves up to LISA_ATTN_QMV_MAX_PROJ projections of the same x
 * (q_proj + k_proj + v_proj as fused3 does; their outputs are what
 * lisa_attn_decode takes as q_gate, k, v with LISA_DTYPE_F32). k must be a
 * multiple of 64 in 64..LISA_ATTN_QMV_MAX_K, x and packed 16-byte aligned,
 * and x must fit in shared memory beside two weight stages (rows x k up to
 * 4 x 6144 or 2 x 8192); LISA_EINVAL otherwise. */
#define LISA_ATTN_QMV_MAX_PROJ 4
#define LISA_ATTN_QMV_MAX_ROWS 4
#define LISA_ATTN_QMV_MAX_K 8192
typedef struct {
  const void* packed;     /* [n][k/8] uint32 */
  const uint16_t* scales; /* [n][k/64] bf16 */
  const uint16_t* biases; /* [n][k/64] bf16 */
  float* out;             /* [rows][n] f32 */
  int n;
} lisa_attn_q4_proj;
int lisa_attn_qmv_u4(int n_proj, const lisa_attn_q4_proj* projs, int rows, int k, const uint16_t* x, void* stream);

/* ---- Gated DeltaNet recurrence ---------------------------------------------
 * The state recurrence of the linear-attention layers (gdn_recurrence,
 * src/kernels/shaders/gdn.metal:245-330), head dim 128 for keys and values,
 * value heads sharing key heads in groups of `repeat` (48 value heads over 16
 * key heads in the model). For each of `steps` tokens t, value head h,
 * value column c, with s = ssm_state[h][c][0..127]:
 *   s *= decay[t][h]; delta = (v - s.k) * beta[t][h]; s += delta * k;
 *   y[t][h*128 + c] = bf16(s.q)  (stored as f32)
 * with k, q = k_norm, q_norm [t][kh*128 ..] (kh = h / repeat) and v =
 * conv_out[t][2*key_dim + h*128 + c] (conv_out rows are 2*key_dim + value_dim
 * floats). ssm_state f32 [value_heads][128][128] is updated in place. With
 * slot_stride > 0 the state after token t is also written to
 * state_slots + t * slot_stride (floats; >= value_heads*128*128). A call over
 * n tokens equals n one-token calls bit for bit. */
int lisa_attn_gdn_recurrence(int steps, int value_heads, int repeat, const float* conv_out, const float* q_norm,
                             const float* k_norm, const float* beta, const float* decay, float* ssm_state, float* y,
                             float* state_slots, size_t slot_stride, void* stream);

/* ---- safetensors shards (weights) ------------------------------------------
 * Host-side reader of the checkpoint container (src/format/safetensor.rs:
 * 1-91): [u64 LE header length][JSON header][tensor bytes], data_offsets
 * relative to the end of the header, top-level keys starting with "__"
 * skipped. The file is memory-mapped read-only. dtype codes follow the
 * reference's names (src/format/dtype.rs:17-31): LISA_ST_* below. Unlike the
 * reference (which panics), a malformed header, an unknown dtype, or a byte
 * range outside the file or not matching the shape gives LISA_EINVAL from
 * lisa_attn_st_open. lisa_attn_st_find returns the index or LISA_EINVAL.
 * lisa_attn_st_upload copies one tensor to device memory (synchronous on
 * `stream`). */
#define LISA_ST_BOOL 0
#define LISA_ST_U8 1
#define LISA_ST_U16 2
#define LISA_ST_I16 3
#define LISA_ST_F16 4
#define LISA_ST_BF16 5
#define LISA_ST_U32 6
#define LISA_ST_I32 7
#define LISA_ST_F32 8
#define LISA_ST_U64 9
#define LISA_ST_F64 10
typedef struct lisa_attn_shard lisa_attn_shard;
int lisa_attn_st_open(const char* path, lisa_attn_shard** out);
int lisa_attn_st_close(lisa_attn_shard* s);
int lisa_attn_st_count(const lisa_attn_shard* s);
int lisa_attn_st_find(const lisa_attn_shard* s, const char* name);
int lisa_attn_st_info(const lisa_attn_shard* s, int index, char* name, size_t name_bytes, int* dtype,
                      uint64_t* shape, int max_dims, int* ndim, uint64_t* data_offset, uint64_t* nbytes);
int lisa_attn_st_host_ptr(const lisa_attn_shard* s, int index, const void** ptr);
int lisa_attn_st_upload(const lisa_attn_shard* s, int index, void* dst, size_t dst_bytes, void* stream);

/* ---- device bridge ----------------------------------------------------------
 * Thin wrappers over the CUDA runtime so a host in another language drives the
 * entry points above with this library alone. They replace lisa-rs's Metal
 * bridge (src/device/metal.rs): MetalDevice::name / max_working_set (160-175)
 * -> lisa_attn_dev_info; new_buffer (176-199) and Drop (414-420) ->
 * lisa_attn_buffer_alloc / _free; new_command_queue (200-206) ->
 * lisa_attn_stream_create; commit + wait_until_completed (314-321) ->
 * lisa_attn_stream_synchronize; MetalBuffer::write_bytes / read_bytes
 * (396-410) -> lisa_attn_copy_h2d / _d2h (device memory is not CPU-visible
 * here, so these are stream-ordered copies; from pinned host memory they are
 * asynchronous). Events order work across streams and time it. A stream
 * argument of NULL is the legacy default stream. All return LISA_OK,
 * LISA_EINVAL (null pointer, bad device) or LISA_ECUDA. */
int lisa_attn_dev_count(int* count);
int lisa_attn_dev_info(int device, char* name, size_t name_bytes, uint64_t* total_bytes, int* sm_count);
int lisa_attn_dev_select(int device);
int lisa_attn_buffer_alloc(int device, size_t bytes, void** ptr);
int lisa_attn_buffer_free(void* ptr);
int lisa_attn_host_alloc(size_t bytes, void** ptr); /* page-locked host memory */
int lisa_attn_host_free(void* ptr);
int lisa_attn_stream_create(int device, void** stream);
int lisa_attn_stream_destroy(void* stream);
int lisa_attn_stream_synchronize(void* stream);
int lisa_attn_event_create(int device, int timing, void** event);
int lisa_attn_event_destroy(void* event);
int lisa_attn_event_record(void* event, void* stream);
int lisa_attn_stream_wait_event(void* stream, void* event);
int lisa_attn_event_synchronize(void* event);
int lisa_attn_event_elapsed_ms(void* start, void* end, float* ms);
int lisa_attn_copy_h2d(void* dst, const void* src, size_t bytes, void* stream);
int lisa_attn_copy_d2h(void* dst, const void* src, size_t bytes, void* stream);
int lisa_attn_copy_d2d(void* dst, const void* src, size_t bytes, void* stream);
int lisa_attn_memset(void* dst, int value, size_t bytes, void* stream);

/* Library build identification (for tests: the .so in use). */
const char* lisa_attn_build_info(void);

#ifdef __cplusplus
}
#endif
#endif /* LISA_ATTN_H */
