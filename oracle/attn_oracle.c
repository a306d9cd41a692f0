/*
 * attn_oracle.c — TEST INFRASTRUCTURE ONLY: the CPU parity checker and the
 * timed CPU baseline for the gated-GQA attention path. Plain C, f32
 * arithmetic, no fast-math. Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load it; the product path never does.
 *
 * Every function restates the reference shader it names
 * (lisa-rs src/kernels/shaders/attention.metal) in scalar C. Two deliberate,
 * documented choices:
 *   - RoPE angles use the reference's f32 product position * inv_freq
 *     (attention.metal:147); inv_freq and cos/sin are evaluated in double and
 *     rounded to f32 (the Metal build uses fast-math approximations, which no
 *     CPU or CUDA build can reproduce; the CUDA kernels use the same rule).
 *   - RMS uses 1/sqrtf where the shader calls rsqrt.
 */
#include "attn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QH 24
#define KVH 4
#define HD 256
#define ROT_PAIRS 32
#define QROW (QH * 512)
#define KROW (KVH * HD)
#define OROW (QH * HD)
#define SLICE 64
static const float LOG2E = 1.4426950408889634f;

float orc_bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t orc_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

uint16_t orc_f32_to_bf16_trunc(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return (uint16_t)(u >> 16);
}

static inline float rbf(float f) { return orc_bf16_to_f32(orc_f32_to_bf16(f)); }

float orc_rope_inv_freq(int pair) { return (float)(1.0 / pow(1.0e7, (double)(2 * pair) / 64.0)); }

/* One head: bf16-round the 256 raw values, RMS-normalise against the gain,
 * rotate pairs (j, j+32) for j < 32 at `pos`, round to bf16.
 * attention.metal:33-60 (rms_norm_rope) and 136-154 (the decode form). */
static void norm_rope_head(const float* src, const uint16_t* w, float eps, uint32_t pos, uint16_t* dst) {
  float x[HD], n[HD];
  float s = 0.0f;
  for (int j = 0; j < HD; j++) {
    x[j] = rbf(src[j]);
    s += x[j] * x[j];
  }
  const float inv = 1.0f / sqrtf(s / 256.0f + eps);
  for (int j = 0; j < HD; j++) n[j] = x[j] * inv * orc_bf16_to_f32(w[j]);
  for (int j = 0; j < ROT_PAIRS; j++) {
    const float angle = (float)pos * orc_rope_inv_freq(j);
    const float c = (float)cos((double)angle), sn = (float)sin((double)angle);
    dst[j] = orc_f32_to_bf16(n[j] * c - n[j + ROT_PAIRS] * sn);
    dst[j + ROT_PAIRS] = orc_f32_to_bf16(n[j + ROT_PAIRS] * c + n[j] * sn);
  }
  for (int j = 2 * ROT_PAIRS; j < HD; j++) dst[j] = orc_f32_to_bf16(n[j]);
}

void orc_q_prologue(const float* q_gate, int rows, uint32_t base, const uint16_t* q_norm_w, float eps,
                    uint16_t* query, float* gate) {
  for (int r = 0; r < rows; r++)
    for (int h = 0; h < QH; h++) {
      const float* src = q_gate + (size_t)r * QROW + h * 512;
      norm_rope_head(src, q_norm_w, eps, base + (uint32_t)r, query + (size_t)r * OROW + h * HD);
      for (int j = 0; j < HD; j++) gate[(size_t)r * OROW + h * HD + j] = rbf(src[HD + j]);
    }
}

void orc_kv_append(const float* k, const float* v, int rows, uint32_t base, const uint16_t* k_norm_w,
                   float eps, uint16_t* k_cache, uint16_t* v_cache, uint32_t capacity) {
  for (int r = 0; r < rows; r++) {
    const uint32_t pos = base + (uint32_t)r;
    if (pos >= capacity) continue; /* attention.metal:172 */
    for (int h = 0; h < KVH; h++) {
      const size_t in = (size_t)r * KROW + h * HD;
      const size_t out = ((size_t)h * capacity + pos) * HD;
      norm_rope_head(k + in, k_norm_w, eps, pos, k_cache + out);
      for (int j = 0; j < HD; j++) v_cache[out + j] = orc_f32_to_bf16(v[in + j]);
    }
  }
}

/* Online softmax over tokens [t0, t1) of one (row, head): the per-token loop of
 * attention.metal:577-594 (and 218-235). Returns the unnormalised accumulator
 * plus {denominator, max}. */
static void online_span(const uint16_t* qv, const uint16_t* kc, const uint16_t* vc, uint32_t t0,
                        uint32_t t1, float* acc, float* den_out, float* max_out) {
  float q[HD];
  for (int d = 0; d < HD; d++) q[d] = orc_bf16_to_f32(qv[d]);
  for (int d = 0; d < HD; d++) acc[d] = 0.0f;
  float m = -INFINITY, den = 0.0f;
  for (uint32_t t = t0; t < t1; t++) {
    const uint16_t* kr = kc + (size_t)t * HD;
    const uint16_t* vr = vc + (size_t)t * HD;
    float dot = 0.0f;
    for (int d = 0; d < HD; d++) dot += q[d] * orc_bf16_to_f32(kr[d]);
    const float score = dot * 0.0625f;
    const float next = score > m ? score : m;
    const float old_scale = exp2f(LOG2E * (m - next));
    const float new_scale = exp2f(LOG2E * (score - next));
    den = den * old_scale + new_scale;
    for (int d = 0; d < HD; d++) acc[d] = acc[d] * old_scale + new_scale * orc_bf16_to_f32(vr[d]);
    m = next;
  }
  *den_out = den;
  *max_out = m;
}

void orc_sdpa_serial(const uint16_t* query, const uint16_t* k_cache, const uint16_t* v_cache,
                     uint32_t capacity, uint32_t base, int rows, float* out) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int rh = 0; rh < rows * QH; rh++) {
    const int r = rh / QH, h = rh % QH, kvh = h / (QH / KVH);
    const uint32_t ctx = base + (uint32_t)r + 1u;
    float* o = out + (size_t)r * OROW + h * HD;
    if (ctx > capacity) { /* attention.metal:328: the reference leaves it unwritten */
      for (int d = 0; d < HD; d++) o[d] = 0.0f;
      continue;
    }
    float acc[HD], den, m;
    online_span(query + (size_t)r * OROW + h * HD, k_cache + (size_t)kvh * capacity * HD,
                v_cache + (size_t)kvh * capacity * HD, 0, ctx, acc, &den, &m);
    const float inv = 1.0f / den;
    for (int d = 0; d < HD; d++) o[d] = acc[d] * inv;
  }
}

void orc_sdpa_sliced(const uint16_t* query, const uint16_t* k_cache, const uint16_t* v_cache,
                     uint32_t capacity, uint32_t base, int rows, float* out) {
  const uint32_t max_ctx = base + (uint32_t)rows;
  const uint32_t slices = (max_ctx + SLICE - 1) / SLICE;
  float* part = (float*)malloc((size_t)rows * QH * slices * HD * sizeof(float));
  float* stat = (float*)malloc((size_t)rows * QH * slices * 2 * sizeof(float));
  const long total = (long)rows * QH * slices;
  /* sdpa_decode_partial (attention.metal:550-604) */
#pragma omp parallel for schedule(dynamic, 4)
  for (long i = 0; i < total; i++) {
    const int s = (int)(i % slices), rh = (int)(i / slices);
    const int r = rh / QH, h = rh % QH, kvh = h / (QH / KVH);
    const uint32_t ctx = base + (uint32_t)r + 1u;
    const uint32_t t0 = (uint32_t)s * SLICE;
    if (ctx > capacity || t0 >= ctx) continue; /* inactive slice: never merged */
    const uint32_t t1 = t0 + SLICE < ctx ? t0 + SLICE : ctx;
    online_span(query + (size_t)r * OROW + h * HD, k_cache + (size_t)kvh * capacity * HD,
                v_cache + (size_t)kvh * capacity * HD, t0, t1, part + (size_t)i * HD,
                &stat[(size_t)i * 2], &stat[(size_t)i * 2 + 1]);
  }
  /* sdpa_decode_final (attention.metal:611-641) */
#pragma omp parallel for schedule(static)
  for (int rh = 0; rh < rows * QH; rh++) {
    const int r = rh / QH, h = rh % QH;
    const uint32_t ctx = base + (uint32_t)r + 1u;
    float* o = out + (size_t)r * OROW + h * HD;
    if (ctx > capacity) {
      for (int d = 0; d < HD; d++) o[d] = 0.0f;
      continue;
    }
    const uint32_t used = (ctx + SLICE - 1) / SLICE;
    const size_t st = (size_t)rh * slices;
    float gmax = -INFINITY;
    for (uint32_t s = 0; s < used; s++) gmax = fmaxf(gmax, stat[(st + s) * 2 + 1]);
    for (int d = 0; d < HD; d++) {
      float total_den = 0.0f, res = 0.0f;
      for (uint32_t s = 0; s < used; s++) {
        const float w = exp2f(LOG2E * (stat[(st + s) * 2 + 1] - gmax));
        total_den += w * stat[(st + s) * 2];
        res += w * part[(st + s) * HD + d];
      }
      o[d] = res / total_den;
    }
  }
  free(part);
  free(stat);
}

void orc_gate(const float* out, const float* gate, int n, uint16_t* gated) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; i++) {
    const float sg = 1.0f / (1.0f + exp2f(-LOG2E * gate[i]));
    gated[i] = orc_f32_to_bf16(out[i] * sg);
  }
}

void orc_attention_layer(const float* q_gate, const float* k, const float* v, int rows, uint32_t base,
                         const uint16_t* q_norm_w, const uint16_t* k_norm_w, float eps,
                         uint16_t* k_cache, uint16_t* v_cache, uint32_t capacity, int sliced,
                         uint16_t* gated) {
  uint16_t* query = (uint16_t*)malloc((size_t)rows * OROW * sizeof(uint16_t));
  float* gate = (float*)malloc((size_t)rows * OROW * sizeof(float));
  float* out = (float*)malloc((size_t)rows * OROW * sizeof(float));
  orc_q_prologue(q_gate, rows, base, q_norm_w, eps, query, gate);
  orc_kv_append(k, v, rows, base, k_norm_w, eps, k_cache, v_cache, capacity);
  if (sliced)
    orc_sdpa_sliced(query, k_cache, v_cache, capacity, base, rows, out);
  else
    orc_sdpa_serial(query, k_cache, v_cache, capacity, base, rows, out);
  orc_gate(out, gate, rows * OROW, gated);
  free(query);
  free(gate);
  free(out);
}

void orc_legacy_batch(const float* q, const float* k, const float* v, int L, const uint16_t* q_norm_w,
                      const uint16_t* k_norm_w, float eps, float* out) {
  uint16_t* qn = (uint16_t*)malloc((size_t)L * OROW * sizeof(uint16_t));
  uint16_t* kn = (uint16_t*)malloc((size_t)L * KROW * sizeof(uint16_t));
  /* qk_norm_gate_rope / k_norm_rope: position = row (attention.metal:64-94) */
  for (int r = 0; r < L; r++) {
    for (int h = 0; h < QH; h++)
      norm_rope_head(q + (size_t)r * QROW + h * 512, q_norm_w, eps, (uint32_t)r, qn + (size_t)r * OROW + h * HD);
    for (int h = 0; h < KVH; h++)
      norm_rope_head(k + (size_t)r * KROW + h * HD, k_norm_w, eps, (uint32_t)r, kn + (size_t)r * KROW + h * HD);
  }
  /* sdpa_scalar (attention.metal:485-517): two-pass softmax, v rounded to bf16 */
  for (int r = 0; r < L; r++)
    for (int h = 0; h < QH; h++) {
      const int kvh = h / (QH / KVH);
      float sc[4096];
      float mx = -1e30f;
      for (int i = 0; i <= r; i++) {
        float acc = 0.0f;
        for (int d = 0; d < HD; d++)
          acc += orc_bf16_to_f32(qn[(size_t)r * OROW + h * HD + d]) * orc_bf16_to_f32(kn[(size_t)i * KROW + kvh * HD + d]);
        sc[i] = acc * 0.0625f;
        if (sc[i] > mx) mx = sc[i];
      }
      float sum = 0.0f;
      for (int i = 0; i <= r; i++) {
        sc[i] = exp2f(LOG2E * (sc[i] - mx));
        sum += sc[i];
      }
      const float iz = 1.0f / sum;
      for (int d = 0; d < HD; d++) {
        float acc = 0.0f;
        for (int i = 0; i <= r; i++) acc += sc[i] * rbf(v[(size_t)i * KROW + kvh * HD + d]);
        out[(size_t)r * OROW + h * HD + d] = acc * iz;
      }
    }
  free(qn);
  free(kn);
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
