/*
 * g4_oracle.h -- CPU restatement of the gemma4-webgpu-engine decode/prefill arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker and the timed CPU baseline. Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arms load it. The
 * product (libgemma4_cuda.so) never links, loads or calls it.
 *
 * Parity pinning: the reference is TypeScript + WGSL and cannot execute here (no JavaScript
 * runtime, no WebGPU). The restatement is pinned to the literal known answers in the
 * reference's source (tests/golden/reference_constants.json, extracted by
 * tests/golden/make_golden.py) and to golden vectors from a second, independent line-by-line
 * Python transliteration of the reference's own CPU oracles (tests/golden/ref_restate.py). The
 * reference's real-checkpoint fixtures are absent from its snapshot, so parity against them is
 * unpinned.
 *
 * Two kinds of function live here:
 *   g4o_ref_*   restate the reference's CPU oracles as written (f64 accumulation where the
 *               reference accumulates in f64), each citing its file:line;
 *   everything else is the exact f32 evaluation order the CUDA kernels use, which is one valid
 *   f32 evaluation of the same reference arithmetic (fixed reduction trees, single correctly
 *   rounded operations). The full forward uses these, so greedy tokens can be compared bit for
 *   bit.
 */
#ifndef G4_ORACLE_H
#define G4_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- scalar arithmetic */
float g4o_exp(float x);
float g4o_tanh(float x);
float g4o_gelu(float x);
int g4o_srq_code(float x, float s);
float g4o_srq_out(float v, float s);
uint16_t g4o_f32_to_f16(float f);
float g4o_f16_to_f32(uint16_t h);
uint16_t g4o_f32_to_bf16(float f);
float g4o_bf16_to_f32(uint16_t h);
uint64_t g4o_hash(uint64_t seed, uint64_t stream, uint64_t i);

/* ------------------------------------------------------------------ per-kernel calls */
/* Calibrated (in_scale != 0) or f32-path linear over `cols` columns. wq row-major packed
 * (bits 4: 2 codes per byte, low nibble first, zero point 8; bits 8: signed bytes). */
void g4o_qgemv(const uint8_t *wq, const uint16_t *scales_f16, const float *x, float in_scale,
               float out_scale, int bits, int N, int K, int cols, float *y, int32_t *acc);
void g4o_gelu_mul(const float *gate, const float *up, float *dst, int n, float srq_scale);
float g4o_rms_inv(const float *v, int n, float eps);
void g4o_rms_norm(const float *src, const float *gain, float *dst, int rows, int width, float eps);
void g4o_norm_residual(const float *src, const float *gain, const float *residual, float *dst,
                       int rows, int width, float eps);
void g4o_norm_residual_norm(const float *src, const float *gain, const float *residual,
                            const float *gain2, float alpha, float *hidden, float *dst,
                            int rows, int width, float eps);
void g4o_rope_tables(int head_dim, int rotary_pairs, double theta, int pos0, int npos,
                     float *cos_tab, float *sin_tab);
void g4o_q_norm_rope(const float *src, const float *gain, const float *cos_tab,
                     const float *sin_tab, float *dst, int rows, int width, int rows_per_pos,
                     float eps);
void g4o_kv_norm_rope_store(const float *k, const float *v, const float *gain,
                            const float *cos_tab, const float *sin_tab, float *cache,
                            int tokens, int head_dim, int start_pos, int max_context, float eps);
void g4o_attention(const float *q, const float *cache, float *out, int heads, int head_dim,
                   int q_count, int q_start, int kv_len, int window, int max_context);
void g4o_embed_gather(const uint8_t *codes, const uint16_t *scales_f16, const int32_t *ids,
                      float *dst, int slots, int cols, int group_size, float out_scale,
                      int slice_start, int slice_rows);
void g4o_dense_bf16(const uint16_t *w, const float *x, float *y, int N, int K, int cols,
                    float alpha);
void g4o_softcap_argmax(const float *logits, float *capped, int32_t *token, int n, float cap);

/* Reference restatements (f64 accumulators as in the TypeScript oracles). */
void g4o_ref_rms_norm(const float *src, const float *gain, float *dst, int rows, int width,
                      float eps);
void g4o_ref_norm_residual(const float *src, const float *gain, const float *residual,
                           float *dst, int rows, int width, float eps);
void g4o_ref_attention(const float *q, const float *k, const float *v, float *out, int heads,
                       int head_dim, int q_count, int q_start, int kv_len, int window,
                       double scale);
void g4o_ref_gelu_mul(const float *gate, const float *up, float *dst, int n, float srq_scale);
void g4o_ref_dense(const float *w, const float *x, float *y, int N, int K, int cols, float alpha);

/* ------------------------------------------------------------------ table split */
int g4o_plan_table_split(uint64_t rows, uint64_t row_bytes, uint64_t limit_bytes,
                         uint64_t slice_bytes, int32_t *n_slices, int32_t *rows_per_slice,
                         int32_t *last_rows);

/* -------------------------------------------------------------------- the model */
typedef struct g4o_arch {
  int32_t layer_count, hidden, q_heads, sliding_hd, global_hd;
  uint64_t global_mask;
  int32_t window, producers, ffn, vocab, ple_dim;
  float eps, softcap, theta_sliding, theta_global, partial_rotary;
  /* The checkpoint's families (src/plan.ts:116-122, src/quant.ts:574-609): consumer layers' MLP
   * width and bits (2: the interleaved 2-bit family), the embedding / tied head bits, and whether
   * the head is calibrated (0: both activation scales 0.0, the f32 path). */
  int32_t consumer_ffn, consumer_mlp_bits, head_bits, head_calibrated;
} g4o_arch;

void g4o_arch_default(g4o_arch *a);

typedef struct g4o_model g4o_model;

/* Generate the seeded synthetic model (the same generator spec the CUDA library implements).
 * Element values do not depend on how the device splits the PLE table. */
g4o_model *g4o_model_synth(const g4o_arch *a, uint64_t seed);
void g4o_model_free(g4o_model *m);
/* Named tensor access (checkpoint names), for checking a device copy. */
const void *g4o_model_tensor(const g4o_model *m, const char *name, uint64_t *bytes);
float g4o_model_scalar(const g4o_model *m, const char *name);

typedef struct g4o_seq g4o_seq;
g4o_seq *g4o_seq_new(const g4o_model *m, int32_t max_context);
void g4o_seq_free(g4o_seq *s);

/*
 * Run `n` tokens at positions start_pos.. through the model. all_layers = 0 runs the producer
 * layers only (the KV-sharing exit of a non-last prefill chunk). When want_head, the head runs
 * on the last position: *token gets the argmax, logits (nullable, vocab floats) the capped
 * logits, top2 (nullable) {v1, i1, v2, i2}.
 */
int g4o_forward(const g4o_model *m, g4o_seq *s, const int32_t *ids, int32_t n, int32_t start_pos,
                int32_t all_layers, int32_t want_head, int32_t *token, float *logits, float *top2);

/* Greedy generation: prompt (prefill = producer-only chunk for positions 0..n-2, then the last
 * position through all layers), then max_new - 1 decode steps. Writes max_new tokens and, per
 * token, the top-2 gap of the capped logits. */
int g4o_generate(const g4o_model *m, const int32_t *prompt, int32_t n_prompt, int32_t max_new,
                 int32_t max_context, int32_t *tokens, float *gaps);

/* Synthetic prompt ids (uniform over the vocabulary from the seed). */
void g4o_synth_prompt(uint64_t seed, int32_t n, int32_t vocab, int32_t *ids);

/* Calibration statistics of the last forward: max |x| per site kind (in, out). */
void g4o_site_stats(float *max_in, float *max_out, int32_t n_sites);
void g4o_threads(int32_t n);

#ifdef __cplusplus
}
#endif
#endif
