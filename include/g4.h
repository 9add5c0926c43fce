/*
 * g4.h -- C ABI of libgemma4_cuda.so, the sm_100a (B200) implementation of the quantized
 * decode/prefill hot path of the gemma4-webgpu-engine (Gemma-4-E2B).
 *
 * Every entry point is plain C: integers, floats, host pointers, device pointers and sizes. No
 * C++ or torch type crosses this line. Each declaration names the reference interface it
 * replaces as `path:line` inside the reference project (TypeScript + WGSL).
 *
 * Conventions (mirroring the reference, src/kernels/registry.ts:23-70 and src/runtime.ts:73-88):
 *   - Every call returns an int status: G4_OK (0) or a negative G4_ERR_* class. The message of
 *     the last failure on a context is g4_last_error(ctx); context-free calls (g4_op_*) report
 *     through g4_last_error(NULL), which is thread-local.
 *   - The context owns all device memory it allocates. Host pointers are borrowed for the call.
 *     Device pointers passed to g4_op_* stay owned by the caller.
 *   - One context per GPU; calls on one context are not re-entrant (the reference serialises its
 *     host side on one encode chain, src/runtime.ts:530-537). Different contexts may run on
 *     different threads or processes.
 *   - Arithmetic contract: calibrated linears accumulate int4/int8 weight codes times int8
 *     activation codes in exact int32 (src/kernels/qgemv.ts:1131-1176); every f32 operation is a
 *     single correctly rounded IEEE operation in a fixed order, so results do not depend on the
 *     batch width, the grid or the stream.
 */
#ifndef G4_H
#define G4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------ status */

#define G4_OK 0
#define G4_ERR_INVALID (-1)     /* bad argument: shape, id, position, null pointer */
#define G4_ERR_CUDA (-2)        /* a CUDA runtime call failed; the message names it */
#define G4_ERR_OOM (-3)         /* device allocation failed */
#define G4_ERR_STATE (-4)       /* call not valid in the current state (no weights, ...) */
#define G4_ERR_UNSUPPORTED (-5) /* a configuration this build does not implement */
#define G4_ERR_NOT_FOUND (-6)   /* unknown tensor or scalar name */
#define G4_ERR_TIMEOUT (-7)     /* a bounded device wait gave up and set the error flag */

typedef struct g4_ctx g4_ctx;

/*
 * Message of the last failure on `ctx`, or of the last context-free call on this thread when
 * `ctx` is NULL. Never NULL; "" when nothing failed. Replaces the thrown Error prose of the
 * reference (src/execute.ts:321-347, src/runtime.ts:415-445).
 */
const char *g4_last_error(const g4_ctx *ctx);

/* Library version string, e.g. "gemma4_cuda 0.1 sm_100a". */
const char *g4_version(void);

/* ------------------------------------------------------------------------ architecture */

/*
 * The architecture contract, GEMMA4_E2B in src/plan.ts:29-82 plus the per-site weight widths of
 * gemvBitsForSite (src/plan.ts:116-120). Global layers are a bit mask over layer indices.
 */
typedef struct g4_arch {
  int32_t layer_count;           /* 35 */
  int32_t hidden_size;           /* 1536 */
  int32_t query_heads;           /* 8 */
  int32_t kv_heads;              /* 1 (multi-query); the only supported value */
  int32_t sliding_head_dim;      /* 256 */
  int32_t global_head_dim;       /* 512 */
  uint64_t global_layer_mask;    /* bits 4, 9, 14, 19, 24, 29, 34 */
  int32_t sliding_window;        /* 512, inclusive of the query position */
  int32_t kv_producer_layers;    /* 15 */
  int32_t producer_intermediate; /* 6144 */
  int32_t consumer_intermediate; /* 6144 in the synthetic model (12288 in the checkpoint) */
  int32_t vocab_size;            /* 262144 */
  int32_t ple_dim;               /* 256 */
  int32_t attn_bits;             /* 4 */
  int32_t mlp_bits;              /* 4: the producer layers' MLP */
  int32_t ple_bits;              /* 8, the I8 PLE linears (src/quant.ts:610-620) */
  int32_t consumer_mlp_bits;     /* 4, or 2: the checkpoint's consumer MLP on the interleaved
                                    2-bit layout (src/plan.ts:116-122, src/quant.ts:598-609) */
  int32_t head_bits;             /* 4, or 2: the embedding and its tied lm_head (src/quant.ts:
                                    550-585; the 2-bit table is gathered from the tile layout) */
  int32_t head_calibrated;       /* 1: the head's SRQ scales are set (integer path); 0: both are
                                    0.0, the f32 path of the checkpoint's head (needs head_bits 2) */
  float rms_eps;                 /* 1e-6 */
  float final_softcap;           /* 30 */
  float rope_theta_sliding;      /* 1e4 */
  float rope_theta_global;       /* 1e6 */
  float partial_rotary_factor;   /* 0.25 */
} g4_arch;

/* Fill `arch` with the Gemma-4-E2B-shaped synthetic architecture of the benchmark configs. */
int g4_arch_default(g4_arch *arch);

/* The checkpoint's layout (google/gemma-4-E2B-it-qat-mobile, src/plan.ts:116-122): as the default
 * but consumer MLP 2-bit at width 12288, and a 2-bit uncalibrated embedding / lm_head. */
int g4_arch_checkpoint(g4_arch *arch);

/* --------------------------------------------------------------------------- context */

typedef struct g4_config {
  g4_arch arch;
  int32_t max_seqs;          /* sequence slots, each with its own KV region */
  int32_t max_context;       /* positions per sequence (kv.ts DEFAULT_MAX_CONTEXT is 2048) */
  int32_t max_step_columns;  /* widest step: a prefill chunk or a decode batch */
  int32_t use_graphs;        /* 1: record decode steps into CUDA graphs (default) */
  uint64_t ple_slice_bytes;  /* 0: PLE table is one buffer; else the vocab-row slice cap */
  int32_t gemm_min_columns;  /* steps this wide or wider run their linears on the tcgen05 int8
                                GEMM (prefill chunks, batched decode); 0: 16 */
  int32_t gemm_shadow_min_columns; /* steps at least this wide run their int4 / 2-bit linears on
                                int8 copies of the weights held beside the packed ones (the GEMM
                                then loads them by TMA with no unpack; same integer sums, about
                                1.3 GB more HBM at the full shape); 0: every tensor-core step;
                                negative: no copies */
  int32_t gemm_split_k;      /* K split of tensor-core launches with fewer tiles than SMs (all
                                bit-identical): 0 (default) over a thread-block cluster, partials
                                summed in distributed shared memory; 1 never; 2 through a global
                                int32 workspace, only for launches of few tiles and long K */
} g4_config;

/* Defaults: g4_arch_default, max_seqs 1, max_context 2048, max_step_columns 64, graphs on,
 * gemm_min_columns 16, gemm_shadow_min_columns 0 (every tensor-core step), gemm_split_k 0. */
int g4_config_default(g4_config *cfg);

/*
 * Create a context on CUDA device `cuda_device`. Allocates activations, KV caches (f32, K then V
 * per producer layer, src/kv.ts:116-148) and rope tables; weights are added afterwards by
 * g4_init_random or g4_upload_weight. Replaces GpuExecutor construction and
 * BufferManager/createKvLayout (src/runtime.ts:193-358, src/buffers.ts:203, src/kv.ts:116).
 */
int g4_ctx_create(int cuda_device, const g4_config *cfg, g4_ctx **out);
void g4_ctx_destroy(g4_ctx *ctx);

/* Bytes of device memory the context holds (weights + KV + activations). */
int g4_ctx_memory(const g4_ctx *ctx, uint64_t *weight_bytes, uint64_t *kv_bytes, uint64_t *other_bytes);

/* ---------------------------------------------------------------------------- weights */

/*
 * Build the seeded synthetic model on the device: int4 linears with f16 row scales, I8 PLE
 * linears, int4 embedding (tied lm_head) and PLE tables, bf16 per_layer_model_projection, f32
 * norm gains, layer scalars and static activation scales. The generator is a counter hash of
 * (seed, tensor, element), so any tensor can be regenerated on the host for checking.
 * Replaces Gemma4Mobile.load's weight stream (src/engine.ts:369-603, src/cache.ts:1057).
 */
int g4_init_random(g4_ctx *ctx, uint64_t seed);

/*
 * Upload bytes [offset, offset + n) of the tensor `name` (checkpoint naming, e.g.
 * "model.language_model.layers.0.self_attn.q_proj.weight"), whose full size is `total` bytes.
 * Mirrors BufferManager.uploadWeight (src/buffers.ts:369-486). Storage per family:
 *   *.weight (linear)           packed codes, row major, packed axis last (src/quant.ts:11-15)
 *   *.weight_scale              f16, one per output row
 *   *.embedding_quantized       int4 rows; *.embedding_scale f16 (embed) or f16 [rows, 35] (PLE)
 *   *norm*.weight               f32 (the reference widens bf16 at load, src/engine.ts:550-556)
 *   per_layer_model_projection  bf16, [8960, 1536] (src/quant.ts:396-398)
 */
int g4_upload_weight(g4_ctx *ctx, const char *name, const void *bytes, uint64_t offset,
                     uint64_t n, uint64_t total);

/* Copy a resident tensor back to the host (for checks). `*n` in: capacity, out: bytes. */
int g4_download_weight(g4_ctx *ctx, const char *name, void *bytes, uint64_t *n);

/*
 * Four-byte checkpoint scalars: `<module>.input_activation_scale`,
 * `<module>.output_activation_scale` and `layers.N.layer_scalar`. 0.0 means uncalibrated.
 * Mirrors the host scalars map (src/engine.ts:547-549, src/runtime.ts:63-70).
 */
int g4_set_scalar(g4_ctx *ctx, const char *name, float value);
int g4_get_scalar(const g4_ctx *ctx, const char *name, float *value);

/*
 * Split the PLE table into vocab-row slices of at most `slice_bytes`, one device buffer per
 * slice, rows aligned to 16 (planTableSplit, src/tableSplit.ts:125-215; declareSplit,
 * src/buffers.ts:291-326). Must precede weight creation. Reports the plan through the out
 * arguments (nullable).
 */
int g4_plan_table_split(uint64_t rows, uint64_t row_bytes, uint64_t limit_bytes,
                        uint64_t slice_bytes, int32_t *n_slices, int32_t *rows_per_slice,
                        int32_t *last_rows);

/* ---------------------------------------------------------------------------- forward */

/*
 * ForwardExecutor.prefill (src/runtime.ts:960-973): run `n` prompt tokens of sequence `seq` at
 * positions start_pos.., storing their KV. A chunk that is not the last runs the 15 KV producer
 * layers only (src/plan.ts:812-824); the last chunk runs all layers and the head and writes the
 * argmax of its final position to *out_token (-1 otherwise).
 */
int g4_prefill(g4_ctx *ctx, int32_t seq, const int32_t *ids, int32_t n, int32_t start_pos,
               int32_t is_last, int32_t *out_token);

/*
 * ForwardExecutor.decode (src/runtime.ts:975-983): one decode step of `seq` with prev_token at
 * `pos`; returns the greedy argmax in *out_token.
 */
int g4_decode(g4_ctx *ctx, int32_t seq, int32_t prev_token, int32_t pos, int32_t *out_token);

/*
 * ForwardExecutor.decodeAhead (src/runtime.ts:1016-1023): as g4_decode, but the input token is
 * the one the previous step of this context left on the device, so the host need not have read
 * it. `*out_token` receives this step's argmax.
 */
int g4_decode_ahead(g4_ctx *ctx, int32_t seq, int32_t pos, int32_t *out_token);

/*
 * GpuExecutor.verify (src/runtime.ts:993-1014), the verify pass of a speculative decode:
 * tokens[0] is the token the model chose last and tokens[1..n-1] a drafted continuation, placed
 * at positions pos..pos+n-1 of `seq`; out_tokens[i] receives the model's argmax after tokens[i].
 * Every column is computed with exactly the arithmetic of a one-token decode step (the
 * column-for-column contract of src/kernels/qgemvWide.ts:8-71), so out_tokens[i] is what
 * g4_decode would answer at pos + i given the same prefix. KV rows of all n positions are
 * written; the caller keeps the accepted prefix with g4_kv_truncate and the next pass overwrites
 * the rest. n is 1 to min(max_step_columns, max(max_seqs, G4_VERIFY_COLS)); the reference's wide
 * kernel caps it at GEMV_WIDE_COLS (2).
 */
#define G4_VERIFY_COLS 8
int g4_verify(g4_ctx *ctx, int32_t seq, const int32_t *tokens, int32_t n, int32_t pos,
              int32_t *out_tokens);

/*
 * Batched decode (new; the reference has no batch dimension): B independent sequences, one
 * column each, every column computed with exactly the arithmetic of a one-sequence step (the
 * column-for-column contract of src/kernels/qgemvWide.ts:8-71).
 */
int g4_decode_batch(g4_ctx *ctx, int32_t B, const int32_t *seqs, const int32_t *tokens,
                    const int32_t *positions, int32_t *out_tokens);

/*
 * Device-resident decode loop (no host copies per step). g4_step_stage copies B columns
 * (sequence, token, position) into the context's device step buffer once; each
 * g4_step_run_device then runs one decode step of those columns without waiting for the host.
 * With `advance` nonzero the step leaves its argmax token and position + 1 in the buffer, so
 * consecutive calls continue every sequence greedily (the decodeAhead chain of
 * src/runtime.ts:518-536, entirely on the device). g4_step_read_tokens waits and returns the
 * last step's tokens.
 */
int g4_step_stage(g4_ctx *ctx, int32_t B, const int32_t *seqs, const int32_t *tokens,
                  const int32_t *positions);
int g4_step_run_device(g4_ctx *ctx, int32_t B, int32_t advance);
int g4_step_read_tokens(g4_ctx *ctx, int32_t B, int32_t *out_tokens);

/* KvCacheState.truncate (src/kv.ts:247-254): host bookkeeping of the valid length of `seq`. */
int g4_kv_truncate(g4_ctx *ctx, int32_t seq, int32_t n);
int g4_kv_length(const g4_ctx *ctx, int32_t seq, int32_t *n);

/*
 * Diagnostics of the last step: the softcapped logits of column `col` (`n` floats, n <= vocab)
 * and its top-2 (value, index) pairs. Mirrors lastLogits (src/engine.ts:820-878).
 */
int g4_read_logits(g4_ctx *ctx, int32_t col, float *out, int32_t n);

/*
 * The PLE code table's layout in this context: the number of vocab-row slices (1 when the table
 * is one buffer), the rows of every slice but the last, and the last slice's rows. The slices a
 * BufferManager.declareSplit would register (src/buffers.ts:291-326).
 */
int g4_ctx_ple_slices(const g4_ctx *ctx, int32_t *n_slices, int32_t *rows_per_slice,
                      int32_t *last_rows);

/* Device stream the context launches on (a cudaStream_t), for callers that time on it. */
void *g4_ctx_stream(g4_ctx *ctx);

/* Launch count of the last forward call, as recorded by the executor. */
int g4_last_launches(const g4_ctx *ctx, int32_t *launches);

/*
 * The launches of the last forward call, one "kernel<TAB>roles" line each in launch order: the
 * kernel family (qgemv-4bit, attention-decode, qgemm-8bit, ...) and the reference modules or roles
 * it covers (e.g. "layers.3.self_attn.q_proj,layers.3.self_attn.k_proj,layers.3.self_attn.v_proj").
 * The executor's compiled plan, for comparison with planDecodeStep's dispatch list (src/plan.ts:
 * 487-859, src/engine.ts:919-922). `*needed` receives the bytes including the terminating NUL;
 * buf may be NULL to ask for that size.
 */
int g4_last_launch_list(const g4_ctx *ctx, char *buf, uint64_t cap, uint64_t *needed);

/* ------------------------------------------------------------------ per-operator calls */
/*
 * The operator API (the registry's Kernel.bind, src/kernels/registry.ts:108-119), one entry per
 * kernel family, on caller-owned device pointers and a caller stream (NULL = default stream).
 * They launch the same kernels the executor records into its graphs.
 */

/*
 * Quantized linear, `cols` activation columns (qgemv-4bit / qgemv-8bit / qgemm-4bit, and the
 * M-wide family: src/kernels/qgemv.ts:413-690, 1131-1176; src/kernels/qgemm.ts:532-552;
 * src/kernels/qgemvWide.ts:452; qgemv-2bit, src/kernels/qgemv.ts:693-868). wq: packed weights
 * [N, K*bits/8] bytes, or at 2 bits the interleaved tile layout [ceil(N/16), K] u32
 * (g4_op_repack_tile16); scales: f16 [N]; x: f32 [cols, K]; y: f32 [cols, N]; acc_out: int32
 * [cols, N] or NULL (the exact integer accumulators on a calibrated site). bits is 2, 4 or 8; K a
 * multiple of 512 (2-bit), 256 (4-bit) or 128 (8-bit) (src/kernels/qgemv.ts:1258, 1305-1310).
 * in_scale 0 selects the f32 path (one column at 4 and 8 bits, K <= 3072 at 2 bits).
 */
int g4_op_qgemv(const void *wq, const void *scales, const float *x, float in_scale,
                float out_scale, int32_t bits, int32_t N, int32_t K, int32_t cols, float *y,
                int32_t *acc_out, void *stream);

/*
 * The same linear on int8 activation codes (the wNa8o8 form of BASELINE config 1: the column
 * already snapped, x = codes * in_scale): codes int8 [cols, K] in K order, in_scale != 0. The
 * accumulators and outputs equal g4_op_qgemv's on x = codes * in_scale; the prologue only loads
 * the codes (no snap).
 */
int g4_op_qgemv_codes(const void *wq, const void *scales, const int8_t *codes, float in_scale,
                      float out_scale, int32_t bits, int32_t N, int32_t K, int32_t cols, float *y,
                      int32_t *acc_out, void *stream);

/*
 * The 2-bit family's layout change (src/kernels/repack.ts:17-209, src/kernels/qlayout.ts:186-227):
 * to_rows 0 repacks the checkpoint's rows (row r: K / 16 u32 words, code k at bits 2 (k % 16) of
 * word k / 16) into the interleaved tiles (word k of tile t holds row 16 t + i at bits 2 i, rows
 * past N zero); to_rows 1 is the inverse. K a multiple of 16. Device pointers.
 */
int g4_op_repack_tile16(const void *row_words, void *tile_words, int32_t N, int32_t K,
                        int32_t to_rows, void *stream);

/*
 * The prefill / batched form (qgemm-4bit, src/kernels/qgemm.ts:76-110, 490-552, 565-636: every
 * column is exactly the qgemv of that column) on the tensor cores: the columns are snapped to
 * int8 codes once, then a tcgen05 int8 GEMM accumulates exact int32 in tensor memory. Same
 * arguments and results as g4_op_qgemv on a calibrated site (in_scale != 0); K a multiple of
 * 128 (and of 256 for 4-bit). Allocates its code scratch stream-ordered (cudaMallocAsync).
 */
int g4_op_qgemm(const void *wq, const void *scales, const float *x, float in_scale,
                float out_scale, int32_t bits, int32_t N, int32_t K, int32_t cols, float *y,
                void *stream);

/* The fused gelu prologue build (qgemv-Nbit-gelu, src/kernels/qgemv.ts:371-400): the GEMV over
 * gelu_tanh(gate) * up[up_offset..], snapped by in_scale. gate/up: f32 [cols, K]. */
int g4_op_qgemv_gelu(const void *wq, const void *scales, const float *gate, const float *up,
                     int32_t up_offset, int32_t up_stride, float in_scale, float out_scale,
                     int32_t bits, int32_t N, int32_t K, int32_t cols, float *y, void *stream);

/* rms-norm / rms-norm-weightless (src/kernels/rmsNorm.ts:131-208): gain NULL = weightless. */
int g4_op_rms_norm(const float *src, const float *gain, float *dst, int32_t rows,
                   int32_t width, float eps, void *stream);

/* norm-residual (src/kernels/mlpEpilogue.ts:109-220): dst = residual + norm(src) * gain. */
int g4_op_norm_residual(const float *src, const float *gain, const float *residual,
                        float *dst, int32_t rows, int32_t width, float eps, void *stream);

/* norm-residual-norm (src/kernels/blockJoin.ts:73-160): hidden = alpha * (residual +
 * norm(src) * gain); dst = norm(hidden) * gain2. */
int g4_op_norm_residual_norm(const float *src, const float *gain, const float *residual,
                             const float *gain2, float alpha, float *hidden, float *dst,
                             int32_t rows, int32_t width, float eps, void *stream);

/* gelu-mul with the SRQ snap (src/kernels/geluMul.ts:101-240). */
int g4_op_gelu_mul(const float *gate, const float *up, float *dst, int32_t n, float srq_scale,
                   void *stream);

/* q-norm-rope (src/kernels/attnPrologue.ts:83-170): rows (position, head) of `width`;
 * cos/sin tables [positions, width/2]; rows_per_position rows share one table row. */
int g4_op_q_norm_rope(const float *src, const float *gain, const float *cos_tab,
                      const float *sin_tab, float *dst, int32_t rows, int32_t width,
                      int32_t rows_per_position, float eps, void *stream);

/* kv-norm-rope-store (src/kernels/attnPrologue.ts:172-260): k, v [tokens, head_dim] into the
 * packed cache [2, max_context, head_dim] at start_pos. */
int g4_op_kv_norm_rope_store(const float *k, const float *v, const float *gain,
                             const float *cos_tab, const float *sin_tab, float *cache,
                             int32_t tokens, int32_t head_dim, int32_t start_pos,
                             int32_t max_context, float eps, void *stream);

/* attention-decode / attention-prefill (src/kernels/attention.ts:339-752, oracle 858-903):
 * q [q_count, heads, head_dim]; cache packed K then V [2, max_context, head_dim]; window 0 =
 * global. Scale 1.0 (src/kernels/attention.ts:81). */
int g4_op_attention(const float *q, const float *cache, float *out, int32_t heads,
                    int32_t head_dim, int32_t q_count, int32_t q_start, int32_t kv_len,
                    int32_t window, int32_t max_context, void *stream);

/* The prefill form of the same attention (src/kernels/attention.ts:339-752 with q_count > 1): the
 * queries are the consecutive positions q_start .. q_start + q_count - 1 of one sequence, tiled
 * so each KV block is read once per query tile. Same arguments and bit-identical results as
 * g4_op_attention; allocates nothing. */
int g4_op_attention_prefill(const float *q, const float *cache, float *out, int32_t heads,
                            int32_t head_dim, int32_t q_count, int32_t q_start, int32_t kv_len,
                            int32_t window, int32_t max_context, void *stream);

/* embed-gather (int4 rows here) and ple-gather-4bit(-sliced) (src/kernels/embedGather.ts:
 * 176-261, 319-344, 547-577). codes: row-major int4; scales f16 [rows, groups]; ids int32
 * [slots]; dst f32 [slots, cols]. A sliced call writes only the slots whose id lies in
 * [slice_start, slice_start + slice_rows) and reads codes relative to slice_start. */
int g4_op_embed_gather(const void *codes, const void *scales, const int32_t *ids, float *dst,
                       int32_t slots, int32_t cols, int32_t group_size, float out_scale,
                       int32_t slice_start, int32_t slice_rows, void *stream);

/* dense-bf16-matmul (src/kernels/denseMatmul.ts:93-222): y[c, r] = alpha * dot(w[r], x[c]). */
int g4_op_dense_bf16(const void *w, const float *x, float *y, int32_t N, int32_t K,
                     int32_t cols, float alpha, void *stream);

/* logit-softcap then the two-stage argmax (src/kernels/logitSoftcap.ts:54-120,
 * src/kernels/argmax.ts:43-310): capped may be NULL; token receives (index, value bits). */
int g4_op_softcap_argmax(const float *logits, float *capped, int32_t *token, int32_t n,
                         float cap, void *stream);

/*
 * g4_op_attention without any device allocation. No counterpart in the reference: the WebGPU
 * engine has no allocator-free path. It exists for callers that cannot allocate device memory
 * (a host that has handed all memory to its own pools, a server that must not block on or fail
 * in the allocator once running, an embedding whose allocator belongs to someone else). Same
 * arguments and results as g4_op_attention; the per-block scratch is a fixed 4 MiB file-scope
 * device array (1,048,576 floats; needed: q_count * blocks * heads * (head_dim + 2), blocks =
 * window ? ceil(window / 64) + 1 : ceil(kv_len / 64)) that each device loading the library keeps until
 * the process exits. Larger requests return G4_ERR_INVALID. q, cache, out (and the stream, when
 * not NULL) must belong to one device; the call makes that device current for its duration and
 * restores the caller's current device before it returns. The first call on a device looks up
 * the array's device address with that device current; make that first call before any stream
 * capture (a lookup that fails is not remembered: the next call tries again). Calls share the
 * array: two calls that overlap on the GPU (different streams, or different host threads) race
 * on it and must be serialised by the caller.
 */
int g4_op_attention_noalloc(const float *q, const float *cache, float *out, int32_t heads,
                            int32_t head_dim, int32_t q_count, int32_t q_start, int32_t kv_len,
                            int32_t window, int32_t max_context, void *stream);

/*
 * Failure detection without a fault (no counterpart in the reference, whose lost-device handling
 * is src/engine.ts:791-798). A one-thread kernel copies `bytes` (16..4096, a multiple of 16) from
 * `src` (16-byte aligned device memory) into shared memory through a bulk copy, and arms a second
 * mbarrier for `missing_bytes` that no copy delivers. With missing_bytes > 0 its bounded wait gives
 * up after `poll_limit` polls, raises the device error flag every library kernel raises when a
 * wait gives up, waits for its own copy and exits; the call then returns G4_ERR_TIMEOUT and the
 * device stays usable. status (device, 3 int32): [second wait completed, copy landed, byte sum].
 * Synchronises `stream`.
 */
int g4_op_wait_probe(const void *src, int32_t bytes, int32_t missing_bytes, int32_t poll_limit,
                     int32_t *status, void *stream);

/*
 * Out-of-memory injection for tests: with nth > 0, the nth device allocation a context makes from
 * now on (g4_ctx_create's arena, tables, caches and activations) fails as cudaMalloc does when
 * the device is out of memory; 0 disarms. The failing call returns G4_ERR_OOM, names the
 * allocation in g4_last_error and releases what it had allocated.
 */
int g4_debug_fail_allocation(int32_t nth);

/*
 * Error-path injection for tests: sets the sticky error flag that one unit of the library's
 * kernels raises when a bounded device wait gives up (0 streaming GEMV and attention, 1 2-bit
 * GEMV, 2 tensor-core GEMM, 3 per-layer-input tail), as if such a wait had run out, without any
 * kernel failing. The next call that returns tokens (g4_decode, g4_decode_batch, g4_verify,
 * g4_prefill with is_last) then returns G4_ERR_TIMEOUT and clears it, as a real timeout does.
 */
int g4_debug_raise_error_flag(g4_ctx *ctx, int32_t unit);

/* Elementwise probes of the library's f32 exp and tanh (used by the attention softmax, GELU
 * and the softcap), for checking them against CUDA's expf/tanhf within error bounds. */
int g4_op_math_probe(const float *x, float *exp_out, float *tanh_out, float *cuda_exp,
                     float *cuda_tanh, int32_t n, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* G4_H */
