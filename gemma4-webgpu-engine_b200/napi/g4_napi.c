/*
 * g4_napi.c -- the Node-API addon a TypeScript host binds (gemma4_cuda.node): every entry point
 * the reference's ForwardExecutor seam needs (src/runtime.ts:73-88: prefill, decode, decodeAhead,
 * verify), the weight and scalar paths of BufferManager / the scalars map (src/buffers.ts:369-377,
 * src/engine.ts:547-549), and the batch, rewind and logits calls, each a thin wrapper over one
 * C-ABI call of include/g4.h. Failures throw a JavaScript Error whose code is "G4_ERR_<class>"
 * and whose message is g4_last_error's prose, as the reference throws Errors naming the kernel and
 * role (src/execute.ts:321-347).
 *
 * The calls are synchronous; a host that must not block its JavaScript thread runs them on a
 * worker (or wraps them in napi_create_async_work), keeping one context's calls serialised as the
 * reference serialises its encode chain (src/runtime.ts:530-537).
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef G4_HAVE_NODE_API_H
#include <node_api.h>
#else
#include "node_api_min.h"
#endif

#include "../../include/g4.h"

/* The context behind a JavaScript external; ctx is cleared by destroyContext so the finalizer
 * does not destroy it twice. */
typedef struct {
  g4_ctx *ctx;
} G4Handle;

static napi_value g4_throw(napi_env env, const g4_ctx *ctx, int rc) {
  static const char *names[] = {"G4_OK", "G4_ERR_INVALID", "G4_ERR_CUDA", "G4_ERR_OOM",
                                "G4_ERR_STATE", "G4_ERR_UNSUPPORTED", "G4_ERR_NOT_FOUND",
                                "G4_ERR_TIMEOUT"};
  const char *code = (rc <= 0 && rc >= -7) ? names[-rc] : "G4_ERR";
  napi_throw_error(env, code, g4_last_error(ctx));
  return NULL;
}

static napi_value g4_throw_arg(napi_env env, const char *msg) {
  napi_throw_error(env, "G4_ERR_INVALID", msg);
  return NULL;
}

static napi_value undefined_value(napi_env env) {
  napi_value u = NULL;
  napi_get_undefined(env, &u);
  return u;
}

static napi_value int_value(napi_env env, int32_t v) {
  napi_value r = NULL;
  napi_create_int32(env, v, &r);
  return r;
}

static napi_value int_array(napi_env env, const int32_t *v, size_t n) {
  napi_value arr = NULL;
  if (napi_create_array_with_length(env, n, &arr) != napi_ok) return NULL;
  for (size_t i = 0; i < n; i++) napi_set_element(env, arr, (uint32_t)i, int_value(env, v[i]));
  return arr;
}

/* Arguments: at least `need` of them. */
static int get_args(napi_env env, napi_callback_info info, size_t need, napi_value *argv, size_t cap) {
  size_t argc = cap;
  if (napi_get_cb_info(env, info, &argc, argv, NULL, NULL) != napi_ok) return 0;
  for (size_t i = argc; i < cap; i++) argv[i] = NULL;
  return argc >= need;
}

static g4_ctx *ctx_of(napi_env env, napi_value v) {
  G4Handle *h = NULL;
  if (!v || napi_get_value_external(env, v, (void **)&h) != napi_ok || !h) return NULL;
  return h->ctx;
}

static int i32_of(napi_env env, napi_value v, int32_t *out) {
  return v && napi_get_value_int32(env, v, out) == napi_ok;
}

/* A typed array of the given kind: its data and element count. */
static int typed_of(napi_env env, napi_value v, napi_typedarray_type want, void **data, size_t *n) {
  napi_typedarray_type t;
  napi_value ab;
  size_t off;
  if (!v || napi_get_typedarray_info(env, v, &t, n, data, &ab, &off) != napi_ok) return 0;
  return t == want;
}

static int str_of(napi_env env, napi_value v, char *buf, size_t cap) {
  size_t len = 0;
  return v && napi_get_value_string_utf8(env, v, buf, cap, &len) == napi_ok && len + 1 < cap;
}

/* Optional numeric option `name` of object `obj` into *dst (unchanged when absent). */
static void opt_num(napi_env env, napi_value obj, const char *name, double *dst) {
  bool has = false;
  napi_value v;
  if (!obj || napi_has_named_property(env, obj, name, &has) != napi_ok || !has) return;
  if (napi_get_named_property(env, obj, name, &v) == napi_ok) napi_get_value_double(env, v, dst);
}

static void opt_i32(napi_env env, napi_value obj, const char *name, int32_t *dst) {
  double d = *dst;
  opt_num(env, obj, name, &d);
  *dst = (int32_t)d;
}

static void ctx_finalize(napi_env env, void *data, void *hint) {
  (void)env;
  (void)hint;
  G4Handle *h = (G4Handle *)data;
  if (h && h->ctx) g4_ctx_destroy(h->ctx);
  free(h);
}

/*
 * createContext(device, options?) -> External. Options (all optional, numbers or booleans):
 * maxSeqs, maxContext, maxStepColumns, pleSliceBytes, useGraphs, gemmMinColumns,
 * gemmShadowMinColumns, gemmSplitK; checkpoint (the checkpoint's 2-bit families,
 * g4_arch_checkpoint); arch overrides layerCount, hiddenSize, globalLayerMask, slidingWindow,
 * kvProducerLayers, producerIntermediate, consumerIntermediate, vocabSize, consumerMlpBits,
 * headBits, headCalibrated. Replaces GpuExecutor construction (src/runtime.ts:193-358).
 */
static napi_value create_context(napi_env env, napi_callback_info info) {
  napi_value argv[2];
  if (!get_args(env, info, 1, argv, 2)) return g4_throw_arg(env, "createContext(device, options?)");
  int32_t device = 0;
  if (!i32_of(env, argv[0], &device)) return g4_throw_arg(env, "createContext: device must be a number");
  g4_config cfg;
  g4_config_default(&cfg);
  napi_value o = argv[1];
  double ckpt = 0;
  opt_num(env, o, "checkpoint", &ckpt);
  if (ckpt != 0) g4_arch_checkpoint(&cfg.arch);
  double graphs = cfg.use_graphs, slice = (double)cfg.ple_slice_bytes, mask = (double)cfg.arch.global_layer_mask;
  opt_i32(env, o, "maxSeqs", &cfg.max_seqs);
  opt_i32(env, o, "maxContext", &cfg.max_context);
  opt_i32(env, o, "maxStepColumns", &cfg.max_step_columns);
  opt_num(env, o, "pleSliceBytes", &slice);
  opt_num(env, o, "useGraphs", &graphs);
  opt_i32(env, o, "gemmMinColumns", &cfg.gemm_min_columns);
  opt_i32(env, o, "gemmShadowMinColumns", &cfg.gemm_shadow_min_columns);
  opt_i32(env, o, "gemmSplitK", &cfg.gemm_split_k);
  opt_i32(env, o, "layerCount", &cfg.arch.layer_count);
  opt_i32(env, o, "hiddenSize", &cfg.arch.hidden_size);
  opt_num(env, o, "globalLayerMask", &mask);
  opt_i32(env, o, "slidingWindow", &cfg.arch.sliding_window);
  opt_i32(env, o, "kvProducerLayers", &cfg.arch.kv_producer_layers);
  opt_i32(env, o, "producerIntermediate", &cfg.arch.producer_intermediate);
  opt_i32(env, o, "consumerIntermediate", &cfg.arch.consumer_intermediate);
  opt_i32(env, o, "vocabSize", &cfg.arch.vocab_size);
  opt_i32(env, o, "consumerMlpBits", &cfg.arch.consumer_mlp_bits);
  opt_i32(env, o, "headBits", &cfg.arch.head_bits);
  opt_i32(env, o, "headCalibrated", &cfg.arch.head_calibrated);
  cfg.use_graphs = graphs != 0;
  cfg.ple_slice_bytes = slice > 0 ? (uint64_t)slice : 0;
  cfg.arch.global_layer_mask = mask > 0 ? (uint64_t)mask : 0;
  g4_ctx *ctx = NULL;
  int rc = g4_ctx_create(device, &cfg, &ctx);
  if (rc) return g4_throw(env, NULL, rc);
  G4Handle *h = (G4Handle *)calloc(1, sizeof(G4Handle));
  h->ctx = ctx;
  napi_value ext;
  if (napi_create_external(env, h, ctx_finalize, NULL, &ext) != napi_ok) {
    g4_ctx_destroy(ctx);
    free(h);
    return g4_throw_arg(env, "createContext: cannot wrap the context");
  }
  return ext;
}

/* destroyContext(ctx): BufferManager.dispose (src/buffers.ts:761-780). */
static napi_value destroy_context(napi_env env, napi_callback_info info) {
  napi_value argv[1];
  G4Handle *h = NULL;
  if (!get_args(env, info, 1, argv, 1) || napi_get_value_external(env, argv[0], (void **)&h) != napi_ok || !h)
    return g4_throw_arg(env, "destroyContext(ctx)");
  if (h->ctx) g4_ctx_destroy(h->ctx);
  h->ctx = NULL;
  return undefined_value(env);
}

/* initRandom(ctx, seed): the seeded synthetic model in place of a checkpoint download. */
static napi_value init_random(napi_env env, napi_callback_info info) {
  napi_value argv[2];
  double seed = 0;
  g4_ctx *ctx;
  if (!get_args(env, info, 2, argv, 2) || !(ctx = ctx_of(env, argv[0])) ||
      napi_get_value_double(env, argv[1], &seed) != napi_ok || seed < 0 || seed > 9007199254740992.0)
    return g4_throw_arg(env, "initRandom(ctx, seed: a non-negative integer below 2^53)");
  int rc = g4_init_random(ctx, (uint64_t)seed);
  return rc ? g4_throw(env, ctx, rc) : undefined_value(env);
}

/* uploadWeight(ctx, name, bytes: Uint8Array, offset, total): BufferManager.uploadWeight pieces. */
static napi_value upload_weight(napi_env env, napi_callback_info info) {
  napi_value argv[5];
  g4_ctx *ctx;
  char name[512];
  void *data;
  size_t n;
  double offset = 0, total = 0;
  if (!get_args(env, info, 5, argv, 5) || !(ctx = ctx_of(env, argv[0])) || !str_of(env, argv[1], name, sizeof name) ||
      !typed_of(env, argv[2], napi_uint8_array, &data, &n) || napi_get_value_double(env, argv[3], &offset) != napi_ok ||
      napi_get_value_double(env, argv[4], &total) != napi_ok || offset < 0 || total < 0)
    return g4_throw_arg(env, "uploadWeight(ctx, name, bytes: Uint8Array, offset, total)");
  int rc = g4_upload_weight(ctx, name, data, (uint64_t)offset, (uint64_t)n, (uint64_t)total);
  return rc ? g4_throw(env, ctx, rc) : undefined_value(env);
}

/* setScalar(ctx, name, value): the scalars map (src/engine.ts:547-549). */
static napi_value set_scalar(napi_env env, napi_callback_info info) {
  napi_value argv[3];
  g4_ctx *ctx;
  char name[512];
  double v = 0;
  if (!get_args(env, info, 3, argv, 3) || !(ctx = ctx_of(env, argv[0])) || !str_of(env, argv[1], name, sizeof name) ||
      napi_get_value_double(env, argv[2], &v) != napi_ok)
    return g4_throw_arg(env, "setScalar(ctx, name, value)");
  int rc = g4_set_scalar(ctx, name, (float)v);
  return rc ? g4_throw(env, ctx, rc) : undefined_value(env);
}

/* prefill(ctx, seq, ids: Int32Array, startPosition, isLast) -> token (-1 unless isLast). */
static napi_value prefill(napi_env env, napi_callback_info info) {
  napi_value argv[5];
  g4_ctx *ctx;
  int32_t seq, start;
  bool last = false;
  void *ids;
  size_t n;
  if (!get_args(env, info, 5, argv, 5) || !(ctx = ctx_of(env, argv[0])) || !i32_of(env, argv[1], &seq) ||
      !typed_of(env, argv[2], napi_int32_array, &ids, &n) || !i32_of(env, argv[3], &start) ||
      napi_get_value_bool(env, argv[4], &last) != napi_ok)
    return g4_throw_arg(env, "prefill(ctx, seq, ids: Int32Array, startPosition, isLast: boolean)");
  int32_t tok = -1;
  int rc = g4_prefill(ctx, seq, (const int32_t *)ids, (int32_t)n, start, last ? 1 : 0, &tok);
  return rc ? g4_throw(env, ctx, rc) : int_value(env, tok);
}

/* decode(ctx, seq, prevToken, position) -> token. */
static napi_value decode(napi_env env, napi_callback_info info) {
  napi_value argv[4];
  g4_ctx *ctx;
  int32_t seq, prev, pos;
  if (!get_args(env, info, 4, argv, 4) || !(ctx = ctx_of(env, argv[0])) || !i32_of(env, argv[1], &seq) ||
      !i32_of(env, argv[2], &prev) || !i32_of(env, argv[3], &pos))
    return g4_throw_arg(env, "decode(ctx, seq, prevToken, position)");
  int32_t tok = -1;
  int rc = g4_decode(ctx, seq, prev, pos, &tok);
  return rc ? g4_throw(env, ctx, rc) : int_value(env, tok);
}

/* decodeAhead(ctx, seq, position) -> token (input: the token the previous step left). */
static napi_value decode_ahead(napi_env env, napi_callback_info info) {
  napi_value argv[3];
  g4_ctx *ctx;
  int32_t seq, pos;
  if (!get_args(env, info, 3, argv, 3) || !(ctx = ctx_of(env, argv[0])) || !i32_of(env, argv[1], &seq) ||
      !i32_of(env, argv[2], &pos))
    return g4_throw_arg(env, "decodeAhead(ctx, seq, position)");
  int32_t tok = -1;
  int rc = g4_decode_ahead(ctx, seq, pos, &tok);
  return rc ? g4_throw(env, ctx, rc) : int_value(env, tok);
}

/* verify(ctx, seq, tokens: Int32Array, position) -> number[] (GpuExecutor.verify). */
static napi_value verify(napi_env env, napi_callback_info info) {
  napi_value argv[4];
  g4_ctx *ctx;
  int32_t seq, pos;
  void *toks;
  size_t n;
  if (!get_args(env, info, 4, argv, 4) || !(ctx = ctx_of(env, argv[0])) || !i32_of(env, argv[1], &seq) ||
      !typed_of(env, argv[2], napi_int32_array, &toks, &n) || !i32_of(env, argv[3], &pos) || n == 0 || n > 4096)
    return g4_throw_arg(env, "verify(ctx, seq, tokens: Int32Array (1 or more), position)");
  int32_t out[4096];
  int rc = g4_verify(ctx, seq, (const int32_t *)toks, (int32_t)n, pos, out);
  return rc ? g4_throw(env, ctx, rc) : int_array(env, out, n);
}

/* decodeBatch(ctx, seqs, tokens, positions: Int32Array) -> number[]. */
static napi_value decode_batch(napi_env env, napi_callback_info info) {
  napi_value argv[4];
  g4_ctx *ctx;
  void *s, *t, *p;
  size_t ns, nt, np;
  if (!get_args(env, info, 4, argv, 4) || !(ctx = ctx_of(env, argv[0])) ||
      !typed_of(env, argv[1], napi_int32_array, &s, &ns) || !typed_of(env, argv[2], napi_int32_array, &t, &nt) ||
      !typed_of(env, argv[3], napi_int32_array, &p, &np) || ns != nt || ns != np || ns == 0)
    return g4_throw_arg(env, "decodeBatch(ctx, seqs, tokens, positions: Int32Arrays of one length)");
  int32_t *out = (int32_t *)calloc(ns, sizeof(int32_t));
  int rc = g4_decode_batch(ctx, (int32_t)ns, (const int32_t *)s, (const int32_t *)t, (const int32_t *)p, out);
  napi_value r = rc ? g4_throw(env, ctx, rc) : int_array(env, out, ns);
  free(out);
  return r;
}

/* kvTruncate(ctx, seq, n): KvCacheState.truncate (src/kv.ts:247-254). */
static napi_value kv_truncate(napi_env env, napi_callback_info info) {
  napi_value argv[3];
  g4_ctx *ctx;
  int32_t seq, n;
  if (!get_args(env, info, 3, argv, 3) || !(ctx = ctx_of(env, argv[0])) || !i32_of(env, argv[1], &seq) ||
      !i32_of(env, argv[2], &n))
    return g4_throw_arg(env, "kvTruncate(ctx, seq, n)");
  int rc = g4_kv_truncate(ctx, seq, n);
  return rc ? g4_throw(env, ctx, rc) : undefined_value(env);
}

/* readLogits(ctx, column, out: Float32Array): lastLogits (src/engine.ts:820-878). */
static napi_value read_logits(napi_env env, napi_callback_info info) {
  napi_value argv[3];
  g4_ctx *ctx;
  int32_t col;
  void *out;
  size_t n;
  if (!get_args(env, info, 3, argv, 3) || !(ctx = ctx_of(env, argv[0])) || !i32_of(env, argv[1], &col) ||
      !typed_of(env, argv[2], napi_float32_array, &out, &n))
    return g4_throw_arg(env, "readLogits(ctx, column, out: Float32Array)");
  int rc = g4_read_logits(ctx, col, (float *)out, (int32_t)n);
  return rc ? g4_throw(env, ctx, rc) : undefined_value(env);
}

/* version() -> string. */
static napi_value version(napi_env env, napi_callback_info info) {
  (void)info;
  napi_value s = NULL;
  napi_create_string_utf8(env, g4_version(), NAPI_AUTO_LENGTH, &s);
  return s;
}

napi_value napi_register_module_v1(napi_env env, napi_value exports) {
  static const struct {
    const char *name;
    napi_callback fn;
  } fns[] = {{"createContext", create_context}, {"destroyContext", destroy_context},
             {"initRandom", init_random},       {"uploadWeight", upload_weight},
             {"setScalar", set_scalar},         {"prefill", prefill},
             {"decode", decode},                {"decodeAhead", decode_ahead},
             {"verify", verify},                {"decodeBatch", decode_batch},
             {"kvTruncate", kv_truncate},       {"readLogits", read_logits},
             {"version", version}};
  for (size_t i = 0; i < sizeof fns / sizeof fns[0]; i++) {
    napi_value f;
    if (napi_create_function(env, fns[i].name, NAPI_AUTO_LENGTH, fns[i].fn, NULL, &f) != napi_ok ||
        napi_set_named_property(env, exports, fns[i].name, f) != napi_ok)
      return NULL;
  }
  return exports;
}
