// g4_runtime.cu -- context, weights, executor and C ABI of libgemma4_cuda.so.
//
// The executor replaces src/execute.ts (resolveStep), src/runtime.ts (GpuExecutor encode and
// submit), src/buffers.ts (slot and weight buffers), src/kv.ts (cache layout) and
// src/tableSplit.ts (PLE vocab-row slices). Steps are recorded once per (columns, layer range,
// head) into CUDA graphs instead of being re-encoded per token (src/runtime.ts:702-770).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/g4.h"
#include "g4_device.cuh"
#include "g4_kernels.cuh"
#include "g4_gemv.cuh"

using namespace g4;

// ================================================================================ errors

static thread_local std::string tl_error;

struct Linear {
  uint8_t *w = nullptr;
  uint16_t *s = nullptr;
  int N = 0, K = 0, bits = 4;
  float in_scale = 0, out_scale = 0;
  std::string module;
  CUtensorMap tmw;          // TMA view of w for the tensor-core path (has_tm)
  bool has_tm = false;
  // Signed int8 copy [N][K] of int4 / 2-bit codes for wide tensor-core steps (no unpack), and its
  // 128-byte-swizzled TMA view.
  int8_t *w8 = nullptr;
  CUtensorMap tmw8;
  bool has_tm8 = false;
};

// The tensor map the tensor-core linear loads weights through: int4 packed rows (box 64 bytes x
// 128 rows, unpacked on chip), 2-bit tiles, or int8 rows (box 128 x 128, 128-byte swizzle).
// Needs K % 128 == 0.
static void linear_tmap(Linear &l) {
  l.has_tm = false;
  if (!l.w || l.K % 128 != 0) return;
  if (l.bits == 2) {
    // 2-bit tiles: u32 words [tiles][K], box 128 words x 8 tiles (128 rows), unpacked on chip.
    l.has_tm = make_tmap_u32(&l.tmw, l.w, (uint64_t)l.K, (uint64_t)((l.N + 15) / 16),
                             (uint64_t)l.K * 4, 128, 8) == 0;
    return;
  }
  if (l.bits != 4 && l.bits != 8) return;
  const uint64_t rb = (uint64_t)l.K * l.bits / 8;
  l.has_tm = make_tmap_u8(&l.tmw, l.w, rb, (uint64_t)l.N, rb, l.bits == 4 ? 64 : 128, 128, l.bits == 8) == 0;
}

struct Layer {
  int hd = 256;
  bool global = false, producer = false;
  int cache_layer = 0;
  Linear q, k, v, o, gate, up, down, pleg, plep;
  float *ln_in, *ln_post_attn, *ln_pre_ffn, *ln_post_ffn, *ln_post_ple, *q_norm, *k_norm;
  float layer_scalar = 1.0f;
};

struct TensorRef {
  void *ptr;
  uint64_t bytes;       // the checkpoint layout's bytes (what upload and download move)
  bool sliced;          // the PLE code table split into vocab-row slices
  int t16_rows = 0;     // > 0: a 2-bit tensor held in the interleaved tile layout (rows x t16_k)
  int t16_k = 0;
};

struct GraphKey {
  int cols, layers, head, advance;
  bool operator<(const GraphKey &o) const {
    return std::tie(cols, layers, head, advance) < std::tie(o.cols, o.layers, o.head, o.advance);
  }
};

struct g4_ctx {
  int dev = 0;
  cudaStream_t st = nullptr;
  g4_config cfg;
  std::string err;
  int H = 0, V = 0, PD = 0, NL = 0, ple_cols = 0, ffn = 0, maxc = 0, head_cols = 0;
  // weights
  void *arena = nullptr;
  size_t arena_bytes = 0, arena_used = 0;
  std::vector<void *> ple_slices;
  uint8_t **d_ple_slices = nullptr;
  int ple_rps = 0;
  uint64_t ple_slice_bytes = 0;
  std::vector<Layer> layers;
  uint8_t *embed_w = nullptr;
  uint16_t *embed_s = nullptr, *ple_s = nullptr, *plmp_w = nullptr;
  float *plmp_norm = nullptr, *final_norm = nullptr;
  Linear lm;
  std::map<std::string, TensorRef> tensors;
  bool weights_ready = false;
  // KV caches, per producer layer [max_seqs][2][max_ctx][hd]
  std::vector<float *> kv;
  std::vector<size_t> kv_stride;
  std::vector<int32_t> kv_len;
  uint64_t kv_bytes = 0;
  // rope tables [max_ctx][pairs]
  float *cos_s = nullptr, *sin_s = nullptr, *cos_g = nullptr, *sin_g = nullptr;
  // activations
  float *res[2] = {nullptr, nullptr};
  float *ple_id, *ple_proj, *ple_in, *q, *k, *v, *qr, *attn, *proj, *gate, *up, *pleg_out;
  float *part_o, *part_m, *part_l;
  int att_blocks_sliding = 0, att_blocks_global = 0;
  int32_t *att_count = nullptr;     // finished attention blocks per column (decode steps)
  // Tensor-core path: activation codes (three input scales at most per launch group), their
  // TMA views by (buffer, K, tile columns), lm_head argmax partials, and the column threshold.
  uint8_t *gq[3] = {nullptr, nullptr, nullptr};
  int gq_ld = 0, gq_rows = 0;
  std::map<std::tuple<int, int, int>, CUtensorMap> tmx;
  float *gpv = nullptr;
  int32_t *gpi = nullptr;
  int32_t *gacc = nullptr, *gcnt = nullptr;   // split-K workspace [maxc][gacc_ld] and tile counts
  int gacc_ld = 0;
  int gemm_split_k = 0;   // g4_config::gemm_split_k
  bool gemm_persist = false;
  // int8 weight copies: steps of at least shadow_min_cols columns run their int4 / 2-bit linears
  // on them; refreshed from the packed weights before the next forward after any weight change.
  uint8_t *shadow = nullptr;
  size_t shadow_bytes = 0;
  int shadow_min_cols = 0;
  bool shadow_dirty = false;
  // Token tile of steps wider than 128 columns: 128 columns at two CTAs per SM (-128), measured
  // 10% faster on a 2048-token prefill than 256-column tiles at one CTA per SM.
  int gemm_wide_bn = -128;
  int gparts = 0, gemm_min_cols = 16;
  // The argmax partials the head of the step being recorded wrote.
  float *cur_pv = nullptr;
  int32_t *cur_pi = nullptr;
  int cur_parts = 0;
  uint8_t *codes_mlp = nullptr;     // down_proj input codes [maxc][ffn_max]
  uint8_t *codes_ple = nullptr;     // per_layer_projection input codes [maxc][PD]
  uint8_t *codes_attn = nullptr;    // o_proj input codes written by attention [maxc][heads * hd]
  int ple_block = -1;               // the fused per-layer-input tail fits this device (-1: not asked)
  int ffn_max = 0;
  float *logits = nullptr;
  float *head_pv = nullptr;
  int32_t *head_pi = nullptr;
  int head_blocks = 0;   // CTAs of the last recorded GEMV head launch
  int head_cap = 0;      // argmax partials allocated per head column
  int gemv_target = 0;   // CTAs a GEMV launch is partitioned for (two per SM)
  int32_t *d_step = nullptr;   // [3][maxc]: seq, pos, token
  int32_t *d_tok_out = nullptr;
  float *d_val_out = nullptr;
  // Pinned staging ring: slot i is reused only after the copy that read it has executed.
  static constexpr int kStageSlots = 4;
  int32_t *h_step[kStageSlots] = {nullptr, nullptr, nullptr, nullptr};
  cudaEvent_t stage_ev[kStageSlots] = {nullptr, nullptr, nullptr, nullptr};
  int stage_next = 0;
  int32_t *h_tok = nullptr;    // pinned token outputs, then the step's error word
  ErrFlags errf = {};          // the kernels' sticky error flags, by device address
  uint64_t other_bytes = 0;
  std::map<GraphKey, cudaGraphExec_t> graphs;
  // 2-bit tensors being uploaded in pieces: the checkpoint bytes so far, repacked when complete.
  std::map<std::string, std::vector<uint8_t>> t16_staging;
  std::map<std::string, uint64_t> t16_received;
  std::map<GraphKey, int> graph_launches;   // kernels in each graph
  std::map<GraphKey, std::vector<std::string>> graph_roles;
  int sms = 148;
  int launches = 0;
  // One "kernel<TAB>role" line per launch of the last forward call, in launch order.
  std::vector<std::string> roles;
  int last_cols = 0;
  int staged_cols = 0;
  std::vector<int32_t> staged_seq, staged_pos;
  int prologue_graphs = 0;
};

static int fail(g4_ctx *c, int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  tl_error = buf;
  return code;
}

#define CK(call)                                                                          \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess)                                                                \
      return fail(ctx, e_ == cudaErrorMemoryAllocation ? G4_ERR_OOM : G4_ERR_CUDA,        \
                  "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
  } while (0)

// For the other translation units of the library: record a context-free error message.
void g4_internal_set_error(const char *msg) { tl_error = msg; }

// Out-of-memory injection for tests: armed with n > 0, the n-th device allocation a context makes
// from then on fails as cudaMalloc does when the device is out of memory.
static std::atomic<int> g_fail_alloc{0};

static cudaError_t ctx_malloc(void **p, size_t bytes) {
  int n = g_fail_alloc.load(std::memory_order_relaxed);
  while (n > 0 && !g_fail_alloc.compare_exchange_weak(n, n - 1)) {
  }
  if (n == 1) {
    *p = nullptr;
    return cudaErrorMemoryAllocation;
  }
  return cudaMalloc(p, bytes);
}

// Record one launch of the step being built: its kernel family and the reference roles it covers
// (module names without the model.language_model. prefix, or the fused step's role).
static void note_launch(g4_ctx *ctx, const std::string &kernel, const std::string &role) {
  ctx->launches++;
  ctx->roles.push_back(kernel + "\t" + role);
}

static std::string short_module(const std::string &m) {
  static const std::string pre = "model.language_model.";
  return m.compare(0, pre.size(), pre) == 0 ? m.substr(pre.size()) : m;
}

extern "C" const char *g4_last_error(const g4_ctx *ctx) {
  return ctx ? ctx->err.c_str() : tl_error.c_str();
}

extern "C" const char *g4_version(void) { return "gemma4_cuda 0.1 sm_100a"; }

// ========================================================================== configuration

extern "C" int g4_arch_default(g4_arch *a) {
  if (!a) return fail(nullptr, G4_ERR_INVALID, "g4_arch_default: null arch");
  memset(a, 0, sizeof(*a));
  a->layer_count = 35;
  a->hidden_size = 1536;
  a->query_heads = 8;
  a->kv_heads = 1;
  a->sliding_head_dim = 256;
  a->global_head_dim = 512;
  a->global_layer_mask = (1ull << 4) | (1ull << 9) | (1ull << 14) | (1ull << 19) | (1ull << 24) |
                         (1ull << 29) | (1ull << 34);
  a->sliding_window = 512;
  a->kv_producer_layers = 15;
  a->producer_intermediate = 6144;
  a->consumer_intermediate = 6144;
  a->vocab_size = 262144;
  a->ple_dim = 256;
  a->attn_bits = 4;
  a->mlp_bits = 4;
  a->ple_bits = 8;
  a->consumer_mlp_bits = 4;
  a->head_bits = 4;
  a->head_calibrated = 1;
  a->rms_eps = 1e-6f;
  a->final_softcap = 30.0f;
  a->rope_theta_sliding = 1e4f;
  a->rope_theta_global = 1e6f;
  a->partial_rotary_factor = 0.25f;
  return G4_OK;
}

extern "C" int g4_arch_checkpoint(g4_arch *a) {
  int rc = g4_arch_default(a);
  if (rc) return rc;
  a->consumer_intermediate = 12288;
  a->consumer_mlp_bits = 2;
  a->head_bits = 2;
  a->head_calibrated = 0;
  return G4_OK;
}

extern "C" int g4_config_default(g4_config *cfg) {
  if (!cfg) return fail(nullptr, G4_ERR_INVALID, "g4_config_default: null config");
  memset(cfg, 0, sizeof(*cfg));
  g4_arch_default(&cfg->arch);
  cfg->max_seqs = 1;
  cfg->max_context = 2048;
  cfg->max_step_columns = 64;
  cfg->use_graphs = 1;
  cfg->ple_slice_bytes = 0;
  cfg->gemm_min_columns = 16;
  cfg->gemm_split_k = 0;
  cfg->gemm_shadow_min_columns = 0;
  return G4_OK;
}

// planTableSplit (src/tableSplit.ts:125-215).
extern "C" int g4_plan_table_split(uint64_t rows, uint64_t row_bytes, uint64_t limit_bytes,
                                   uint64_t slice_bytes, int32_t *n_slices,
                                   int32_t *rows_per_slice, int32_t *last_rows) {
  if (row_bytes == 0) return fail(nullptr, G4_ERR_INVALID, "plan_table_split: row_bytes 0");
  uint64_t total = rows * row_bytes;
  bool fits = total > 0 && total <= limit_bytes;
  uint64_t cap = slice_bytes < limit_bytes ? slice_bytes : limit_bytes;
  if (cap < 1) cap = 1;
  uint64_t per = (fits ? limit_bytes : cap) / row_bytes;
  if (per < 1)
    return fail(nullptr, G4_ERR_INVALID, "plan_table_split: one row of %llu bytes exceeds the cap",
                (unsigned long long)row_bytes);
  uint64_t aligned = per >= 16 ? per - (per % 16) : per;
  uint64_t ps = rows < aligned ? rows : aligned;
  uint64_t n = ps ? (rows + ps - 1) / ps : 1;
  if (n == 0) n = 1;
  if (n_slices) *n_slices = (int32_t)n;
  if (rows_per_slice) *rows_per_slice = (int32_t)ps;
  if (last_rows) *last_rows = (int32_t)(rows - (n - 1) * ps);
  return G4_OK;
}

static bool is_global(const g4_arch &a, int L) { return (a.global_layer_mask >> L) & 1ull; }

// =============================================================================== context

static void *arena_take(g4_ctx *c, size_t bytes) {
  size_t off = (c->arena_used + 255) & ~(size_t)255;
  if (off + bytes > c->arena_bytes) return nullptr;
  c->arena_used = off + bytes;
  return (uint8_t *)c->arena + off;
}

static const char *LMP = "model.language_model.";

static std::string layer_name(int L, const char *suffix) {
  return std::string(LMP) + "layers." + std::to_string(L) + "." + suffix;
}

// Device bytes of a linear's codes: row-major packed, or the interleaved tiles at 2 bits.
static size_t linear_bytes(size_t N, size_t K, int bits) {
  return bits == 2 ? tile16_bytes((int)N, (int)K) : N * K * bits / 8;
}

static int make_linear(g4_ctx *ctx, Linear &lin, const std::string &module, int N, int K, int bits) {
  lin.N = N;
  lin.K = K;
  lin.bits = bits;
  lin.module = module;
  lin.w = (uint8_t *)arena_take(ctx, linear_bytes(N, K, bits));
  lin.s = (uint16_t *)arena_take(ctx, (size_t)N * 2);
  if (!lin.w || !lin.s) return fail(ctx, G4_ERR_OOM, "weight arena exhausted at %s", module.c_str());
  TensorRef tr{lin.w, (uint64_t)N * K * bits / 8, false};
  if (bits == 2) {
    tr.t16_rows = N;
    tr.t16_k = K;
  }
  ctx->tensors[module + ".weight"] = tr;
  ctx->tensors[module + ".weight_scale"] = {lin.s, (uint64_t)N * 2, false};
  return G4_OK;
}

static float *make_f32(g4_ctx *ctx, const std::string &name, size_t n) {
  float *p = (float *)arena_take(ctx, n * 4);
  if (p) ctx->tensors[name] = {p, n * 4, false};
  return p;
}

static size_t weight_arena_bytes(const g4_arch &a) {
  size_t H = a.hidden_size, total = 0;
  auto lin = [&](size_t N, size_t K, int bits) { total += ((linear_bytes(N, K, bits) + 255) & ~255ull) + ((N * 2 + 255) & ~255ull); };
  for (int L = 0; L < a.layer_count; L++) {
    size_t hd = is_global(a, L) ? a.global_head_dim : a.sliding_head_dim;
    bool prod = L < a.kv_producer_layers;
    size_t ffn = prod ? a.producer_intermediate : a.consumer_intermediate;
    const int mb = prod ? a.mlp_bits : a.consumer_mlp_bits;
    lin(a.query_heads * hd, H, 4);
    if (prod) {
      lin(hd, H, 4);
      lin(hd, H, 4);
    }
    lin(H, a.query_heads * hd, 4);
    lin(ffn, H, mb);
    lin(ffn, H, mb);
    lin(H, ffn, mb);
    lin(a.ple_dim, H, 8);
    lin(H, a.ple_dim, 8);
    total += 5 * ((H * 4 + 255) & ~255ull) + 2 * ((hd * 4 + 255) & ~255ull);
  }
  size_t V = a.vocab_size, ple_cols = (size_t)a.layer_count * a.ple_dim;
  total += linear_bytes(V, H, a.head_bits) + 256 + V * 2 + 256;   // embed (tied lm_head)
  total += V * a.layer_count * 2 + 256;                    // PLE scales
  total += ple_cols * H * 2 + 256;                         // PLMP bf16
  total += a.ple_dim * 4 + 256 + H * 4 + 256;              // norms
  return total + (1 << 20);
}

static int alloc_weights(g4_ctx *ctx) {
  const g4_arch &a = ctx->cfg.arch;
  ctx->arena_bytes = weight_arena_bytes(a);
  CK(ctx_malloc((void **)&ctx->arena, ctx->arena_bytes));
  ctx->arena_used = 0;
  const int H = ctx->H;
  ctx->layers.assign(a.layer_count, Layer());
  for (int L = 0; L < a.layer_count; L++) {
    Layer &ly = ctx->layers[L];
    ly.global = is_global(a, L);
    ly.producer = L < a.kv_producer_layers;
    ly.hd = ly.global ? a.global_head_dim : a.sliding_head_dim;
    int ffn = ly.producer ? a.producer_intermediate : a.consumer_intermediate;
    const int mb = ly.producer ? a.mlp_bits : a.consumer_mlp_bits;
    int qrows = a.query_heads * ly.hd;
    int rc;
    if ((rc = make_linear(ctx, ly.q, layer_name(L, "self_attn.q_proj"), qrows, H, 4))) return rc;
    if (ly.producer) {
      if ((rc = make_linear(ctx, ly.k, layer_name(L, "self_attn.k_proj"), ly.hd, H, 4))) return rc;
      if ((rc = make_linear(ctx, ly.v, layer_name(L, "self_attn.v_proj"), ly.hd, H, 4))) return rc;
    }
    if ((rc = make_linear(ctx, ly.o, layer_name(L, "self_attn.o_proj"), H, qrows, 4))) return rc;
    if ((rc = make_linear(ctx, ly.gate, layer_name(L, "mlp.gate_proj"), ffn, H, mb))) return rc;
    if ((rc = make_linear(ctx, ly.up, layer_name(L, "mlp.up_proj"), ffn, H, mb))) return rc;
    if ((rc = make_linear(ctx, ly.down, layer_name(L, "mlp.down_proj"), H, ffn, mb))) return rc;
    if ((rc = make_linear(ctx, ly.pleg, layer_name(L, "per_layer_input_gate"), a.ple_dim, H, 8))) return rc;
    if ((rc = make_linear(ctx, ly.plep, layer_name(L, "per_layer_projection"), H, a.ple_dim, 8))) return rc;
    ly.ln_in = make_f32(ctx, layer_name(L, "input_layernorm.weight"), H);
    ly.ln_post_attn = make_f32(ctx, layer_name(L, "post_attention_layernorm.weight"), H);
    ly.ln_pre_ffn = make_f32(ctx, layer_name(L, "pre_feedforward_layernorm.weight"), H);
    ly.ln_post_ffn = make_f32(ctx, layer_name(L, "post_feedforward_layernorm.weight"), H);
    ly.ln_post_ple = make_f32(ctx, layer_name(L, "post_per_layer_input_norm.weight"), H);
    ly.q_norm = make_f32(ctx, layer_name(L, "self_attn.q_norm.weight"), ly.hd);
    ly.k_norm = make_f32(ctx, layer_name(L, "self_attn.k_norm.weight"), ly.hd);
    if (!ly.ln_in || !ly.ln_post_attn || !ly.ln_pre_ffn || !ly.ln_post_ffn || !ly.ln_post_ple ||
        !ly.q_norm || !ly.k_norm)
      return fail(ctx, G4_ERR_OOM, "weight arena exhausted at layer %d norms", L);
    // kvRoleForLayer (src/kv.ts:76-88): consumers read the last producer of their type.
    if (ly.producer) {
      ly.cache_layer = L;
    } else {
      int last = -1;
      for (int p = 0; p < a.kv_producer_layers; p++)
        if (is_global(a, p) == ly.global) last = p;
      ly.cache_layer = last;
    }
  }
  size_t V = ctx->V;
  const int hb = a.head_bits;
  ctx->embed_w = (uint8_t *)arena_take(ctx, linear_bytes(V, H, hb));
  ctx->embed_s = (uint16_t *)arena_take(ctx, V * 2);
  ctx->ple_s = (uint16_t *)arena_take(ctx, V * ctx->NL * 2);
  ctx->plmp_w = (uint16_t *)arena_take(ctx, (size_t)ctx->ple_cols * H * 2);
  ctx->plmp_norm = make_f32(ctx, std::string(LMP) + "per_layer_projection_norm.weight", ctx->PD);
  ctx->final_norm = make_f32(ctx, std::string(LMP) + "norm.weight", H);
  if (!ctx->embed_w || !ctx->embed_s || !ctx->ple_s || !ctx->plmp_w || !ctx->plmp_norm || !ctx->final_norm)
    return fail(ctx, G4_ERR_OOM, "weight arena exhausted at the embedding tables");
  {
    TensorRef tr{ctx->embed_w, V * H * hb / 8, false};
    if (hb == 2) {
      tr.t16_rows = (int)V;
      tr.t16_k = H;
    }
    ctx->tensors[std::string(LMP) + "embed_tokens.embedding_quantized"] = tr;
  }
  ctx->tensors[std::string(LMP) + "embed_tokens.embedding_scale"] = {ctx->embed_s, V * 2, false};
  ctx->tensors[std::string(LMP) + "embed_tokens_per_layer.embedding_scale"] = {ctx->ple_s, V * ctx->NL * 2, false};
  ctx->tensors[std::string(LMP) + "per_layer_model_projection.weight"] = {ctx->plmp_w, (uint64_t)ctx->ple_cols * H * 2, false};
  // lm_head is tied to embed_tokens (src/execute.ts:207-214).
  ctx->lm.w = ctx->embed_w;
  ctx->lm.s = ctx->embed_s;
  ctx->lm.N = ctx->V;
  ctx->lm.K = H;
  ctx->lm.bits = hb;
  ctx->lm.module = "lm_head";
  for (Layer &ly : ctx->layers)
    for (Linear *l : {&ly.q, &ly.k, &ly.v, &ly.o, &ly.gate, &ly.up, &ly.down, &ly.pleg, &ly.plep})
      linear_tmap(*l);
  linear_tmap(ctx->lm);
  // int8 copies of the int4 / 2-bit linears for tensor-core steps (about 1.3 GB at the full
  // shape; HBM is plentiful, and without them the GEMM is bound by the unpack: a 2048-token prefill
  // 4% and a B=64 decode step 6% slower). 0: every tensor-core step uses them.
  ctx->shadow_min_cols = ctx->cfg.gemm_shadow_min_columns == 0 ? 1 : ctx->cfg.gemm_shadow_min_columns;
  if (ctx->shadow_min_cols > 0) {
    std::vector<Linear *> ls;
    for (Layer &ly : ctx->layers)
      for (Linear *l : {&ly.q, &ly.k, &ly.v, &ly.o, &ly.gate, &ly.up, &ly.down})
        if (l->w && l->bits != 8 && l->K % 128 == 0) ls.push_back(l);
    if (ctx->lm.K % 128 == 0) ls.push_back(&ctx->lm);
    size_t total = 0;
    for (Linear *l : ls) total += ((size_t)l->N * l->K + 255) & ~(size_t)255;
    CK(ctx_malloc((void **)&ctx->shadow, total));
    ctx->shadow_bytes = total;
    size_t off = 0;
    for (Linear *l : ls) {
      l->w8 = (int8_t *)(ctx->shadow + off);
      off += ((size_t)l->N * l->K + 255) & ~(size_t)255;
      l->has_tm8 = make_tmap_u8(&l->tmw8, l->w8, (uint64_t)l->K, (uint64_t)l->N, (uint64_t)l->K, 128, 128, true) == 0;
    }
  }
  // The PLE code table: one buffer or vocab-row slices (src/tableSplit.ts:125-215).
  const uint64_t row_bytes = (uint64_t)ctx->ple_cols / 2;
  const uint64_t total = row_bytes * V;
  int32_t n = 1, rps = ctx->V, last = ctx->V;
  if (ctx->cfg.ple_slice_bytes > 0) {
    int rc = g4_plan_table_split(V, row_bytes, ctx->cfg.ple_slice_bytes, ctx->cfg.ple_slice_bytes, &n, &rps, &last);
    if (rc) return fail(ctx, rc, "%s", tl_error.c_str());
  }
  ctx->ple_rps = rps;
  ctx->ple_slices.assign(n, nullptr);
  for (int i = 0; i < n; i++) {
    size_t rows = i + 1 < n ? (size_t)rps : (size_t)last;
    CK(ctx_malloc((void **)&ctx->ple_slices[i], rows * row_bytes));
  }
  CK(ctx_malloc((void **)&ctx->d_ple_slices, sizeof(uint8_t *) * n));
  CK(cudaMemcpy(ctx->d_ple_slices, ctx->ple_slices.data(), sizeof(uint8_t *) * n, cudaMemcpyHostToDevice));
  ctx->ple_slice_bytes = total;
  ctx->tensors[std::string(LMP) + "embed_tokens_per_layer.embedding_quantized"] = {nullptr, total, true};
  return G4_OK;
}

static int alloc_runtime(g4_ctx *ctx) {
  const g4_arch &a = ctx->cfg.arch;
  const int maxc = ctx->maxc, H = ctx->H, mctx = ctx->cfg.max_context;
  // KV caches.
  ctx->kv.assign(a.kv_producer_layers, nullptr);
  ctx->kv_stride.assign(a.kv_producer_layers, 0);
  for (int L = 0; L < a.kv_producer_layers; L++) {
    size_t hd = ctx->layers[L].hd;
    ctx->kv_stride[L] = 2 * (size_t)mctx * hd;
    size_t bytes = ctx->kv_stride[L] * ctx->cfg.max_seqs * 4;
    CK(ctx_malloc((void **)&ctx->kv[L], bytes));
    CK(cudaMemset(ctx->kv[L], 0, bytes));
    ctx->kv_bytes += bytes;
  }
  ctx->kv_len.assign(ctx->cfg.max_seqs, 0);
  // Rope tables (ropeTables, src/kernels/rope.ts:149-191), f64 on the host, f32 on the device.
  auto tables = [&](int hd, int rot_pairs, double theta, float **cd, float **sd) -> int {
    int pairs = hd / 2;
    std::vector<float> cs((size_t)mctx * pairs), sn((size_t)mctx * pairs);
    for (int p = 0; p < mctx; p++)
      for (int i = 0; i < pairs; i++) {
        double inv = i < rot_pairs ? std::pow(theta, (-2.0 * i) / (double)hd) : 0.0;
        double ang = (double)p * inv;
        cs[(size_t)p * pairs + i] = (float)std::cos(ang);
        sn[(size_t)p * pairs + i] = (float)std::sin(ang);
      }
    CK(ctx_malloc((void **)cd, cs.size() * 4));
    CK(ctx_malloc((void **)sd, sn.size() * 4));
    CK(cudaMemcpy(*cd, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(*sd, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    ctx->other_bytes += cs.size() * 8;
    return G4_OK;
  };
  int rc;
  if ((rc = tables(a.sliding_head_dim, a.sliding_head_dim / 2, (double)a.rope_theta_sliding, &ctx->cos_s, &ctx->sin_s))) return rc;
  int grot = (int)(a.partial_rotary_factor * a.global_head_dim / 2);
  if ((rc = tables(a.global_head_dim, grot, (double)a.rope_theta_global, &ctx->cos_g, &ctx->sin_g))) return rc;
  // Activation slots, sized once for the widest step (src/execute.ts:248-317).
  const size_t ghd = a.global_head_dim, nh = a.query_heads, ffn = std::max(a.producer_intermediate, a.consumer_intermediate);
  auto take = [&](float **p, size_t n) -> int {
    CK(ctx_malloc((void **)p, n * 4));
    CK(cudaMemset(*p, 0, n * 4));
    ctx->other_bytes += n * 4;
    return G4_OK;
  };
  if ((rc = take(&ctx->res[0], (size_t)maxc * H))) return rc;
  if ((rc = take(&ctx->res[1], (size_t)maxc * H))) return rc;
  if ((rc = take(&ctx->ple_id, (size_t)maxc * ctx->ple_cols))) return rc;
  if ((rc = take(&ctx->ple_proj, (size_t)maxc * ctx->ple_cols))) return rc;
  if ((rc = take(&ctx->ple_in, (size_t)maxc * ctx->ple_cols))) return rc;
  if ((rc = take(&ctx->q, (size_t)maxc * nh * ghd))) return rc;
  if ((rc = take(&ctx->k, (size_t)maxc * ghd))) return rc;
  if ((rc = take(&ctx->v, (size_t)maxc * ghd))) return rc;
  if ((rc = take(&ctx->qr, (size_t)maxc * nh * ghd))) return rc;
  if ((rc = take(&ctx->attn, (size_t)maxc * nh * ghd))) return rc;
  if ((rc = take(&ctx->proj, (size_t)maxc * H))) return rc;
  if ((rc = take(&ctx->gate, (size_t)maxc * ffn))) return rc;
  if ((rc = take(&ctx->up, (size_t)maxc * ffn))) return rc;
  if ((rc = take(&ctx->pleg_out, (size_t)maxc * a.ple_dim))) return rc;
  ctx->att_blocks_sliding = (a.sliding_window + 63) / 64 + 1;
  ctx->att_blocks_global = (mctx + 63) / 64;
  int mb = std::max(ctx->att_blocks_sliding, ctx->att_blocks_global);
  if ((rc = take(&ctx->part_o, (size_t)maxc * mb * nh * ghd))) return rc;
  if ((rc = take(&ctx->part_m, (size_t)maxc * mb * nh))) return rc;
  if ((rc = take(&ctx->part_l, (size_t)maxc * mb * nh))) return rc;
  ctx->gq_ld = (int)((std::max<size_t>({(size_t)ctx->H, ffn, nh * ghd}) + 127) & ~(size_t)127);
  ctx->gq_rows = std::max(maxc, 256);
  for (int i = 0; i < 3; i++) {
    CK(ctx_malloc((void **)&ctx->gq[i], (size_t)ctx->gq_rows * ctx->gq_ld));
    CK(cudaMemset(ctx->gq[i], 0, (size_t)ctx->gq_rows * ctx->gq_ld));
  }
  ctx->gacc_ld = ctx->gq_ld;
  CK(ctx_malloc((void **)&ctx->gacc, (size_t)maxc * ctx->gacc_ld * 4));
  CK(cudaMemset(ctx->gacc, 0, (size_t)maxc * ctx->gacc_ld * 4));
  CK(ctx_malloc((void **)&ctx->gcnt, 8192 * 4));
  CK(cudaMemset(ctx->gcnt, 0, 8192 * 4));
  ctx->gparts = (int)((a.vocab_size + 127) / 128);
  CK(ctx_malloc((void **)&ctx->gpv, (size_t)maxc * ctx->gparts * 4));
  CK(ctx_malloc((void **)&ctx->gpi, (size_t)maxc * ctx->gparts * 4));
  ctx->gemm_min_cols = ctx->cfg.gemm_min_columns > 0 ? ctx->cfg.gemm_min_columns : 16;
  ctx->gemm_split_k = ctx->cfg.gemm_split_k;
  ctx->ffn_max = (ffn + 15) & ~15;
  CK(ctx_malloc((void **)&ctx->codes_mlp, (size_t)maxc * ctx->ffn_max));
  CK(ctx_malloc((void **)&ctx->codes_ple, (size_t)maxc * ctx->PD));
  CK(ctx_malloc((void **)&ctx->codes_attn, (size_t)maxc * a.query_heads * std::max(a.sliding_head_dim, a.global_head_dim)));
  CK(ctx_malloc((void **)&ctx->att_count, (size_t)maxc * 8 * 4));
  CK(cudaMemset(ctx->att_count, 0, (size_t)maxc * 8 * 4));
  // Logit rows: one per sequence of a decode batch, and at least G4_VERIFY_COLS for the
  // positions of a verify pass.
  ctx->head_cols = std::min(maxc, std::max(ctx->cfg.max_seqs, (int)G4_VERIFY_COLS));
  if ((rc = take(&ctx->logits, (size_t)ctx->head_cols * ctx->V))) return rc;
  CK(cudaDeviceGetAttribute(&ctx->sms, cudaDevAttrMultiProcessorCount, ctx->dev));
  ctx->gemv_target = 2 * ctx->sms;
  // A GEMV launch has at most gemv_target CTAs (gemv_stream_partition), each writing one argmax
  // partial per column in the head.
  ctx->head_cap = std::min(ctx->gemv_target, ctx->V);
  ctx->head_blocks = ctx->head_cap;
  if ((rc = take(&ctx->head_pv, (size_t)ctx->head_cols * ctx->head_cap))) return rc;
  CK(ctx_malloc((void **)&ctx->head_pi, (size_t)ctx->head_cols * ctx->head_cap * 4));
  CK(ctx_malloc((void **)&ctx->d_step, (size_t)3 * maxc * 4));
  CK(cudaMemset(ctx->d_step, 0, (size_t)3 * maxc * 4));
  // The tokens of a step, then one word: the OR of the error flags (k_argmax_final).
  CK(ctx_malloc((void **)&ctx->d_tok_out, (size_t)(maxc + 1) * 4));
  CK(ctx_malloc((void **)&ctx->d_val_out, (size_t)maxc * 4));
  for (int i = 0; i < g4_ctx::kStageSlots; i++) {
    CK(cudaMallocHost(&ctx->h_step[i], (size_t)3 * maxc * 4));
    CK(cudaEventCreateWithFlags(&ctx->stage_ev[i], cudaEventDisableTiming));
  }
  CK(cudaMallocHost(&ctx->h_tok, (size_t)(maxc + 1) * 4));
  int *fl[4] = {dev_error_addr(), gemv2_error_addr(), gemm_error_addr(), ple_error_addr()};
  for (int i = 0; i < 4; i++) {
    if (!fl[i]) return fail(ctx, G4_ERR_CUDA, "cannot resolve the device address of an error flag");
    ctx->errf.p[i] = fl[i];
  }
  return G4_OK;
}

extern "C" int g4_ctx_create(int cuda_device, const g4_config *cfg_in, g4_ctx **out) {
  if (!out) return fail(nullptr, G4_ERR_INVALID, "g4_ctx_create: null out");
  *out = nullptr;
  g4_config cfg;
  if (cfg_in) cfg = *cfg_in; else g4_config_default(&cfg);
  const g4_arch &a = cfg.arch;
  if (a.kv_heads != 1) return fail(nullptr, G4_ERR_UNSUPPORTED, "only one KV head is supported");
  if (a.query_heads != 8) return fail(nullptr, G4_ERR_UNSUPPORTED, "the attention kernels are built for 8 query heads");
  if (a.attn_bits != 4 || a.mlp_bits != 4 || a.ple_bits != 8 ||
      (a.consumer_mlp_bits != 4 && a.consumer_mlp_bits != 2) || (a.head_bits != 4 && a.head_bits != 2))
    return fail(nullptr, G4_ERR_UNSUPPORTED, "weight widths: attn 4, producer MLP 4, PLE 8, consumer MLP 4 or 2, head 4 or 2");
  if (!a.head_calibrated && a.head_bits != 2)
    return fail(nullptr, G4_ERR_UNSUPPORTED, "an uncalibrated (f32-path) head is built for the 2-bit family only");
  if ((a.consumer_mlp_bits == 2 || a.head_bits == 2) && a.hidden_size % 128 != 0)
    return fail(nullptr, G4_ERR_UNSUPPORTED, "the 2-bit family needs the hidden size a multiple of 128");
  if (a.hidden_size % 256 != 0 || a.hidden_size > 2048)
    return fail(nullptr, G4_ERR_UNSUPPORTED, "hidden size must be a multiple of 256 up to 2048");
  if ((a.sliding_head_dim != 256 && a.sliding_head_dim != 512) || (a.global_head_dim != 256 && a.global_head_dim != 512))
    return fail(nullptr, G4_ERR_UNSUPPORTED, "head dims 256 or 512 only");
  if (a.ple_dim % 256 != 0 || a.layer_count > 64 || a.kv_producer_layers < 1 || a.kv_producer_layers > a.layer_count)
    return fail(nullptr, G4_ERR_INVALID, "bad PLE or layer geometry");
  if (cfg.max_seqs < 1 || cfg.max_context < 1 || cfg.max_step_columns < 1)
    return fail(nullptr, G4_ERR_INVALID, "max_seqs, max_context and max_step_columns must be positive");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || cuda_device < 0 || cuda_device >= ndev)
    return fail(nullptr, G4_ERR_CUDA, "CUDA device %d is not available", cuda_device);
  g4_ctx *ctx = new g4_ctx();
  ctx->dev = cuda_device;
  ctx->cfg = cfg;
  ctx->H = a.hidden_size;
  ctx->V = a.vocab_size;
  ctx->PD = a.ple_dim;
  ctx->NL = a.layer_count;
  ctx->ple_cols = a.layer_count * a.ple_dim;
  ctx->ffn = std::max(a.producer_intermediate, a.consumer_intermediate);
  ctx->maxc = cfg.max_step_columns;
  int rc = G4_OK;
  if (cudaSetDevice(cuda_device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->st, cudaStreamNonBlocking) != cudaSuccess) {
    rc = fail(ctx, G4_ERR_CUDA, "cannot initialise device %d", cuda_device);
  }
  if (!rc) rc = alloc_weights(ctx);
  if (!rc) rc = alloc_runtime(ctx);
  if (rc) {
    std::string msg = ctx->err;
    g4_ctx_destroy(ctx);
    return fail(nullptr, rc, "%s", msg.c_str());
  }
  *out = ctx;
  return G4_OK;
}

#ifdef G4_TRACE
// Diagnostic builds only (not part of include/g4.h): drop the records so far.
extern "C" int g4_trace_reset(void) {
  unsigned long long dummy[2];
  trace_take(dummy, 0);
  gemm_trace_take(dummy, 0);
  ple_trace_take(dummy, 0);
  return 0;
}
#endif

extern "C" void g4_ctx_destroy(g4_ctx *ctx) {
#ifdef G4_TRACE
  if (const char *path = getenv("G4_TRACE_FILE")) {
    std::vector<unsigned long long> rec(2 << 15);
    const int n = trace_take(rec.data(), 1 << 15);
    if (FILE *f = fopen(path, "w")) {
      for (int i = 0; i < n; i++) fprintf(f, "%llu %llu\n", rec[2 * i], rec[2 * i + 1]);
      const int gm = gemm_trace_take(rec.data(), 1 << 15);
      for (int i = 0; i < gm; i++) fprintf(f, "%llu %llu\n", rec[2 * i], rec[2 * i + 1]);
      const int pm = ple_trace_take(rec.data(), 1 << 15);
      for (int i = 0; i < pm; i++) fprintf(f, "%llu %llu\n", rec[2 * i], rec[2 * i + 1]);
      fclose(f);
    }
  }
#endif
  if (!ctx) return;
  cudaSetDevice(ctx->dev);
  if (ctx->st) cudaStreamSynchronize(ctx->st);
  for (auto &kv : ctx->graphs) cudaGraphExecDestroy(kv.second);
  cudaFree(ctx->arena);
  cudaFree(ctx->shadow);
  for (void *p : ctx->ple_slices) cudaFree(p);
  cudaFree(ctx->d_ple_slices);
  for (float *p : ctx->kv) cudaFree(p);
  float *fs[] = {ctx->cos_s, ctx->sin_s, ctx->cos_g, ctx->sin_g, ctx->res[0], ctx->res[1],
                 ctx->ple_id, ctx->ple_proj, ctx->ple_in, ctx->q, ctx->k, ctx->v, ctx->qr,
                 ctx->attn, ctx->proj, ctx->gate, ctx->up, ctx->pleg_out, ctx->part_o,
                 ctx->part_m, ctx->part_l, ctx->logits, ctx->head_pv, ctx->d_val_out};
  for (float *p : fs) cudaFree(p);
  cudaFree(ctx->head_pi);
  cudaFree(ctx->att_count);
  cudaFree(ctx->codes_mlp);
  cudaFree(ctx->codes_attn);
  for (int i = 0; i < 3; i++) cudaFree(ctx->gq[i]);
  cudaFree(ctx->gpv);
  cudaFree(ctx->gpi);
  cudaFree(ctx->gacc);
  cudaFree(ctx->gcnt);
  cudaFree(ctx->codes_ple);
  cudaFree(ctx->d_step);
  cudaFree(ctx->d_tok_out);
  for (int i = 0; i < g4_ctx::kStageSlots; i++) {
    cudaFreeHost(ctx->h_step[i]);
    if (ctx->stage_ev[i]) cudaEventDestroy(ctx->stage_ev[i]);
  }
  cudaFreeHost(ctx->h_tok);
  if (ctx->st) cudaStreamDestroy(ctx->st);
  delete ctx;
  cudaGetLastError();   // a failed release must not surface in the next context's first launch
}

extern "C" int g4_ctx_memory(const g4_ctx *ctx, uint64_t *w, uint64_t *kvb, uint64_t *o) {
  if (!ctx) return fail(nullptr, G4_ERR_INVALID, "null context");
  if (w) *w = ctx->arena_bytes + ctx->ple_slice_bytes;
  if (kvb) *kvb = ctx->kv_bytes;
  if (o) *o = ctx->other_bytes;
  return G4_OK;
}

extern "C" int g4_ctx_ple_slices(const g4_ctx *ctx, int32_t *n_slices, int32_t *rows_per_slice,
                                 int32_t *last_rows) {
  if (!ctx) return fail(nullptr, G4_ERR_INVALID, "null context");
  const int32_t n = (int32_t)ctx->ple_slices.size();
  if (n_slices) *n_slices = n;
  if (rows_per_slice) *rows_per_slice = ctx->ple_rps;
  if (last_rows) *last_rows = n > 0 ? ctx->V - (n - 1) * ctx->ple_rps : 0;
  return G4_OK;
}

extern "C" int g4_debug_fail_allocation(int32_t nth) {
  g_fail_alloc.store(nth > 0 ? nth : 0);
  return G4_OK;
}

extern "C" int g4_debug_raise_error_flag(g4_ctx *ctx, int32_t unit) {
  if (!ctx || unit < 0 || unit > 3) return fail(ctx, G4_ERR_INVALID, "g4_debug_raise_error_flag: unit %d outside 0..3", unit);
  CK(cudaSetDevice(ctx->dev));
  const int one = 1;
  CK(cudaMemcpy(const_cast<int *>(ctx->errf.p[unit]), &one, sizeof(int), cudaMemcpyHostToDevice));
  return G4_OK;
}

extern "C" void *g4_ctx_stream(g4_ctx *ctx) { return ctx ? (void *)ctx->st : nullptr; }

extern "C" int g4_last_launch_list(const g4_ctx *ctx, char *buf, uint64_t cap, uint64_t *needed) {
  if (!ctx || !needed) return fail(nullptr, G4_ERR_INVALID, "null argument");
  std::string all;
  for (const std::string &r : ctx->roles) all += r + "\n";
  *needed = all.size() + 1;
  if (buf) {
    if (cap < all.size() + 1) return fail(nullptr, G4_ERR_INVALID, "launch list needs %llu bytes", (unsigned long long)(all.size() + 1));
    memcpy(buf, all.c_str(), all.size() + 1);
  }
  return G4_OK;
}

extern "C" int g4_last_launches(const g4_ctx *ctx, int32_t *n) {
  if (!ctx || !n) return fail(nullptr, G4_ERR_INVALID, "null argument");
  *n = ctx->launches;
  return G4_OK;
}

// ================================================================================ weights

// Synthetic tensor kinds; a layer tensor's hash stream is ((layer + 1) << 8) | kind.
enum {
  TK_Q_W = 0, TK_Q_S, TK_K_W, TK_K_S, TK_V_W, TK_V_S, TK_O_W, TK_O_S,
  TK_GATE_W, TK_GATE_S, TK_UP_W, TK_UP_S, TK_DOWN_W, TK_DOWN_S,
  TK_PLEG_W, TK_PLEG_S, TK_PLEP_W, TK_PLEP_S,
  TK_LN_IN, TK_LN_POST_ATTN, TK_LN_PRE_FFN, TK_LN_POST_FFN, TK_LN_POST_PLE,
  TK_QNORM, TK_KNORM, TK_LAYER_SCALAR, TK_SRQ,
  TK_EMBED_W = 40, TK_EMBED_S, TK_PLE_W, TK_PLE_S, TK_PLMP_W, TK_PLMP_NORM, TK_FINAL_NORM
};
enum { S_Q = 0, S_K, S_V, S_O, S_GATE, S_UP, S_DOWN, S_PLEG, S_PLEP, S_LM, N_SITES };
// Static activation scales: max |x| / 127 of a seeded 16-token warm-up forward per site, each
// layer's value jittered by (0.9 + 0.2 u). lm_head's output is not snapped.
static const double SRQ_BASE_IN[N_SITES] = {0.04, 0.04, 0.04, 0.04, 0.033, 0.033, 1.0, 0.085, 0.34, 0.024};
static const double SRQ_BASE_OUT[N_SITES] = {0.11, 0.097, 0.092, 0.2, 0.108, 0.11, 3.9, 0.225, 0.085, 0.0};

static uint64_t layer_stream(int L, int kind) { return ((uint64_t)(L + 1) << 8) | (uint64_t)kind; }

static float synth_srq(uint64_t seed, int L, int site, int out) {
  double base = out ? SRQ_BASE_OUT[site] : SRQ_BASE_IN[site];
  if (base == 0.0) return 0.0f;
  uint64_t h = keyed(stream_key(seed, layer_stream(L, TK_SRQ)), (uint64_t)(site * 2 + out));
  return (float)(base * (0.9 + 0.2 * unit24(h)));
}

static float bf16_round(float f) {
  uint32_t b = (uint32_t)f32_to_bf16_bits(f) << 16;
  float r;
  memcpy(&r, &b, 4);
  return r;
}

// The checkpoint layout's words of a 2-bit tensor, generated into a staging buffer and repacked
// into the tile layout the kernels read (src/kernels/repack.ts:17-209).
static int gen_tile16(g4_ctx *ctx, void *dst, int N, int K, uint64_t key) {
  const size_t wb = (size_t)N * K / 4;
  void *tmp = nullptr;
  CK(ctx_malloc(&tmp, wb));
  cudaError_t e = launch_gen_words((uint32_t *)tmp, wb / 4, key, 0, ctx->st);
  if (e == cudaSuccess) e = launch_repack_tile16(tmp, dst, N, K, ctx->st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->st);
  cudaFree(tmp);
  CK(e);
  return G4_OK;
}

static int gen_linear(g4_ctx *ctx, Linear &lin, uint64_t seed, int L, int kw, int ks, int site) {
  size_t wb = (size_t)lin.N * lin.K * lin.bits / 8;
  if (lin.bits == 2) {
    int rc = gen_tile16(ctx, lin.w, lin.N, lin.K, stream_key(seed, layer_stream(L, kw)));
    if (rc) return rc;
  } else {
    CK(launch_gen_words((uint32_t *)lin.w, wb / 4, stream_key(seed, layer_stream(L, kw)), 0, ctx->st));
  }
  // Row scales keep activations O(1): int8 codes are 16x larger than int4, 2-bit ones 4x smaller.
  double div = lin.bits == 8 ? 16.0 : (lin.bits == 2 ? 0.25 : 1.0);
  CK(launch_gen_f16(lin.s, (size_t)lin.N, stream_key(seed, layer_stream(L, ks)), 1e-3 / div, 1e-2 / div, ctx->st));
  lin.in_scale = synth_srq(seed, L, site, 0);
  lin.out_scale = synth_srq(seed, L, site, 1);
  return G4_OK;
}

static int gen_gain(g4_ctx *ctx, float *p, size_t n, uint64_t seed, int L, int kind) {
  CK(launch_gen_bf16_f32(p, n, stream_key(seed, layer_stream(L, kind)), 0.5, 1.5, ctx->st));
  return G4_OK;
}

extern "C" int g4_init_random(g4_ctx *ctx, uint64_t seed) {
  if (!ctx) return fail(nullptr, G4_ERR_INVALID, "null context");
  CK(cudaSetDevice(ctx->dev));
  const int H = ctx->H;
  int rc;
  for (int L = 0; L < ctx->NL; L++) {
    Layer &ly = ctx->layers[L];
    if ((rc = gen_linear(ctx, ly.q, seed, L, TK_Q_W, TK_Q_S, S_Q))) return rc;
    if (ly.producer) {
      if ((rc = gen_linear(ctx, ly.k, seed, L, TK_K_W, TK_K_S, S_K))) return rc;
      if ((rc = gen_linear(ctx, ly.v, seed, L, TK_V_W, TK_V_S, S_V))) return rc;
    }
    if ((rc = gen_linear(ctx, ly.o, seed, L, TK_O_W, TK_O_S, S_O))) return rc;
    if ((rc = gen_linear(ctx, ly.gate, seed, L, TK_GATE_W, TK_GATE_S, S_GATE))) return rc;
    if ((rc = gen_linear(ctx, ly.up, seed, L, TK_UP_W, TK_UP_S, S_UP))) return rc;
    if ((rc = gen_linear(ctx, ly.down, seed, L, TK_DOWN_W, TK_DOWN_S, S_DOWN))) return rc;
    if ((rc = gen_linear(ctx, ly.pleg, seed, L, TK_PLEG_W, TK_PLEG_S, S_PLEG))) return rc;
    if ((rc = gen_linear(ctx, ly.plep, seed, L, TK_PLEP_W, TK_PLEP_S, S_PLEP))) return rc;
    if ((rc = gen_gain(ctx, ly.ln_in, H, seed, L, TK_LN_IN))) return rc;
    if ((rc = gen_gain(ctx, ly.ln_post_attn, H, seed, L, TK_LN_POST_ATTN))) return rc;
    if ((rc = gen_gain(ctx, ly.ln_pre_ffn, H, seed, L, TK_LN_PRE_FFN))) return rc;
    if ((rc = gen_gain(ctx, ly.ln_post_ffn, H, seed, L, TK_LN_POST_FFN))) return rc;
    if ((rc = gen_gain(ctx, ly.ln_post_ple, H, seed, L, TK_LN_POST_PLE))) return rc;
    if ((rc = gen_gain(ctx, ly.q_norm, ly.hd, seed, L, TK_QNORM))) return rc;
    if ((rc = gen_gain(ctx, ly.k_norm, ly.hd, seed, L, TK_KNORM))) return rc;
    double u = unit24(keyed(stream_key(seed, layer_stream(L, TK_LAYER_SCALAR)), 0));
    ly.layer_scalar = bf16_round((float)(0.03 + (0.9 - 0.03) * u));
  }
  const size_t V = ctx->V;
  const uint64_t ekey = stream_key(seed, layer_stream(-1, TK_EMBED_W));
  const double ediv = ctx->lm.bits == 2 ? 0.25 : 1.0;
  if (ctx->lm.bits == 2) {
    if ((rc = gen_tile16(ctx, ctx->embed_w, (int)V, H, ekey))) return rc;
  } else {
    CK(launch_gen_words((uint32_t *)ctx->embed_w, V * H / 8, ekey, 0, ctx->st));
  }
  CK(launch_gen_f16(ctx->embed_s, V, stream_key(seed, layer_stream(-1, TK_EMBED_S)), 1e-3 / ediv, 1e-2 / ediv, ctx->st));
  CK(launch_gen_f16(ctx->ple_s, V * ctx->NL, stream_key(seed, layer_stream(-1, TK_PLE_S)), 1e-3, 1e-2, ctx->st));
  CK(launch_gen_plmp(ctx->plmp_w, (size_t)ctx->ple_cols * H, stream_key(seed, layer_stream(-1, TK_PLMP_W)), 0.04419417382415922, ctx->st));
  if ((rc = gen_gain(ctx, ctx->plmp_norm, ctx->PD, seed, -1, TK_PLMP_NORM))) return rc;
  if ((rc = gen_gain(ctx, ctx->final_norm, H, seed, -1, TK_FINAL_NORM))) return rc;
  // The PLE table by absolute word index, into whichever slice holds the row.
  {
    const size_t words_per_row = (size_t)ctx->ple_cols / 8;
    const uint64_t key = stream_key(seed, layer_stream(-1, TK_PLE_W));
    size_t n = ctx->ple_slices.size();
    for (size_t i = 0; i < n; i++) {
      size_t row0 = i * (size_t)ctx->ple_rps;
      size_t rows = std::min((size_t)ctx->ple_rps, V - row0);
      // Each slice starts at word row0 * words_per_row of the table's counter stream.
      uint32_t *dst = (uint32_t *)ctx->ple_slices[i];
      size_t nw = rows * words_per_row;
      CK(launch_gen_words(dst, nw, key, row0 * words_per_row, ctx->st));
    }
  }
  // An uncalibrated head (the checkpoint's, src/quant.ts:574-585) keeps both scales 0.0.
  ctx->lm.in_scale = ctx->cfg.arch.head_calibrated ? synth_srq(seed, -1, S_LM, 0) : 0.0f;
  ctx->lm.out_scale = ctx->cfg.arch.head_calibrated ? synth_srq(seed, -1, S_LM, 1) : 0.0f;
  CK(cudaStreamSynchronize(ctx->st));
  ctx->weights_ready = true;
  ctx->shadow_dirty = ctx->shadow != nullptr;
  for (auto &kv : ctx->graphs) cudaGraphExecDestroy(kv.second);
  ctx->graphs.clear();
  return G4_OK;
}

static int find_tensor(g4_ctx *ctx, const char *name, TensorRef *ref) {
  auto it = ctx->tensors.find(name);
  if (it == ctx->tensors.end()) return fail(ctx, G4_ERR_NOT_FOUND, "unknown tensor %s", name);
  *ref = it->second;
  return G4_OK;
}

extern "C" int g4_upload_weight(g4_ctx *ctx, const char *name, const void *bytes, uint64_t offset,
                                uint64_t n, uint64_t total) {
  if (!ctx || !name || (!bytes && n)) return fail(ctx, G4_ERR_INVALID, "g4_upload_weight: null argument");
  TensorRef r;
  int rc = find_tensor(ctx, name, &r);
  if (rc) return rc;
  if (total != r.bytes) return fail(ctx, G4_ERR_INVALID, "%s holds %llu bytes, upload says %llu", name, (unsigned long long)r.bytes, (unsigned long long)total);
  if (offset + n > total) return fail(ctx, G4_ERR_INVALID, "%s: bytes [%llu, %llu) past the end", name, (unsigned long long)offset, (unsigned long long)(offset + n));
  CK(cudaSetDevice(ctx->dev));
  if (r.t16_rows > 0) {
    // The checkpoint layout arrives in pieces; once the last byte is in, it is repacked into the
    // tile layout (src/kernels/repack.ts:17-209).
    std::vector<uint8_t> &st = ctx->t16_staging[name];
    st.resize(total);
    memcpy(st.data() + offset, bytes, n);
    uint64_t &got = ctx->t16_received[name];
    got += n;
    if (got >= total) {
      void *tmp = nullptr;
      CK(ctx_malloc(&tmp, total));
      cudaError_t e = cudaMemcpy(tmp, st.data(), total, cudaMemcpyHostToDevice);
      if (e == cudaSuccess) e = launch_repack_tile16(tmp, r.ptr, r.t16_rows, r.t16_k, ctx->st);
      if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->st);
      cudaFree(tmp);
      ctx->t16_staging.erase(name);
      ctx->t16_received.erase(name);
      CK(e);
    }
  } else if (!r.sliced) {
    CK(cudaMemcpy((uint8_t *)r.ptr + offset, bytes, n, cudaMemcpyHostToDevice));
  } else {
    const uint64_t slice_bytes = (uint64_t)ctx->ple_rps * (ctx->ple_cols / 2);
    uint64_t done = 0;
    while (done < n) {
      uint64_t pos = offset + done;
      uint64_t si = pos / slice_bytes, so = pos % slice_bytes;
      uint64_t take = std::min(n - done, slice_bytes - so);
      CK(cudaMemcpy((uint8_t *)ctx->ple_slices[si] + so, (const uint8_t *)bytes + done, take, cudaMemcpyHostToDevice));
      done += take;
    }
  }
  ctx->shadow_dirty = ctx->shadow != nullptr;
  ctx->weights_ready = true;
  return G4_OK;
}

extern "C" int g4_download_weight(g4_ctx *ctx, const char *name, void *bytes, uint64_t *n) {
  if (!ctx || !name || !n) return fail(ctx, G4_ERR_INVALID, "g4_download_weight: null argument");
  TensorRef r;
  int rc = find_tensor(ctx, name, &r);
  if (rc) return rc;
  if (!bytes || *n < r.bytes) {
    *n = r.bytes;
    return bytes ? fail(ctx, G4_ERR_INVALID, "%s needs %llu bytes", name, (unsigned long long)r.bytes) : G4_OK;
  }
  CK(cudaSetDevice(ctx->dev));
  CK(cudaStreamSynchronize(ctx->st));
  if (r.t16_rows > 0) {
    void *tmp = nullptr;
    CK(ctx_malloc(&tmp, r.bytes));
    cudaError_t e = launch_tile16_to_rows(r.ptr, tmp, r.t16_rows, r.t16_k, ctx->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->st);
    if (e == cudaSuccess) e = cudaMemcpy(bytes, tmp, r.bytes, cudaMemcpyDeviceToHost);
    cudaFree(tmp);
    CK(e);
  } else if (!r.sliced) {
    CK(cudaMemcpy(bytes, r.ptr, r.bytes, cudaMemcpyDeviceToHost));
  } else {
    const uint64_t row_bytes = ctx->ple_cols / 2;
    uint64_t off = 0;
    for (size_t i = 0; i < ctx->ple_slices.size(); i++) {
      uint64_t rows = std::min((uint64_t)ctx->ple_rps, (uint64_t)ctx->V - i * ctx->ple_rps);
      CK(cudaMemcpy((uint8_t *)bytes + off, ctx->ple_slices[i], rows * row_bytes, cudaMemcpyDeviceToHost));
      off += rows * row_bytes;
    }
  }
  *n = r.bytes;
  return G4_OK;
}

static Linear *linear_by_module(g4_ctx *ctx, const std::string &mod) {
  if (mod == "lm_head") return &ctx->lm;
  for (int L = 0; L < ctx->NL; L++) {
    Layer &ly = ctx->layers[L];
    Linear *all[] = {&ly.q, &ly.k, &ly.v, &ly.o, &ly.gate, &ly.up, &ly.down, &ly.pleg, &ly.plep};
    for (Linear *l : all)
      if (l->w && l->module == mod) return l;
  }
  return nullptr;
}

static bool parse_scalar(g4_ctx *ctx, const std::string &name, float **slot) {
  static const char *sfx[] = {".input_activation_scale", ".output_activation_scale"};
  for (int i = 0; i < 2; i++) {
    size_t ls = strlen(sfx[i]);
    if (name.size() > ls && name.compare(name.size() - ls, ls, sfx[i]) == 0) {
      Linear *l = linear_by_module(ctx, name.substr(0, name.size() - ls));
      if (!l) return false;
      *slot = i == 0 ? &l->in_scale : &l->out_scale;
      return true;
    }
  }
  int L;
  char tail[64];
  if (sscanf(name.c_str(), "model.language_model.layers.%d.%63s", &L, tail) == 2 &&
      strcmp(tail, "layer_scalar") == 0 && L >= 0 && L < ctx->NL) {
    *slot = &ctx->layers[L].layer_scalar;
    return true;
  }
  return false;
}

extern "C" int g4_set_scalar(g4_ctx *ctx, const char *name, float value) {
  if (!ctx || !name) return fail(ctx, G4_ERR_INVALID, "g4_set_scalar: null argument");
  float *slot;
  if (!parse_scalar(ctx, name, &slot)) return fail(ctx, G4_ERR_NOT_FOUND, "unknown scalar %s", name);
  *slot = value;
  for (auto &kv : ctx->graphs) cudaGraphExecDestroy(kv.second);
  ctx->graphs.clear();
  return G4_OK;
}

extern "C" int g4_get_scalar(const g4_ctx *cctx, const char *name, float *value) {
  g4_ctx *ctx = const_cast<g4_ctx *>(cctx);
  if (!ctx || !name || !value) return fail(ctx, G4_ERR_INVALID, "g4_get_scalar: null argument");
  float *slot;
  if (!parse_scalar(ctx, name, &slot)) return fail(ctx, G4_ERR_NOT_FOUND, "unknown scalar %s", name);
  *value = *slot;
  return G4_OK;
}

// =============================================================================== executor

struct Seg {
  const Linear *lin;
  float *y;
};

static std::string seg_roles(std::initializer_list<Seg> segs) {
  std::string r;
  for (auto &sg : segs) r += (r.empty() ? "" : ",") + short_module(sg.lin->module);
  return r;
}

static std::string layer_role(int L, bool kv_store) {
  return "layers." + std::to_string(L) + ".self_attn" + (kv_store ? ",kv_store" : "");
}

static std::string bits_name(const char *family, int bits, bool head = false) {
  return std::string(family) + "-" + std::to_string(bits) + "bit" + (head ? "-head" : "");
}

struct WRef {
  const void *p;
  uint64_t bytes;
};

static WRef wref(const Linear &l) {
  return {l.w, l.w ? (uint64_t)l.N * l.K * l.bits / 8 : 0};
}

// One quantized linear launch (or several, 8 columns each) with a fused prologue, streaming its
// weights; `prefetch` names weights of later launches to pull into L2 meanwhile.
static const CUtensorMap *codes_tmap(g4_ctx *ctx, int buf, int K, int bn) {
  auto key = std::make_tuple(buf, K, bn);
  auto it = ctx->tmx.find(key);
  if (it != ctx->tmx.end()) return &it->second;
  CUtensorMap m;
  if (make_tmap_u8(&m, ctx->gq[buf], (uint64_t)K, (uint64_t)ctx->gq_rows, (uint64_t)ctx->gq_ld, 128, bn, true))
    return nullptr;
  return &(ctx->tmx[key] = m);
}

// The tensor-core path of a linear launch group: the prologue runs once per column into int8
// codes (one code vector per distinct input scale), then one tcgen05 GEMM per segment.
static bool gemm_eligible(g4_ctx *ctx, std::initializer_list<Seg> segs, int cols, const GemvArgs &p) {
  // Precomputed codes reach the tensor-core path only in its own code buffer (attention writes
  // o_proj's there).
  if (cols < ctx->gemm_min_cols || (p.pro == PRO_CODES && p.src_codes != ctx->gq[0]) || p.epi != EPI_Y || p.pair)
    return false;
  for (auto &sg : segs)
    if (!sg.lin->has_tm || sg.lin->in_scale == 0.0f || sg.lin->K % 128 != 0) return false;
  return true;
}

static int run_linear_gemm(g4_ctx *ctx, std::initializer_list<Seg> segs, int cols, GemvArgs q, bool head) {
  const int K = segs.begin()->lin->K;
  float sc[3];
  int nsc = 0, which[3];
  int i = 0;
  for (auto &sg : segs) {
    int j = 0;
    while (j < nsc && sc[j] != sg.lin->in_scale) j++;
    if (j == nsc) sc[nsc++] = sg.lin->in_scale;
    which[i++] = j;
  }
  q.K = K;
  q.cols = cols;
  // Wide steps read the int8 copies (no unpack in the GEMM); the int32 sums are the same.
  bool sh = ctx->shadow && !ctx->shadow_dirty && cols >= ctx->shadow_min_cols;
  for (auto &sg : segs) sh = sh && sg.lin->w8 && sg.lin->has_tm8;
  auto wmap = [&](const Linear &l) -> const CUtensorMap & { return sh ? l.tmw8 : l.tmw; };
  auto wbits = [&](const Linear &l) { return sh ? 8 : l.bits; };
  if (q.pro != PRO_CODES) {
    CK(launch_quantize(q, ctx->gq[0], ctx->gq_ld, sc[0], nsc > 1 ? ctx->gq[1] : nullptr, nsc > 1 ? sc[1] : 0.0f,
                       ctx->st, true));
    note_launch(ctx, "quantize", seg_roles(segs));
  }
  if (nsc > 2) {
    q.hidden_out = nullptr;
    CK(launch_quantize(q, ctx->gq[2], ctx->gq_ld, sc[2], nullptr, 0.0f, ctx->st, true));
    note_launch(ctx, "quantize", seg_roles(segs));
  }
  // Token tile: 64 or 128 columns; wider steps use 128-column tiles at two CTAs per SM (one
  // CTA's epilogue runs while the other's MMAs do), or 256-column tiles one per SM.
  int bn = cols <= 64 || cols > 128 && cols <= 512 ? 64 : (cols <= 128 ? 128 : ctx->gemm_wide_bn);
  if (cols > 128 && bn == 64) {
    // 129-512 columns: 64-token tiles where the launch is small enough to split K or to merge
    // segments; a group with two SMs' worth of 64-token tiles or more (a box step's gate/up)
    // keeps 128-token tiles, which unpack each weight tile for twice the tokens.
    int xt = 0;
    for (auto &sg : segs) xt += (sg.lin->N + 127) / 128;
    if (xt * ((cols + 63) / 64) >= 2 * ctx->sms) bn = ctx->gemm_wide_bn;
  }
  const int nseg = (int)segs.size();
  bool same_bits = true;
  for (auto &sg : segs) same_bits = same_bits && wbits(*sg.lin) == wbits(*segs.begin()->lin);
  if (nseg > 1 && nseg <= 3 && !head && (bn == 64 || bn == -128) && same_bits && ctx->gemm_split_k != 2) {
    // q/k/v or gate/up: one launch, the segments' tiles end to end along x, each CTA with its
    // segment's weight and code tensor maps; with 64-token tiles, few tiles split K over a cluster.
    GemmMaps m;
    memset(&m, 0, sizeof(m));
    GemmArgs g;
    memset(&g, 0, sizeof(g));
    int tb = 0, si = 0;
    for (auto &sg : segs) {
      const Linear &l = *sg.lin;
      const CUtensorMap *tx = codes_tmap(ctx, which[si], K, bn < 0 ? -bn : bn);
      if (!tx) return fail(ctx, G4_ERR_CUDA, "activation-code tensor map for K %d failed", K);
      m.w[si] = wmap(l);
      m.x[si] = *tx;
      if (si == 0) {
        g.N = l.N;
        g.s = l.s;
        g.in_scale = l.in_scale;
        g.out_scale = l.out_scale;
        g.y = sg.y;
        g.ld_y = l.N;
      } else {
        g.more[si - 1] = {l.N, l.s, l.in_scale, l.out_scale, sg.y, l.N};
      }
      g.tile_begin[si] = tb;
      tb += (l.N + 127) / 128;
      si++;
    }
    g.tile_begin[nseg] = tb;
    g.nseg = nseg;
    g.K = K;
    g.M = cols;
    // Up to two CTAs per SM over all (row, token) tiles (the cluster kernel drops to three
    // stages past one per SM).
    const int all_tiles = tb * ((cols + 63) / 64);
    int splits = 1;
    if (ctx->gemm_split_k == 0 && bn == 64)
      while (splits < 8 && 2 * splits * all_tiles <= 2 * ctx->sms && 2 * splits <= K / 128) splits *= 2;
    g.splits = splits;
    CK(launch_qgemm_multi(m, g, wbits(*segs.begin()->lin), bn, ctx->st, true));
    note_launch(ctx, bits_name("qgemm", wbits(*segs.begin()->lin)), seg_roles(segs));
    return G4_OK;
  }
  i = 0;
  for (auto &sg : segs) {
    const Linear &l = *sg.lin;
    const CUtensorMap *tx = codes_tmap(ctx, which[i++], K, bn < 0 ? -bn : bn);
    if (!tx) return fail(ctx, G4_ERR_CUDA, "activation-code tensor map for K %d failed", K);
    GemmArgs g;
    memset(&g, 0, sizeof(g));
    g.N = l.N;
    g.K = K;
    g.M = cols;
    g.s = l.s;
    g.in_scale = l.in_scale;
    g.out_scale = l.out_scale;
    g.y = sg.y;
    g.ld_y = l.N;
    const int tiles = ((l.N + 127) / 128) * ((cols + std::abs(bn) - 1) / std::abs(bn));
    const int kts = K / 128;
    if (ctx->gemm_split_k == 0 && !head && bn == 64 && tiles < ctx->sms) {
      // A launch of fewer tiles than SMs (a decode batch: 2 to 48 tiles) splits K over a cluster
      // of 2, 4 or 8 CTAs per tile, as many as two per SM hold, each with at least one K stage.
      int splits = 1;
      while (splits < 8 && 2 * splits * tiles <= 2 * ctx->sms && 2 * splits <= kts) splits *= 2;
      if (splits > 1) {
        g.splits = splits;
        CK(launch_qgemm_cluster(wmap(l), *tx, g, wbits(l), ctx->st, true));
        note_launch(ctx, bits_name("qgemm", wbits(l)), short_module(l.module));
        continue;
      }
    }
    // The workspace form (int32 atomics into a global buffer, the tile's last split finishes)
    // pays only where a launch has very few tiles and a long K loop (the down projection of a
    // decode batch: 12 tiles x 48 K stages).
    const bool few_long = tiles <= 24 && kts >= 16;
    if (ctx->gemm_split_k == 2 && few_long && !head && tiles < ctx->sms && l.N <= ctx->gacc_ld && tiles <= 8192) {
      g.splits = std::min(kts, (ctx->sms + tiles - 1) / tiles);
      if (g.splits > 1) {
        g.acc_ws = ctx->gacc;
        g.ld_ws = ctx->gacc_ld;
        g.tile_cnt = ctx->gcnt;
      }
    }
    if (head) {
      g.head = 1;
      g.softcap = q.softcap;
      g.logits = ctx->logits;
      g.ld_logits = ctx->V;
      g.part_val = ctx->gpv;
      g.part_idx = ctx->gpi;
      g.n_parts = (l.N + gemm_tile_rows() - 1) / gemm_tile_rows();
      ctx->cur_pv = ctx->gpv;
      ctx->cur_pi = ctx->gpi;
      ctx->cur_parts = g.n_parts;
    }
    // The persistent tile loop (epilogue overlapping the next tile's MMAs) measured 6% slower on a
    // 2048-token prefill than two per-tile CTAs per SM (tail imbalance, twice the DRAM reads), so
    // the executor keeps the per-tile kernel; g4_op_qgemm uses the loop for wide calls.
    const int tiles128 = ((l.N + 127) / 128) * ((cols + 127) / 128);
    if (ctx->gemm_persist && !head && g.splits <= 1 && tiles128 > ctx->sms && wbits(l) != 2) {
      const CUtensorMap *tx128 = codes_tmap(ctx, which[i - 1], K, 128);
      if (!tx128) return fail(ctx, G4_ERR_CUDA, "activation-code tensor map for K %d failed", K);
      CK(launch_qgemm_persist(wmap(l), *tx128, g, wbits(l), std::min(tiles128, ctx->sms), ctx->st, true));
    } else {
      // Many 64-token tiles (the lm_head of a decode batch: 2,048): three stages, two CTAs per SM,
      // so one CTA's epilogue runs beside the other's main loop.
      const int bn_l = bn == 64 && tiles >= 2 * ctx->sms ? -64 : bn;
      CK(launch_qgemm(wmap(l), *tx, g, wbits(l), bn_l, ctx->st, true));
    }
    note_launch(ctx, bits_name("qgemm", wbits(l), head), short_module(l.module));
  }
  return G4_OK;
}

static int run_linear(g4_ctx *ctx, std::initializer_list<Seg> segs, int cols, GemvArgs proto,
                      bool head = false, std::initializer_list<WRef> prefetch = {}) {
  if (gemm_eligible(ctx, segs, cols, proto)) return run_linear_gemm(ctx, segs, cols, proto, head);
  const Linear *l0 = segs.begin()->lin;
  for (int c0 = 0; c0 < cols; c0 += 8) {
    GemvArgs a = proto;
    a.K = l0->K;
    a.cols = std::min(8, cols - c0);
    a.nseg = 0;
    for (auto &s : segs) {
      GemvSeg &g = a.seg[a.nseg++];
      g.w = s.lin->w;
      g.s = s.lin->s;
      g.y = s.y ? s.y + (size_t)c0 * s.lin->N : nullptr;
      g.acc_out = nullptr;
      g.N = s.lin->N;
      g.in_scale = s.lin->in_scale;
      g.out_scale = s.lin->out_scale;
    }
    const int blocks = l0->bits == 2 ? gemv2_partition(a, ctx->gemv_target)
                                     : gemv_stream_partition(a, ctx->gemv_target);
    int np = 0;
    if (c0 == 0)
      for (auto &w : prefetch)
        if (np < 4 && w.p) {
          a.prefetch[np] = w.p;
          a.prefetch_bytes[np++] = w.bytes;
        }
    if (a.src) a.src += (size_t)c0 * a.ld_src;
    if (a.res) a.res += (size_t)c0 * a.ld_res;
    if (a.hidden_out) a.hidden_out += (size_t)c0 * a.ld_res;
    if (a.up) a.up += (size_t)c0 * a.ld_up;
    if (a.epi_up) a.epi_up += (size_t)c0 * a.epi_ld_up;
    if (a.codes_out) a.codes_out += (size_t)c0 * a.codes_ld;
    if (a.src_codes) a.src_codes += (size_t)c0 * a.ld_codes;
    if (head) {
      if (blocks > ctx->head_cap || c0 + a.cols > ctx->head_cols)
        return fail(ctx, G4_ERR_STATE, "head launch of %d CTAs x %d columns exceeds its partial buffers (%d x %d)",
                    blocks, c0 + a.cols, ctx->head_cap, ctx->head_cols);
      a.head = 1;
      a.logits = ctx->logits + (size_t)c0 * ctx->V;
      a.ld_logits = ctx->V;
      a.part_val = ctx->head_pv + (size_t)c0 * blocks;
      a.part_idx = ctx->head_pi + (size_t)c0 * blocks;
      ctx->head_blocks = blocks;
      ctx->cur_pv = ctx->head_pv;
      ctx->cur_pi = ctx->head_pi;
      ctx->cur_parts = blocks;
    }
    CK(launch_gemv(a, l0->bits, ctx->st, true));
    note_launch(ctx, bits_name("qgemv", l0->bits, head), seg_roles(segs));
  }
  return G4_OK;
}

static GemvArgs pro_args(int pro) {
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.pro = pro;
  a.alpha = 1.0f;
  return a;
}

// Record the launches of one step: `cols` columns (already staged in d_step), layers
// [0, n_layers), then the head when asked. Step order is planDecodeStep / planPrefillChunk
// (src/plan.ts:487-824) with the fusions of the decode plan.
// One forward step over `cols` columns through `n_layers` layers. head: every column runs the
// lm_head and its argmax. wide: the columns are consecutive positions of one sequence (a prefill
// chunk, or a verify pass when head is set), so attention stores every column's KV row first and
// then attends causally; otherwise (a decode step) each column is its own sequence and one fused
// launch per layer stores and attends.
static int record_step(g4_ctx *ctx, int cols, int n_layers, bool head, bool advance = false,
                       bool wide = false) {
  const g4_arch &a = ctx->cfg.arch;
  const bool fused_attn = head && !wide;
  const int H = ctx->H, PD = ctx->PD;
  const float eps = a.rms_eps;
  int32_t *d_seq = ctx->d_step, *d_pos = ctx->d_step + ctx->maxc, *d_tok = ctx->d_step + 2 * ctx->maxc;
  ctx->launches = 0;
  ctx->roles.clear();
  // ---- embed phase (planEmbed, src/plan.ts:727-736)
  CK(launch_embed(d_tok, cols, ctx->embed_w, ctx->embed_s, (float)std::sqrt((double)H),
                  (const uint8_t *const *)ctx->d_ple_slices, ctx->ple_rps, ctx->ple_s, H,
                  ctx->ple_cols, PD, ctx->res[0], ctx->ple_id, ctx->st, true, ctx->lm.bits));
  // Per-layer inputs of the layers this step runs (rows are layer-major): a prefill chunk's
  // producer-only columns need the first n_layers groups only.
  CK(launch_dense_bf16(ctx->plmp_w, ctx->res[0], H, ctx->ple_proj, ctx->ple_cols, n_layers * PD, H, cols,
                       (float)std::pow((double)H, -0.5), ctx->st, true));
  CK(launch_ple_combine(ctx->ple_proj, ctx->ple_id, ctx->plmp_norm, ctx->ple_in, cols, n_layers, PD,
                        ctx->ple_cols, eps, (float)0.7071067811865476, ctx->st, true));
  note_launch(ctx, "embed-gather", "embed_tokens,embed_tokens_per_layer");
  note_launch(ctx, "dense-bf16", "per_layer_model_projection");
  note_launch(ctx, "ple-combine", "per_layer_projection_norm");
  int cur = 0;
  int rc;
  for (int L = 0; L < n_layers; L++) {
    Layer &ly = ctx->layers[L];
    const int hd = ly.hd, nh = a.query_heads, qrows = nh * hd;
    // ---- q, k, v with the input norm (layer 0) or the previous layer's tail join fused in
    {
      GemvArgs p;
      if (L == 0) {
        p = pro_args(PRO_NORM);
        p.src = ctx->res[cur];
        p.ld_src = H;
        p.g1 = ly.ln_in;
      } else {
        Layer &pv = ctx->layers[L - 1];
        p = pro_args(PRO_JOIN);
        p.src = ctx->proj;
        p.ld_src = H;
        p.res = ctx->res[cur];
        p.ld_res = H;
        p.g1 = pv.ln_post_ple;
        p.g2 = ly.ln_in;
        p.alpha = pv.layer_scalar;
        p.hidden_out = ctx->res[cur ^ 1];
      }
      p.eps = eps;
      if (ly.producer)
        rc = run_linear(ctx, {{&ly.q, ctx->q}, {&ly.k, ctx->k}, {&ly.v, ctx->v}}, cols, p, false,
                        {wref(ly.gate), wref(ly.up)});
      else
        rc = run_linear(ctx, {{&ly.q, ctx->q}}, cols, p, false, {wref(ly.gate), wref(ly.up)});
      if (rc) return rc;
      if (L > 0) cur ^= 1;
    }
    // o_proj's input codes come straight from the attention kernel (fused decode, query-tiled
    // prefill): into the tensor-core path's code buffer, or in the streaming GEMV's order.
    const bool o_gemm = gemm_eligible(ctx, {{&ly.o, ctx->proj}}, cols, pro_args(PRO_X));
    AttnCodes oc;
    memset(&oc, 0, sizeof(oc));
    if (ly.o.in_scale != 0.0f && (fused_attn || cols > 1) && (o_gemm || ly.o.bits == 4 || ly.o.bits == 8))
      oc = o_gemm ? AttnCodes{ctx->gq[0], ctx->gq_ld, ly.o.in_scale, 8}
                  : AttnCodes{ctx->codes_attn, qrows, ly.o.in_scale, ly.o.bits};
    // ---- decode steps: prologue, attention and merge in one launch per layer
    if (fused_attn) {
      AttnDec ad;
      memset(&ad, 0, sizeof(ad));
      ad.cols = cols;
      ad.hd = hd;
      ad.window = ly.global ? 0 : a.sliding_window;
      ad.max_ctx = ctx->cfg.max_context;
      ad.max_seqs = ctx->cfg.max_seqs;
      ad.max_blocks = ly.global ? ctx->att_blocks_global : ctx->att_blocks_sliding;
      ad.q = ctx->q;
      ad.q_ld = qrows;
      ad.k = ly.producer ? ctx->k : nullptr;
      ad.v = ly.producer ? ctx->v : nullptr;
      ad.qgain = ly.q_norm;
      ad.kgain = ly.k_norm;
      ad.cos_tab = ly.global ? ctx->cos_g : ctx->cos_s;
      ad.sin_tab = ly.global ? ctx->sin_g : ctx->sin_s;
      ad.cache = ctx->kv[ly.cache_layer];
      ad.seq_stride = ctx->kv_stride[ly.cache_layer];
      ad.refs.seq = d_seq;
      ad.refs.pos = d_pos;
      ad.part_o = ctx->part_o;
      ad.part_m = ctx->part_m;
      ad.part_l = ctx->part_l;
      ad.counter = ctx->att_count;
      ad.out = ctx->attn;
      ad.eps = eps;
      ad.codes = oc;
      CK(launch_attn_decode(ad, ctx->st, true));
      note_launch(ctx, "attention-decode", layer_role(L, ly.producer));
    }
    // ---- attention prologue: q-norm-rope, kv-norm-rope-store (src/kernels/attnPrologue.ts)
    if (!fused_attn) {
      AttnPro ap;
      memset(&ap, 0, sizeof(ap));
      ap.cols = cols;
      ap.heads = nh;
      ap.hd = hd;
      ap.q = ctx->q;
      ap.q_ld = qrows;
      ap.k = ly.producer ? ctx->k : nullptr;
      ap.v = ly.producer ? ctx->v : nullptr;
      ap.kv_ld = hd;
      ap.qgain = ly.q_norm;
      ap.kgain = ly.k_norm;
      ap.cos_tab = ly.global ? ctx->cos_g : ctx->cos_s;
      ap.sin_tab = ly.global ? ctx->sin_g : ctx->sin_s;
      ap.tab_row = d_pos;
      ap.rows_per_col_tab = 1;
      ap.qr = ctx->qr;
      ap.cache = ly.producer ? ctx->kv[L] : nullptr;
      ap.seq_stride = ly.producer ? ctx->kv_stride[L] : 0;
      ap.max_ctx = ctx->cfg.max_context;
      ap.refs.seq = d_seq;
      ap.refs.pos = d_pos;
      ap.eps = eps;
      CK(launch_attn_prologue(ap, ctx->st, true));
      note_launch(ctx, "attn-prologue", layer_role(L, ly.producer));
    }
    // ---- attention over the producer cache (kvRoleForLayer)
    if (!fused_attn) {
      AttnArgs at;
      memset(&at, 0, sizeof(at));
      at.cols = cols;
      at.heads = nh;
      at.hd = hd;
      at.window = ly.global ? 0 : a.sliding_window;
      at.max_ctx = ctx->cfg.max_context;
      at.kv_cap = 0;
      at.qr = ctx->qr;
      at.cache = ctx->kv[ly.cache_layer];
      at.seq_stride = ctx->kv_stride[ly.cache_layer];
      at.refs.seq = d_seq;
      at.refs.pos = d_pos;
      at.max_blocks = ly.global ? ctx->att_blocks_global : ctx->att_blocks_sliding;
      at.part_o = ctx->part_o;
      at.part_m = ctx->part_m;
      at.part_l = ctx->part_l;
      at.out = ctx->attn;
      if (cols > 1) {
        at.codes = oc;
        // A prefill chunk: consecutive positions of one sequence, query-tiled.
        CK(launch_attention_prefill(at, ctx->st, true));
        note_launch(ctx, "attention-prefill", layer_role(L, false));
      } else {
        CK(launch_attention(at, ctx->st, true));
        note_launch(ctx, "attention-blocks", layer_role(L, false));
        note_launch(ctx, "attention-merge", layer_role(L, false));
      }
    }
    // ---- o_proj
    {
      GemvArgs p = pro_args(oc.out ? PRO_CODES : PRO_X);
      p.src = ctx->attn;
      p.ld_src = qrows;
      if (oc.out) {
        p.src = nullptr;
        p.src_codes = oc.out;
        p.ld_codes = oc.ld;
      }
      if ((rc = run_linear(ctx, {{&ly.o, ctx->proj}}, cols, p, false, {wref(ly.down)}))) return rc;
    }
    // gelu(gate) * up is formed once, by the gate/up launch (each CTA owns the same rows of
    // both), and handed to down_proj as its int8 codes; likewise gelu(pleg) * per-layer input
    // for per_layer_projection. Needs calibrated scales on all three linears.
    const bool gemm_step = cols >= ctx->gemm_min_cols;
    const bool mlp_codes = !gemm_step && ly.gate.N == ly.up.N && ly.gate.bits == ly.up.bits &&
                           ly.gate.in_scale != 0.0f && ly.up.in_scale != 0.0f &&
                           ly.down.in_scale != 0.0f && ly.down.K <= ctx->ffn_max;
    const bool ple_codes = !gemm_step && ly.pleg.in_scale != 0.0f && ly.plep.in_scale != 0.0f && ly.plep.K == PD;
    // ---- gate, up with the post-attention join fused in (alpha 1)
    {
      GemvArgs p = pro_args(PRO_JOIN);
      if (mlp_codes) {
        p.pair = 1;
        p.epi = EPI_GELU_CODES;
        p.codes_out = ctx->codes_mlp;
        p.codes_ld = ctx->ffn_max;
        p.codes_scale = ly.down.in_scale;
        p.codes_bits = ly.down.bits;
      }
      p.src = ctx->proj;
      p.ld_src = H;
      p.res = ctx->res[cur];
      p.ld_res = H;
      p.g1 = ly.ln_post_attn;
      p.g2 = ly.ln_pre_ffn;
      p.alpha = 1.0f;
      p.hidden_out = ctx->res[cur ^ 1];
      p.eps = eps;
      if ((rc = run_linear(ctx, {{&ly.gate, ctx->gate}, {&ly.up, ctx->up}}, cols, p, false,
                           {wref(ly.pleg), wref(ly.plep)})))
        return rc;
      cur ^= 1;
    }
    // ---- down_proj over gelu(gate) * up (codes from the gate/up launch, or the gelu prologue)
    {
      GemvArgs p = pro_args(mlp_codes ? PRO_CODES : PRO_GELU);
      p.src = ctx->gate;
      p.ld_src = ly.gate.N;
      p.up = ctx->up;
      p.ld_up = ly.up.N;
      p.up_off = 0;
      if (mlp_codes) {
        p.src = nullptr;
        p.up = nullptr;
        p.src_codes = ctx->codes_mlp;
        p.ld_codes = ctx->ffn_max;
      }
      const Layer *nx = L + 1 < n_layers ? &ctx->layers[L + 1] : nullptr;
      if ((rc = run_linear(ctx, {{&ly.down, ctx->proj}}, cols, p, false,
                           {nx ? wref(nx->q) : WRef{nullptr, 0}, nx ? wref(nx->k) : WRef{nullptr, 0},
                            nx ? wref(nx->v) : WRef{nullptr, 0}})))
        return rc;
    }
    // A decode step of 1..16 columns on the GEMV path runs the per-layer-input tail (post-FFN
    // norm-residual, gate, gelu x per-layer input, projection) as one cluster launch
    // (g4_ple.cu); it gives the two GEMVs' bits.
    bool ple_fused = ple_codes && cols <= 16 && ly.pleg.bits == 8 && ly.plep.bits == 8 &&
                     ly.pleg.N == PD && ly.pleg.K == H && ly.plep.N == H && ly.plep.K == PD;
    if (ple_fused && ctx->ple_block < 0) ctx->ple_block = ple_block_fits(H, PD, 16) ? 1 : 0;
    ple_fused = ple_fused && ctx->ple_block == 1;
    if (ple_fused) {
      PleArgs pa;
      memset(&pa, 0, sizeof(pa));
      pa.src = ctx->proj;
      pa.ld_src = H;
      pa.res = ctx->res[cur];
      pa.ld_res = H;
      pa.g1 = ly.ln_post_ffn;
      pa.eps = eps;
      pa.hidden_out = ctx->res[cur ^ 1];
      pa.w1 = ly.pleg.w;
      pa.s1 = ly.pleg.s;
      pa.in1 = ly.pleg.in_scale;
      pa.out1 = ly.pleg.out_scale;
      pa.w2 = ly.plep.w;
      pa.s2 = ly.plep.s;
      pa.in2 = ly.plep.in_scale;
      pa.out2 = ly.plep.out_scale;
      pa.ple_in = ctx->ple_in;
      pa.ld_ple = ctx->ple_cols;
      pa.ple_off = L * PD;
      pa.y = ctx->proj;
      pa.ld_y = H;
      pa.cols = cols;
      pa.H = H;
      const Layer *nx = L + 1 < n_layers ? &ctx->layers[L + 1] : nullptr;
      if (nx) {
        const WRef pf[3] = {wref(nx->o), wref(nx->gate), wref(nx->up)};
        for (int i = 0; i < 3; i++) {
          pa.prefetch[i] = pf[i].p;
          pa.prefetch_bytes[i] = pf[i].bytes;
        }
      }
      CK(launch_ple_block(pa, ctx->st, true));
      note_launch(ctx, "ple-block", short_module(ly.pleg.module) + "," + short_module(ly.plep.module));
      cur ^= 1;
    }
    // ---- per_layer_input_gate over the post-FFN norm-residual (the residual itself)
    if (!ple_fused) {
      GemvArgs p = pro_args(PRO_NORMRES);
      p.src = ctx->proj;
      p.ld_src = H;
      p.res = ctx->res[cur];
      p.ld_res = H;
      p.g1 = ly.ln_post_ffn;
      p.hidden_out = ctx->res[cur ^ 1];
      p.eps = eps;
      if (ple_codes) {
        p.epi = EPI_GELU_CODES;
        p.epi_up = ctx->ple_in;
        p.epi_ld_up = ctx->ple_cols;
        p.epi_up_off = L * PD;
        p.codes_out = ctx->codes_ple;
        p.codes_ld = PD;
        p.codes_scale = ly.plep.in_scale;
        p.codes_bits = ly.plep.bits;
      }
      const Layer *nx = L + 1 < n_layers ? &ctx->layers[L + 1] : nullptr;
      if ((rc = run_linear(ctx, {{&ly.pleg, ctx->pleg_out}}, cols, p, false,
                           {nx ? wref(nx->o) : WRef{nullptr, 0}})))
        return rc;
      cur ^= 1;
    }
    // ---- per_layer_projection over gelu(gate) * the layer's per-layer input row
    if (!ple_fused) {
      GemvArgs p = pro_args(ple_codes ? PRO_CODES : PRO_GELU);
      p.src = ctx->pleg_out;
      p.ld_src = PD;
      p.up = ctx->ple_in;
      p.ld_up = ctx->ple_cols;
      p.up_off = L * PD;
      if (ple_codes) {
        p.src = nullptr;
        p.up = nullptr;
        p.src_codes = ctx->codes_ple;
        p.ld_codes = PD;
      }
      const Layer *nx = L + 1 < n_layers ? &ctx->layers[L + 1] : nullptr;
      if ((rc = run_linear(ctx, {{&ly.plep, ctx->proj}}, cols, p, false,
                           {nx ? wref(nx->gate) : WRef{nullptr, 0}, nx ? wref(nx->up) : WRef{nullptr, 0}})))
        return rc;
    }
  }
  if (head) {
    Layer &last = ctx->layers[n_layers - 1];
    GemvArgs p = pro_args(PRO_JOIN);
    p.src = ctx->proj;
    p.ld_src = H;
    p.res = ctx->res[cur];
    p.ld_res = H;
    p.g1 = last.ln_post_ple;
    p.g2 = ctx->final_norm;
    p.alpha = last.layer_scalar;
    p.hidden_out = ctx->res[cur ^ 1];
    p.eps = eps;
    p.softcap = a.final_softcap;
    if ((rc = run_linear(ctx, {{&ctx->lm, nullptr}}, cols, p, true))) return rc;
    CK(launch_argmax_final(ctx->cur_pv, ctx->cur_pi, ctx->cur_parts, cols, d_tok,
                           ctx->d_tok_out, ctx->d_val_out, ctx->st, true, &ctx->errf, ctx->d_tok_out + cols));
    if (advance) CK(launch_advance(d_pos, cols, ctx->st, true));
    note_launch(ctx, "argmax-final", "argmax");
    if (advance) note_launch(ctx, "advance", "position advance");
  }
  return G4_OK;
}

static int run_step(g4_ctx *ctx, int cols, int n_layers, bool head, bool advance = false,
                    bool wide = false) {
  if (!ctx->cfg.use_graphs) return record_step(ctx, cols, n_layers, head, advance, wide);
  GraphKey key{cols, n_layers, head ? (wide ? 2 : 1) : 0, advance ? 1 : 0};
  auto it = ctx->graphs.find(key);
  if (it == ctx->graphs.end()) {
    // First use: run eagerly (sets kernel attributes, validates), then capture.
    int rc = record_step(ctx, cols, n_layers, head, advance, wide);
    if (rc) return rc;
    int launches = ctx->launches;
    std::vector<std::string> roles = ctx->roles;
    CK(cudaStreamSynchronize(ctx->st));
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(ctx->st, cudaStreamCaptureModeThreadLocal));
    rc = record_step(ctx, cols, n_layers, head, advance, wide);
    cudaError_t e = cudaStreamEndCapture(ctx->st, &g);
    if (rc) return rc;
    CK(e);
    cudaGraphExec_t ex;
    CK(cudaGraphInstantiate(&ex, g, 0));
    cudaGraphDestroy(g);
    ctx->graphs[key] = ex;
    ctx->graph_launches[key] = launches;
    ctx->graph_roles[key] = roles;
    ctx->launches = launches;
    ctx->roles = roles;
    // The eager run already advanced the step; the graph serves the next calls.
    return G4_OK;
  }
  CK(cudaGraphLaunch(it->second, ctx->st));
  ctx->launches = ctx->graph_launches[key];
  ctx->roles = ctx->graph_roles[key];
  return G4_OK;
}

static int check_seq_pos(g4_ctx *ctx, int32_t seq, int32_t pos, int32_t n) {
  if (!ctx->weights_ready) return fail(ctx, G4_ERR_STATE, "no weights: call g4_init_random or g4_upload_weight first");
  if (seq < 0 || seq >= ctx->cfg.max_seqs) return fail(ctx, G4_ERR_INVALID, "sequence %d outside 0..%d", seq, ctx->cfg.max_seqs - 1);
  if (pos < 0 || n < 1 || pos + n > ctx->cfg.max_context)
    return fail(ctx, G4_ERR_INVALID, "positions %d..%d outside the context of %d", pos, pos + n - 1, ctx->cfg.max_context);
  if (pos > ctx->kv_len[seq])
    return fail(ctx, G4_ERR_INVALID, "position %d leaves a gap after the %d cached positions of sequence %d", pos, ctx->kv_len[seq], seq);
  return G4_OK;
}

// Rebuild the int8 weight copies after a weight change (before any step uses them).
static int refresh_shadows(g4_ctx *ctx) {
  if (!ctx->shadow_dirty) return G4_OK;
  auto widen = [&](Linear &l) -> cudaError_t {
    return l.w8 ? launch_widen_weights(l.w, l.bits, l.N, l.K, l.w8, ctx->st) : cudaSuccess;
  };
  for (Layer &ly : ctx->layers)
    for (Linear *l : {&ly.q, &ly.k, &ly.v, &ly.o, &ly.gate, &ly.up, &ly.down}) CK(widen(*l));
  CK(widen(ctx->lm));
  ctx->shadow_dirty = false;
  return G4_OK;
}

// Copy one step's columns into the device step buffer. The pinned source slot is rewritten only
// once the copy that last read it has executed on the stream (consecutive prefill chunks are
// enqueued without a host wait).
static int stage(g4_ctx *ctx, int cols, const int32_t *seqs, const int32_t *pos, const int32_t *toks,
                 bool tokens_too) {
  int rc = refresh_shadows(ctx);
  if (rc) return rc;
  const int slot = ctx->stage_next;
  ctx->stage_next = (slot + 1) % g4_ctx::kStageSlots;
  CK(cudaEventSynchronize(ctx->stage_ev[slot]));
  int32_t *h = ctx->h_step[slot];
  for (int i = 0; i < cols; i++) {
    h[i] = seqs[i];
    h[ctx->maxc + i] = pos[i];
    if (tokens_too) h[2 * ctx->maxc + i] = toks[i];
  }
  CK(cudaMemcpyAsync(ctx->d_step, h, (size_t)ctx->maxc * 4 * (tokens_too ? 3 : 2), cudaMemcpyHostToDevice, ctx->st));
  CK(cudaEventRecord(ctx->stage_ev[slot], ctx->st));
  return G4_OK;
}

// The step's tokens and its error word in one copy; the flags themselves are read (and cleared)
// only when the word says one is set.
static int fetch_tokens(g4_ctx *ctx, int cols, int32_t *out) {
  CK(cudaMemcpyAsync(ctx->h_tok, ctx->d_tok_out, (size_t)(cols + 1) * 4, cudaMemcpyDeviceToHost, ctx->st));
  CK(cudaStreamSynchronize(ctx->st));
  if (ctx->h_tok[cols] != 0 && (device_error_take() > 0 || gemm_error_take() > 0 || ple_error_take() > 0)) {
    // A block that gave up may have left its column's finished-block count behind.
    cudaMemsetAsync(ctx->att_count, 0, (size_t)ctx->maxc * 8 * 4, ctx->st);
    cudaStreamSynchronize(ctx->st);
    return fail(ctx, G4_ERR_TIMEOUT, "a bounded device wait gave up (a bulk copy never completed)");
  }
  for (int i = 0; i < cols; i++) out[i] = ctx->h_tok[i];
  return G4_OK;
}

extern "C" int g4_prefill(g4_ctx *ctx, int32_t seq, const int32_t *ids, int32_t n, int32_t start_pos,
                          int32_t is_last, int32_t *out_token) {
  if (!ctx || !ids) return fail(ctx, G4_ERR_INVALID, "g4_prefill: null argument");
  int rc = check_seq_pos(ctx, seq, start_pos, n);
  if (rc) return rc;
  for (int i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= ctx->V) return fail(ctx, G4_ERR_INVALID, "token id %d outside the vocabulary", ids[i]);
  CK(cudaSetDevice(ctx->dev));
  const int nl_all = ctx->NL, nl_prod = ctx->cfg.arch.kv_producer_layers;
  std::vector<int32_t> sq(ctx->maxc, seq), ps(ctx->maxc);
  // A last chunk runs every layer and the head on its final position; the positions before it
  // need all layers only for their KV (which only producers write), so they run as the
  // producer-only chunk (src/plan.ts:160-192, 812-824).
  int body = is_last ? n - 1 : n;
  int launches = 0;
  std::vector<std::string> roles;
  for (int c0 = 0; c0 < body; c0 += ctx->maxc) {
    int cols = std::min(ctx->maxc, body - c0);
    for (int i = 0; i < cols; i++) ps[i] = start_pos + c0 + i;
    if ((rc = stage(ctx, cols, sq.data(), ps.data(), ids + c0, true))) return rc;
    if ((rc = record_step(ctx, cols, nl_prod, false))) return rc;
    launches += ctx->launches;
    roles.insert(roles.end(), ctx->roles.begin(), ctx->roles.end());
  }
  ctx->launches = launches;
  ctx->roles = roles;
  if (is_last) {
    ps[0] = start_pos + n - 1;
    if ((rc = stage(ctx, 1, sq.data(), ps.data(), ids + n - 1, true))) return rc;
    if ((rc = run_step(ctx, 1, nl_all, true))) return rc;
    ctx->launches += launches;
    roles.insert(roles.end(), ctx->roles.begin(), ctx->roles.end());
    ctx->roles = roles;
    int32_t tok;
    if ((rc = fetch_tokens(ctx, 1, &tok))) return rc;
    if (out_token) *out_token = tok;
  } else {
    CK(cudaStreamSynchronize(ctx->st));
    if (out_token) *out_token = -1;
  }
  ctx->kv_len[seq] = start_pos + n;
  ctx->last_cols = 1;
  return G4_OK;
}

extern "C" int g4_decode(g4_ctx *ctx, int32_t seq, int32_t prev_token, int32_t pos, int32_t *out_token) {
  if (!ctx || !out_token) return fail(ctx, G4_ERR_INVALID, "g4_decode: null argument");
  int rc = check_seq_pos(ctx, seq, pos, 1);
  if (rc) return rc;
  if (prev_token < 0 || prev_token >= ctx->V) return fail(ctx, G4_ERR_INVALID, "token id %d outside the vocabulary", prev_token);
  CK(cudaSetDevice(ctx->dev));
  if ((rc = stage(ctx, 1, &seq, &pos, &prev_token, true))) return rc;
  if ((rc = run_step(ctx, 1, ctx->NL, true))) return rc;
  if ((rc = fetch_tokens(ctx, 1, out_token))) return rc;
  ctx->kv_len[seq] = pos + 1;
  ctx->last_cols = 1;
  return G4_OK;
}

extern "C" int g4_decode_ahead(g4_ctx *ctx, int32_t seq, int32_t pos, int32_t *out_token) {
  if (!ctx || !out_token) return fail(ctx, G4_ERR_INVALID, "g4_decode_ahead: null argument");
  int rc = check_seq_pos(ctx, seq, pos, 1);
  if (rc) return rc;
  CK(cudaSetDevice(ctx->dev));
  if ((rc = stage(ctx, 1, &seq, &pos, nullptr, false))) return rc;
  if ((rc = run_step(ctx, 1, ctx->NL, true))) return rc;
  if ((rc = fetch_tokens(ctx, 1, out_token))) return rc;
  ctx->kv_len[seq] = pos + 1;
  ctx->last_cols = 1;
  return G4_OK;
}

extern "C" int g4_verify(g4_ctx *ctx, int32_t seq, const int32_t *tokens, int32_t n, int32_t pos,
                         int32_t *out_tokens) {
  if (!ctx || !tokens || !out_tokens) return fail(ctx, G4_ERR_INVALID, "g4_verify: null argument");
  const int max_n = std::min(ctx->maxc, ctx->head_cols);
  if (n < 1 || n > max_n)
    return fail(ctx, G4_ERR_INVALID, "gemma4 engine: a verify pass takes 1 to %d tokens, got %d", max_n, n);
  int rc = check_seq_pos(ctx, seq, pos, n);
  if (rc) return rc;
  for (int i = 0; i < n; i++)
    if (tokens[i] < 0 || tokens[i] >= ctx->V) return fail(ctx, G4_ERR_INVALID, "token id %d outside the vocabulary", tokens[i]);
  CK(cudaSetDevice(ctx->dev));
  std::vector<int32_t> sq(n, seq), ps(n);
  for (int i = 0; i < n; i++) ps[i] = pos + i;
  if ((rc = stage(ctx, n, sq.data(), ps.data(), tokens, true))) return rc;
  if ((rc = run_step(ctx, n, ctx->NL, true, false, n > 1))) return rc;
  if ((rc = fetch_tokens(ctx, n, out_tokens))) return rc;
  ctx->kv_len[seq] = pos + n;
  ctx->last_cols = n;
  return G4_OK;
}

extern "C" int g4_decode_batch(g4_ctx *ctx, int32_t B, const int32_t *seqs, const int32_t *tokens,
                               const int32_t *positions, int32_t *out_tokens) {
  if (!ctx || !seqs || !tokens || !positions || !out_tokens) return fail(ctx, G4_ERR_INVALID, "g4_decode_batch: null argument");
  if (B < 1 || B > ctx->maxc || B > ctx->head_cols)
    return fail(ctx, G4_ERR_INVALID, "batch %d outside 1..%d", B, std::min(ctx->maxc, ctx->head_cols));
  int rc;
  for (int i = 0; i < B; i++) {
    if ((rc = check_seq_pos(ctx, seqs[i], positions[i], 1))) return rc;
    if (tokens[i] < 0 || tokens[i] >= ctx->V) return fail(ctx, G4_ERR_INVALID, "token id %d outside the vocabulary", tokens[i]);
    for (int j = 0; j < i; j++)
      if (seqs[j] == seqs[i]) return fail(ctx, G4_ERR_INVALID, "sequence %d appears twice in one batch", seqs[i]);
  }
  CK(cudaSetDevice(ctx->dev));
  if ((rc = stage(ctx, B, seqs, positions, tokens, true))) return rc;
  if ((rc = run_step(ctx, B, ctx->NL, true))) return rc;
  if ((rc = fetch_tokens(ctx, B, out_tokens))) return rc;
  for (int i = 0; i < B; i++) ctx->kv_len[seqs[i]] = positions[i] + 1;
  ctx->last_cols = B;
  return G4_OK;
}

extern "C" int g4_step_stage(g4_ctx *ctx, int32_t B, const int32_t *seqs, const int32_t *tokens,
                             const int32_t *positions) {
  if (!ctx || !seqs || !tokens || !positions) return fail(ctx, G4_ERR_INVALID, "g4_step_stage: null argument");
  if (B < 1 || B > ctx->maxc || B > ctx->head_cols) return fail(ctx, G4_ERR_INVALID, "batch %d too wide", B);
  int rc;
  for (int i = 0; i < B; i++) {
    if ((rc = check_seq_pos(ctx, seqs[i], positions[i], 1))) return rc;
    for (int j = 0; j < i; j++)
      if (seqs[j] == seqs[i]) return fail(ctx, G4_ERR_INVALID, "sequence %d appears twice in one batch", seqs[i]);
  }
  CK(cudaSetDevice(ctx->dev));
  if ((rc = stage(ctx, B, seqs, positions, tokens, true))) return rc;
  CK(cudaStreamSynchronize(ctx->st));
  ctx->staged_cols = B;
  ctx->staged_seq.assign(seqs, seqs + B);
  ctx->staged_pos.assign(positions, positions + B);
  return G4_OK;
}

extern "C" int g4_step_run_device(g4_ctx *ctx, int32_t B, int32_t advance) {
  if (!ctx) return fail(nullptr, G4_ERR_INVALID, "null context");
  if (B < 1 || B > ctx->maxc || B > ctx->head_cols) return fail(ctx, G4_ERR_INVALID, "batch %d too wide", B);
  if (B != ctx->staged_cols) return fail(ctx, G4_ERR_STATE, "g4_step_stage staged %d columns, not %d", ctx->staged_cols, B);
  for (int i = 0; i < B; i++) {
    int32_t s = ctx->staged_seq[i], p = ctx->staged_pos[i];
    if (p >= ctx->cfg.max_context)
      return fail(ctx, G4_ERR_INVALID, "sequence %d would step past the context of %d", s, ctx->cfg.max_context);
  }
  int rc = run_step(ctx, B, ctx->NL, true, advance != 0);
  if (rc) return rc;
  for (int i = 0; i < B; i++) {
    ctx->kv_len[ctx->staged_seq[i]] = std::max(ctx->kv_len[ctx->staged_seq[i]], ctx->staged_pos[i] + 1);
    if (advance) ctx->staged_pos[i]++;
  }
  ctx->last_cols = B;
  return G4_OK;
}

extern "C" int g4_step_read_tokens(g4_ctx *ctx, int32_t B, int32_t *out_tokens) {
  if (!ctx || !out_tokens) return fail(ctx, G4_ERR_INVALID, "null argument");
  return fetch_tokens(ctx, B, out_tokens);
}

extern "C" int g4_kv_truncate(g4_ctx *ctx, int32_t seq, int32_t n) {
  if (!ctx) return fail(nullptr, G4_ERR_INVALID, "null context");
  if (seq < 0 || seq >= ctx->cfg.max_seqs) return fail(ctx, G4_ERR_INVALID, "sequence %d out of range", seq);
  if (n < 0 || n > ctx->kv_len[seq]) return fail(ctx, G4_ERR_INVALID, "truncate %d outside 0..%d", n, ctx->kv_len[seq]);
  ctx->kv_len[seq] = n;
  return G4_OK;
}

extern "C" int g4_kv_length(const g4_ctx *ctx, int32_t seq, int32_t *n) {
  if (!ctx || !n) return fail(nullptr, G4_ERR_INVALID, "null argument");
  if (seq < 0 || seq >= ctx->cfg.max_seqs) return fail(const_cast<g4_ctx *>(ctx), G4_ERR_INVALID, "sequence %d out of range", seq);
  *n = ctx->kv_len[seq];
  return G4_OK;
}

extern "C" int g4_read_logits(g4_ctx *ctx, int32_t col, float *out, int32_t n) {
  if (!ctx || !out) return fail(ctx, G4_ERR_INVALID, "g4_read_logits: null argument");
  if (col < 0 || col >= ctx->head_cols || n < 0 || n > ctx->V) return fail(ctx, G4_ERR_INVALID, "bad column or count");
  CK(cudaStreamSynchronize(ctx->st));
  CK(cudaMemcpy(out, ctx->logits + (size_t)col * ctx->V, (size_t)n * 4, cudaMemcpyDeviceToHost));
  return G4_OK;
}

// ============================================================================ operator API

#define OPCK(call)                                                                           \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess) return fail(nullptr, G4_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

static int device_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

extern "C" int g4_op_qgemv(const void *wq, const void *scales, const float *x, float in_scale,
                           float out_scale, int32_t bits, int32_t N, int32_t K, int32_t cols, float *y,
                           int32_t *acc_out, void *stream) {
  if (!wq || !scales || !x || !y) return fail(nullptr, G4_ERR_INVALID, "g4_op_qgemv: null pointer");
  if (bits != 2 && bits != 4 && bits != 8) return fail(nullptr, G4_ERR_INVALID, "bits must be 2, 4 or 8");
  // The K spans of src/kernels/qgemv.ts:1258, 1305-1310.
  const int span = bits == 2 ? 512 : (bits == 4 ? 256 : 128);
  if (N < 1 || K < span || K % span != 0 || cols < 1)
    return fail(nullptr, G4_ERR_INVALID, "qgemv-%dbit needs K a multiple of %d, got %d (N %d, cols %d)", bits, span, K, N, cols);
  if (bits == 2) {
    // The interleaved tile layout (g4_op_repack_tile16 makes it from the checkpoint's rows).
    if (K > 16384 || (in_scale == 0.0f && K > 3072))
      return fail(nullptr, G4_ERR_UNSUPPORTED, "K %d too wide for qgemv-2bit", K);
  } else {
    if (in_scale == 0.0f && cols != 1) return fail(nullptr, G4_ERR_UNSUPPORTED, "the f32 path takes one column");
    if ((size_t)K * bits / 8 > 4096 || (size_t)8 * K > 64 * 1024) return fail(nullptr, G4_ERR_UNSUPPORTED, "K %d too wide", K);
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int sms = device_sms();
  for (int c0 = 0; c0 < cols; c0 += 8) {
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    a.pro = PRO_X;
    a.alpha = 1.0f;
    a.K = K;
    a.cols = std::min(8, cols - c0);
    a.nseg = 1;
    a.seg[0].w = (const uint8_t *)wq;
    a.seg[0].s = (const uint16_t *)scales;
    a.seg[0].y = y + (size_t)c0 * N;
    a.seg[0].acc_out = acc_out ? acc_out + (size_t)c0 * N : nullptr;
    a.seg[0].N = N;
    a.seg[0].in_scale = in_scale;
    a.seg[0].out_scale = out_scale;
    a.src = x + (size_t)c0 * K;
    a.ld_src = K;
    if (bits == 2)
      gemv2_partition(a, 2 * sms);
    else
      gemv_stream_partition(a, 2 * sms);
    OPCK(launch_gemv(a, bits, st, true));
  }
  OPCK(cudaGetLastError());
  return G4_OK;
}

extern "C" int g4_op_qgemv_codes(const void *wq, const void *scales, const int8_t *codes, float in_scale,
                                 float out_scale, int32_t bits, int32_t N, int32_t K, int32_t cols, float *y,
                                 int32_t *acc_out, void *stream) {
  if (!wq || !scales || !codes || !y) return fail(nullptr, G4_ERR_INVALID, "g4_op_qgemv_codes: null pointer");
  if (bits != 2 && bits != 4 && bits != 8) return fail(nullptr, G4_ERR_INVALID, "bits must be 2, 4 or 8");
  if (in_scale == 0.0f) return fail(nullptr, G4_ERR_INVALID, "int8 activation codes need their scale (in_scale != 0)");
  const int span = bits == 2 ? 512 : (bits == 4 ? 256 : 128);
  if (N < 1 || K < span || K % span != 0 || cols < 1)
    return fail(nullptr, G4_ERR_INVALID, "qgemv-%dbit needs K a multiple of %d, got %d (N %d, cols %d)", bits, span, K, N, cols);
  if (K > 16384 || (bits != 2 && (size_t)K * bits / 8 > 4096))
    return fail(nullptr, G4_ERR_UNSUPPORTED, "K %d too wide", K);
  cudaStream_t st = (cudaStream_t)stream;
  const int sms = device_sms();
  for (int c0 = 0; c0 < cols; c0 += 8) {
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    a.pro = PRO_CODES;
    a.alpha = 1.0f;
    a.K = K;
    a.cols = std::min(8, cols - c0);
    a.nseg = 1;
    a.seg[0].w = (const uint8_t *)wq;
    a.seg[0].s = (const uint16_t *)scales;
    a.seg[0].y = y + (size_t)c0 * N;
    a.seg[0].acc_out = acc_out ? acc_out + (size_t)c0 * N : nullptr;
    a.seg[0].N = N;
    a.seg[0].in_scale = in_scale;
    a.seg[0].out_scale = out_scale;
    a.src_codes = (const uint8_t *)codes + (size_t)c0 * K;
    a.ld_codes = K;
    a.codes_plain = 1;
    if (bits == 2)
      gemv2_partition(a, 2 * sms);
    else
      gemv_stream_partition(a, 2 * sms);
    OPCK(launch_gemv(a, bits, st, true));
  }
  OPCK(cudaGetLastError());
  return G4_OK;
}

extern "C" int g4_op_qgemm(const void *wq, const void *scales, const float *x, float in_scale,
                           float out_scale, int32_t bits, int32_t N, int32_t K, int32_t cols, float *y,
                           void *stream) {
  if (!wq || !scales || !x || !y) return fail(nullptr, G4_ERR_INVALID, "g4_op_qgemm: null pointer");
  if (bits != 2 && bits != 4 && bits != 8) return fail(nullptr, G4_ERR_INVALID, "bits must be 2, 4 or 8");
  const int span = bits == 2 ? 512 : (bits == 4 ? 256 : 128);
  if (N < 1 || K < span || K % span != 0 || cols < 1)
    return fail(nullptr, G4_ERR_INVALID, "qgemm-%dbit needs K a multiple of %d, got %d (N %d, cols %d)", bits, span, K, N, cols);
  if (in_scale == 0.0f) return fail(nullptr, G4_ERR_UNSUPPORTED, "the tensor-core path needs a calibrated site");
  if (K > 16384) return fail(nullptr, G4_ERR_UNSUPPORTED, "K %d too wide", K);
  cudaStream_t st = (cudaStream_t)stream;
  const int rows = std::max(cols, 256);
  uint8_t *codes = nullptr;
  OPCK(cudaMallocAsync(&codes, (size_t)rows * K, st));
  OPCK(cudaMemsetAsync(codes, 0, (size_t)rows * K, st));
  GemvArgs q;
  memset(&q, 0, sizeof(q));
  q.pro = PRO_X;
  q.alpha = 1.0f;
  q.K = K;
  q.cols = cols;
  q.src = x;
  q.ld_src = K;
  cudaError_t e = launch_quantize(q, codes, K, in_scale, nullptr, 0.0f, st, false);
  CUtensorMap tw, tx;
  // Token tiles: 64, 128, 128 at two CTAs per SM (up to 256 columns), then the persistent tile
  // loop (128-column tiles).
  const bool persist = cols > 256 && bits != 2;
  const int bn = cols <= 64 ? 64 : (cols <= 128 ? 128 : -128);
  const int bnv = bn < 0 ? -bn : bn;
  const uint64_t rb = (uint64_t)K * bits / 8;
  int rc = G4_OK;
  if (e == cudaSuccess) {
    const int wmap = bits == 2 ? make_tmap_u32(&tw, wq, (uint64_t)K, (uint64_t)((N + 15) / 16), (uint64_t)K * 4, 128, 8)
                               : make_tmap_u8(&tw, wq, rb, (uint64_t)N, rb, bits == 4 ? 64 : 128, 128, bits == 8);
    if (wmap ||
        make_tmap_u8(&tx, codes, (uint64_t)K, (uint64_t)rows, (uint64_t)K, 128, bnv, true)) {
      rc = fail(nullptr, G4_ERR_CUDA, "tensor map encoding failed");
    } else {
      GemmArgs g;
      memset(&g, 0, sizeof(g));
      g.N = N;
      g.K = K;
      g.M = cols;
      g.s = (const uint16_t *)scales;
      g.in_scale = in_scale;
      g.out_scale = out_scale;
      g.y = y;
      g.ld_y = N;
      // The executor's rule: fewer tiles than SMs split K, over a thread-block cluster for
      // 64-token tiles, else through an int32 workspace (both exact).
      const int tiles = ((N + 127) / 128) * ((cols + bnv - 1) / bnv);
      const int sms = device_sms();
      int32_t *ws = nullptr;
      bool cluster = false;
      if (bn == 64 && tiles < sms) {
        int splits = 1;
        while (splits < 8 && 2 * splits * tiles <= sms && 2 * splits <= K / 128) splits *= 2;
        if (splits > 1) {
          g.splits = splits;
          cluster = true;
        }
      } else if (tiles < sms && tiles <= 8192) {
        g.splits = std::min(K / 128, (sms + tiles - 1) / tiles);
        if (g.splits > 1) {
          e = cudaMallocAsync(&ws, ((size_t)cols * N + 8192) * 4, st);
          if (e == cudaSuccess) e = cudaMemsetAsync(ws, 0, ((size_t)cols * N + 8192) * 4, st);
          g.acc_ws = ws;
          g.ld_ws = N;
          g.tile_cnt = ws + (size_t)cols * N;
        }
      }
      if (e == cudaSuccess) {
        if (cluster)
          e = launch_qgemm_cluster(tw, tx, g, bits, st, false);
        else if (persist && g.splits <= 1)
          e = launch_qgemm_persist(tw, tx, g, bits, std::min(tiles, sms), st, false);
        else
          e = launch_qgemm(tw, tx, g, bits, bn == 64 && tiles >= 2 * sms ? -64 : bn, st, false);
      }
      if (ws) cudaFreeAsync(ws, st);
    }
  }
  cudaFreeAsync(codes, st);
  if (rc) return rc;
  OPCK(e);
  OPCK(cudaGetLastError());
  return G4_OK;
}

extern "C" int g4_op_repack_tile16(const void *row_words, void *tile_words, int32_t N, int32_t K,
                                   int32_t to_rows, void *stream) {
  if (!row_words || !tile_words || N < 1 || K < 16 || K % 16)
    return fail(nullptr, G4_ERR_INVALID, "g4_op_repack_tile16: bad argument (N %d, K %d)", N, K);
  cudaStream_t st = (cudaStream_t)stream;
  if (to_rows)
    OPCK(launch_tile16_to_rows(tile_words, (void *)row_words, N, K, st));
  else
    OPCK(launch_repack_tile16(row_words, tile_words, N, K, st));
  return G4_OK;
}

extern "C" int g4_op_qgemv_gelu(const void *wq, const void *scales, const float *gate, const float *up,
                                int32_t up_offset, int32_t up_stride, float in_scale, float out_scale,
                                int32_t bits, int32_t N, int32_t K, int32_t cols, float *y, void *stream) {
  if (!wq || !scales || !gate || !up || !y) return fail(nullptr, G4_ERR_INVALID, "g4_op_qgemv_gelu: null pointer");
  const int span = bits == 4 ? 256 : 128;
  if ((bits != 4 && bits != 8) || N < 1 || K < span || K % span || cols < 1)
    return fail(nullptr, G4_ERR_INVALID, "bad qgemv-gelu shape");
  if (in_scale == 0.0f && cols != 1) return fail(nullptr, G4_ERR_UNSUPPORTED, "the f32 path takes one column");
  if ((size_t)K * bits / 8 > 4096 || (size_t)8 * K > 64 * 1024) return fail(nullptr, G4_ERR_UNSUPPORTED, "K %d too wide", K);
  cudaStream_t st = (cudaStream_t)stream;
  const int sms = device_sms();
  for (int c0 = 0; c0 < cols; c0 += 8) {
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    a.pro = PRO_GELU;
    a.alpha = 1.0f;
    a.K = K;
    a.cols = std::min(8, cols - c0);
    a.nseg = 1;
    a.seg[0].w = (const uint8_t *)wq;
    a.seg[0].s = (const uint16_t *)scales;
    a.seg[0].y = y + (size_t)c0 * N;
    a.seg[0].N = N;
    a.seg[0].in_scale = in_scale;
    a.seg[0].out_scale = out_scale;
    a.src = gate + (size_t)c0 * K;
    a.ld_src = K;
    a.up = up + (size_t)c0 * up_stride;
    a.ld_up = up_stride;
    a.up_off = up_offset;
    gemv_stream_partition(a, 2 * sms);
    OPCK(launch_gemv(a, bits, st, true));
  }
  return G4_OK;
}

static int check_width(int width) {
  if (width < 4 || width % 4 != 0) return fail(nullptr, G4_ERR_INVALID, "width %d must be a positive multiple of 4", width);
  return G4_OK;
}

extern "C" int g4_op_rms_norm(const float *src, const float *gain, float *dst, int32_t rows,
                              int32_t width, float eps, void *stream) {
  if (!src || !dst || rows < 1) return fail(nullptr, G4_ERR_INVALID, "g4_op_rms_norm: bad argument");
  if (int rc = check_width(width)) return rc;
  OPCK(launch_rms_norm(src, gain, dst, rows, width, eps, (cudaStream_t)stream));
  return G4_OK;
}

extern "C" int g4_op_norm_residual(const float *src, const float *gain, const float *residual,
                                   float *dst, int32_t rows, int32_t width, float eps, void *stream) {
  if (!src || !gain || !residual || !dst || rows < 1) return fail(nullptr, G4_ERR_INVALID, "g4_op_norm_residual: bad argument");
  if (int rc = check_width(width)) return rc;
  OPCK(launch_norm_residual(src, gain, residual, dst, rows, width, eps, (cudaStream_t)stream));
  return G4_OK;
}

extern "C" int g4_op_norm_residual_norm(const float *src, const float *gain, const float *residual,
                                        const float *gain2, float alpha, float *hidden, float *dst,
                                        int32_t rows, int32_t width, float eps, void *stream) {
  if (!src || !gain || !residual || !gain2 || !hidden || !dst || rows < 1)
    return fail(nullptr, G4_ERR_INVALID, "g4_op_norm_residual_norm: bad argument");
  if (int rc = check_width(width)) return rc;
  OPCK(launch_norm_residual_norm(src, gain, residual, gain2, alpha, hidden, dst, rows, width, eps, (cudaStream_t)stream));
  return G4_OK;
}

extern "C" int g4_op_gelu_mul(const float *gate, const float *up, float *dst, int32_t n, float srq_scale,
                              void *stream) {
  if (!gate || !up || !dst || n < 1) return fail(nullptr, G4_ERR_INVALID, "g4_op_gelu_mul: bad argument");
  OPCK(launch_gelu_mul(gate, up, dst, n, srq_scale, (cudaStream_t)stream));
  return G4_OK;
}

extern "C" int g4_op_q_norm_rope(const float *src, const float *gain, const float *cos_tab,
                                 const float *sin_tab, float *dst, int32_t rows, int32_t width,
                                 int32_t rows_per_position, float eps, void *stream) {
  if (!src || !gain || !cos_tab || !sin_tab || !dst || rows < 1 || rows_per_position < 1)
    return fail(nullptr, G4_ERR_INVALID, "g4_op_q_norm_rope: bad argument");
  if (width % 8 != 0 || width > 4096) return fail(nullptr, G4_ERR_INVALID, "width %d unsupported", width);
  AttnPro a;
  memset(&a, 0, sizeof(a));
  a.cols = rows;
  a.heads = 1;
  a.hd = width;
  a.q = src;
  a.q_ld = width;
  a.qgain = gain;
  a.cos_tab = cos_tab;
  a.sin_tab = sin_tab;
  a.rows_per_col_tab = rows_per_position;
  a.qr = dst;
  a.eps = eps;
  OPCK(launch_attn_prologue(a, (cudaStream_t)stream, false));
  return G4_OK;
}

extern "C" int g4_op_kv_norm_rope_store(const float *k, const float *v, const float *gain,
                                        const float *cos_tab, const float *sin_tab, float *cache,
                                        int32_t tokens, int32_t head_dim, int32_t start_pos,
                                        int32_t max_context, float eps, void *stream) {
  if (!k || !v || !gain || !cos_tab || !sin_tab || !cache || tokens < 1)
    return fail(nullptr, G4_ERR_INVALID, "g4_op_kv_norm_rope_store: bad argument");
  if (start_pos < 0 || start_pos + tokens > max_context)
    return fail(nullptr, G4_ERR_INVALID, "rows %d..%d outside 0..%d", start_pos, start_pos + tokens - 1, max_context - 1);
  if (head_dim % 8 != 0 || head_dim > 4096) return fail(nullptr, G4_ERR_INVALID, "head_dim %d unsupported", head_dim);
  AttnPro a;
  memset(&a, 0, sizeof(a));
  a.cols = tokens;
  a.heads = 0;
  a.hd = head_dim;
  a.k = k;
  a.v = v;
  a.kv_ld = head_dim;
  a.kgain = gain;
  a.cos_tab = cos_tab;
  a.sin_tab = sin_tab;
  a.rows_per_col_tab = 1;
  a.cache = cache;
  a.seq_stride = 0;
  a.max_ctx = max_context;
  a.refs.pos_base = start_pos;
  a.eps = eps;
  OPCK(launch_attn_prologue(a, (cudaStream_t)stream, false));
  return G4_OK;
}

extern "C" int g4_op_attention(const float *q, const float *cache, float *out, int32_t heads,
                               int32_t head_dim, int32_t q_count, int32_t q_start, int32_t kv_len,
                               int32_t window, int32_t max_context, void *stream) {
  if (!q || !cache || !out) return fail(nullptr, G4_ERR_INVALID, "g4_op_attention: null pointer");
  if (heads != 8) return fail(nullptr, G4_ERR_UNSUPPORTED, "the attention kernel is built for 8 query heads");
  if (head_dim != 256 && head_dim != 512) return fail(nullptr, G4_ERR_UNSUPPORTED, "head_dim 256 or 512");
  if (q_count < 1 || q_start < 0 || kv_len < 1 || q_start + q_count > kv_len || kv_len > max_context)
    return fail(nullptr, G4_ERR_INVALID, "attention: query positions extend past kv_len; store KV before attending");
  int max_blocks = window > 0 ? (window + 63) / 64 + 1 : (kv_len + 63) / 64;
  cudaStream_t st = (cudaStream_t)stream;
  float *scratch = nullptr;
  size_t n_o = (size_t)q_count * max_blocks * heads * head_dim, n_ml = (size_t)q_count * max_blocks * heads;
  OPCK(cudaMallocAsync((void **)&scratch, (n_o + 2 * n_ml) * 4, st));
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.cols = q_count;
  a.heads = heads;
  a.hd = head_dim;
  a.window = window;
  a.max_ctx = max_context;
  a.kv_cap = kv_len;
  a.qr = q;
  a.cache = cache;
  a.seq_stride = 0;
  a.refs.pos_base = q_start;
  a.max_blocks = max_blocks;
  a.part_o = scratch;
  a.part_m = scratch + n_o;
  a.part_l = scratch + n_o + n_ml;
  a.out = out;
  cudaError_t e = launch_attention(a, st, false);
  cudaFreeAsync(scratch, st);
  OPCK(e);
  return G4_OK;
}

extern "C" int g4_op_attention_prefill(const float *q, const float *cache, float *out, int32_t heads,
                                       int32_t head_dim, int32_t q_count, int32_t q_start, int32_t kv_len,
                                       int32_t window, int32_t max_context, void *stream) {
  if (!q || !cache || !out) return fail(nullptr, G4_ERR_INVALID, "g4_op_attention_prefill: null pointer");
  if (heads != 8) return fail(nullptr, G4_ERR_UNSUPPORTED, "the attention kernel is built for 8 query heads");
  if (head_dim != 256 && head_dim != 512) return fail(nullptr, G4_ERR_UNSUPPORTED, "head_dim 256 or 512");
  if (q_count < 1 || q_start < 0 || kv_len < 1 || q_start + q_count > kv_len || kv_len > max_context)
    return fail(nullptr, G4_ERR_INVALID, "attention: query positions extend past kv_len; store KV before attending");
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.cols = q_count;
  a.heads = heads;
  a.hd = head_dim;
  a.window = window;
  a.max_ctx = max_context;
  a.qr = q;
  a.cache = cache;
  a.refs.pos_base = q_start;
  a.out = out;
  OPCK(launch_attention_prefill(a, (cudaStream_t)stream, false));
  return G4_OK;
}

extern "C" int g4_op_embed_gather(const void *codes, const void *scales, const int32_t *ids, float *dst,
                                  int32_t slots, int32_t cols, int32_t group_size, float out_scale,
                                  int32_t slice_start, int32_t slice_rows, void *stream) {
  if (!codes || !scales || !ids || !dst || slots < 1) return fail(nullptr, G4_ERR_INVALID, "g4_op_embed_gather: bad argument");
  if (cols % 8 != 0 || group_size < 8 || group_size % 8 != 0 || cols % group_size != 0)
    return fail(nullptr, G4_ERR_INVALID, "embed gather: cols %d / group %d", cols, group_size);
  OPCK(launch_embed_op((const uint8_t *)codes, (const uint16_t *)scales, ids, dst, slots, cols,
                       group_size, out_scale, slice_start, slice_rows, (cudaStream_t)stream, false));
  return G4_OK;
}

extern "C" int g4_op_dense_bf16(const void *w, const float *x, float *y, int32_t N, int32_t K,
                                int32_t cols, float alpha, void *stream) {
  if (!w || !x || !y || N < 1 || cols < 1) return fail(nullptr, G4_ERR_INVALID, "g4_op_dense_bf16: bad argument");
  if (K % 8 != 0 || K > 2048) return fail(nullptr, G4_ERR_UNSUPPORTED, "dense K %d (multiple of 8 up to 2048)", K);
  OPCK(launch_dense_bf16((const uint16_t *)w, x, K, y, N, N, K, cols, alpha, (cudaStream_t)stream, false));
  return G4_OK;
}

extern "C" int g4_op_softcap_argmax(const float *logits, float *capped, int32_t *token, int32_t n,
                                    float cap, void *stream) {
  if (!logits || !token || n < 1) return fail(nullptr, G4_ERR_INVALID, "g4_op_softcap_argmax: bad argument");
  cudaStream_t st = (cudaStream_t)stream;
  int parts = (n + 4095) / 4096;
  float *pv = nullptr;
  OPCK(cudaMallocAsync((void **)&pv, (size_t)parts * 8, st));
  int32_t *pi = (int32_t *)(pv + parts);
  cudaError_t e = launch_softcap_partials(logits, capped, n, cap, pv, pi, parts, st);
  // token[0] = index, token[1] = the value's bits.
  if (e == cudaSuccess) e = launch_argmax_final(pv, pi, parts, 1, nullptr, token, (float *)(token + 1), st, false);
  cudaFreeAsync(pv, st);
  OPCK(e);
  return G4_OK;
}

extern "C" int g4_op_wait_probe(const void *src, int32_t bytes, int32_t missing_bytes,
                                int32_t poll_limit, int32_t *status, void *stream) {
  if (!src || !status || bytes < 16 || bytes > 4096 || bytes % 16 || ((uintptr_t)src & 15) ||
      missing_bytes < 0 || missing_bytes > (1 << 20) || poll_limit < 1 || poll_limit > (1 << 22))
    return fail(nullptr, G4_ERR_INVALID, "g4_op_wait_probe: bad argument");
  if (device_error_take() < 0) return fail(nullptr, G4_ERR_CUDA, "g4_op_wait_probe: cannot read the device error flag");
  OPCK(launch_wait_probe(src, bytes, missing_bytes, poll_limit, status, (cudaStream_t)stream));
  OPCK(cudaStreamSynchronize((cudaStream_t)stream));
  if (device_error_take() > 0)
    return fail(nullptr, G4_ERR_TIMEOUT, "a bounded device wait gave up after %d polls (its barrier "
                "expected %d bytes that no copy delivers)", poll_limit, missing_bytes);
  return G4_OK;
}

extern "C" int g4_op_math_probe(const float *x, float *exp_out, float *tanh_out, float *cuda_exp,
                                float *cuda_tanh, int32_t n, void *stream) {
  if (!x || !exp_out || !tanh_out || !cuda_exp || !cuda_tanh || n < 1)
    return fail(nullptr, G4_ERR_INVALID, "g4_op_math_probe: bad argument");
  OPCK(launch_math_probe(x, exp_out, tanh_out, cuda_exp, cuda_tanh, n, (cudaStream_t)stream));
  return G4_OK;
}
