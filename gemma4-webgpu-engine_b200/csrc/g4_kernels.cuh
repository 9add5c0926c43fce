// g4_kernels.cuh -- launch interface of the sm_100a kernels (internal to libgemma4_cuda.so).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

namespace g4 {

// Runs a set-up function once per (call site, CUDA device). Function attributes such as the
// dynamic shared-memory limit belong to the device that is current when they are set, so a
// process that drives several devices must set them on each. Thread-safe; device ordinals past
// 63 run the set-up on every call.
struct DeviceOnce {
  std::atomic<uint64_t> done{0};
  std::mutex m;
  template <class F>
  void operator()(F &&f) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
      f();
      return;
    }
    const uint64_t bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return;
    std::lock_guard<std::mutex> g(m);
    if (done.load(std::memory_order_relaxed) & bit) return;
    f();
    done.fetch_or(bit, std::memory_order_release);
  }
};

// A kernel launch, chained to the previous kernel of the stream by programmatic dependent launch
// when `pdl` is set (the kernel then calls griddepcontrol.wait before reading its inputs).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t st, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// Activation prologue a quantized linear applies before snapping its input to int8 codes.
enum Prologue : int {
  PRO_X = 0,        // x = src
  PRO_NORM = 1,     // x = norm(src) * g1
  PRO_JOIN = 2,     // h = (res + norm(src) * g1) * alpha -> hidden_out; x = norm(h) * g2
  PRO_NORMRES = 3,  // h = res + norm(src) * g1 -> hidden_out; x = h
  PRO_GELU = 4,     // x = gelu(src) * up[up_off + k]
  PRO_CODES = 5,    // the int8 codes themselves, precomputed by the producing launch
};

// Epilogues of the streaming GEMV.
enum Epilogue : int {
  EPI_Y = 0,           // y rows to seg.y
  EPI_GELU_CODES = 1,  // h = gelu(y0) * (pair ? y1 : epi_up[epi_up_off + r]), stored as the
                       // next linear's int8 codes (codes_scale, codes_bits layout)
  EPI_HEAD = 2,        // lm_head: softcap, logits, per-CTA argmax partials (set through `head`)
};

// Byte offset of activation element k inside a column's code vector. int8 and 2-bit weights read
// codes in order; int4 weights read each 8-element group as [x0 x2 x4 x6 | x1 x3 x5 x7] (even and
// odd nibbles of a packed word).
__host__ __device__ __forceinline__ int code_pos(int k, int bits) {
  if (bits != 4) return k;
  return (k & ~7) + 2 * ((k >> 2) & 1) + 4 * (k & 1) + ((k >> 1) & 1);
}

struct GemvSeg {
  const uint8_t *w;    // packed codes, row-major [N, K * bits / 8]
  const uint16_t *s;   // f16 row scales [N]
  float *y;            // [cols, N]
  int32_t *acc_out;    // optional exact accumulators [cols, N]
  int N;
  int block_begin;     // first block index of this segment in the launch
  float in_scale, out_scale;
};

struct GemvArgs {
  GemvSeg seg[3];
  int nseg;
  int K;
  int cols;
  int pro;
  const float *src; int ld_src;
  const float *res; int ld_res;
  const float *g1; const float *g2; float alpha; float eps;
  float *hidden_out;   // PRO_JOIN / PRO_NORMRES: written by block 0, ld = ld_res
  const float *up; int ld_up; int up_off;
  // lm_head epilogue: softcap, optional logits store, per-block argmax partials
  int head;
  float softcap;
  float *logits; int ld_logits;
  float *part_val; int32_t *part_idx; int n_blocks_total;
  // Weights of later steps to pull into L2 while this launch runs (split across its CTAs).
  const void *prefetch[4]; uint64_t prefetch_bytes[4];
  // Set by launch_gemv_stream: shared-memory ring bytes and the most rows any CTA owns.
  int ring_bytes; int max_rows;
  // pair: seg[0] and seg[1] have the same N and every CTA owns the same rows of both.
  int pair;
  int epi;
  const float *epi_up; int epi_ld_up; int epi_up_off;
  uint8_t *codes_out; int codes_ld; float codes_scale; int codes_bits;
  const uint8_t *src_codes; int ld_codes;   // PRO_CODES
  int codes_plain;   // PRO_CODES at 4 bits: src_codes in K order (the operator API), else dp4a order
};

// The streaming GEMV: one CTA per SM (or fewer), each streaming a contiguous row slice of one
// segment through a shared-memory ring filled by TMA bulk copies. Fills seg[i].block_begin and
// n_blocks_total for `sms` CTAs and returns the CTA count.
int gemv_stream_partition(GemvArgs &a, int sms);
cudaError_t launch_gemv_stream(const GemvArgs &a, int bits, cudaStream_t st, bool pdl);
// Nonzero when a bounded device wait gave up since the last call (then cleared).
int device_error_take();
cudaError_t launch_wait_probe(const void *src, int bytes, int missing, int limit, int32_t *status,
                              cudaStream_t st);
#ifdef G4_TRACE
// Diagnostic build only: the (kernel id, time) records since the last call, then cleared.
int trace_take(unsigned long long *out, int max_records);
int gemm_trace_take(unsigned long long *out, int max_records);
int ple_trace_take(unsigned long long *out, int max_records);
#endif

// A quantized linear launch (the streaming kernel, or the f32 path when in_scale is 0).
// Calibrated launches need gemv_stream_partition first.
cudaError_t launch_gemv(const GemvArgs &a, int bits, cudaStream_t st, bool pdl);

// The 2-bit family on the interleaved 16-row tile layout: tile t (rows 16t .. 16t + 15) is K u32
// words, word k holding row 16t + i at bits 2i (src/kernels/qlayout.ts:160-234). Weight bytes of
// a 2-bit linear are ceil(N / 16) * K * 4. launch_gemv2 needs gemv2_partition first; a segment
// with in_scale 0.0 runs the f32 path.
cudaError_t launch_repack_tile16(const void *row_words, void *tile_words, int N, int K, cudaStream_t st);
cudaError_t launch_tile16_to_rows(const void *tile_words, void *row_words, int N, int K, cudaStream_t st);
int gemv2_partition(GemvArgs &a, int sms);
// Signed int8 row-major copy [N][K] (code - zero point) of int4 rows or 2-bit tiles.
cudaError_t launch_widen_weights(const void *w, int bits, int N, int K, void *w8, cudaStream_t st);
cudaError_t launch_gemv2(const GemvArgs &a, cudaStream_t st, bool pdl);
__host__ __device__ __forceinline__ size_t tile16_bytes(int N, int K) {
  return (size_t)((N + 15) / 16) * (size_t)K * 4;
}

// Per-column step addressing shared by the embed, attention and head kernels.
struct ColRefs {
  const int32_t *seq;   // sequence slot per column (nullable: 0)
  const int32_t *pos;   // absolute position per column (nullable: pos_base + c)
  int pos_base;
};

cudaError_t launch_embed(const int32_t *tokens, int cols, const uint8_t *embed_w,
                         const uint16_t *embed_s, float embed_scale, const uint8_t *const *ple_slices,
                         int ple_rows_per_slice, const uint16_t *ple_s, int H, int ple_cols,
                         int ple_group, float *residual, float *ple_id, cudaStream_t st, bool pdl,
                         int embed_bits = 4);

cudaError_t launch_embed_op(const uint8_t *codes, const uint16_t *scales, const int32_t *ids,
                            float *dst, int slots, int cols, int group, float out_scale,
                            int slice_start, int slice_rows, cudaStream_t st, bool pdl);

cudaError_t launch_dense_bf16(const uint16_t *w, const float *x, int ld_x, float *y, int ld_y, int N, int K,
                              int cols, float alpha, cudaStream_t st, bool pdl);

cudaError_t launch_ple_combine(const float *proj, const float *identity, const float *gain,
                               float *out, int cols, int groups, int group_dim, int row_width, float eps,
                               float scale, cudaStream_t st, bool pdl);

struct AttnPro {
  int cols, heads, hd;
  const float *q; int q_ld;          // [cols, q_ld], head h at h * hd
  const float *k; const float *v; int kv_ld;  // nullable: no KV store
  const float *qgain; const float *kgain;
  const float *cos_tab; const float *sin_tab;  // [rows, hd / 2]
  const int32_t *tab_row;            // nullable: row = c
  float *qr;                         // [cols, heads * hd]
  int rows_per_col_tab;              // op use: q rows per table row (engine: 1 column = 1 row)
  float *cache; size_t seq_stride;   // packed [2, max_ctx, hd] per sequence
  int max_ctx;
  ColRefs refs;
  float eps;
};
cudaError_t launch_attn_prologue(const AttnPro &a, cudaStream_t st, bool pdl);

// The next linear's int8 input codes, written by an attention kernel beside its f32 output
// (o_proj's snap to its input scale): out [cols][ld] at code_pos(k, bits) (bits 4: the int4
// streaming GEMV's dp4a order; 8: K order, for the tensor-core path). out NULL: not written.
struct AttnCodes {
  uint8_t *out; int ld; float scale; int bits;
};

struct AttnArgs {
  int cols, heads, hd, window, max_ctx;
  int kv_cap;                        // > 0: attend j < kv_cap as well as j <= p
  const float *qr;                   // [cols, heads * hd]
  const float *cache; size_t seq_stride;
  ColRefs refs;
  int max_blocks;                    // partial slots per column
  float *part_o; float *part_m; float *part_l;
  float *out;                        // [cols, heads * hd]
  AttnCodes codes;                   // prefill kernel only
};
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st, bool pdl);
// The same attention for a prefill chunk (columns = consecutive positions of one sequence),
// query-tiled: bit-identical to launch_attention on such a chunk.
cudaError_t launch_attention_prefill(const AttnArgs &a, cudaStream_t st, bool pdl);

// Activation codes for the tensor-core path: one CTA per column runs the GEMV prologue `a.pro`
// (norm / join / norm-residual / gelu / x) once and writes the column's int8 codes in K order
// for in_scale s1 (and s2 into codes2 when non-null); a.hidden_out, when set, gets the join.
cudaError_t launch_quantize(const GemvArgs &a, uint8_t *codes, int ld, float s1, uint8_t *codes2,
                           float s2, cudaStream_t st, bool pdl);

// Tensor-core quantized linear (g4_gemm.cu): y[M tokens][ld_y] rows < N, from weights (tensor
// map tmW: int4 packed [N][K/2] box 64 x 128, or int8 [N][K] box 128 x 128 swizzled) and the
// activation codes (tmX: int8 [tokens][K] box 128 x bn swizzled). K a multiple of 128; bn 64,
// 128 or 256. head: softcap, logits and per-128-row argmax partials [token][n_parts].
struct GemmArgs {
  int N, K, M;
  const uint16_t *s;
  float in_scale, out_scale;
  float *y; int ld_y;
  int head; float softcap;
  float *logits; int ld_logits;
  float *part_val; int32_t *part_idx; int n_parts;
  // Split K (splits > 1): each CTA adds its exact int32 partial into acc_ws[token][ld_ws] (zero on
  // entry, left zero), and the last of a tile's splits to finish (tile_cnt) runs the epilogue.
  int splits; int32_t *acc_ws; int ld_ws; int32_t *tile_cnt;
  // Several linears over the same codes width in one launch (nseg > 1, no head, no workspace
  // split): blockIdx.x in [tile_begin[i], tile_begin[i + 1]) is a 128-row tile of segment i,
  // with tensor maps GemmMaps::w[i] / x[i]. Segment 0 is N, s, in_scale, out_scale, y, ld_y
  // above; segments 1 and 2 are more[0], more[1].
  int nseg; int tile_begin[4];
  struct Seg { int N; const uint16_t *s; float in_scale, out_scale; float *y; int ld_y; } more[2];
};
struct GemmMaps {
  CUtensorMap w[3];   // weights of each segment
  CUtensorMap x[3];   // activation codes each segment reads
};
int make_tmap_u32(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer,
                  uint64_t row_stride, uint32_t box_inner, uint32_t box_outer);
int make_tmap_u8(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer,
                 uint64_t row_stride, uint32_t box_inner, uint32_t box_outer, bool swizzle128);
cudaError_t launch_qgemm(const CUtensorMap &tmW, const CUtensorMap &tmX, const GemmArgs &a, int bits,
                         int bn, cudaStream_t st, bool pdl);
// Persistent form (one CTA per SM looping over 128 x 128 tiles, two TMEM accumulators so the
// epilogue overlaps the next tile's MMAs): tmX with box rows 128; no split K.
cudaError_t launch_qgemm_persist(const CUtensorMap &tmW, const CUtensorMap &tmX, const GemmArgs &a,
                                 int bits, int grid, cudaStream_t st, bool pdl);
// K split over a thread-block cluster of a.splits (2, 4 or 8) CTAs per 128-row x 64-token tile: the
// int32 partials are reduced through distributed shared memory, no workspace. tmX: box rows 64.
cudaError_t launch_qgemm_cluster(const CUtensorMap &tmW, const CUtensorMap &tmX, const GemmArgs &a,
                                 int bits, cudaStream_t st, bool pdl);
// One launch over a.nseg segments (maps m.w[i], m.x[i]); token tile bn 64 (a.splits 2/4/8 splits
// K over a cluster) or -128 (128-token tiles, two CTAs per SM, no split).
cudaError_t launch_qgemm_multi(const GemmMaps &m, const GemmArgs &a, int bits, int bn, cudaStream_t st, bool pdl);
int gemm_error_take();
int gemm_tile_rows();

// Decode attention in one launch (every column a distinct sequence at one new position): the
// q-norm-rope of all heads, the K/V row of the new position (producer layers: k != nullptr),
// the 64-position blocks, and the merge, done by the last block of a column to finish
// (counter[c] counts finished blocks and is left at 0).
struct AttnDec {
  int cols, hd, window, max_ctx, max_seqs, max_blocks;
  const float *q; int q_ld;          // raw q rows [cols, q_ld]
  const float *k; const float *v;    // raw k / v rows [cols, hd]; nullable: cache already holds p
  const float *qgain; const float *kgain;
  const float *cos_tab; const float *sin_tab;  // row = position
  float *cache; size_t seq_stride;   // this layer's (or its producer's) cache
  ColRefs refs;
  float *part_o; float *part_m; float *part_l;
  int32_t *counter;                  // [cols][8]
  float *out;                        // [cols, 8 * hd]
  float eps;
  AttnCodes codes;
};
cudaError_t launch_attn_decode(const AttnDec &a, cudaStream_t st, bool pdl);

// The per-layer-input tail of a decode step (g4_ple.cu): the post-FFN norm-residual,
// per_layer_input_gate, gelu(gate) x the layer's per-layer input, per_layer_projection, on one
// cluster of 16 CTAs. Both linears int8, PD = 256, H a multiple of 256 up to 2048, 1..16 columns.
struct PleArgs {
  // The post-FFN norm-residual: h = res + rms_norm(src) * g1 (written to hidden_out by one CTA)
  // is the gate's input.
  const float *src; int ld_src;
  const float *res; int ld_res;                              // hidden_out has ld_res too
  const float *g1; float eps;
  float *hidden_out;
  const uint8_t *w1; const uint16_t *s1; float in1, out1;   // per_layer_input_gate [PD][H]
  const uint8_t *w2; const uint16_t *s2; float in2, out2;   // per_layer_projection [H][PD]
  const float *ple_in; int ld_ple; int ple_off;              // per-layer inputs [cols][ld_ple]
  float *y; int ld_y;                                        // [cols][H]
  const void *prefetch[4]; uint64_t prefetch_bytes[4];       // later weights to pull into L2
  int cols, H;
};
// The per-layer-input tail of a decode step of 1..16 columns as one cluster launch (g4_ple.cu).
bool ple_block_fits(int H, int PD, int cols);
size_t ple_block_smem(int H, int cols);
cudaError_t launch_ple_block(const PleArgs &a, cudaStream_t st, bool pdl);
int ple_error_take();

// Decode chain: position[c] += 1 after a step (its argmax already sits in the token slot).
cudaError_t launch_advance(int32_t *pos, int cols, cudaStream_t st, bool pdl);

// The sticky error flags of the library's kernels (one per translation unit: streaming GEMV and
// attention, 2-bit GEMV, tensor-core GEMM, per-layer-input tail), by device address.
struct ErrFlags {
  const int *p[4];
};
int *dev_error_addr();
int *gemv2_error_addr();
int *gemm_error_addr();
int *ple_error_addr();
// flag_out (optional): the OR of the flags, written once the step's earlier kernels are complete,
// so a host reads tokens and flags with one copy.
cudaError_t launch_argmax_final(const float *part_val, const int32_t *part_idx, int n_parts,
                                int cols, int32_t *token_dev, int32_t *token_out,
                                float *value_out, cudaStream_t st, bool pdl,
                                const ErrFlags *flags = nullptr, int32_t *flag_out = nullptr);

// Standalone norm / elementwise kernels (operator API).
cudaError_t launch_rms_norm(const float *src, const float *gain, float *dst, int rows, int width,
                            float eps, cudaStream_t st);
cudaError_t launch_norm_residual(const float *src, const float *gain, const float *res,
                                 float *dst, int rows, int width, float eps, cudaStream_t st);
cudaError_t launch_norm_residual_norm(const float *src, const float *gain, const float *res,
                                      const float *gain2, float alpha, float *hidden, float *dst,
                                      int rows, int width, float eps, cudaStream_t st);
cudaError_t launch_gelu_mul(const float *gate, const float *up, float *dst, int n, float srq,
                            cudaStream_t st);
cudaError_t launch_softcap_partials(const float *logits, float *capped, int n, float cap,
                                    float *part_val, int32_t *part_idx, int n_parts,
                                    cudaStream_t st);
cudaError_t launch_math_probe(const float *x, float *e, float *t, float *ce, float *ct, int n,
                              cudaStream_t st);

// Synthetic weight generators (counter hash of seed, tensor stream and element index).
cudaError_t launch_gen_words(uint32_t *dst, size_t n_words, uint64_t key, size_t index0,
                             cudaStream_t st);
cudaError_t launch_gen_f16(uint16_t *dst, size_t n, uint64_t key, double lo, double hi,
                           cudaStream_t st);
cudaError_t launch_gen_bf16_f32(float *dst, size_t n, uint64_t key, double lo, double hi,
                                cudaStream_t st);
cudaError_t launch_gen_plmp(uint16_t *dst, size_t n, uint64_t key, double amp, cudaStream_t st);

}  // namespace g4
