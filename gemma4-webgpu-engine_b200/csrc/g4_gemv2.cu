// g4_gemv2.cu -- the 2-bit weight family (the checkpoint's consumer MLP and logit head) on the
// interleaved 16-row layout of src/kernels/qlayout.ts:160-234.
//
// Codes are unsigned 0..3 with zero point 2. The checkpoint stores a row as K / 16 u32 words,
// code k at bits 2 (k % 16) of word k / 16. The kernels read the tile layout the reference
// repacks to at load (src/kernels/repack.ts:17-209): rows grouped in tiles of 16, a tile is K
// words, and word k of tile t holds row 16 t + i at bits 2 i, so one word meets one activation.
// Rows past N pad the last tile with zero codes; every store is guarded by the true row count.
//
// The GEMV (decode, up to eight columns) follows src/kernels/qgemv.ts:693-868:
//   * integer path (calibrated): pair m of a word, (w >> 2m) & 0x00030003, holds rows m and
//     m + 8 in its two 16-bit halves, and one int32 multiply by the activation code forms both
//     products. 16 k-blocks (64 words) per lane add at most 64 x 384 per half, inside 16 bits, before
//     the halves are split (sign-extend the low half, shift the rest), so every lane partial is
//     exact; sum((u - 2) x) = sum(u x) - 2 sum(x) with the column's code sum;
//   * f32 path (uncalibrated: the logit head, both scales 0.0): lane l accumulates k = 128 b +
//     4 l + j in ascending b then j with one fused multiply-add per row, keeps its own activation
//     sum, takes 2 x that sum off every row, and the lanes close with the descending XOR
//     butterfly (masks 16, 8, 4, 2, 1). The reference's WGSL has its own order here; this order
//     is fixed and stated, and the reference's f64 sum bounds both within a tolerance.
// Each CTA streams a contiguous run of tiles through a shared-memory ring filled by bulk copies
// issued before the dependency wait; a warp owns one tile (or a K-interleaved share of one when a
// stage holds fewer tiles than warps), integer shares adding exactly.
#include <cuda_fp16.h>
#include <float.h>

#include <algorithm>

#include "g4_device.cuh"
#include "g4_gemv.cuh"
#include "g4_kernels.cuh"

namespace g4 {

// Raised when a bounded wait on a weight copy gives up (device variables are per translation
// unit here, so this file keeps its own; device_error_take reads both).
__device__ int g4_gemv2_error;
#ifdef G4_TRACE
// Diagnostic build: this unit's own record buffer (device variables are per unit); its records
// are not collected.
__device__ unsigned long long g4_trace_buf[1 << 16];
__device__ unsigned int g4_trace_n;
#endif

int *gemv2_error_addr() {
  void *p = nullptr;
  return cudaGetSymbolAddress(&p, g4_gemv2_error) == cudaSuccess ? (int *)p : nullptr;
}

int gemv2_error_take() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g4_gemv2_error, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g4_gemv2_error, &zero, sizeof(int));
  return v;
}

// ------------------------------------------------------------------ layout conversion

// Row layout -> tile layout (rowWordsToTile16, src/kernels/qlayout.ts:186-206): one thread per
// tile word (tile t, column k).
__global__ void __launch_bounds__(256) k_repack_tile16(const uint32_t *row_words, uint32_t *tile_words,
                                                       int N, int K) {
  const size_t i = (size_t)blockIdx.x * 256 + threadIdx.x;
  const int tiles = (N + 15) / 16;
  if (i >= (size_t)tiles * K) return;
  const int t = (int)(i / K), k = (int)(i % K);
  const int kw = K / 16;
  uint32_t out = 0;
#pragma unroll 4
  for (int r = 0; r < 16; r++) {
    const int row = 16 * t + r;
    if (row < N) out |= ((row_words[(size_t)row * kw + k / 16] >> (2 * (k & 15))) & 3u) << (2 * r);
  }
  tile_words[i] = out;
}

// Tile layout -> row layout (tile16ToRowWords, src/kernels/qlayout.ts:209-227): one thread per
// row word.
__global__ void __launch_bounds__(256) k_tile16_to_rows(const uint32_t *tile_words, uint32_t *row_words,
                                                        int N, int K) {
  const size_t i = (size_t)blockIdx.x * 256 + threadIdx.x;
  const int kw = K / 16;
  if (i >= (size_t)N * kw) return;
  const int row = (int)(i / kw), w = (int)(i % kw);
  const uint32_t *tw = tile_words + (size_t)(row / 16) * K + 16 * w;
  const int shift = 2 * (row % 16);
  uint32_t out = 0;
#pragma unroll
  for (int j = 0; j < 16; j++) out |= ((tw[j] >> shift) & 3u) << (2 * j);
  row_words[i] = out;
}

cudaError_t launch_repack_tile16(const void *row_words, void *tile_words, int N, int K, cudaStream_t st) {
  if (N < 1 || K < 16 || K % 16) return cudaErrorInvalidValue;
  const size_t n = (size_t)((N + 15) / 16) * K;
  k_repack_tile16<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const uint32_t *)row_words,
                                                                (uint32_t *)tile_words, N, K);
  return cudaGetLastError();
}

cudaError_t launch_tile16_to_rows(const void *tile_words, void *row_words, int N, int K, cudaStream_t st) {
  if (N < 1 || K < 16 || K % 16) return cudaErrorInvalidValue;
  const size_t n = (size_t)N * (K / 16);
  k_tile16_to_rows<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const uint32_t *)tile_words,
                                                                 (uint32_t *)row_words, N, K);
  return cudaGetLastError();
}

// Signed int8 copies of packed weights for the tensor-core path (row-major [N][K], code - zero
// point): the GEMM then loads them by TMA straight into its swizzled tile with no unpack.
// int4: one thread per packed u32 (8 codes, low nibble first); 2-bit tiles: one thread per 4
// consecutive k of a row.
__global__ void __launch_bounds__(256) k_widen_int4(const uint32_t *w4, uint2 *w8, size_t words) {
  const size_t i = (size_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= words) return;
  const uint32_t w = w4[i];
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    lo |= (uint32_t)(uint8_t)((int)((w >> (4 * j)) & 15u) - 8) << (8 * j);
    hi |= (uint32_t)(uint8_t)((int)((w >> (4 * j + 16)) & 15u) - 8) << (8 * j);
  }
  w8[i] = make_uint2(lo, hi);
}

__global__ void __launch_bounds__(256) k_widen_tile16(const uint32_t *tiles, uint32_t *w8, int N, int K) {
  const size_t i = (size_t)blockIdx.x * 256 + threadIdx.x;
  const int kq = K / 4;
  if (i >= (size_t)N * kq) return;
  const int row = (int)(i / kq), k = 4 * (int)(i % kq);
  const uint32_t *tw = tiles + (size_t)(row / 16) * K + k;
  const int shift = 2 * (row % 16);
  uint32_t out = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) out |= (uint32_t)(uint8_t)((int)((tw[j] >> shift) & 3u) - 2) << (8 * j);
  w8[i] = out;
}

cudaError_t launch_widen_weights(const void *w, int bits, int N, int K, void *w8, cudaStream_t st) {
  if (N < 1 || K < 16 || K % 16) return cudaErrorInvalidValue;
  if (bits == 4) {
    const size_t words = (size_t)N * K / 8;
    k_widen_int4<<<(unsigned)((words + 255) / 256), 256, 0, st>>>((const uint32_t *)w, (uint2 *)w8, words);
  } else if (bits == 2) {
    const size_t n = (size_t)N * (K / 4);
    k_widen_tile16<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const uint32_t *)w, (uint32_t *)w8, N, K);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------ the GEMV

// Shared memory of one CTA: the ring, barriers, column sums, reduction scratch, per-warp argmax
// candidates, per-warp tile partials, the row scales of the CTA's rows, the y rows a gelu-codes
// epilogue keeps, and the activation codes (or f32 activations).
struct G2Layout {
  int bars, xsum, red, cand_v, cand_i, wpart, scales, ybuf, x, total;
};
__host__ __device__ __forceinline__ G2Layout g2_layout(int ring, int cols, int max_rows, int nsub,
                                                       bool keep_y, int K, bool f32) {
  G2Layout l;
  l.bars = ring;
  l.xsum = l.bars + GS_MAX_STAGES * 8;
  l.red = l.xsum + 16 * 4;
  l.cand_v = l.red + 8 * 4;
  l.cand_i = l.cand_v + 8 * 8 * 4;
  l.wpart = l.cand_i + 8 * 8 * 4;
  l.scales = l.wpart + 8 * 16 * 4;
  l.ybuf = l.scales + nsub * max_rows * 4;
  l.x = (l.ybuf + (keep_y ? nsub * cols * max_rows * 4 : 0) + 15) & ~15;
  l.total = l.x + (f32 ? cols * K * 4 : nsub * cols * K);
  return l;
}
constexpr int G2_MAX_SMEM = 227 * 1024;

// Sixteen per-lane row values reduced over the warp with the descending butterfly, transposed:
// at each step a lane keeps half of its rows and takes its partner's share of them. Lane l ends
// with row ((l >> 4) & 1) * 8 + ((l >> 3) & 1) * 4 + ((l >> 2) & 1) * 2 + ((l >> 1) & 1), as do
// lanes l and l ^ 1. Every row is the tree ((v0 + v16) + (v8 + v24)) + ... of its lane values.
template <typename T>
__device__ __forceinline__ T reduce16_rows(const T (&v)[16], int lane, int *row) {
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4, h2 = lane & 2;
  T a8[8], a4[4], a2[2];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const T mine = h16 ? v[i + 8] : v[i], other = h16 ? v[i] : v[i + 8];
    a8[i] = mine + __shfl_xor_sync(0xffffffffu, other, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const T mine = h8 ? a8[i + 4] : a8[i], other = h8 ? a8[i] : a8[i + 4];
    a4[i] = mine + __shfl_xor_sync(0xffffffffu, other, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const T mine = h4 ? a4[i + 2] : a4[i], other = h4 ? a4[i] : a4[i + 2];
    a2[i] = mine + __shfl_xor_sync(0xffffffffu, other, 4);
  }
  T a1 = (h2 ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, h2 ? a2[0] : a2[1], 2);
  a1 = a1 + __shfl_xor_sync(0xffffffffu, a1, 1);
  *row = (h16 ? 8 : 0) + (h8 ? 4 : 0) + (h4 ? 2 : 0) + (h2 ? 1 : 0);
  return a1;
}

// One word of the integer path: the pair products of four k (x0..x3 against words w.x..w.w).
__device__ __forceinline__ void pair_products(int (&p)[8], uint4 w, int x0, int x1, int x2, int x3) {
#pragma unroll
  for (int m = 0; m < 8; m++) {
    const uint32_t M = 0x00030003u;
    p[m] += (int)((w.x >> (2 * m)) & M) * x0 + (int)((w.y >> (2 * m)) & M) * x1 +
            (int)((w.z >> (2 * m)) & M) * x2 + (int)((w.w >> (2 * m)) & M) * x3;
  }
}
__device__ __forceinline__ void pair_flush(int (&p)[8], int (&acc)[16]) {
#pragma unroll
  for (int m = 0; m < 8; m++) {
    const int lo = (int)((uint32_t)p[m] << 16) >> 16;
    acc[m] += lo;
    acc[m + 8] += (p[m] - lo) >> 16;
    p[m] = 0;
  }
}
__device__ __forceinline__ void f32_word(float (&acc)[16], float &sx, uint32_t w, float x) {
  sx = __fadd_rn(sx, x);
#pragma unroll
  for (int r = 0; r < 16; r++) acc[r] = fmaf((float)((w >> (2 * r)) & 3u), x, acc[r]);
}

// ct: tiles per ring stage (1, 2, 4 or 8; 8 on the f32 path, where a warp owns whole tiles).
template <int PRO, int EPI, bool F32>
__global__ void __launch_bounds__(256) k_qgemv2(const GemvArgs a, int ct) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr bool pair = EPI == EPI_GELU_CODES && PRO == PRO_JOIN;
  constexpr int nsub = pair ? 2 : 1;
  constexpr bool keep_y = EPI == EPI_GELU_CODES;
  const int K = a.K, cols = a.cols;
  const G2Layout lay = g2_layout(a.ring_bytes, cols, a.max_rows, nsub, keep_y, K, F32);
  uint8_t *ring = smem;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + lay.bars);
  int *xsum = reinterpret_cast<int *>(smem + lay.xsum);
  float *red = reinterpret_cast<float *>(smem + lay.red);
  float *cand_v = reinterpret_cast<float *>(smem + lay.cand_v);
  int *cand_i = reinterpret_cast<int *>(smem + lay.cand_i);
  int *wpart = reinterpret_cast<int *>(smem + lay.wpart);
  float *wpartf = reinterpret_cast<float *>(smem + lay.wpart);
  float *rscale = reinterpret_cast<float *>(smem + lay.scales);
  float *ybuf = reinterpret_cast<float *>(smem + lay.ybuf);
  uint8_t *codes = smem + lay.x;
  float *xf = reinterpret_cast<float *>(smem + lay.x);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int bid = blockIdx.x;
  int s = 0;
  if (!pair && a.nseg > 1 && bid >= a.seg[1].block_begin) s = 1;
  if (!pair && a.nseg > 2 && bid >= a.seg[2].block_begin) s = 2;
  const GemvSeg sg = a.seg[s];
  const int nb = pair ? a.n_blocks_total
                      : (s + 1 < a.nseg ? a.seg[s + 1].block_begin : a.n_blocks_total) - sg.block_begin;
  const int ib = pair ? bid : bid - sg.block_begin;
  const int ntiles = (sg.N + 15) / 16;
  const int t0 = (int)(((long long)ntiles * ib) / nb), t1 = (int)(((long long)ntiles * (ib + 1)) / nb);
  const int r0 = 16 * t0;
  const int rows = min(16 * t1, sg.N) - r0;
  const int tile_bytes = 4 * K;
  const int stage_bytes = ct * tile_bytes;
  int nstages = a.ring_bytes / stage_bytes;
  if (nstages > GS_MAX_STAGES) nstages = GS_MAX_STAGES;
  const int nch1 = (t1 - t0 + ct - 1) / ct;
  const int nchunks = nsub * nch1;

  if (t == 0) {
    for (int i = 0; i < nstages; i++) mbar_init(&bars[i], 1);
    mbar_fence_init();
  }
  if (t < 16) xsum[t] = 0;
  __syncthreads();
  auto issue = [&](int c) {
    const int st = c % nstages;
    const int sub = c / nch1;
    const int ctile = t0 + (c - sub * nch1) * ct;
    const int n = min(ct, t1 - ctile);
    const uint32_t bytes = (uint32_t)(n * tile_bytes);
    mbar_expect_tx(&bars[st], bytes);
    bulk_g2s(ring + st * stage_bytes, a.seg[pair ? sub : s].w + (size_t)ctile * tile_bytes, bytes, &bars[st]);
  };
  if (t == 0)
    for (int c = 0; c < nchunks && c < nstages; c++) issue(c);
  if (t == 32)
    for (int i = 0; i < 4; i++) l2_prefetch_share(a.prefetch[i], a.prefetch_bytes[i], bid, gridDim.x);
  for (int i = t; i < nsub * rows; i += 256) {
    const int sub = i / rows;
    rscale[sub * a.max_rows + i - sub * rows] =
        f16_bits_to_f32(__ldg(a.seg[pair ? sub : s].s + r0 + i - sub * rows));
  }
  ProGains pg;
  prologue_gains<PRO>(a, pg);
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(1000 + 200 + PRO * 10 + EPI);

#pragma unroll 1
  for (int c = 0; c < cols; c++) {
    if (F32) {
      gemv_prologue_f32<PRO>(a, pg, c, xf + (size_t)c * K, red, bid == 0 && a.hidden_out != nullptr);
    } else {
      int x2 = 0;
      const int v = warp_sum_int(gemv_prologue_col<2, PRO>(
          a, pg, c, sg.in_scale, codes + (size_t)c * K, red, bid == 0 && a.hidden_out != nullptr,
          pair ? a.seg[1].in_scale : 0.0f, pair ? codes + (size_t)(cols + c) * K : nullptr, &x2));
      if (lane == 0) atomicAdd(&xsum[c], v);
      if (pair) {
        x2 = warp_sum_int(x2);
        if (lane == 0) atomicAdd(&xsum[8 + c], x2);
      }
    }
  }
  __syncthreads();

  float best_v[8];
  int best_i[8];
#pragma unroll
  for (int c = 0; c < 8; c++) {
    best_v[c] = -FLT_MAX;
    best_i[c] = 0x7fffffff;
  }
  const int wpt = 8 / ct;              // warps per tile
  const int my_tile = warp / wpt, part = warp % wpt;
  const int KB = K / 128;
  for (int ch = 0; ch < nchunks; ch++) {
    const int st = ch % nstages;
    const bool ok = mbar_wait(&bars[st], (uint32_t)((ch / nstages) & 1));
    if (!__syncthreads_and(ok)) {
      if (t == 0) {
        atomicExch(&g4_gemv2_error, 1);
        for (int c2 = ch; c2 < nchunks && c2 < ch + nstages; c2++)
          mbar_wait(&bars[c2 % nstages], (uint32_t)((c2 / nstages) & 1));
      }
      __syncthreads();
      return;
    }
    const int sub = ch / nch1;
    const int ctile = t0 + (ch - sub * nch1) * ct;
    const int ntile = min(ct, t1 - ctile);
    const GemvSeg &g = a.seg[pair ? sub : s];
    const float out_r = g.out_scale != 0.0f ? __fdiv_rn(1.0f, g.out_scale) : 0.0f;
    const uint4 *wt = reinterpret_cast<const uint4 *>(ring + st * stage_bytes + (size_t)my_tile * tile_bytes);
    for (int c = 0; c < cols; c++) {
      if (my_tile < ntile) {
        int row;
        if (F32) {
          float acc[16];
#pragma unroll
          for (int r = 0; r < 16; r++) acc[r] = 0.0f;
          float sx = 0.0f;
          const float4 *xc = reinterpret_cast<const float4 *>(xf + (size_t)c * K);
          for (int kb = part; kb < KB; kb += wpt) {
            const uint4 w = wt[32 * kb + lane];
            const float4 x = xc[32 * kb + lane];
            f32_word(acc, sx, w.x, x.x);
            f32_word(acc, sx, w.y, x.y);
            f32_word(acc, sx, w.z, x.z);
            f32_word(acc, sx, w.w, x.w);
          }
          const float sx2 = __fmul_rn(2.0f, sx);
#pragma unroll
          for (int r = 0; r < 16; r++) acc[r] = __fsub_rn(acc[r], sx2);
          const float v = reduce16_rows(acc, lane, &row);
          if (!(lane & 1)) wpartf[warp * 16 + row] = v;
        } else {
          int p[8], acc[16];
#pragma unroll
          for (int m = 0; m < 8; m++) p[m] = 0;
#pragma unroll
          for (int r = 0; r < 16; r++) acc[r] = 0;
          const uint32_t *xc = reinterpret_cast<const uint32_t *>(codes + (size_t)(sub * cols + c) * K);
          int n = 0;
          for (int kb = part; kb < KB; kb += wpt) {
            const uint4 w = wt[32 * kb + lane];
            const uint32_t xw = xc[32 * kb + lane];
            pair_products(p, w, (int)(xw << 24) >> 24, (int)(xw << 16) >> 24, (int)(xw << 8) >> 24,
                          (int)xw >> 24);
            if (++n == 16) {
              pair_flush(p, acc);
              n = 0;
            }
          }
          pair_flush(p, acc);
          const int v = reduce16_rows(acc, lane, &row);
          if (!(lane & 1)) wpart[warp * 16 + row] = v;
        }
      }
      __syncthreads();
      // Epilogue: one thread per row of the stage (tile lt, row i), its warps' shares in order.
      if (t < ntile * 16) {
        const int lt = t >> 4, i = t & 15;
        const int row = 16 * (ctile + lt) + i;
        if (row < g.N) {
          const float wscale = rscale[sub * a.max_rows + row - r0];
          float y;
          int exact = 0;
          if (F32) {
            y = __fmul_rn(__fmul_rn(1.0f, wscale), wpartf[lt * wpt * 16 + i]);
          } else {
            int sum = 0;
            for (int q = 0; q < wpt; q++) sum += wpart[(lt * wpt + q) * 16 + i];
            exact = sum - 2 * xsum[sub * 8 + c];
            y = __fmul_rn(__fmul_rn(g.in_scale, wscale), (float)exact);
          }
          y = srq_out_r(y, g.out_scale, out_r);
          if (g.acc_out) g.acc_out[(size_t)c * g.N + row] = exact;
          if (keep_y) {
            ybuf[(sub * cols + c) * a.max_rows + row - r0] = y;
          } else if (EPI == EPI_HEAD) {
            if (a.softcap != 0.0f) y = __fmul_rn(g4_tanh(__fdiv_rn(y, a.softcap)), a.softcap);
            if (a.logits) a.logits[(size_t)c * a.ld_logits + row] = y;
#pragma unroll
            for (int cc = 0; cc < 8; cc++)
              if (cc == c && (y > best_v[cc] || (y == best_v[cc] && row < best_i[cc]))) {
                best_v[cc] = y;
                best_i[cc] = row;
              }
          } else {
            g.y[(size_t)c * g.N + row] = y;
          }
        }
      }
      __syncthreads();
    }
    if (t == 0 && ch + nstages < nchunks) issue(ch + nstages);
  }
  G4_TRACE_POINT(200000 + 1000 + 200 + PRO * 10 + EPI);
  if constexpr (keep_y) {
    // h = gelu(gate) * up (src/kernels/geluMul.ts:67-115), snapped to the next linear's codes.
    const float cr = __fdiv_rn(1.0f, a.codes_scale);
    for (int i = t; i < rows * cols; i += 256) {
      const int c = i / rows, r = i - c * rows;
      const float gv = ybuf[c * a.max_rows + r];
      const float u = pair ? ybuf[(cols + c) * a.max_rows + r]
                           : a.epi_up[(size_t)c * a.epi_ld_up + a.epi_up_off + r0 + r];
      const float h = __fmul_rn(g4_gelu(gv), u);
      a.codes_out[(size_t)c * a.codes_ld + code_pos(r0 + r, a.codes_bits)] =
          (uint8_t)(srq_code_r(h, a.codes_scale, cr) & 255);
    }
  }
  if constexpr (EPI == EPI_HEAD) {
#pragma unroll
    for (int c = 0; c < 8; c++) {
      if (c < cols) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, best_v[c], o);
          const int oi = __shfl_xor_sync(0xffffffffu, best_i[c], o);
          if (ov > best_v[c] || (ov == best_v[c] && oi < best_i[c])) {
            best_v[c] = ov;
            best_i[c] = oi;
          }
        }
        if (lane == 0) {
          cand_v[warp * 8 + c] = best_v[c];
          cand_i[warp * 8 + c] = best_i[c];
        }
      }
    }
    __syncthreads();
    if (t < cols) {
      float bv = -FLT_MAX;
      int bi = 0x7fffffff;
      for (int w = 0; w < 8; w++) {
        const float v = cand_v[w * 8 + t];
        const int i = cand_i[w * 8 + t];
        if (v > bv || (v == bv && i < bi)) {
          bv = v;
          bi = i;
        }
      }
      a.part_val[(size_t)t * a.n_blocks_total + bid] = bv;
      a.part_idx[(size_t)t * a.n_blocks_total + bid] = bi;
    }
  }
}

// Tiles of the segments over at most `sms` CTAs (a pair: the same tiles of both).
int gemv2_partition(GemvArgs &a, int sms) {
  if (a.pair) {
    const int tiles = (a.seg[0].N + 15) / 16;
    const int nb = tiles < sms ? tiles : sms;
    a.seg[0].block_begin = 0;
    a.seg[1].block_begin = 0;
    a.n_blocks_total = nb;
    return nb;
  }
  long long tiles[3], nb[3];
  for (int i = 0; i < a.nseg; i++) tiles[i] = (a.seg[i].N + 15) / 16;
  split_ctas(tiles, a.nseg, sms, nb);
  int begin = 0;
  for (int i = 0; i < a.nseg; i++) {
    a.seg[i].block_begin = begin;
    begin += (int)nb[i];
  }
  a.n_blocks_total = begin;
  return begin;
}

template <int PRO, int EPI, bool F32>
static cudaError_t launch_g2_t(const GemvArgs &a, int ct, size_t smem, cudaStream_t st, bool pdl) {
  auto k = k_qgemv2<PRO, EPI, F32>;
  static DeviceOnce attr;
  attr([&] { cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, G2_MAX_SMEM); });
  return launch_k(k, dim3(a.n_blocks_total), dim3(256), smem, st, pdl, a, ct);
}

template <bool F32>
static cudaError_t launch_g2_f(const GemvArgs &a, int epi, int ct, size_t smem, cudaStream_t st, bool pdl) {
  if (epi == EPI_Y) {
    switch (a.pro) {
      case PRO_X: return launch_g2_t<PRO_X, EPI_Y, F32>(a, ct, smem, st, pdl);
      case PRO_NORM: return launch_g2_t<PRO_NORM, EPI_Y, F32>(a, ct, smem, st, pdl);
      case PRO_JOIN: return launch_g2_t<PRO_JOIN, EPI_Y, F32>(a, ct, smem, st, pdl);
      case PRO_NORMRES: return launch_g2_t<PRO_NORMRES, EPI_Y, F32>(a, ct, smem, st, pdl);
      case PRO_GELU: return launch_g2_t<PRO_GELU, EPI_Y, F32>(a, ct, smem, st, pdl);
      case PRO_CODES:
        if (!F32) return launch_g2_t<PRO_CODES, EPI_Y, false>(a, ct, smem, st, pdl);
        break;
    }
  } else if (epi == EPI_HEAD) {
    if (a.pro == PRO_JOIN) return launch_g2_t<PRO_JOIN, EPI_HEAD, F32>(a, ct, smem, st, pdl);
    if (a.pro == PRO_NORM) return launch_g2_t<PRO_NORM, EPI_HEAD, F32>(a, ct, smem, st, pdl);
    if (a.pro == PRO_X) return launch_g2_t<PRO_X, EPI_HEAD, F32>(a, ct, smem, st, pdl);
  } else if (epi == EPI_GELU_CODES && !F32) {
    if (a.pro == PRO_JOIN && a.pair && a.nseg == 2 && a.seg[0].N == a.seg[1].N)
      return launch_g2_t<PRO_JOIN, EPI_GELU_CODES, false>(a, ct, smem, st, pdl);
  }
  return cudaErrorInvalidConfiguration;
}

// Needs gemv2_partition first. Uncalibrated (seg 0 in_scale 0.0) selects the f32 path.
cudaError_t launch_gemv2(const GemvArgs &a0, cudaStream_t st, bool pdl) {
  GemvArgs a = a0;
  const bool f32 = a.seg[0].in_scale == 0.0f;
  if (a.K < 128 || a.K % 128 || a.K > 16384 || a.cols < 1 || a.cols > 8 || a.nseg < 1)
    return cudaErrorInvalidConfiguration;
  for (int i = 1; i < a.nseg; i++)
    if ((a.seg[i].in_scale == 0.0f) != f32) return cudaErrorInvalidConfiguration;
  const int epi = a.head ? EPI_HEAD : a.epi;
  const bool pair = epi == EPI_GELU_CODES && a.pro == PRO_JOIN;
  if (f32 && (pair || epi == EPI_GELU_CODES || a.pro == PRO_NORMRES)) return cudaErrorInvalidConfiguration;
  const int tile_bytes = 4 * a.K;
  int ct = 8;
  if (!f32)
    while (ct > 1 && ct * tile_bytes > 24 * 1024) ct >>= 1;
  const int stage_bytes = ct * tile_bytes;
  if (stage_bytes > GS_RING) return cudaErrorInvalidConfiguration;
  const int nsub = pair ? 2 : 1;
  int max_tiles = 1;
  for (int i = 0; i < (pair ? 1 : a.nseg); i++) {
    const int nb = pair ? a.n_blocks_total
                        : (i + 1 < a.nseg ? a.seg[i + 1].block_begin : a.n_blocks_total) - a.seg[i].block_begin;
    const int tiles = (a.seg[i].N + 15) / 16;
    max_tiles = std::max(max_tiles, (tiles + nb - 1) / nb);
  }
  const int chunks = nsub * ((max_tiles + ct - 1) / ct);
  int nstages = std::min(std::min(chunks, GS_RING / stage_bytes), GS_MAX_STAGES);
  if (nstages < 1) nstages = 1;
  a.ring_bytes = nstages * stage_bytes;
  a.max_rows = 16 * max_tiles;
  const G2Layout lay = g2_layout(a.ring_bytes, a.cols, a.max_rows, nsub, epi == EPI_GELU_CODES, a.K, f32);
  if (lay.total > G2_MAX_SMEM) return cudaErrorInvalidConfiguration;
  return f32 ? launch_g2_f<true>(a, epi, ct, (size_t)lay.total, st, pdl)
             : launch_g2_f<false>(a, epi, ct, (size_t)lay.total, st, pdl);
}

}  // namespace g4
