// g4_kernels.cu -- sm_100a kernels of the Gemma-4-E2B quantized decode/prefill path.
//
// Reference citations are path:line inside the reference project (TypeScript + WGSL).
#include <cuda_fp16.h>
#include <float.h>
#include <map>
#include <mutex>

#include "g4_device.cuh"
#include "g4_kernels.cuh"
#include "g4_gemv.cuh"

namespace g4 {

#ifdef G4_TRACE
__device__ unsigned long long g4_trace_buf[1 << 16];
__device__ unsigned int g4_trace_n;
#endif


// =====================================================================================
// Quantized linear (qgemv / qgemm column contract, src/kernels/qgemv.ts:413-690 and
// 1131-1176): int4 (zero point 8) or int8 weight codes against int8 activation codes, exact
// int32 accumulation with dp4a, y = srqOut((inScale * scale[r]) * f32(acc)).
//
// Layout: 256 threads = 8 warps; warp w owns RPW consecutive rows; lane l reads the 16-byte
// pieces l*16 + 512 i (i < PPR) of each of its rows, all loads issued before the dependency
// wait so the weight stream overlaps the previous kernel (programmatic dependent launch).
// int4 words are split into even and odd nibble bytes (w & 0x0F0F0F0F, (w >> 4) & 0x0F0F0F0F),
// multiplied as unsigned codes against activation codes stored in matching even/odd order, and
// the zero point comes off once per row: sum((u - 8) x) = sum(u x) - 8 sum(x).
// =====================================================================================

// Activation codes for the tensor-core path (one CTA per column, plain K order).
template <int PRO>
__global__ void __launch_bounds__(256) k_quantize(const GemvArgs a, uint8_t *codes, int ld, float s1,
                                                  uint8_t *codes2, float s2) {
  __shared__ float red[8];
  ProGains pg;
  prologue_gains<PRO>(a, pg);
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(4000 + PRO);
  const int c = blockIdx.x;
  int x2 = 0;
  gemv_prologue_col<8, PRO>(a, pg, c, s1, codes + (size_t)c * ld, red, a.hidden_out != nullptr, s2,
                            codes2 ? codes2 + (size_t)c * ld : nullptr, &x2);
}

// The elementwise prologues (x, gelu(x) * u) need no per-column reduction: grid (column, chunk
// block), one vec4 chunk per thread, so a wide column (down_proj's 6144) spreads over many SMs.
template <int PRO>
__global__ void __launch_bounds__(256) k_quantize_elem(const GemvArgs a, uint8_t *codes, int ld, float s1,
                                                       uint8_t *codes2, float s2) {
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(4000 + PRO);
  const int c = blockIdx.x, ch = blockIdx.y * 256 + threadIdx.x;
  if (ch >= (a.K >> 2)) return;
  float4 x = reinterpret_cast<const float4 *>(a.src + (size_t)c * a.ld_src)[ch];
  if (PRO == PRO_GELU)
    x = f4_gelu_mul(x, reinterpret_cast<const float4 *>(a.up + (size_t)c * a.ld_up + a.up_off)[ch]);
  ChunkPro::store<8>(codes + (size_t)c * ld, ch, x, s1, __fdiv_rn(1.0f, s1));
  if (codes2) ChunkPro::store<8>(codes2 + (size_t)c * ld, ch, x, s2, __fdiv_rn(1.0f, s2));
}

cudaError_t launch_quantize(const GemvArgs &a, uint8_t *codes, int ld, float s1, uint8_t *codes2,
                           float s2, cudaStream_t st, bool pdl) {
  if (a.cols < 1 || (a.K & 15) || s1 == 0.0f || (codes2 && s2 == 0.0f)) return cudaErrorInvalidValue;
  const dim3 g(a.cols), b(256), ge(a.cols, ((a.K >> 2) + 255) / 256);
  switch (a.pro) {
    case PRO_X: return launch_k(k_quantize_elem<PRO_X>, ge, b, 0, st, pdl, a, codes, ld, s1, codes2, s2);
    case PRO_NORM: return launch_k(k_quantize<PRO_NORM>, g, b, 0, st, pdl, a, codes, ld, s1, codes2, s2);
    case PRO_JOIN: return launch_k(k_quantize<PRO_JOIN>, g, b, 0, st, pdl, a, codes, ld, s1, codes2, s2);
    case PRO_NORMRES: return launch_k(k_quantize<PRO_NORMRES>, g, b, 0, st, pdl, a, codes, ld, s1, codes2, s2);
    case PRO_GELU: return launch_k(k_quantize_elem<PRO_GELU>, ge, b, 0, st, pdl, a, codes, ld, s1, codes2, s2);
  }
  return cudaErrorInvalidValue;
}

// The f32 path of an uncalibrated site (in_scale == 0, src/kernels/qgemv.ts:666-675), one column:
// lane l accumulates the row's 16-byte chunks l, l + 32, ... in k order with fused multiply-adds,
// the lanes close with the butterfly, y = srqOut((1 * scale) * sum).
template <int BITS>
__global__ void __launch_bounds__(256) k_gemv_f32(const GemvArgs a) {
  extern __shared__ __align__(16) float xf[];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const GemvSeg sg = a.seg[0];
  const int K = a.K, row_bytes = K * BITS / 8;
  const int row = blockIdx.x * 8 + warp;
  grid_launch_dependents();
  grid_wait();
  const int nc = K >> 2;
  const float4 *src = reinterpret_cast<const float4 *>(a.src);
  const float4 *up = a.pro == PRO_GELU ? reinterpret_cast<const float4 *>(a.up + a.up_off) : nullptr;
  for (int ch = t; ch < nc; ch += 256) {
    float4 x = src[ch];
    if (a.pro == PRO_GELU) x = f4_gelu_mul(x, up[ch]);
    reinterpret_cast<float4 *>(xf)[ch] = x;
  }
  __syncthreads();
  if (row >= sg.N) return;
  const int per = 16 * 8 / BITS;
  float accf = 0.0f;
  for (int off = lane * 16; off < row_bytes; off += 512) {
    const uint8_t *p = sg.w + (size_t)row * row_bytes + off;
    const int k0 = off * 8 / BITS;
    for (int j = 0; j < per; j++) {
      int code;
      if (BITS == 4) {
        uint8_t b = p[j >> 1];
        code = (int)((j & 1) ? (b >> 4) : (b & 15)) - 8;
      } else {
        code = (int)(int8_t)p[j];
      }
      accf = fmaf((float)code, xf[k0 + j], accf);
    }
  }
  float sum = warp_sum_bfly(accf);
  if (lane == 0) {
    float scale = f16_bits_to_f32(sg.s[row]);
    float y = __fmul_rn(__fmul_rn(1.0f, scale), sum);
    sg.y[row] = srq_out(y, sg.out_scale);
    if (sg.acc_out) sg.acc_out[row] = 0;
  }
}

// =====================================================================================
// Streaming quantized linear. One CTA per SM (or fewer): CTA i of a segment owns the contiguous
// rows [N i / nb, N (i + 1) / nb), a contiguous byte range of the packed weights, and streams it
// through a shared-memory ring with TMA bulk copies (cp.async.bulk, completion on an mbarrier).
// The first stages are requested before the programmatic-dependency wait, so a launch's weight
// stream starts while the previous kernel is still finishing; the CTA may also pull the weights
// of later launches into L2 (cp.async.bulk.prefetch.L2). Arithmetic is k_gemv's: exact int32
// dp4a code dots and the same epilogue.
// =====================================================================================

__device__ int g4_dev_error;

// Shared memory of one streaming-GEMV CTA: the ring, then the barriers, the column sums, the
// reduction and argmax scratch, the row scales of the CTA's slice (per sub-slice), the y rows
// an EPI_GELU_CODES epilogue keeps, and the activation codes.
struct GsLayout {
  int bars, xsum, red, cand_v, cand_i, scales, ybuf, codes, total;
};
__host__ __device__ __forceinline__ GsLayout gs_layout(int ring, int cols, int max_rows, int nsub,
                                                       bool keep_y, int K) {
  GsLayout l;
  l.bars = ring;
  l.xsum = l.bars + GS_MAX_STAGES * 8;
  l.red = l.xsum + 16 * 4;
  l.cand_v = l.red + 8 * 4;
  l.cand_i = l.cand_v + 8 * cols * 4;
  l.scales = l.cand_i + 8 * cols * 4;
  l.ybuf = l.scales + nsub * max_rows * 4;
  l.codes = (l.ybuf + (keep_y ? nsub * cols * max_rows * 4 : 0) + 15) & ~15;
  l.total = l.codes + nsub * cols * K;
  return l;
}

// Resident CTAs per SM the register allocation is bounded for.
#ifndef G4_GEMV_MIN_BLOCKS
#define G4_GEMV_MIN_BLOCKS 2
#endif

template <int BITS, int COLS, int RS, int PRO, int EPI>
__global__ void __launch_bounds__(256, ((PRO == PRO_X || PRO == PRO_CODES) && EPI == EPI_Y && COLS == 1)
                                           ? 4 : G4_GEMV_MIN_BLOCKS)
    k_qgemv_stream(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int ring_bytes = a.ring_bytes;
  // gate/up: both sub-slices of one CTA, each with its own input codes.
  constexpr bool pair = EPI == EPI_GELU_CODES && PRO == PRO_JOIN;
  constexpr int nsub = pair ? 2 : 1;
  constexpr bool keep_y = EPI == EPI_GELU_CODES;
  const GsLayout lay = gs_layout(ring_bytes, COLS, a.max_rows, nsub, keep_y, a.K);
  uint8_t *ring = smem;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + lay.bars);
  int *xsum = reinterpret_cast<int *>(smem + lay.xsum);
  float *red = reinterpret_cast<float *>(smem + lay.red);
  float *cand_v = reinterpret_cast<float *>(smem + lay.cand_v);
  int *cand_i = reinterpret_cast<int *>(smem + lay.cand_i);
  float *rscale = reinterpret_cast<float *>(smem + lay.scales);
  float *ybuf = reinterpret_cast<float *>(smem + lay.ybuf);
  uint8_t *codes = smem + lay.codes;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int bid = blockIdx.x;
  int s = 0;
  if (!pair && a.nseg > 1 && bid >= a.seg[1].block_begin) s = 1;
  if (!pair && a.nseg > 2 && bid >= a.seg[2].block_begin) s = 2;
  const GemvSeg sg = a.seg[s];
  const int nb = pair ? a.n_blocks_total
                      : (s + 1 < a.nseg ? a.seg[s + 1].block_begin : a.n_blocks_total) - sg.block_begin;
  const int ib = pair ? bid : bid - sg.block_begin;
  const int r0 = (int)(((long long)sg.N * ib) / nb);
  const int r1 = (int)(((long long)sg.N * (ib + 1)) / nb);
  const int K = a.K;
  const int row_bytes = K * BITS / 8;
  const int vb = row_bytes / RS;                 // bytes per virtual row
  int srows = gs_stage_vrows(vb) / RS;           // real rows per stage
  if (srows > a.max_rows) srows = a.max_rows;    // a chunk never spans two sub-slices
  if (srows * row_bytes > ring_bytes) srows = ring_bytes / row_bytes;
  const int stage_bytes = srows * row_bytes;
  int nstages = ring_bytes / stage_bytes;
  if (nstages > GS_MAX_STAGES) nstages = GS_MAX_STAGES;
  const int nch1 = (r1 - r0 + srows - 1) / srows;   // chunks per sub-slice
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
    const int cr0 = r0 + (c - sub * nch1) * srows;
    const int rows = min(srows, r1 - cr0);
    const uint32_t bytes = (uint32_t)(rows * row_bytes);
    mbar_expect_tx(&bars[st], bytes);
    bulk_g2s(ring + st * stage_bytes, a.seg[pair ? sub : s].w + (size_t)cr0 * row_bytes, bytes, &bars[st]);
  };
  if (t == 0)
    for (int c = 0; c < nchunks && c < nstages; c++) issue(c);
  if (t == 32)
    for (int i = 0; i < 4; i++) l2_prefetch_share(a.prefetch[i], a.prefetch_bytes[i], bid, gridDim.x);
  // Row scales and norm gains are weights too: read them before the wait.
  for (int i = t; i < nsub * (r1 - r0); i += 256) {
    const int sub = i / (r1 - r0);
    rscale[sub * a.max_rows + i - sub * (r1 - r0)] =
        f16_bits_to_f32(__ldg(a.seg[pair ? sub : s].s + r0 + i - sub * (r1 - r0)));
  }
  ProGains pg;
  prologue_gains<PRO>(a, pg);
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(1000 + BITS * 100 + PRO * 10 + EPI);

#pragma unroll 1
  for (int c = 0; c < a.cols; c++) {
    int x2 = 0;
    const int v = warp_sum_int(gemv_prologue_col<BITS, PRO>(
        a, pg, c, sg.in_scale, codes + c * K, red, bid == 0 && a.hidden_out != nullptr,
        pair ? a.seg[1].in_scale : 0.0f, pair ? codes + (COLS + c) * K : nullptr, &x2));
    if (lane == 0) atomicAdd(&xsum[c], v);
    if (pair) {
      x2 = warp_sum_int(x2);
      if (lane == 0) atomicAdd(&xsum[8 + c], x2);
    }
  }
  __syncthreads();
  G4_TRACE_POINT(100000 + 1000 + BITS * 100 + PRO * 10 + EPI);

  float best_v[COLS];
  int best_i[COLS];
#pragma unroll
  for (int c = 0; c < COLS; c++) {
    best_v[c] = -FLT_MAX;
    best_i[c] = 0x7fffffff;
  }
  const float out_r0 = sg.out_scale != 0.0f ? __fdiv_rn(1.0f, sg.out_scale) : 0.0f;
  const float out_r1 = pair && a.seg[1].out_scale != 0.0f ? __fdiv_rn(1.0f, a.seg[1].out_scale) : 0.0f;
  for (int ch = 0; ch < nchunks; ch++) {
    const int st = ch % nstages;
    const bool ok = mbar_wait(&bars[st], (uint32_t)((ch / nstages) & 1));
    if (!__syncthreads_and(ok)) {
      // A copy never completed: record it, give the copies still in flight a bounded wait so
      // none lands in released shared memory, and leave.
      if (t == 0) {
        atomicExch(&g4_dev_error, 1);
        for (int c2 = ch; c2 < nchunks && c2 < ch + nstages; c2++)
          mbar_wait(&bars[c2 % nstages], (uint32_t)((c2 / nstages) & 1));
      }
      __syncthreads();
      return;
    }
    const int sub = ch / nch1;
    const int cr0 = r0 + (ch - sub * nch1) * srows;
    const int vrows = min(srows, r1 - cr0) * RS;
    const uint8_t *sw = ring + st * stage_bytes;
    const float out_scale = sub ? a.seg[1].out_scale : sg.out_scale;
    const float out_r = sub ? out_r1 : out_r0;
    const float in_scale = sub ? a.seg[1].in_scale : sg.in_scale;
    const uint8_t *ccodes = codes + sub * COLS * K;
    // Each warp takes groups of four virtual rows; the four dot products run as independent
    // chains and close with one transposed reduction, after which lanes 0, 8, 16 and 24 hold
    // the four totals; the parts of a split row are then added and its lanes finish the rows
    // in parallel.
    for (int g0 = warp * 4; g0 < vrows; g0 += 32) {
      int acc[4][COLS];
#pragma unroll
      for (int q = 0; q < 4; q++)
#pragma unroll
        for (int c = 0; c < COLS; c++) acc[q][c] = 0;
      for (int off = lane * 16; off < vb; off += 512) {
        uint4 w[4];
        int koff[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const int vr = g0 + q;
          koff[q] = (vr % RS) * vb + off;  // byte offset of this piece inside its real row
          w[q] = vr < vrows ? *reinterpret_cast<const uint4 *>(sw + (size_t)vr * vb + off)
                            : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int c = 0; c < COLS; c++) {
          // RS == 1: all four rows read the same activation codes; RS == 2: rows 0/2 and 1/3.
          constexpr int NX = RS == 1 ? 1 : (RS == 2 ? 2 : 4);
          uint4 xa[NX], xb[NX];
#pragma unroll
          for (int j = 0; j < NX; j++) {
            if (BITS == 4) {
              const uint4 *xp = reinterpret_cast<const uint4 *>(ccodes + c * K + 2 * koff[j]);
              xa[j] = xp[0];
              xb[j] = xp[1];
            } else {
              xa[j] = *reinterpret_cast<const uint4 *>(ccodes + c * K + koff[j]);
            }
          }
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const uint4 x01 = xa[q % NX];
            int v = acc[q][c];
            if (BITS == 4) {
              const uint4 x23 = xb[q % NX];
              const uint32_t M = 0x0F0F0F0Fu;
              v = dp4a_us(w[q].x & M, x01.x, v);
              v = dp4a_us((w[q].x >> 4) & M, x01.y, v);
              v = dp4a_us(w[q].y & M, x01.z, v);
              v = dp4a_us((w[q].y >> 4) & M, x01.w, v);
              v = dp4a_us(w[q].z & M, x23.x, v);
              v = dp4a_us((w[q].z >> 4) & M, x23.y, v);
              v = dp4a_us(w[q].w & M, x23.z, v);
              v = dp4a_us((w[q].w >> 4) & M, x23.w, v);
            } else {
              v = dp4a_ss(w[q].x, x01.x, v);
              v = dp4a_ss(w[q].y, x01.y, v);
              v = dp4a_ss(w[q].z, x01.z, v);
              v = dp4a_ss(w[q].w, x01.w, v);
            }
            acc[q][c] = v;
          }
        }
      }
      // Transposed reduction of four rows: lanes < 16 keep rows 0-1, lanes >= 16 rows 2-3;
      // bit 3 of the lane then picks one row; three more butterflies close it. Integer adds,
      // so the grouping cannot change the sum.
      const bool hi16 = lane >= 16, hi8 = (lane & 8) != 0;
      const int my_vrow = (hi16 ? 2 : 0) + (hi8 ? 1 : 0);
#pragma unroll
      for (int c = 0; c < COLS; c++) {
        int b0 = (hi16 ? acc[2][c] : acc[0][c]) + __shfl_xor_sync(0xffffffffu, hi16 ? acc[0][c] : acc[2][c], 16);
        int b1 = (hi16 ? acc[3][c] : acc[1][c]) + __shfl_xor_sync(0xffffffffu, hi16 ? acc[1][c] : acc[3][c], 16);
        int v = (hi8 ? b1 : b0) + __shfl_xor_sync(0xffffffffu, hi8 ? b0 : b1, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        if (RS >= 2) v += __shfl_xor_sync(0xffffffffu, v, 8);   // parts 0+1 (and 2+3)
        if (RS >= 4) v += __shfl_xor_sync(0xffffffffu, v, 16);  // parts (0+1)+(2+3)
        acc[0][c] = v;
      }
      const int vr = g0 + my_vrow;
      if ((lane & (8 * RS - 1)) == 0 && vr < vrows) {
        const int row = cr0 + vr / RS;
        const float wscale = rscale[sub * a.max_rows + row - r0];
#pragma unroll
        for (int c = 0; c < COLS; c++) {
          if (c < a.cols) {
            const int exact = BITS == 4 ? acc[0][c] - 8 * xsum[sub * 8 + c] : acc[0][c];
            float y = __fmul_rn(__fmul_rn(in_scale, wscale), (float)exact);
            y = srq_out_r(y, out_scale, out_r);
            if (sg.acc_out) sg.acc_out[(size_t)c * sg.N + row] = exact;
            if (keep_y) {
              ybuf[(sub * COLS + c) * a.max_rows + row - r0] = y;
            } else if (EPI == EPI_HEAD) {
              if (a.softcap != 0.0f) y = __fmul_rn(g4_tanh(__fdiv_rn(y, a.softcap)), a.softcap);
              if (a.logits) a.logits[(size_t)c * a.ld_logits + row] = y;
              if (y > best_v[c] || (y == best_v[c] && row < best_i[c])) {
                best_v[c] = y;
                best_i[c] = row;
              }
            } else {
              sg.y[(size_t)c * sg.N + row] = y;
            }
          }
        }
      }
    }
    __syncthreads();
    if (t == 0 && ch + nstages < nchunks) issue(ch + nstages);
  }
  G4_TRACE_POINT(200000 + 1000 + BITS * 100 + PRO * 10 + EPI);
  if constexpr (keep_y) {
    // h = gelu(y0) * u (gelu-mul, src/kernels/geluMul.ts:67-115), snapped to the next linear's
    // input codes exactly as its own prologue would (src/kernels/qgemv.ts:371-400, 624-626).
    const int rows = r1 - r0;
    const float cr = __fdiv_rn(1.0f, a.codes_scale);
    for (int i = t; i < rows * COLS; i += 256) {
      const int c = i / rows, r = i - c * rows;
      if (c < a.cols) {
        const float g = ybuf[c * a.max_rows + r];
        const float u = pair ? ybuf[(COLS + c) * a.max_rows + r]
                             : a.epi_up[(size_t)c * a.epi_ld_up + a.epi_up_off + r0 + r];
        const float h = __fmul_rn(g4_gelu(g), u);
        a.codes_out[(size_t)c * a.codes_ld + code_pos(r0 + r, a.codes_bits)] =
            (uint8_t)(srq_code_r(h, a.codes_scale, cr) & 255);
      }
    }
  }
  if constexpr (EPI == EPI_HEAD) {
#pragma unroll
    for (int c = 0; c < COLS; c++) {
      // The candidates sit in lanes 0, 8, 16, 24 of each warp; every other lane carries -FLT_MAX.
#pragma unroll
      for (int o = 8; o < 32; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best_v[c], o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i[c], o);
        if (ov > best_v[c] || (ov == best_v[c] && oi < best_i[c])) {
          best_v[c] = ov;
          best_i[c] = oi;
        }
      }
      if (lane == 0) {
        cand_v[warp * COLS + c] = best_v[c];
        cand_i[warp * COLS + c] = best_i[c];
      }
    }
    __syncthreads();
    if (t < COLS && t < a.cols) {
      float bv = -FLT_MAX;
      int bi = 0x7fffffff;
      for (int w = 0; w < 8; w++) {
        const float v = cand_v[w * COLS + t];
        const int i = cand_i[w * COLS + t];
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

int gemv_stream_partition(GemvArgs &a, int sms) {
  if (a.pair) {
    // Every CTA owns the same rows of both segments.
    const int nb = a.seg[0].N < sms ? a.seg[0].N : sms;
    a.seg[0].block_begin = 0;
    a.seg[1].block_begin = 0;
    a.n_blocks_total = nb;
    return nb;
  }
  long long rows[3], nb[3];
  for (int i = 0; i < a.nseg; i++) rows[i] = a.seg[i].N;
  split_ctas(rows, a.nseg, sms, nb);
  int begin = 0;
  for (int i = 0; i < a.nseg; i++) {
    a.seg[i].block_begin = begin;
    begin += (int)nb[i];
  }
  a.n_blocks_total = begin;
  return begin;
}

template <int BITS, int COLS, int RS, int PRO, int EPI>
static cudaError_t launch_stream_t(const GemvArgs &a0, cudaStream_t st, bool pdl) {
  // The ring holds the slice a CTA owns (both sub-slices for a pair) when that fits in GS_RING
  // (then the whole slice is requested before the dependency wait), else GS_RING. A small ring
  // lets the next launch's CTAs sit on the SM beside this one's and start their copies early.
  GemvArgs a = a0;
  const int row_bytes = a.K * BITS / 8;
  const int nsub = (EPI == EPI_GELU_CODES && PRO == PRO_JOIN) ? 2 : 1;
  int max_rows = 1;
  if (nsub == 2) {
    max_rows = (a.seg[0].N + a.n_blocks_total - 1) / a.n_blocks_total;
  } else {
    for (int i = 0; i < a.nseg; i++) {
      const int nb = (i + 1 < a.nseg ? a.seg[i + 1].block_begin : a.n_blocks_total) - a.seg[i].block_begin;
      max_rows = std::max(max_rows, (a.seg[i].N + nb - 1) / nb);
    }
  }
  const long long slice = (long long)nsub * max_rows * row_bytes;
  a.ring_bytes = slice < GS_RING ? (int)((slice + 127) & ~127LL) : GS_RING;
#ifdef G4_GEMV_FULL_RING
  a.ring_bytes = GS_RING;
#endif
  if (a.ring_bytes < row_bytes) a.ring_bytes = (row_bytes + 127) & ~127;
  a.max_rows = max_rows;
  const GsLayout lay = gs_layout(a.ring_bytes, COLS, max_rows, nsub, EPI == EPI_GELU_CODES, a.K);
  if (lay.total > 200 * 1024) return cudaErrorInvalidConfiguration;
  auto k = k_qgemv_stream<BITS, COLS, RS, PRO, EPI>;
  static DeviceOnce attr_set;
  attr_set([&] {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  });
  return launch_k(k, dim3(a.n_blocks_total), dim3(256), (size_t)lay.total, st, pdl, a);
}

// Each (prologue, epilogue) pair is its own kernel: a launch runs a short straight path, which
// matters because every launch starts with a cold instruction cache. One column or up to eight.
template <int BITS, int PRO, int EPI>
static cudaError_t launch_stream_b(const GemvArgs &a, int rs, cudaStream_t st, bool pdl) {
  if (a.cols == 1) {
    if (rs == 1) return launch_stream_t<BITS, 1, 1, PRO, EPI>(a, st, pdl);
    if (rs == 2) return launch_stream_t<BITS, 1, 2, PRO, EPI>(a, st, pdl);
    return launch_stream_t<BITS, 1, 4, PRO, EPI>(a, st, pdl);
  }
  if (rs == 1) return launch_stream_t<BITS, 8, 1, PRO, EPI>(a, st, pdl);
  if (rs == 2) return launch_stream_t<BITS, 8, 2, PRO, EPI>(a, st, pdl);
  return launch_stream_t<BITS, 8, 4, PRO, EPI>(a, st, pdl);
}

template <int PRO, int EPI>
static cudaError_t launch_stream_pe(const GemvArgs &a, int bits, int rs, cudaStream_t st, bool pdl) {
  return bits == 4 ? launch_stream_b<4, PRO, EPI>(a, rs, st, pdl) : launch_stream_b<8, PRO, EPI>(a, rs, st, pdl);
}

cudaError_t launch_gemv_stream(const GemvArgs &a, int bits, cudaStream_t st, bool pdl) {
  const int row_bytes = a.K * bits / 8;
  const int rs = gs_row_split(row_bytes);
  if (row_bytes % 16 != 0 || row_bytes % rs != 0 || row_bytes / rs > 1024 || (row_bytes / rs) % 16 != 0)
    return cudaErrorInvalidConfiguration;
  if (a.cols < 1 || a.cols > 8 || (bits != 4 && bits != 8)) return cudaErrorInvalidConfiguration;
  const int epi = a.head ? EPI_HEAD : a.epi;
  if (epi == EPI_Y) {
    switch (a.pro) {
      case PRO_X: return launch_stream_pe<PRO_X, EPI_Y>(a, bits, rs, st, pdl);
      case PRO_NORM: return launch_stream_pe<PRO_NORM, EPI_Y>(a, bits, rs, st, pdl);
      case PRO_JOIN: return launch_stream_pe<PRO_JOIN, EPI_Y>(a, bits, rs, st, pdl);
      case PRO_NORMRES: return launch_stream_pe<PRO_NORMRES, EPI_Y>(a, bits, rs, st, pdl);
      case PRO_GELU: return launch_stream_pe<PRO_GELU, EPI_Y>(a, bits, rs, st, pdl);
      case PRO_CODES: return launch_stream_pe<PRO_CODES, EPI_Y>(a, bits, rs, st, pdl);
    }
  } else if (epi == EPI_GELU_CODES) {
    // join: the gate/up pair; norm-residual: one linear times the per-layer input row.
    if (a.pro == PRO_JOIN && a.pair && a.nseg == 2 && a.seg[0].N == a.seg[1].N)
      return launch_stream_pe<PRO_JOIN, EPI_GELU_CODES>(a, bits, rs, st, pdl);
    if (a.pro == PRO_NORMRES && !a.pair)
      return launch_stream_pe<PRO_NORMRES, EPI_GELU_CODES>(a, bits, rs, st, pdl);
  } else if (epi == EPI_HEAD) {
    if (a.pro == PRO_JOIN) return launch_stream_pe<PRO_JOIN, EPI_HEAD>(a, bits, rs, st, pdl);
    if (a.pro == PRO_NORM) return launch_stream_pe<PRO_NORM, EPI_HEAD>(a, bits, rs, st, pdl);
    if (a.pro == PRO_X) return launch_stream_pe<PRO_X, EPI_HEAD>(a, bits, rs, st, pdl);
  }
  return cudaErrorInvalidConfiguration;
}

#ifdef G4_TRACE
int trace_take(unsigned long long *out, int max_records) {
  unsigned int n = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&n, g4_trace_n, sizeof(n)) != cudaSuccess) return -1;
  if (n > (1u << 15)) n = 1u << 15;
  if ((int)n > max_records) n = (unsigned int)max_records;
  if (n && cudaMemcpyFromSymbol(out, g4_trace_buf, (size_t)n * 16) != cudaSuccess) return -1;
  cudaMemcpyToSymbol(g4_trace_n, &zero, sizeof(zero));
  return (int)n;
}
#endif

// Failure-detection probe: thread 0 copies `bytes` into shared memory by a bulk copy completing
// on one mbarrier, and arms a second mbarrier for `missing` bytes that no copy delivers. With
// missing > 0 the bounded wait on the second barrier gives up after `limit` polls and raises the
// device error flag, exactly as a kernel whose weight copy never lands does; the thread then waits
// (bounded) for its own copy before the CTA exits. status: [second wait completed, copy landed,
// byte sum of the copy].
__global__ void k_wait_probe(const uint8_t *src, int bytes, int missing, int limit, int32_t *status) {
  __shared__ __align__(128) uint8_t buf[4096];
  __shared__ __align__(8) uint64_t bars[2];
  if (threadIdx.x != 0) return;
  mbar_init(&bars[0], 1);
  mbar_init(&bars[1], 1);
  mbar_fence_init();
  mbar_expect_tx(&bars[0], (uint32_t)bytes);
  bulk_g2s(buf, src, (uint32_t)bytes, &bars[0]);
  mbar_expect_tx(&bars[1], (uint32_t)missing);
  const bool done = mbar_wait_n(&bars[1], 0, limit);
  if (!done) atomicExch(&g4_dev_error, 4);
  const bool landed = mbar_wait(&bars[0], 0);
  uint32_t sum = 0;
  if (landed)
    for (int i = 0; i < bytes; i++) sum += buf[i];
  status[0] = done ? 1 : 0;
  status[1] = landed ? 1 : 0;
  status[2] = (int32_t)sum;
}

cudaError_t launch_wait_probe(const void *src, int bytes, int missing, int limit, int32_t *status,
                              cudaStream_t st) {
  k_wait_probe<<<1, 32, 0, st>>>((const uint8_t *)src, bytes, missing, limit, status);
  return cudaGetLastError();
}

int gemv2_error_take();

int *dev_error_addr() {
  void *p = nullptr;
  return cudaGetSymbolAddress(&p, g4_dev_error) == cudaSuccess ? (int *)p : nullptr;
}

int device_error_take() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g4_dev_error, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g4_dev_error, &zero, sizeof(int));
  const int v2 = gemv2_error_take();
  if (v2 < 0) return -1;
  return v ? v : v2;
}

cudaError_t launch_gemv(const GemvArgs &a, int bits, cudaStream_t st, bool pdl) {
  if (bits == 2) return launch_gemv2(a, st, pdl);
  if (a.seg[0].in_scale == 0.0f) {
    // Uncalibrated f32 path: one column, one segment, x or gelu prologue only.
    if (a.cols != 1 || a.nseg != 1 || !(a.pro == PRO_X || a.pro == PRO_GELU) || a.head)
      return cudaErrorInvalidConfiguration;
    size_t smem = (size_t)a.K * 4;
    int blocks = (a.seg[0].N + 7) / 8;
    if (bits == 4) {
      cudaFuncSetAttribute(k_gemv_f32<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
      return launch_k(k_gemv_f32<4>, dim3(blocks), dim3(256), smem, st, pdl, a);
    }
    cudaFuncSetAttribute(k_gemv_f32<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    return launch_k(k_gemv_f32<8>, dim3(blocks), dim3(256), smem, st, pdl, a);
  }
  return launch_gemv_stream(a, bits, st, pdl);
}

// =====================================================================================
// Gathers (embed-gather / ple-gather-4bit(-sliced), src/kernels/embedGather.ts:176-261,
// 547-577): one thread per 8 columns of a row; the embed scale folds into the row scale first,
// then one multiply per element. The embedding is int4 rows (zero point 8) or the 2-bit family's
// interleaved tiles (zero point 2: column k of row r at bits 2 (r % 16) of word (r / 16) H + k).
// =====================================================================================

__global__ void __launch_bounds__(256)
k_embed(const int32_t *tokens, const uint8_t *embed_w, const uint16_t *embed_s, float embed_scale,
        const uint8_t *const *ple_slices, int ple_rps, const uint16_t *ple_s, int H, int ple_cols,
        int ple_group, float *residual, float *ple_id, int embed_bits) {
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(3001);
  const int c = blockIdx.y;
  const int w = blockIdx.x * 256 + threadIdx.x;
  const int hw = H / 8, pw = ple_cols / 8;
  if (w >= hw + pw) return;
  const int row = tokens[c];
  uint32_t word;
  float scale;
  float *dst;
  if (w < hw && embed_bits == 2) {
    const uint4 *tw = reinterpret_cast<const uint4 *>(embed_w + ((size_t)(row / 16) * H + 8 * w) * 4);
    const uint4 q0 = tw[0], q1 = tw[1];
    const int sh = 2 * (row % 16);
    scale = __fmul_rn(embed_scale, f16_bits_to_f32(embed_s[row]));
    const uint32_t cw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __fmul_rn((float)((int)((cw[j] >> sh) & 3u) - 2), scale);
    dst = residual + (size_t)c * H + 8 * w;
    reinterpret_cast<float4 *>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4 *>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
    return;
  }
  if (w < hw) {
    word = reinterpret_cast<const uint32_t *>(embed_w)[(size_t)row * hw + w];
    scale = __fmul_rn(embed_scale, f16_bits_to_f32(embed_s[row]));
    dst = residual + (size_t)c * H + 8 * w;
  } else {
    const int wp = w - hw;
    const int slice = row / ple_rps, local = row - slice * ple_rps;
    word = reinterpret_cast<const uint32_t *>(ple_slices[slice])[(size_t)local * pw + wp];
    const int groups = ple_cols / ple_group;
    scale = __fmul_rn(16.0f, f16_bits_to_f32(ple_s[(size_t)row * groups + (8 * wp) / ple_group]));
    dst = ple_id + (size_t)c * ple_cols + 8 * wp;
  }
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] = __fmul_rn((float)((int)((word >> (4 * j)) & 15u) - 8), scale);
  reinterpret_cast<float4 *>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4 *>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

cudaError_t launch_embed(const int32_t *tokens, int cols, const uint8_t *embed_w,
                         const uint16_t *embed_s, float embed_scale, const uint8_t *const *ple_slices,
                         int ple_rps, const uint16_t *ple_s, int H, int ple_cols, int ple_group,
                         float *residual, float *ple_id, cudaStream_t st, bool pdl, int embed_bits) {
  int words = H / 8 + ple_cols / 8;
  dim3 grid((words + 255) / 256, cols);
  return launch_k(k_embed, grid, dim3(256), 0, st, pdl, tokens, embed_w, embed_s, embed_scale,
                  ple_slices, ple_rps, ple_s, H, ple_cols, ple_group, residual, ple_id, embed_bits);
}

// Operator form: one table (or one slice of it), arbitrary group size.
__global__ void __launch_bounds__(256)
k_embed_op(const uint8_t *codes, const uint16_t *scales, const int32_t *ids, float *dst, int cols,
           int group, float out_scale, int slice_start, int slice_rows) {
  grid_wait();
  const int s = blockIdx.y;
  const int w = blockIdx.x * 256 + threadIdx.x;
  if (w >= cols / 8) return;
  const int row = ids[s];
  int local = row;
  if (slice_rows > 0) {
    if (row < slice_start || row - slice_start >= slice_rows) return;
    local = row - slice_start;
  }
  const uint32_t word = reinterpret_cast<const uint32_t *>(codes)[(size_t)local * (cols / 8) + w];
  const int groups = cols / group;
  const float scale = __fmul_rn(out_scale, f16_bits_to_f32(scales[(size_t)row * groups + (8 * w) / group]));
  float *d = dst + (size_t)s * cols + 8 * w;
#pragma unroll
  for (int j = 0; j < 8; j++) d[j] = __fmul_rn((float)((int)((word >> (4 * j)) & 15u) - 8), scale);
}

cudaError_t launch_embed_op(const uint8_t *codes, const uint16_t *scales, const int32_t *ids,
                            float *dst, int slots, int cols, int group, float out_scale,
                            int slice_start, int slice_rows, cudaStream_t st, bool pdl) {
  dim3 grid((cols / 8 + 255) / 256, slots);
  return launch_k(k_embed_op, grid, dim3(256), 0, st, pdl, codes, scales, ids, dst, cols, group,
                  out_scale, slice_start, slice_rows);
}

// =====================================================================================
// Dense bf16 linear, per_layer_model_projection (src/kernels/denseMatmul.ts:93-222): warp per
// row; lane l walks the row's 8-element chunks l, l + 32, ... with an fma per element; the
// butterfly closes the row; one multiply by alpha.
// =====================================================================================

template <int COLS>
__global__ void __launch_bounds__(256)
k_dense_bf16(const uint16_t *w, const float *x, int ld_x, float *y, int ld_y, int N, int K, int cols,
             float alpha) {
  extern __shared__ __align__(16) float xs[];  // [COLS][K]
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int row = blockIdx.x * 8 + warp;
  const int nch = K / 8;
  constexpr int MAXCH = 8;  // K <= 8 * 32 * 8 = 2048
  uint4 wv[MAXCH];
#pragma unroll
  for (int i = 0; i < MAXCH; i++) {
    int ch = lane + 32 * i;
    wv[i] = (row < N && ch < nch) ? ldg_stream(w + (size_t)row * K + 8 * ch) : make_uint4(0, 0, 0, 0);
  }
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(3002);
  for (int c = 0; c < cols; c++)
    for (int i = t; i < K / 4; i += 256)
      reinterpret_cast<float4 *>(xs + c * K)[i] = reinterpret_cast<const float4 *>(x + (size_t)c * ld_x)[i];
  __syncthreads();
  if (row >= N) return;
  float acc[COLS];
#pragma unroll
  for (int c = 0; c < COLS; c++) acc[c] = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXCH; i++) {
    int ch = lane + 32 * i;
    if (ch < nch) {
      const uint32_t ww[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
      for (int c = 0; c < COLS; c++) {
        if (c < cols) {
          const float4 xa = reinterpret_cast<const float4 *>(xs + c * K + 8 * ch)[0];
          const float4 xb = reinterpret_cast<const float4 *>(xs + c * K + 8 * ch)[1];
          const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
          float v = acc[c];
#pragma unroll
          for (int j = 0; j < 8; j++) {
            float wf = (j & 1) ? __uint_as_float(ww[j >> 1] & 0xffff0000u) : __uint_as_float(ww[j >> 1] << 16);
            v = fmaf(wf, xv[j], v);
          }
          acc[c] = v;
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < COLS; c++) {
    float sum = warp_sum_bfly(acc[c]);
    if (lane == 0 && c < cols) y[(size_t)c * ld_y + row] = __fmul_rn(alpha, sum);
  }
}

__device__ __forceinline__ void cp_async16(void *dst_smem, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Many columns (prefill, wide batches): warp w of a CTA keeps rows R (8 b + w) .. + R - 1 in
// registers (read once, before the dependency wait) and walks the columns in tiles of 8 staged
// in shared memory, double-buffered: the next tile's copy (cp.async) runs under this tile's
// FMAs. Each (row, column) sum is the same per-lane chunk order and butterfly as k_dense_bf16.
template <int MAXCH>
__global__ void __launch_bounds__(256)
k_dense_bf16_wide(const uint16_t *w, const float *x, int ld_x, float *y, int ld_y, int N, int K, int cols,
                  float alpha) {
  constexpr int R = MAXCH <= 6 ? 4 : 2, T = 8;
  extern __shared__ __align__(16) float xs_both[];  // [2][T][K]
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int row0 = (blockIdx.x * 8 + warp) * R;
  const int nch = K / 8;
  uint4 wv[R][MAXCH];
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int i = 0; i < MAXCH; i++) {
      const int ch = lane + 32 * i;
      wv[r][i] = (row0 + r < N && ch < nch) ? ldg_stream(w + (size_t)(row0 + r) * K + 8 * ch)
                                            : make_uint4(0, 0, 0, 0);
    }
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(3002);
  // This CTA's columns: grid.y splits them into ranges of whole tiles.
  const int span = ((cols + (int)gridDim.y - 1) / (int)gridDim.y + T - 1) / T * T;
  const int c_begin = (int)blockIdx.y * span, c_end = min(cols, c_begin + span);
  auto stage = [&](int c0) {   // request tile c0 into buffer (c0 / T) & 1
    float *dst = xs_both + ((c0 / T) & 1) * T * K;
    const int nc = min(T, c_end - c0);
    for (int i = t; i < nc * (K / 4); i += 256) {
      const int c = i / (K / 4), k4 = i - c * (K / 4);
      cp_async16(dst + c * K + 4 * k4, x + (size_t)(c0 + c) * ld_x + 4 * k4);
    }
    cp_async_commit();
  };
  if (c_begin < c_end) stage(c_begin);
  for (int c0 = c_begin; c0 < c_end; c0 += T) {
    const int nc = min(T, c_end - c0);
    const float *xs = xs_both + ((c0 / T) & 1) * T * K;
    if (c0 + T < c_end) stage(c0 + T);
    else cp_async_commit();   // an empty group keeps the wait below uniform
    cp_async_wait_1();        // this tile's copies (all but the newest group) have landed
    __syncthreads();
    float acc[R][T];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int c = 0; c < T; c++) acc[r][c] = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXCH; i++) {
      const int ch = lane + 32 * i;
      if (ch < nch) {
#pragma unroll
        for (int c = 0; c < T; c++) {
          if (c < nc) {
            const float4 xa = reinterpret_cast<const float4 *>(xs + c * K + 8 * ch)[0];
            const float4 xb = reinterpret_cast<const float4 *>(xs + c * K + 8 * ch)[1];
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int r = 0; r < R; r++) {
              const uint32_t ww[4] = {wv[r][i].x, wv[r][i].y, wv[r][i].z, wv[r][i].w};
              float v = acc[r][c];
#pragma unroll
              for (int j = 0; j < 8; j++) {
                const float wf = (j & 1) ? __uint_as_float(ww[j >> 1] & 0xffff0000u)
                                         : __uint_as_float(ww[j >> 1] << 16);
                v = fmaf(wf, xv[j], v);
              }
              acc[r][c] = v;
            }
          }
        }
      }
    }
    // Close the 32 sums; lane 8 r + c stores (row0 + r, column c0 + c).
    float mine = 0.0f;
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int c = 0; c < T; c++) {
        const float sum = warp_sum_bfly(acc[r][c]);
        if (lane == r * T + c) mine = sum;
      }
    const int r = lane / T, c = lane % T;
    if (r < R && row0 + r < N && c < nc) y[(size_t)(c0 + c) * ld_y + row0 + r] = __fmul_rn(alpha, mine);
    __syncthreads();   // the next iteration's copy overwrites the buffer read here
  }
}

cudaError_t launch_dense_bf16(const uint16_t *w, const float *x, int ld_x, float *y, int ld_y, int N, int K,
                              int cols, float alpha, cudaStream_t st, bool pdl) {
  if (K % 8 != 0 || K > 2048) return cudaErrorInvalidValue;
  if (cols > 8) {
    const size_t smem = (size_t)2 * 8 * K * 4;   // two tiles of 8 columns
    // Column ranges along grid.y: the split (up to 16, at least two tiles each) that fills the
    // SMs' waves best (one CTA per SM).
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int row_ctas = K <= 1536 ? (N + 31) / 32 : (N + 15) / 16;
    int gy = 1;
    double best = 0.0;
    for (int split = 1; split <= 16 && (split == 1 || cols / split >= 16); split++) {
      const int ctas = row_ctas * split, waves = (ctas + sms - 1) / sms;
      const double eff = (double)ctas / ((double)waves * sms) - 0.01 * split;   // small cost per split
      if (eff > best) {
        best = eff;
        gy = split;
      }
    }
    if (K <= 1536) {
      const dim3 grid((N + 31) / 32, gy);
      cudaFuncSetAttribute(k_dense_bf16_wide<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 1024);
      return launch_k(k_dense_bf16_wide<6>, grid, dim3(256), smem, st, pdl, w, x, ld_x, y, ld_y, N, K, cols, alpha);
    }
    const dim3 grid((N + 15) / 16, gy);
    cudaFuncSetAttribute(k_dense_bf16_wide<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 1024);
    return launch_k(k_dense_bf16_wide<8>, grid, dim3(256), smem, st, pdl, w, x, ld_x, y, ld_y, N, K, cols, alpha);
  }
  cudaError_t e = cudaSuccess;
  for (int c0 = 0; c0 < cols && e == cudaSuccess; c0 += 8) {
    int nc = cols - c0 < 8 ? cols - c0 : 8;
    size_t smem = (size_t)nc * K * 4;
    dim3 grid((N + 7) / 8);
    const float *xc = x + (size_t)c0 * ld_x;
    float *yc = y + (size_t)c0 * ld_y;
    if (nc <= 1) e = launch_k(k_dense_bf16<1>, grid, dim3(256), smem, st, pdl, w, xc, ld_x, yc, ld_y, N, K, nc, alpha);
    else if (nc <= 2) e = launch_k(k_dense_bf16<2>, grid, dim3(256), smem, st, pdl, w, xc, ld_x, yc, ld_y, N, K, nc, alpha);
    else if (nc <= 4) e = launch_k(k_dense_bf16<4>, grid, dim3(256), smem, st, pdl, w, xc, ld_x, yc, ld_y, N, K, nc, alpha);
    else {
      cudaFuncSetAttribute(k_dense_bf16<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
      e = launch_k(k_dense_bf16<8>, grid, dim3(256), smem, st, pdl, w, xc, ld_x, yc, ld_y, N, K, nc, alpha);
    }
  }
  return e;
}

// Per-layer input combine (src/plan.ts:669-749, src/execute.ts:540-556): per 256-wide group,
// normed = norm(proj) * gain; sum = normed + identity; out = 2^-0.5 * sum.
__global__ void __launch_bounds__(256)
k_ple_combine(const float *proj, const float *identity, const float *gain, float *out,
              int row_width, int group_dim, float eps, float scale) {
  __shared__ float red[8];
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(3003);
  const int c = blockIdx.x, g = blockIdx.y, t = threadIdx.x;
  const size_t base = (size_t)c * row_width + (size_t)g * group_dim;
  const float inv = rms_inv(block_sumsq256(proj + base, group_dim, red), group_dim, eps);
  for (int ch = t; ch < group_dim / 4; ch += 256) {
    float4 p = reinterpret_cast<const float4 *>(proj + base)[ch];
    float4 id = reinterpret_cast<const float4 *>(identity + base)[ch];
    float4 gg = reinterpret_cast<const float4 *>(gain)[ch];
    float4 n = f4_norm_apply(p, inv, gg);
    float4 r = f4_scale(f4_add(n, id), scale);
    reinterpret_cast<float4 *>(out + base)[ch] = r;
  }
}

cudaError_t launch_ple_combine(const float *proj, const float *identity, const float *gain,
                               float *out, int cols, int groups, int group_dim, int row_width, float eps,
                               float scale, cudaStream_t st, bool pdl) {
  return launch_k(k_ple_combine, dim3(cols, groups), dim3(256), 0, st, pdl, proj, identity, gain,
                  out, row_width, group_dim, eps, scale);
}

// =====================================================================================
// Attention prologue (q-norm-rope and kv-norm-rope-store, src/kernels/attnPrologue.ts:83-260):
// block y < heads normalises and rotates query head y of column x; y == heads the K row (gain,
// rotation, store), y == heads + 1 the V row (weightless norm, store).
// =====================================================================================

__global__ void __launch_bounds__(256) k_attn_prologue(const AttnPro a) {
  extern __shared__ __align__(16) float nrm[];  // [hd]
  __shared__ float red[8];
  grid_launch_dependents();
  grid_wait();
  const int c = blockIdx.x, role = blockIdx.y, t = threadIdx.x;
  const int hd = a.hd, pairs = hd / 2;
  const int tab = a.tab_row ? a.tab_row[c] : c / a.rows_per_col_tab;
  const float *src;
  const float *gain;
  if (role < a.heads) {
    src = a.q + (size_t)c * a.q_ld + (size_t)role * hd;
    gain = a.qgain;
  } else if (role == a.heads) {
    src = a.k + (size_t)c * a.kv_ld;
    gain = a.kgain;
  } else {
    src = a.v + (size_t)c * a.kv_ld;
    gain = nullptr;
  }
  const float inv = rms_inv(block_sumsq256(src, hd, red), hd, a.eps);
  for (int i = t; i < hd; i += 256) {
    float v = __fmul_rn(src[i], inv);
    nrm[i] = gain ? __fmul_rn(v, gain[i]) : v;
  }
  __syncthreads();
  const int seq = a.refs.seq ? a.refs.seq[c] : 0;
  const int cpos = a.refs.pos ? a.refs.pos[c] : a.refs.pos_base + c;
  float *vbase = a.cache ? a.cache + (size_t)seq * a.seq_stride : nullptr;
  if (role == a.heads + 1) {
    float *dst = vbase + (size_t)a.max_ctx * hd + (size_t)cpos * hd;
    for (int i = t; i < hd; i += 256) dst[i] = nrm[i];
    return;
  }
  float *dst = role < a.heads ? a.qr + (size_t)c * a.heads * hd + (size_t)role * hd
                              : vbase + (size_t)cpos * hd;
  const float *ct = a.cos_tab + (size_t)tab * pairs;
  const float *stb = a.sin_tab + (size_t)tab * pairs;
  for (int i = t; i < pairs; i += 256) {
    float lo = nrm[i], hi = nrm[i + pairs], cc = ct[i], ss = stb[i];
    dst[i] = __fsub_rn(__fmul_rn(lo, cc), __fmul_rn(hi, ss));
    dst[i + pairs] = __fadd_rn(__fmul_rn(hi, cc), __fmul_rn(lo, ss));
  }
}

// The same prologue at head dim 256 / 512 with one warp per (column, role) row (eight rows per
// CTA, no block barriers): head_norm_rope_warp's sum of squares follows block_sumsq256's order,
// so the results are the block kernel's bit for bit.
template <int HD>
__global__ void __launch_bounds__(256) k_attn_prologue_w(const AttnPro a) {
  grid_launch_dependents();
  grid_wait();
  const int lane = threadIdx.x & 31;
  const int roles = a.heads + (a.k ? 2 : 0);
  const int gw = (int)blockIdx.x * 8 + (int)(threadIdx.x >> 5);
  if (gw >= a.cols * roles) return;
  const int c = gw / roles, role = gw - c * roles;
  const int tab = a.tab_row ? a.tab_row[c] : c / a.rows_per_col_tab;
  const float *ct = a.cos_tab + (size_t)tab * (HD / 2);
  const float *stb = a.sin_tab + (size_t)tab * (HD / 2);
  if (role < a.heads) {
    head_norm_rope_warp<HD>(a.q + (size_t)c * a.q_ld + (size_t)role * HD, a.qgain, ct, stb, a.eps,
                            a.qr + (size_t)c * a.heads * HD + (size_t)role * HD, nullptr, lane);
    return;
  }
  const int seq = a.refs.seq ? a.refs.seq[c] : 0;
  const int cpos = a.refs.pos ? a.refs.pos[c] : a.refs.pos_base + c;
  float *kbase = a.cache + (size_t)seq * a.seq_stride;
  if (role == a.heads)
    head_norm_rope_warp<HD>(a.k + (size_t)c * a.kv_ld, a.kgain, ct, stb, a.eps, kbase + (size_t)cpos * HD,
                            nullptr, lane);
  else
    head_norm_rope_warp<HD>(a.v + (size_t)c * a.kv_ld, nullptr, nullptr, nullptr, a.eps,
                            kbase + (size_t)a.max_ctx * HD + (size_t)cpos * HD, nullptr, lane);
}

cudaError_t launch_attn_prologue(const AttnPro &a, cudaStream_t st, bool pdl) {
  int roles = a.heads + (a.k ? 2 : 0);
  if ((a.hd == 256 || a.hd == 512) && (!a.k || a.cache)) {
    const dim3 grid((a.cols * roles + 7) / 8);
    if (a.hd == 256) return launch_k(k_attn_prologue_w<256>, grid, dim3(256), 0, st, pdl, a);
    return launch_k(k_attn_prologue_w<512>, grid, dim3(256), 0, st, pdl, a);
  }
  return launch_k(k_attn_prologue, dim3(a.cols, roles), dim3(256), (size_t)a.hd * 4, st, pdl, a);
}

// =====================================================================================
// Attention (src/kernels/attention.ts:339-752): scale 1.0, window [p - W + 1, p] or global,
// one KV head shared by every query head. Block (c, b) takes the 64 positions of absolute block
// b0 + b for all heads: four lanes per position split the head into the reference's four score
// accumulators (vec4 chunk i feeds accumulator i mod 4; s = (a0 + a1) + (a2 + a3)); the block max
// m, p_j = exp(s_j - m), l = sum p_j and o = sum p_j v_j in ascending j are written as a partial.
// The merge folds the block partials in ascending order with the flash rescale.
// =====================================================================================

template <int HD>
__global__ void __launch_bounds__(256) k_attn_blocks(const AttnArgs a) {
  constexpr int NH = 8;
  constexpr int NC = HD / 4;          // vec4 chunks per row
  constexpr int HPG = HD / 128;       // heads per PV thread group
  extern __shared__ __align__(16) float sm[];
  float *qs = sm;                     // [NH][HD]
  float *ss = qs + NH * HD;           // [NH][64]
  float *ps = ss + NH * ATT_BLK;      // [NH][64]
  float *ms = ps + NH * ATT_BLK;      // [NH]
  float *vs = ms + 4 * NH;            // [64][HD]: the block's V rows (16-byte aligned)
  grid_launch_dependents();
  grid_wait();
  const int c = blockIdx.x, bi = blockIdx.y, t = threadIdx.x;
  int p, lo, hi;
  attn_range(a, c, &p, &lo, &hi);
  const int b = lo / ATT_BLK + bi;
  if (b * ATT_BLK > hi) return;
  const int j0 = max(b * ATT_BLK, lo), j1 = min(b * ATT_BLK + ATT_BLK - 1, hi);
  const int seq = a.refs.seq ? a.refs.seq[c] : 0;
  const float *K = a.cache + (size_t)seq * a.seq_stride;
  const float *V = K + (size_t)a.max_ctx * HD;

  const float4 *qsrc = reinterpret_cast<const float4 *>(a.qr + (size_t)c * NH * HD);
  for (int i = t; i < NH * NC; i += 256) reinterpret_cast<float4 *>(qs)[i] = qsrc[i];
  // V rows j0..j1 into shared memory: independent loads, consumed after the scores.
  {
    const int nrow = j1 - j0 + 1;
    const float4 *vsrc = reinterpret_cast<const float4 *>(V + (size_t)j0 * HD);
    float4 *vdst = reinterpret_cast<float4 *>(vs + (size_t)(j0 - b * ATT_BLK) * HD);
    for (int i = t; i < nrow * NC; i += 256) vdst[i] = vsrc[i];
  }
  __syncthreads();

  // Scores: thread (jl, m) with m = t & 3 computes accumulator m of position jl for all heads.
  {
    const int jl = t >> 2, m = t & 3;
    const int j = b * ATT_BLK + jl;
    const bool valid = j >= j0 && j <= j1;
    float acc[NH];
#pragma unroll
    for (int h = 0; h < NH; h++) acc[h] = 0.0f;
    if (valid) {
      const float4 *kr = reinterpret_cast<const float4 *>(K + (size_t)j * HD);
#pragma unroll 4
      for (int cc = m; cc < NC; cc += 4) {
        const float4 k4 = kr[cc];
#pragma unroll
        for (int h = 0; h < NH; h++) {
          const float4 q4 = reinterpret_cast<const float4 *>(qs + h * HD)[cc];
          float v = acc[h];
          v = fmaf(q4.x, k4.x, v);
          v = fmaf(q4.y, k4.y, v);
          v = fmaf(q4.z, k4.z, v);
          v = fmaf(q4.w, k4.w, v);
          acc[h] = v;
        }
      }
    }
#pragma unroll
    for (int h = 0; h < NH; h++) {
      float v1 = __fadd_rn(acc[h], __shfl_xor_sync(0xffffffffu, acc[h], 1));
      float v2 = __fadd_rn(v1, __shfl_xor_sync(0xffffffffu, v1, 2));
      if (m == 0) ss[h * ATT_BLK + jl] = valid ? v2 : -FLT_MAX;
    }
  }
  __syncthreads();
  // Block max and probabilities: warp h handles head h.
  {
    const int h = t >> 5, lane = t & 31;
    float s0 = ss[h * ATT_BLK + lane], s1 = ss[h * ATT_BLK + lane + 32];
    float mx = fmaxf(s0, s1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int ja = b * ATT_BLK + lane, jb = ja + 32;
    ps[h * ATT_BLK + lane] = (ja >= j0 && ja <= j1) ? g4_exp(__fsub_rn(s0, mx)) : 0.0f;
    ps[h * ATT_BLK + lane + 32] = (jb >= j0 && jb <= j1) ? g4_exp(__fsub_rn(s1, mx)) : 0.0f;
    if (lane == 0) ms[h] = mx;
  }
  __syncthreads();
  // Weighted V: thread (hg, dc) owns vec4 chunk dc of heads hg * HPG .. + HPG - 1.
  {
    const int dc = t % NC, hg = t / NC;
    float4 o[HPG];
    float l[HPG];
#pragma unroll
    for (int hh = 0; hh < HPG; hh++) {
      o[hh] = make_float4(0.f, 0.f, 0.f, 0.f);
      l[hh] = 0.0f;
    }
#pragma unroll 4
    for (int j = j0; j <= j1; j++) {
      const int jl = j - b * ATT_BLK;
      const float4 v4 = reinterpret_cast<const float4 *>(vs + (size_t)jl * HD)[dc];
#pragma unroll
      for (int hh = 0; hh < HPG; hh++) {
        const float pj = ps[(hg * HPG + hh) * ATT_BLK + jl];
        o[hh].x = fmaf(pj, v4.x, o[hh].x);
        o[hh].y = fmaf(pj, v4.y, o[hh].y);
        o[hh].z = fmaf(pj, v4.z, o[hh].z);
        o[hh].w = fmaf(pj, v4.w, o[hh].w);
        l[hh] = __fadd_rn(l[hh], pj);
      }
    }
#pragma unroll
    for (int hh = 0; hh < HPG; hh++) {
      const int h = hg * HPG + hh;
      const size_t slot = ((size_t)c * a.max_blocks + bi) * NH + h;
      reinterpret_cast<float4 *>(a.part_o + slot * HD)[dc] = o[hh];
      if (dc == 0) {
        a.part_m[slot] = ms[h];
        a.part_l[slot] = l[hh];
      }
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(256) k_attn_merge(const AttnArgs a) {
  constexpr int NH = 8;
  grid_launch_dependents();
  grid_wait();
  const int c = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
  int p, lo, hi;
  attn_range(a, c, &p, &lo, &hi);
  const int nb = hi / ATT_BLK - lo / ATT_BLK + 1;
  constexpr int DPT = HD / 256;  // dims per thread
  size_t slot = ((size_t)c * a.max_blocks) * NH + h;
  float M = a.part_m[slot], L = a.part_l[slot];
  float O[DPT];
#pragma unroll
  for (int d = 0; d < DPT; d++) O[d] = a.part_o[slot * HD + t + 256 * d];
  for (int bi = 1; bi < nb; bi++) {
    slot = ((size_t)c * a.max_blocks + bi) * NH + h;
    const float m = a.part_m[slot], l = a.part_l[slot];
    const float Mn = fmaxf(M, m);
    const float ea = g4_exp(__fsub_rn(M, Mn)), ec = g4_exp(__fsub_rn(m, Mn));
    L = __fadd_rn(__fmul_rn(L, ea), __fmul_rn(l, ec));
#pragma unroll
    for (int d = 0; d < DPT; d++)
      O[d] = __fadd_rn(__fmul_rn(O[d], ea), __fmul_rn(a.part_o[slot * HD + t + 256 * d], ec));
    M = Mn;
  }
  float *out = a.out + (size_t)c * NH * HD + (size_t)h * HD;
#pragma unroll
  for (int d = 0; d < DPT; d++) out[t + 256 * d] = __fdiv_rn(O[d], L);
}

// Prefill attention (a chunk of consecutive positions of one sequence): CTA = QT consecutive
// queries x 8 heads = NP (query, head) pairs. It walks the 64-position blocks in ascending order
// and folds each block into a running (M, L, O) right away. Per (query, block) the arithmetic is
// k_attn_blocks' (four-accumulator scores, block max, exp, ascending l and o chains) and the fold
// is k_attn_merge's in the same ascending block order, so the result is bit-identical.
//
// Register micro-tiles keep the shared-memory traffic below the FMA rate: a score thread owns
// accumulator m (chunks m, m + 4, ...) of PA pairs x 8 positions, loading PA q and 8 K vectors
// per chunk for PA x 8 x 4 FMAs; a PV thread owns 8 pairs x 2 vec4 columns. K and V rows are
// staged KVR at a time (all 64 at head dim 256, 32 at 512) in one padded buffer; the positions
// of score group jg are jg, jg + 8, ... so the padded rows a warp reads fall in distinct banks.
// Four consecutive outputs k0 .. k0 + 3 of column col, snapped to the next linear's codes
// (srq_code_r, the snap every prologue uses).
// k0 is a multiple of 4: K order takes one 32-bit store; the int4 GEMV's order keeps codes k0 and
// k0 + 2 adjacent, and k0 + 1 and k0 + 3 (two 16-bit stores, as the GEMV prologue writes them).
__device__ __forceinline__ void attn_codes4(const AttnCodes &cd, int col, int k0, float4 v) {
  if (!cd.out) return;
  const float r = __fdiv_rn(1.0f, cd.scale);
  const uint32_t q0 = srq_code_r(v.x, cd.scale, r) & 255, q1 = srq_code_r(v.y, cd.scale, r) & 255;
  const uint32_t q2 = srq_code_r(v.z, cd.scale, r) & 255, q3 = srq_code_r(v.w, cd.scale, r) & 255;
  uint8_t *o = cd.out + (size_t)col * cd.ld;
  if (cd.bits == 4) {
    *reinterpret_cast<uint16_t *>(o + code_pos(k0, 4)) = (uint16_t)(q0 | (q2 << 8));
    *reinterpret_cast<uint16_t *>(o + code_pos(k0 + 1, 4)) = (uint16_t)(q1 | (q3 << 8));
  } else {
    *reinterpret_cast<uint32_t *>(o + k0) = q0 | (q1 << 8) | (q2 << 16) | (q3 << 24);
  }
}

template <int HD>
__global__ void __launch_bounds__(256, 1) k_attn_prefill(const AttnArgs a) {
  constexpr int NH = 8, NC = HD / 4, QT = 2048 / HD, NP = QT * NH;   // pairs per CTA
  constexpr int PA = NP / 8;                   // score micro-tile pairs (8 pair groups)
  constexpr int KVR = HD <= 256 ? 64 : 32;     // K / V rows staged at a time
  // Padded row (floats): a quarter warp's score loads read two adjacent rows x four 16-byte
  // columns, and a 64-byte row shift puts those eight pieces in eight different bank groups.
  constexpr int LDK = HD + 16;
  constexpr int PB = 8, DB = 2;                // PV micro-tile: pairs x vec4 columns
  constexpr int NDG = NC / DB;                 // PV column groups
  static_assert((NP / PB) * NDG == 256, "PV tiling covers the CTA");
  extern __shared__ __align__(16) float sm[];
  float *qs = sm;                              // [NP][HD]
  float *kv = qs + NP * HD;                    // [2][KVR][LDK] K / V stages, double-buffered
  float *ss = kv + 2 * KVR * LDK;              // [NP][64] scores, then probabilities
  float *mb = ss + NP * ATT_BLK;               // [NP] block max
  float *lb = mb + NP;                         // [NP] block sum
  float *RM = lb + NP;                         // [NP] running max
  float *RL = RM + NP;                         // [NP] running sum
  float *ea = RL + NP;                         // [NP]
  float *ec = ea + NP;                         // [NP]
  uint64_t *sbar = reinterpret_cast<uint64_t *>(ec + NP);   // [2] stage buffers' copies
  int *mode = reinterpret_cast<int *>(sbar + 2);  // [NP] 0 skip, 1 copy, 2 fold
  int *qp = mode + NP;                         // [QT] positions
  int *qlo = qp + QT;                          // [QT] window start
  grid_launch_dependents();
  const int t = threadIdx.x;
  if (t == 0) {
    mbar_init(&sbar[0], 1);
    mbar_init(&sbar[1], 1);
    mbar_fence_init();
  }
  grid_wait();
  G4_TRACE_POINT(2100 + HD);
  // The last query tiles of a chunk see the most keys: they start first (longest work first).
  const int c0 = ((int)gridDim.x - 1 - (int)blockIdx.x) * QT;
  const int nq = min(QT, a.cols - c0);
  const int seq = a.refs.seq ? a.refs.seq[c0] : 0;
  const float *K = a.cache + (size_t)seq * a.seq_stride;
  const float *V = K + (size_t)a.max_ctx * HD;
  if (t < QT) {
    int p = -1, lo = 0, hi = -1;
    if (t < nq) attn_range(a, c0 + t, &p, &lo, &hi);
    qp[t] = t < nq ? hi : -1;
    qlo[t] = t < nq ? lo : 1 << 30;
  }
  for (int i = t; i < NP; i += 256) {
    RM[i] = -FLT_MAX;
    RL[i] = 0.0f;
  }
  for (int i = t; i < nq * NH * NC; i += 256)
    reinterpret_cast<float4 *>(qs)[i] = reinterpret_cast<const float4 *>(a.qr + (size_t)c0 * NH * HD)[i];
  for (int i = nq * NH * NC + t; i < NP * NC; i += 256)
    reinterpret_cast<float4 *>(qs)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  int ulo = 1 << 30, uhi = -1;
#pragma unroll
  for (int q = 0; q < QT; q++) {
    ulo = min(ulo, qlo[q]);
    uhi = max(uhi, qp[q]);
  }
  // K and V rows reach shared memory by one bulk copy per row into the padded layout, a stage
  // ahead: stage s (block b0 + s / SPB; its K halves, then its V halves) lands in buffer s & 1
  // while stage s - 1 is computed. Only the rows some query of the tile can see are copied; the
  // other rows of a stage keep stale values, whose scores are masked and whose V rows are never
  // read.
  constexpr int SPB = 2 * (ATT_BLK / KVR);     // stages per block
  const int b0 = ulo / ATT_BLK;
  const int nstage = (uhi / ATT_BLK - b0 + 1) * SPB;
  auto issue = [&](int st) {
    const int b = b0 + st / SPB, w = st % SPB, r0 = (w % (SPB / 2)) * KVR;
    const int jb = b * ATT_BLK;
    const int j0 = max(max(jb, ulo), jb + r0), j1 = min(min(jb + ATT_BLK - 1, uhi), jb + r0 + KVR - 1);
    const int n = j1 >= j0 ? j1 - j0 + 1 : 0;
    const float *src = w < SPB / 2 ? K : V;
    float *dst = kv + (size_t)(st & 1) * KVR * LDK;
    const int lane = t & 31;
    if (lane == 0) mbar_expect_tx(&sbar[st & 1], (uint32_t)n * HD * 4);
    __syncwarp();
    for (int i = lane; i < n; i += 32)
      bulk_g2s(dst + (size_t)(j0 + i - jb - r0) * LDK, src + (size_t)(j0 + i) * HD, HD * 4, &sbar[st & 1]);
  };
  // Bounded wait for stage st; on a timeout the flag is raised and the stage is used as it is.
  auto stage_wait = [&](int st) {
    if (!mbar_wait(&sbar[st & 1], (uint32_t)((st >> 1) & 1)) && t == 0) atomicExch(&g4_dev_error, 2);
  };
  if (t < 32) issue(0);
  int stg = 0;
  // Score thread: accumulator m, pair group pg (pairs pg*PA ..), position group jg.
  const int m = t & 3, mt = t >> 2, pg = mt >> 3, jg = mt & 7;
  // PV thread: pairs pb*PB .., vec4 columns dg + NDG * d.
  const int pb = t / NDG, dg = t % NDG;
  float4 O[PB][DB];
#pragma unroll
  for (int i = 0; i < PB; i++)
#pragma unroll
    for (int d = 0; d < DB; d++) O[i][d] = make_float4(0.f, 0.f, 0.f, 0.f);

  for (int b = ulo / ATT_BLK; b * ATT_BLK <= uhi; b++) {
    const int jb = b * ATT_BLK;
    const int jlo = max(jb, ulo), jhi = min(jb + ATT_BLK - 1, uhi);
    // ---- scores, KVR rows of K at a time
#pragma unroll 1
    for (int r0 = 0; r0 < ATT_BLK; r0 += KVR) {
      __syncthreads();   // the previous stage's rows are no longer read: its buffer takes the next
      if (t < 32 && stg + 1 < nstage) issue(stg + 1);
      stage_wait(stg);
      const float *kvs = kv + (size_t)(stg & 1) * KVR * LDK;
      stg++;
      constexpr int JB = KVR / 8;               // this stage's positions per score thread
      float acc[PA][JB];
#pragma unroll
      for (int x = 0; x < PA; x++)
#pragma unroll
        for (int y = 0; y < JB; y++) acc[x][y] = 0.0f;
#pragma unroll 2
      for (int cc = m; cc < NC; cc += 4) {
        float4 qv[PA], kk[JB];
#pragma unroll
        for (int x = 0; x < PA; x++) qv[x] = reinterpret_cast<const float4 *>(qs + (size_t)(pg * PA + x) * HD)[cc];
#pragma unroll
        for (int y = 0; y < JB; y++) kk[y] = reinterpret_cast<const float4 *>(kvs + (size_t)(jg + 8 * y) * LDK)[cc];
#pragma unroll
        for (int x = 0; x < PA; x++)
#pragma unroll
          for (int y = 0; y < JB; y++) {
            float v = acc[x][y];
            v = fmaf(qv[x].x, kk[y].x, v);
            v = fmaf(qv[x].y, kk[y].y, v);
            v = fmaf(qv[x].z, kk[y].z, v);
            v = fmaf(qv[x].w, kk[y].w, v);
            acc[x][y] = v;
          }
      }
#pragma unroll
      for (int x = 0; x < PA; x++)
#pragma unroll
        for (int y = 0; y < JB; y++) {
          const float v1 = __fadd_rn(acc[x][y], __shfl_xor_sync(0xffffffffu, acc[x][y], 1));
          const float v2 = __fadd_rn(v1, __shfl_xor_sync(0xffffffffu, v1, 2));
          const int pi = pg * PA + x, q = pi / NH, jl = r0 + jg + 8 * y, j = jb + jl;
          if (m == 0) ss[pi * ATT_BLK + jl] = (j >= qlo[q] && j <= qp[q]) ? v2 : -FLT_MAX;
        }
    }
    __syncthreads();
    // ---- block max and probabilities per pair (warp w: pairs w, w + 8, ...)
    {
      const int lane = t & 31, warp = t >> 5;
      for (int i = warp; i < NP; i += 8) {
        const int q = i / NH;
        const float s0 = ss[i * ATT_BLK + lane], s1 = ss[i * ATT_BLK + lane + 32];
        float mx = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const int ja = jb + lane, jc = ja + 32;
        ss[i * ATT_BLK + lane] = (ja >= qlo[q] && ja <= qp[q]) ? g4_exp(__fsub_rn(s0, mx)) : 0.0f;
        ss[i * ATT_BLK + lane + 32] = (jc >= qlo[q] && jc <= qp[q]) ? g4_exp(__fsub_rn(s1, mx)) : 0.0f;
        if (lane == 0) mb[i] = mx;
      }
    }
    // ---- weighted V and the probability sums, ascending j, KVR rows of V at a time
    float4 o[PB][DB];
    float l[PB];
#pragma unroll
    for (int i = 0; i < PB; i++) {
      l[i] = 0.0f;
#pragma unroll
      for (int d = 0; d < DB; d++) o[i][d] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll 1
    for (int r0 = 0; r0 < ATT_BLK; r0 += KVR) {
      __syncthreads();   // scores / the previous stage are no longer read: its buffer takes the next
      const int slo = max(jlo - jb, r0), shi = min(jhi - jb, r0 + KVR - 1);
      if (t < 32 && stg + 1 < nstage) issue(stg + 1);
      stage_wait(stg);
      const float *kvs = kv + (size_t)(stg & 1) * KVR * LDK;
      stg++;
      // Ascending rows; the probabilities of four aligned rows come in one 16-byte load per pair.
      auto pv_row = [&](int jl, const float *pj) {
        float4 v4[DB];
#pragma unroll
        for (int d = 0; d < DB; d++) v4[d] = reinterpret_cast<const float4 *>(kvs + (size_t)(jl - r0) * LDK)[dg + NDG * d];
#pragma unroll
        for (int i = 0; i < PB; i++) {
#pragma unroll
          for (int d = 0; d < DB; d++) {
            o[i][d].x = fmaf(pj[i], v4[d].x, o[i][d].x);
            o[i][d].y = fmaf(pj[i], v4[d].y, o[i][d].y);
            o[i][d].z = fmaf(pj[i], v4[d].z, o[i][d].z);
            o[i][d].w = fmaf(pj[i], v4[d].w, o[i][d].w);
          }
          l[i] = __fadd_rn(l[i], pj[i]);
        }
      };
      int jl = slo;
      for (; jl <= shi && (jl & 3); jl++) {
        float pj[PB];
#pragma unroll
        for (int i = 0; i < PB; i++) pj[i] = ss[(pb * PB + i) * ATT_BLK + jl];
        pv_row(jl, pj);
      }
#pragma unroll 1
      for (; jl + 3 <= shi; jl += 4) {
        float4 p4[PB];
#pragma unroll
        for (int i = 0; i < PB; i++) p4[i] = *reinterpret_cast<const float4 *>(ss + (pb * PB + i) * ATT_BLK + jl);
        float pj[PB];
#pragma unroll
        for (int i = 0; i < PB; i++) pj[i] = p4[i].x;
        pv_row(jl, pj);
#pragma unroll
        for (int i = 0; i < PB; i++) pj[i] = p4[i].y;
        pv_row(jl + 1, pj);
#pragma unroll
        for (int i = 0; i < PB; i++) pj[i] = p4[i].z;
        pv_row(jl + 2, pj);
#pragma unroll
        for (int i = 0; i < PB; i++) pj[i] = p4[i].w;
        pv_row(jl + 3, pj);
      }
      for (; jl <= shi; jl++) {
        float pj[PB];
#pragma unroll
        for (int i = 0; i < PB; i++) pj[i] = ss[(pb * PB + i) * ATT_BLK + jl];
        pv_row(jl, pj);
      }
    }
    if (dg == 0) {
#pragma unroll
      for (int i = 0; i < PB; i++) lb[pb * PB + i] = l[i];
    }
    __syncthreads();
    // ---- the fold of this block into each pair's running (M, L): k_attn_merge's formula
    for (int i = t; i < NP; i += 256) {
      const int q = i / NH;
      const bool valid = jb <= qp[q] && jb + ATT_BLK - 1 >= qlo[q];
      if (!valid) {
        mode[i] = 0;
      } else if (RM[i] == -FLT_MAX && RL[i] == 0.0f) {
        mode[i] = 1;
        RM[i] = mb[i];
        RL[i] = lb[i];
      } else {
        mode[i] = 2;
        const float Mn = fmaxf(RM[i], mb[i]);
        const float e1 = g4_exp(__fsub_rn(RM[i], Mn)), e2 = g4_exp(__fsub_rn(mb[i], Mn));
        RL[i] = __fadd_rn(__fmul_rn(RL[i], e1), __fmul_rn(lb[i], e2));
        RM[i] = Mn;
        ea[i] = e1;
        ec[i] = e2;
      }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < PB; i++) {
      const int pi = pb * PB + i, md = mode[pi];
#pragma unroll
      for (int d = 0; d < DB; d++) {
        if (md == 1) {
          O[i][d] = o[i][d];
        } else if (md == 2) {
          const float e1 = ea[pi], e2 = ec[pi];
          O[i][d].x = __fadd_rn(__fmul_rn(O[i][d].x, e1), __fmul_rn(o[i][d].x, e2));
          O[i][d].y = __fadd_rn(__fmul_rn(O[i][d].y, e1), __fmul_rn(o[i][d].y, e2));
          O[i][d].z = __fadd_rn(__fmul_rn(O[i][d].z, e1), __fmul_rn(o[i][d].z, e2));
          O[i][d].w = __fadd_rn(__fmul_rn(O[i][d].w, e1), __fmul_rn(o[i][d].w, e2));
        }
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < PB; i++) {
    const int pi = pb * PB + i, q = pi / NH, h = pi % NH;
    if (q < nq) {
      const float L = RL[pi];
#pragma unroll
      for (int d = 0; d < DB; d++) {
        float4 r;
        r.x = __fdiv_rn(O[i][d].x, L);
        r.y = __fdiv_rn(O[i][d].y, L);
        r.z = __fdiv_rn(O[i][d].z, L);
        r.w = __fdiv_rn(O[i][d].w, L);
        reinterpret_cast<float4 *>(a.out + (size_t)(c0 + q) * NH * HD + (size_t)h * HD)[dg + NDG * d] = r;
        attn_codes4(a.codes, c0 + q, h * HD + 4 * (dg + NDG * d), r);
      }
    }
  }
}

template <int HD>
static size_t attn_prefill_smem() {
  constexpr int NP = (2048 / HD) * 8, KVR = HD <= 256 ? 64 : 32;
  return ((size_t)NP * HD + 2 * (size_t)KVR * (HD + 16) + (size_t)NP * ATT_BLK + 6 * NP + 4 + NP +
          2 * (2048 / HD)) * 4;
}

cudaError_t launch_attention_prefill(const AttnArgs &a, cudaStream_t st, bool pdl) {
  if (a.heads != 8 || a.kv_cap != 0) return cudaErrorInvalidValue;
  static DeviceOnce attr;
  attr([&] {
    cudaFuncSetAttribute(k_attn_prefill<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_prefill_smem<256>());
    cudaFuncSetAttribute(k_attn_prefill<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_prefill_smem<512>());
  });
  if (a.hd == 256)
    return launch_k(k_attn_prefill<256>, dim3((a.cols + 7) / 8), dim3(256), attn_prefill_smem<256>(), st, pdl, a);
  if (a.hd == 512)
    return launch_k(k_attn_prefill<512>, dim3((a.cols + 3) / 4), dim3(256), attn_prefill_smem<512>(), st, pdl, a);
  return cudaErrorInvalidValue;
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st, bool pdl) {
  if (a.heads != 8) return cudaErrorInvalidValue;
  size_t smem = ((size_t)8 * a.hd + 8 * ATT_BLK * 2 + 32 + (size_t)ATT_BLK * a.hd) * 4;
  static DeviceOnce attr;
  attr([&] {
    cudaFuncSetAttribute(k_attn_blocks<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(k_attn_blocks<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  dim3 g1(a.cols, a.max_blocks), g2(a.cols, 8);
  cudaError_t e;
  if (a.hd == 256) {
    e = launch_k(k_attn_blocks<256>, g1, dim3(256), smem, st, pdl, a);
    if (e == cudaSuccess) e = launch_k(k_attn_merge<256>, g2, dim3(256), 0, st, pdl, a);
  } else if (a.hd == 512) {
    e = launch_k(k_attn_blocks<512>, g1, dim3(256), smem, st, pdl, a);
    if (e == cudaSuccess) e = launch_k(k_attn_merge<512>, g2, dim3(256), 0, st, pdl, a);
  } else {
    e = cudaErrorInvalidValue;
  }
  return e;
}

// =====================================================================================
// Decode attention, fused (src/kernels/attnPrologue.ts:83-260 then src/kernels/attention.ts:
// 339-752 for a step whose columns are distinct sequences at one new position each). Block
// (c, bi) of a column:
//   * before the dependency wait, pulls its K and V rows into L2 (a prefetch only: the
//     position read there may be stale, which costs nothing but a wasted prefetch);
//   * requests its V rows (all but the new position) as bulk copies into shared memory: the
//     whole block at once (per-head CTAs), or in two 32-row halves through one half-size buffer
//     (8-head CTAs, so that two CTAs fit an SM at head dim 512);
//   * normalises and rotates the 8 query heads itself (warp h: head h; the sum of squares
//     follows block_sumsq256's chunk order exactly), and, in the block holding the new position
//     of a producer layer, the K row (gain, rotation) and V row (weightless norm), which it
//     stores to the cache and keeps in shared memory;
//   * scores, block max, exp, and the weighted V sum exactly as k_attn_blocks;
//   * writes its partial; the last block of the column to finish folds the partials in
//     ascending block order exactly as k_attn_merge (a single block divides directly).
// =====================================================================================

// Shared memory of one CTA: V staging, query rows, the new K / V rows, scores, probabilities,
// maxima, barriers and a flag; with CL, then the cluster's block partials (held by the leader).
template <int HD, int NHL>
__host__ __device__ constexpr size_t attn_decode_smem_base() {
  return ((size_t)(NHL == 8 ? ATT_BLK / 2 : ATT_BLK) * HD + NHL * HD + 2 * HD + 2 * NHL * ATT_BLK + 8) * 4 + 32;
}
constexpr int ATT_CL_MAX = 16;   // blocks of one (column, head) in one cluster, at most

__device__ __forceinline__ uint32_t att_mapa(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void att_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
}

// CL (one head per CTA, a launch's blocks of one (column, head) forming one thread-block cluster
// along y): each block's partial goes into the shared memory of the cluster's first block by
// distributed-shared-memory stores, one cluster barrier replaces the global partials, the fence,
// the finished-block count and the L2 reads of the merge, and the first block merges in the same
// order. Every CTA of the cluster takes that barrier exactly once, blocks past the context too.
template <int HD, int NHL, bool CL = false>
__global__ void __launch_bounds__(256) k_attn_decode(const AttnDec a) {
  // NHL query heads per CTA: 8 (one CTA per (column, block)) or 1 (grid z = head).
  constexpr int NH = 8;
  constexpr int NC = HD / 4;
  constexpr int NOUT = NHL * NC;                       // float4 outputs of the PV step
  constexpr int HPT = NOUT >= 256 ? NOUT / 256 : 1;    // heads per PV thread
  constexpr int NCH = NOUT >= 256 ? 256 / NC : NHL;    // PV head groups
  constexpr int VH = NHL == 8 ? 2 : 1;                 // V staging phases
  constexpr int VROWS = ATT_BLK / VH;
  extern __shared__ __align__(16) float sm[];
  float *vs = sm;                     // [VROWS][HD] (bulk copy destination)
  float *qs = vs + VROWS * HD;        // [NHL][HD]
  float *kc = qs + NHL * HD;          // [HD]       K row of the new position
  float *vn = kc + HD;                // [HD]       V row of the new position
  float *ss = vn + HD;                // [NHL][64]
  float *ps = ss + NHL * ATT_BLK;     // [NHL][64]
  float *ms = ps + NHL * ATT_BLK;     // [8]
  uint64_t *bar = reinterpret_cast<uint64_t *>(ms + 8);    // [VH], 8-byte aligned: offsets above
  int *flag = reinterpret_cast<int *>(bar + VH);           // are multiples of 8 floats
  // CL: [ATT_CL_MAX][HD] partial outputs, then ATT_CL_MAX maxima and ATT_CL_MAX sums.
  float *cpart = reinterpret_cast<float *>(reinterpret_cast<char *>(sm) + attn_decode_smem_base<HD, NHL>());
  float *cm = cpart + ATT_CL_MAX * HD, *cl = cm + ATT_CL_MAX;
  const int c = blockIdx.x, bi = blockIdx.y, t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int h0 = blockIdx.z * NHL;    // first head of this CTA

  grid_launch_dependents();
  if (t == 0) {
    for (int i = 0; i < VH; i++) mbar_init(&bar[i], 1);
    mbar_fence_init();
    // L2 prefetch of this block's rows from a possibly stale position (clamped in bounds).
    int p = a.refs.pos ? a.refs.pos[c] : a.refs.pos_base + c;
    int sq = a.refs.seq ? a.refs.seq[c] : 0;
    if (p >= 0 && p < a.max_ctx && sq >= 0 && sq < a.max_seqs && blockIdx.z == 0) {
      const int lo = a.window > 0 ? max(0, p - a.window + 1) : 0;
      const int b = lo / ATT_BLK + bi;
      if (b * ATT_BLK <= p) {
        const int j0 = max(b * ATT_BLK, lo), j1 = min(b * ATT_BLK + ATT_BLK - 1, p);
        const float *K = a.cache + (size_t)sq * a.seq_stride;
        const uint32_t bytes = (uint32_t)(j1 - j0 + 1) * HD * 4;
        l2_prefetch(K + (size_t)j0 * HD, bytes);
        l2_prefetch(K + (size_t)a.max_ctx * HD + (size_t)j0 * HD, bytes);
      }
    }
  }
  grid_wait();
  G4_TRACE_POINT(2000 + HD);
  int p, lo, hi;
  {
    AttnArgs r;
    r.refs = a.refs;
    r.window = a.window;
    r.kv_cap = 0;
    attn_range(r, c, &p, &lo, &hi);
  }
  const int b = lo / ATT_BLK + bi;
  if (b * ATT_BLK > hi) {
    if constexpr (CL) att_cluster_sync();
    return;
  }
  const int nb = hi / ATT_BLK - lo / ATT_BLK + 1;
  const int j0 = max(b * ATT_BLK, lo), j1 = min(b * ATT_BLK + ATT_BLK - 1, hi);
  const int seq = a.refs.seq ? a.refs.seq[c] : 0;
  float *K = a.cache + (size_t)seq * a.seq_stride;
  float *V = K + (size_t)a.max_ctx * HD;
  const bool cur = a.k != nullptr && j1 == p;     // this block writes and uses row p itself
  const bool store_kv = cur && blockIdx.z == 0;   // one CTA of the block stores the new row
  const int jv1 = cur ? p - 1 : j1;
  // Staging phase ph covers rows [b * 64 + ph * VROWS, + VROWS) of [j0, jv1].
  auto vfirst = [&](int ph) { return max(j0, b * ATT_BLK + ph * VROWS); };
  auto vbytes = [&](int ph) {
    const int r1 = min(jv1, b * ATT_BLK + ph * VROWS + VROWS - 1);
    return r1 >= vfirst(ph) ? (uint32_t)(r1 - vfirst(ph) + 1) * HD * 4 : 0u;
  };
  auto vissue = [&](int ph) {
    const uint32_t nbytes = vbytes(ph);
    if (nbytes) {
      mbar_expect_tx(&bar[ph], nbytes);
      bulk_g2s(vs + (size_t)(vfirst(ph) - b * ATT_BLK - ph * VROWS) * HD, V + (size_t)vfirst(ph) * HD,
               nbytes, &bar[ph]);
    }
  };
  // Bounded wait on phase ph's copy; on a timeout the error flag is raised, the copy is waited
  // for once more (bounded), and the block finishes with whatever arrived.
  auto vwait = [&](int ph) {
    if (vbytes(ph) && !mbar_wait(&bar[ph], 0)) {
      if (t == 0) atomicExch(&g4_dev_error, 2);
      mbar_wait(&bar[ph], 0);
    }
  };
  __syncthreads();   // barriers initialised
  if (t == 0) vissue(0);

  // Query heads (warp w < NHL: head h0 + w), then the new position's K and V rows (the warps
  // after them).
  {
    const float *ct = a.cos_tab + (size_t)p * (HD / 2);
    const float *stb = a.sin_tab + (size_t)p * (HD / 2);
    if (w < NHL)
      head_norm_rope_warp<HD>(a.q + (size_t)c * a.q_ld + (size_t)(h0 + w) * HD, a.qgain, ct, stb,
                              a.eps, qs + w * HD, nullptr, lane);
    constexpr int WK = NHL < 8 ? NHL : 0, WV = NHL < 7 ? NHL + 1 : 1;
    if (cur && w == WK)
      head_norm_rope_warp<HD>(a.k + (size_t)c * HD, a.kgain, ct, stb, a.eps, kc,
                              store_kv ? K + (size_t)p * HD : nullptr, lane);
    if (cur && w == WV)
      head_norm_rope_warp<HD>(a.v + (size_t)c * HD, nullptr, nullptr, nullptr, a.eps, vn,
                              store_kv ? V + (size_t)p * HD : nullptr, lane);
  }
  __syncthreads();
  G4_TRACE_POINT(102000 + HD);

  // Scores (as k_attn_blocks).
  {
    const int jl = t >> 2, m = t & 3;
    const int j = b * ATT_BLK + jl;
    const bool valid = j >= j0 && j <= j1;
    float acc[NHL];
#pragma unroll
    for (int h = 0; h < NHL; h++) acc[h] = 0.0f;
    if (valid) {
      const float4 *kr = reinterpret_cast<const float4 *>(cur && j == p ? kc : K + (size_t)j * HD);
      constexpr int PER = NC / 4, BATCH = PER < 16 ? PER : 16;
#pragma unroll
      for (int i0 = 0; i0 < PER; i0 += BATCH) {
        float4 k4[BATCH];
#pragma unroll
        for (int i = 0; i < BATCH; i++) k4[i] = kr[m + 4 * (i0 + i)];
#pragma unroll
        for (int i = 0; i < BATCH; i++) {
          const int cc = m + 4 * (i0 + i);
#pragma unroll
          for (int h = 0; h < NHL; h++) {
            const float4 q4 = reinterpret_cast<const float4 *>(qs + h * HD)[cc];
            float v = acc[h];
            v = fmaf(q4.x, k4[i].x, v);
            v = fmaf(q4.y, k4[i].y, v);
            v = fmaf(q4.z, k4[i].z, v);
            v = fmaf(q4.w, k4[i].w, v);
            acc[h] = v;
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < NHL; h++) {
      float v1 = __fadd_rn(acc[h], __shfl_xor_sync(0xffffffffu, acc[h], 1));
      float v2 = __fadd_rn(v1, __shfl_xor_sync(0xffffffffu, v1, 2));
      if (m == 0) ss[h * ATT_BLK + jl] = valid ? v2 : -FLT_MAX;
    }
  }
  __syncthreads();
  if (w < NHL) {
    const int h = w;
    float s0 = ss[h * ATT_BLK + lane], s1 = ss[h * ATT_BLK + lane + 32];
    float mx = fmaxf(s0, s1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int ja = b * ATT_BLK + lane, jb = ja + 32;
    ps[h * ATT_BLK + lane] = (ja >= j0 && ja <= j1) ? g4_exp(__fsub_rn(s0, mx)) : 0.0f;
    ps[h * ATT_BLK + lane + 32] = (jb >= j0 && jb <= j1) ? g4_exp(__fsub_rn(s1, mx)) : 0.0f;
    if (lane == 0) ms[h] = mx;
  }
  G4_TRACE_POINT(202000 + HD);
  vwait(0);
  __syncthreads();
  const int dc = t % NC, hg = t / NC;
  const bool pv = hg < NCH;
  float4 o[HPT];
  float l[HPT];
#pragma unroll
  for (int hh = 0; hh < HPT; hh++) {
    o[hh] = make_float4(0.f, 0.f, 0.f, 0.f);
    l[hh] = 0.0f;
  }
#pragma unroll 1
  for (int ph = 0; ph < VH; ph++) {
    if (ph > 0) {
      __syncthreads();   // every thread is done with the previous phase's rows
      if (t == 0) vissue(ph);
      vwait(ph);
    }
    const int r0 = b * ATT_BLK + ph * VROWS;
    const int ja = max(j0, r0), jb = min(j1, r0 + VROWS - 1);
    if (pv) {
      // Ascending rows; the probabilities of four aligned rows come in one 16-byte load per head.
      auto pv_row = [&](int j, const float *pj) {
        const float *vrow = cur && j == p ? vn : vs + (size_t)(j - r0) * HD;
        const float4 v4 = reinterpret_cast<const float4 *>(vrow)[dc];
#pragma unroll
        for (int hh = 0; hh < HPT; hh++) {
          o[hh].x = fmaf(pj[hh], v4.x, o[hh].x);
          o[hh].y = fmaf(pj[hh], v4.y, o[hh].y);
          o[hh].z = fmaf(pj[hh], v4.z, o[hh].z);
          o[hh].w = fmaf(pj[hh], v4.w, o[hh].w);
          l[hh] = __fadd_rn(l[hh], pj[hh]);
        }
      };
      const float *pbase = ps + (size_t)hg * HPT * ATT_BLK - b * ATT_BLK;   // indexed by j
      int j = ja;
      for (; j <= jb && (j & 3); j++) {
        float pj[HPT];
#pragma unroll
        for (int hh = 0; hh < HPT; hh++) pj[hh] = pbase[hh * ATT_BLK + j];
        pv_row(j, pj);
      }
#pragma unroll 1
      for (; j + 3 <= jb; j += 4) {
        float4 p4[HPT];
#pragma unroll
        for (int hh = 0; hh < HPT; hh++) p4[hh] = *reinterpret_cast<const float4 *>(pbase + hh * ATT_BLK + j);
        float pj[HPT];
#pragma unroll
        for (int hh = 0; hh < HPT; hh++) pj[hh] = p4[hh].x;
        pv_row(j, pj);
#pragma unroll
        for (int hh = 0; hh < HPT; hh++) pj[hh] = p4[hh].y;
        pv_row(j + 1, pj);
#pragma unroll
        for (int hh = 0; hh < HPT; hh++) pj[hh] = p4[hh].z;
        pv_row(j + 2, pj);
#pragma unroll
        for (int hh = 0; hh < HPT; hh++) pj[hh] = p4[hh].w;
        pv_row(j + 3, pj);
      }
      for (; j <= jb; j++) {
        float pj[HPT];
#pragma unroll
        for (int hh = 0; hh < HPT; hh++) pj[hh] = pbase[hh * ATT_BLK + j];
        pv_row(j, pj);
      }
    }
  }
  G4_TRACE_POINT(302000 + HD);
  if (nb == 1) {
    if (pv) {
#pragma unroll
      for (int hh = 0; hh < HPT; hh++) {
        const int h = h0 + hg * HPT + hh;
        float4 r;
        r.x = __fdiv_rn(o[hh].x, l[hh]);
        r.y = __fdiv_rn(o[hh].y, l[hh]);
        r.z = __fdiv_rn(o[hh].z, l[hh]);
        r.w = __fdiv_rn(o[hh].w, l[hh]);
        reinterpret_cast<float4 *>(a.out + (size_t)c * NH * HD + (size_t)h * HD)[dc] = r;
        attn_codes4(a.codes, c, h * HD + 4 * dc, r);
      }
    }
    if constexpr (CL) att_cluster_sync();
    return;
  }
  int *cnt = a.counter + c * (NH / NHL) + blockIdx.z;
  if constexpr (CL) {
    // One head per CTA (HPT 1): the partial into the first block's shared memory, then the barrier.
    if (pv) {
      const uint32_t dst = att_mapa(cpart + (size_t)bi * HD + 4 * dc, 0);
      asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "f"(o[0].x), "f"(o[0].y),
                   "f"(o[0].z), "f"(o[0].w)
                   : "memory");
      if (dc == 0) {
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(att_mapa(cm + bi, 0)), "f"(ms[0]) : "memory");
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(att_mapa(cl + bi, 0)), "f"(l[0]) : "memory");
      }
    }
    att_cluster_sync();
    G4_TRACE_POINT(402000 + HD);
    if (bi != 0) return;
  } else {
    if (pv) {
#pragma unroll
      for (int hh = 0; hh < HPT; hh++) {
        const int hl = hg * HPT + hh, h = h0 + hl;
        const size_t slot = ((size_t)c * a.max_blocks + bi) * NH + h;
        reinterpret_cast<float4 *>(a.part_o + slot * HD)[dc] = o[hh];
        if (dc == 0) {
          a.part_m[slot] = ms[hl];
          a.part_l[slot] = l[hh];
        }
      }
    }
    __threadfence();
    __syncthreads();
    if (t == 0) *flag = atomicAdd(cnt, 1) == nb - 1;
    __syncthreads();
    G4_TRACE_POINT(402000 + HD);
    if (!*flag) return;
    __threadfence();
  }
#ifdef G4_TRACE
  if (blockIdx.x == 0 && blockIdx.z == 0 && t == 0) {   // the merge of column 0, head group 0
    unsigned long long now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    G4_TRACE_REC(502000 + HD, now);
  }
#endif
  // The merge, in k_attn_merge's order, for this CTA's heads. Per head, M_k = max(m_0..m_k) is
  // an exact prefix max, so lane k of warp hl computes ea_k = exp(M_{k-1} - M_k),
  // ec_k = exp(m_k - M_k) and l_k * ec_k in parallel; lane 0 then runs
  // L_k = L_{k-1} * ea_k + l_k * ec_k. Each thread folds its vec4s of the partial outputs block
  // after block with the same factors.
  const size_t base = (size_t)c * a.max_blocks * NH;
  float *fa = vs;                                  // [nb][8] ea_k  (vs is free after the PV loop)
  float *fc = vs + (size_t)a.max_blocks * NH;      // [nb][8] ec_k
  float *fl = fc + (size_t)a.max_blocks * NH;      // [nb][8] l_k * ec_k
  float *Lh = fl + (size_t)a.max_blocks * NH;      // [8] final L
  constexpr int NV = NHL * HD / 4;                 // float4 outputs of this CTA per block
  constexpr int F = (NV + 255) / 256;              // per thread
  constexpr int KB = F <= 2 ? 8 : 16 / F;          // blocks loaded per round
  float4 O[F];
  float4 nx[KB][F];
  const float4 *po = reinterpret_cast<const float4 *>(a.part_o + (base + h0) * HD);
  // Block k's partial output, vec4 i (CL: from this CTA's shared memory).
  auto ld_o = [&](int k, int i) -> float4 {
    if constexpr (CL) return reinterpret_cast<const float4 *>(cpart)[(size_t)k * (HD / 4) + i];
    else return __ldcg(po + (size_t)k * NH * HD / 4 + i);
  };
#pragma unroll
  for (int i = 0; i < F; i++)
    if (t + 256 * i < NV) O[i] = ld_o(0, t + 256 * i);
#pragma unroll
  for (int kk = 0; kk < KB; kk++)
    if (1 + kk < nb) {
#pragma unroll
      for (int i = 0; i < F; i++)
        if (t + 256 * i < NV) nx[kk][i] = ld_o(1 + kk, t + 256 * i);
    }
  if (w < NHL) {
    const int h = h0 + w;
    float carry = -FLT_MAX, Lrun = 0.0f;
    for (int k0 = 0; k0 < nb; k0 += 32) {
      const int k = k0 + lane;
      float mk = -FLT_MAX, lk = 0.0f;
      if (k < nb) {
        if constexpr (CL) {
          mk = cm[k];
          lk = cl[k];
        } else {
          mk = __ldcg(a.part_m + base + (size_t)k * NH + h);
          lk = __ldcg(a.part_l + base + (size_t)k * NH + h);
        }
      }
      float Mk = mk;   // inclusive prefix max within the chunk, then with the carry
#pragma unroll
      for (int o2 = 1; o2 < 32; o2 <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, Mk, o2);
        if (lane >= o2) Mk = fmaxf(Mk, u);
      }
      Mk = fmaxf(Mk, carry);
      float Mp = __shfl_up_sync(0xffffffffu, Mk, 1);
      if (lane == 0) Mp = carry;
      if (k < nb) {
        if (k == 0) {
          fl[h] = lk;
        } else {
          const float e1 = g4_exp(__fsub_rn(Mp, Mk)), e2 = g4_exp(__fsub_rn(mk, Mk));
          fa[k * NH + h] = e1;
          fc[k * NH + h] = e2;
          fl[k * NH + h] = __fmul_rn(lk, e2);
        }
      }
      carry = __shfl_sync(0xffffffffu, Mk, 31);
      __syncwarp();
      if (lane == 0) {
        const int kend = min(nb, k0 + 32);
        for (int kk = k0; kk < kend; kk++)
          Lrun = kk == 0 ? fl[h] : __fadd_rn(__fmul_rn(Lrun, fa[kk * NH + h]), fl[kk * NH + h]);
      }
      __syncwarp();
    }
    if (lane == 0) Lh[h] = Lrun;
  }
  __syncthreads();
  for (int k0 = 1; k0 < nb; k0 += KB) {
#pragma unroll
    for (int kk = 0; kk < KB; kk++) {
      const int k = k0 + kk;
      if (k < nb) {
#pragma unroll
        for (int i = 0; i < F; i++) {
          if (t + 256 * i < NV) {
            const int h = h0 + (4 * (t + 256 * i)) / HD;
            const float e1 = fa[k * NH + h], e2 = fc[k * NH + h];
            O[i].x = __fadd_rn(__fmul_rn(O[i].x, e1), __fmul_rn(nx[kk][i].x, e2));
            O[i].y = __fadd_rn(__fmul_rn(O[i].y, e1), __fmul_rn(nx[kk][i].y, e2));
            O[i].z = __fadd_rn(__fmul_rn(O[i].z, e1), __fmul_rn(nx[kk][i].z, e2));
            O[i].w = __fadd_rn(__fmul_rn(O[i].w, e1), __fmul_rn(nx[kk][i].w, e2));
          }
        }
      }
    }
    // next round's partials
#pragma unroll
    for (int kk = 0; kk < KB; kk++)
      if (k0 + KB + kk < nb) {
#pragma unroll
        for (int i = 0; i < F; i++)
          if (t + 256 * i < NV)
            nx[kk][i] = ld_o(k0 + KB + kk, t + 256 * i);
      }
  }
#pragma unroll
  for (int i = 0; i < F; i++) {
    if (t + 256 * i < NV) {
      const int h = h0 + (4 * (t + 256 * i)) / HD;
      const float L = Lh[h];
      float4 r;
      r.x = __fdiv_rn(O[i].x, L);
      r.y = __fdiv_rn(O[i].y, L);
      r.z = __fdiv_rn(O[i].z, L);
      r.w = __fdiv_rn(O[i].w, L);
      reinterpret_cast<float4 *>(a.out + (size_t)c * NH * HD + (size_t)h0 * HD)[t + 256 * i] = r;
      attn_codes4(a.codes, c, h0 * HD + 4 * (t + 256 * i), r);
    }
  }
#ifdef G4_TRACE
  if (blockIdx.x == 0 && blockIdx.z == 0 && t == 0) {
    unsigned long long now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    G4_TRACE_REC(602000 + HD, now);
  }
#endif
  if (!CL && t == 0) *cnt = 0;
}

template <int HD, int NHL, bool CL = false>
static size_t attn_decode_smem() {
  return attn_decode_smem_base<HD, NHL>() + (CL ? ((size_t)ATT_CL_MAX * HD + 2 * ATT_CL_MAX) * 4 : 0);
}

template <int HD, int NHL>
static cudaError_t launch_attn_decode_t(const AttnDec &a, cudaStream_t st, bool pdl) {
  static DeviceOnce attr_set;
  attr_set([&] {
    cudaFuncSetAttribute(k_attn_decode<HD, NHL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)attn_decode_smem<HD, NHL>());
    cudaFuncSetAttribute(k_attn_decode<HD, NHL>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  });
  return launch_k(k_attn_decode<HD, NHL>, dim3(a.cols, a.max_blocks, 8 / NHL), dim3(256),
                  attn_decode_smem<HD, NHL>(), st, pdl, a);
}

// One-head CTAs whose blocks of one (column, head) form a cluster of a.max_blocks along y.
template <int HD>
static cudaLaunchConfig_t attn_cl_config(const AttnDec &a, cudaStream_t st, cudaLaunchAttribute *attr, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.cols, a.max_blocks, 8);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = attn_decode_smem<HD, 1, true>();
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = a.max_blocks;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cfg;
}

template <int HD>
static cudaError_t attn_cl_attrs() {
  cudaError_t e = cudaFuncSetAttribute(k_attn_decode<HD, 1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)attn_decode_smem<HD, 1, true>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_attn_decode<HD, 1, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}

// Whether a cluster of a.max_blocks such CTAs can be resident on the current device (asked once
// per device and block count).
template <int HD>
static bool attn_cl_fits(const AttnDec &a) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, bool> known;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  auto it = known.find({dev, a.max_blocks});
  if (it != known.end()) return it->second;
  bool ok = attn_cl_attrs<HD>() == cudaSuccess;
  if (ok) {
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = attn_cl_config<HD>(a, nullptr, attr, false);
    int n = 0;
    ok = cudaOccupancyMaxActiveClusters(&n, k_attn_decode<HD, 1, true>, &cfg) == cudaSuccess && n >= 1;
  }
  if (!ok) cudaGetLastError();
  known[{dev, a.max_blocks}] = ok;
  return ok;
}

template <int HD>
static cudaError_t launch_attn_decode_cl(const AttnDec &a, cudaStream_t st, bool pdl) {
  static DeviceOnce attr_set;
  attr_set([&] { attn_cl_attrs<HD>(); });
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = attn_cl_config<HD>(a, st, attr, pdl);
  return cudaLaunchKernelEx(&cfg, k_attn_decode<HD, 1, true>, a);
}

cudaError_t launch_attn_decode(const AttnDec &a, cudaStream_t st, bool pdl) {
  // The merge keeps three factors per (block, head) in the (32- or 64-row) V buffer.
  if ((size_t)3 * a.max_blocks * 8 + 8 > (size_t)(ATT_BLK / 2) * a.hd) return cudaErrorInvalidValue;
  // Few columns: one CTA per (column, block, head) spreads a latency-bound step over more SMs;
  // a wide batch keeps all 8 heads of a block in one CTA (the V block is staged once for them).
  const bool split = a.cols * a.max_blocks <= 64;
  // One-head CTAs of 2..16 blocks merge inside a thread-block cluster.
  if (split && a.max_blocks >= 2 && a.max_blocks <= ATT_CL_MAX) {
    if (a.hd == 256 && attn_cl_fits<256>(a)) return launch_attn_decode_cl<256>(a, st, pdl);
    if (a.hd == 512 && attn_cl_fits<512>(a)) return launch_attn_decode_cl<512>(a, st, pdl);
  }
  if (a.hd == 256) return split ? launch_attn_decode_t<256, 1>(a, st, pdl) : launch_attn_decode_t<256, 8>(a, st, pdl);
  if (a.hd == 512) return split ? launch_attn_decode_t<512, 1>(a, st, pdl) : launch_attn_decode_t<512, 8>(a, st, pdl);
  return cudaErrorInvalidValue;
}

// =====================================================================================
// Argmax final stage (src/kernels/argmax.ts:43-310): greatest value, lowest index on ties.
// =====================================================================================

__device__ __forceinline__ void amax_take(float &bv, int &bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

__global__ void __launch_bounds__(256)
k_argmax_final(const float *part_val, const int32_t *part_idx, int n_parts, int32_t *token_dev,
               int32_t *token_out, float *value_out, const ErrFlags flags, int32_t *flag_out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(3004);
  const int c = blockIdx.x, t = threadIdx.x, lane = t & 31;
  if (flag_out && c == 0 && t == 32) {
    // Every earlier kernel of the step has completed (each waited on the one before it).
    int v = 0;
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (flags.p[i]) v |= __ldcg(flags.p[i]);
    flag_out[0] = v;
  }
  float bv = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = t; i < n_parts; i += 256)
    amax_take(bv, bi, part_val[(size_t)c * n_parts + i], part_idx[(size_t)c * n_parts + i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    amax_take(bv, bi, ov, oi);
  }
  if (lane == 0) {
    sv[t >> 5] = bv;
    si[t >> 5] = bi;
  }
  __syncthreads();
  if (t == 0) {
    for (int w = 1; w < 8; w++) amax_take(bv, bi, sv[w], si[w]);
    if (token_dev) token_dev[c] = bi;
    if (token_out) token_out[c] = bi;
    if (value_out) value_out[c] = bv;
  }
}

cudaError_t launch_argmax_final(const float *part_val, const int32_t *part_idx, int n_parts,
                                int cols, int32_t *token_dev, int32_t *token_out,
                                float *value_out, cudaStream_t st, bool pdl,
                                const ErrFlags *flags, int32_t *flag_out) {
  ErrFlags f = {};
  if (flags) f = *flags;
  return launch_k(k_argmax_final, dim3(cols), dim3(256), 0, st, pdl, part_val, part_idx, n_parts,
                  token_dev, token_out, value_out, f, flags ? flag_out : nullptr);
}

__global__ void k_advance(int32_t *pos, int cols) {
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(3005);
  int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c < cols) pos[c] += 1;
}

cudaError_t launch_advance(int32_t *pos, int cols, cudaStream_t st, bool pdl) {
  return launch_k(k_advance, dim3((cols + 255) / 256), dim3(256), 0, st, pdl, pos, cols);
}

// Operator form of logit-softcap + argmax stage one: capped = tanh(l / cap) * cap, 4096-wide
// segments reduced to (value, index) partials.
__global__ void __launch_bounds__(256)
k_softcap_partials(const float *logits, float *capped, int n, float cap, float *part_val,
                   int32_t *part_idx) {
  __shared__ float sv[8];
  __shared__ int si[8];
  grid_wait();
  const int seg = blockIdx.x, t = threadIdx.x, lane = t & 31;
  float bv = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = seg * 4096 + t; i < min(n, (seg + 1) * 4096); i += 256) {
    float v = logits[i];
    if (cap != 0.0f) v = __fmul_rn(g4_tanh(__fdiv_rn(v, cap)), cap);
    if (capped) capped[i] = v;
    amax_take(bv, bi, v, i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    amax_take(bv, bi, ov, oi);
  }
  if (lane == 0) {
    sv[t >> 5] = bv;
    si[t >> 5] = bi;
  }
  __syncthreads();
  if (t == 0) {
    for (int w = 1; w < 8; w++) amax_take(bv, bi, sv[w], si[w]);
    part_val[seg] = bv;
    part_idx[seg] = bi;
  }
}

cudaError_t launch_softcap_partials(const float *logits, float *capped, int n, float cap,
                                    float *part_val, int32_t *part_idx, int n_parts,
                                    cudaStream_t st) {
  return launch_k(k_softcap_partials, dim3(n_parts), dim3(256), 0, st, false, logits, capped, n,
                  cap, part_val, part_idx);
}

// =====================================================================================
// Standalone norms and elementwise kernels (operator API).
// =====================================================================================

__global__ void __launch_bounds__(256)
k_norm_op(int kind, const float *src, const float *gain, const float *res, const float *gain2,
          float alpha, float *hidden, float *dst, int width, float eps) {
  __shared__ float red[8];
  grid_wait();
  const int r = blockIdx.x, t = threadIdx.x;
  const float *s = src + (size_t)r * width;
  const float inv = rms_inv(block_sumsq256(s, width, red), width, eps);
  const int nc = width / 4;
  if (kind == 0) {  // rms-norm (gain nullable)
    for (int ch = t; ch < nc; ch += 256) {
      float4 v = reinterpret_cast<const float4 *>(s)[ch];
      float4 o = gain ? f4_norm_apply(v, inv, reinterpret_cast<const float4 *>(gain)[ch])
                      : f4_scale(v, inv);
      reinterpret_cast<float4 *>(dst + (size_t)r * width)[ch] = o;
    }
    return;
  }
  float *hrow = (kind == 1 ? dst : hidden) + (size_t)r * width;
  for (int ch = t; ch < nc; ch += 256) {
    float4 v = reinterpret_cast<const float4 *>(s)[ch];
    float4 h = f4_add(reinterpret_cast<const float4 *>(res + (size_t)r * width)[ch],
                      f4_norm_apply(v, inv, reinterpret_cast<const float4 *>(gain)[ch]));
    if (kind == 2) h = f4_scale(h, alpha);
    reinterpret_cast<float4 *>(hrow)[ch] = h;
  }
  if (kind == 1) return;
  __syncthreads();
  const float inv2 = rms_inv(block_sumsq256(hrow, width, red), width, eps);
  for (int ch = t; ch < nc; ch += 256) {
    float4 h = reinterpret_cast<const float4 *>(hrow)[ch];
    reinterpret_cast<float4 *>(dst + (size_t)r * width)[ch] =
        f4_norm_apply(h, inv2, reinterpret_cast<const float4 *>(gain2)[ch]);
  }
}

cudaError_t launch_rms_norm(const float *src, const float *gain, float *dst, int rows, int width,
                            float eps, cudaStream_t st) {
  return launch_k(k_norm_op, dim3(rows), dim3(256), 0, st, false, 0, src, gain,
                  (const float *)nullptr, (const float *)nullptr, 1.0f, (float *)nullptr, dst,
                  width, eps);
}
cudaError_t launch_norm_residual(const float *src, const float *gain, const float *res,
                                 float *dst, int rows, int width, float eps, cudaStream_t st) {
  return launch_k(k_norm_op, dim3(rows), dim3(256), 0, st, false, 1, src, gain, res,
                  (const float *)nullptr, 1.0f, (float *)nullptr, dst, width, eps);
}
cudaError_t launch_norm_residual_norm(const float *src, const float *gain, const float *res,
                                      const float *gain2, float alpha, float *hidden, float *dst,
                                      int rows, int width, float eps, cudaStream_t st) {
  return launch_k(k_norm_op, dim3(rows), dim3(256), 0, st, false, 2, src, gain, res, gain2, alpha,
                  hidden, dst, width, eps);
}

__global__ void k_gelu_mul(const float *gate, const float *up, float *dst, int n, float srq) {
  grid_wait();
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = __fmul_rn(g4_gelu(gate[i]), up[i]);
  if (srq != 0.0f) v = __fmul_rn((float)srq_code(v, srq), srq);
  dst[i] = v;
}

cudaError_t launch_gelu_mul(const float *gate, const float *up, float *dst, int n, float srq,
                            cudaStream_t st) {
  return launch_k(k_gelu_mul, dim3((n + 255) / 256), dim3(256), 0, st, false, gate, up, dst, n, srq);
}

__global__ void k_math_probe(const float *x, float *e, float *th, float *ce, float *ct, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = x[i];
  e[i] = g4_exp(v);
  th[i] = g4_tanh(v);
  ce[i] = expf(v);
  ct[i] = tanhf(v);
}

cudaError_t launch_math_probe(const float *x, float *e, float *t, float *ce, float *ct, int n,
                              cudaStream_t st) {
  k_math_probe<<<(n + 255) / 256, 256, 0, st>>>(x, e, t, ce, ct, n);
  return cudaGetLastError();
}

// =====================================================================================
// Synthetic weight generators: a counter hash of (seed, tensor, element), so any element can be
// regenerated independently for checking.
// =====================================================================================

__global__ void k_gen_words(uint32_t *dst, size_t n, uint64_t key, size_t index0) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = (uint32_t)(keyed(key, index0 + i) >> 32);
}
__global__ void k_gen_f16(uint16_t *dst, size_t n, uint64_t key, double lo, double hi) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    double v = lo + (hi - lo) * unit24(keyed(key, i));
    dst[i] = f32_to_f16_bits(__double2float_rn(v));
  }
}
__global__ void k_gen_bf16_f32(float *dst, size_t n, uint64_t key, double lo, double hi) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    double v = lo + (hi - lo) * unit24(keyed(key, i));
    dst[i] = __uint_as_float((uint32_t)f32_to_bf16_bits(__double2float_rn(v)) << 16);
  }
}
__global__ void k_gen_plmp(uint16_t *dst, size_t n, uint64_t key, double amp) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    double v = (2.0 * unit24(keyed(key, i)) - 1.0) * amp;
    dst[i] = f32_to_bf16_bits(__double2float_rn(v));
  }
}

static unsigned gen_blocks(size_t n) {
  size_t b = (n + 255) / 256;
  return (unsigned)(b < 148 * 64 ? b : 148 * 64);
}

cudaError_t launch_gen_words(uint32_t *dst, size_t n, uint64_t key, size_t index0, cudaStream_t st) {
  k_gen_words<<<gen_blocks(n), 256, 0, st>>>(dst, n, key, index0);
  return cudaGetLastError();
}
cudaError_t launch_gen_f16(uint16_t *dst, size_t n, uint64_t key, double lo, double hi, cudaStream_t st) {
  k_gen_f16<<<gen_blocks(n), 256, 0, st>>>(dst, n, key, lo, hi);
  return cudaGetLastError();
}
cudaError_t launch_gen_bf16_f32(float *dst, size_t n, uint64_t key, double lo, double hi, cudaStream_t st) {
  k_gen_bf16_f32<<<gen_blocks(n), 256, 0, st>>>(dst, n, key, lo, hi);
  return cudaGetLastError();
}
cudaError_t launch_gen_plmp(uint16_t *dst, size_t n, uint64_t key, double amp, cudaStream_t st) {
  k_gen_plmp<<<gen_blocks(n), 256, 0, st>>>(dst, n, key, amp);
  return cudaGetLastError();
}

}  // namespace g4
