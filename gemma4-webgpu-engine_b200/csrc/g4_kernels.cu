// g4_kernels.cu -- sm_100a kernels of the Gemma-4-E2B quantized decode/prefill path.
//
// Reference citations are path:line inside the reference project (TypeScript + WGSL).
#include <cuda_fp16.h>
#include <float.h>

#include "g4_device.cuh"
#include "g4_kernels.cuh"

namespace g4 {

template <typename... KArgs, typename... Args>
static cudaError_t launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
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

struct ChunkPro {
  // Snap four activations of column c at chunk ch to codes and store them in the dp4a layout.
  template <int BITS>
  static __device__ __forceinline__ int store(uint8_t *codes, int ch, float4 x, float s) {
    int q0 = srq_code(x.x, s), q1 = srq_code(x.y, s), q2 = srq_code(x.z, s), q3 = srq_code(x.w, s);
    if (BITS == 4) {
      uint16_t *cw = reinterpret_cast<uint16_t *>(codes);
      int g = ch >> 1, half = ch & 1;
      cw[4 * g + half] = (uint16_t)((q0 & 255) | ((q2 & 255) << 8));
      cw[4 * g + 2 + half] = (uint16_t)((q1 & 255) | ((q3 & 255) << 8));
    } else {
      reinterpret_cast<uint32_t *>(codes)[ch] =
          (uint32_t)((q0 & 255) | ((q1 & 255) << 8) | ((q2 & 255) << 16) | ((uint32_t)(q3 & 255) << 24));
    }
    return q0 + q1 + q2 + q3;
  }
};

__device__ __forceinline__ float4 f4_norm_apply(float4 v, float inv, float4 g) {
  return make_float4(__fmul_rn(__fmul_rn(v.x, inv), g.x), __fmul_rn(__fmul_rn(v.y, inv), g.y),
                     __fmul_rn(__fmul_rn(v.z, inv), g.z), __fmul_rn(__fmul_rn(v.w, inv), g.w));
}
__device__ __forceinline__ float4 f4_add(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}
__device__ __forceinline__ float4 f4_scale(float4 a, float s) {
  return make_float4(__fmul_rn(a.x, s), __fmul_rn(a.y, s), __fmul_rn(a.z, s), __fmul_rn(a.w, s));
}
__device__ __forceinline__ float4 f4_gelu_mul(float4 g, float4 u) {
  return make_float4(__fmul_rn(g4_gelu(g.x), u.x), __fmul_rn(g4_gelu(g.y), u.y),
                     __fmul_rn(g4_gelu(g.z), u.z), __fmul_rn(g4_gelu(g.w), u.w));
}

// Compute column c's activation vector through the prologue and store its int8 codes.
// Returns this thread's share of the code sum.
template <int BITS>
__device__ __forceinline__ int gemv_prologue_col(const GemvArgs &a, int c, float in_scale,
                                                 uint8_t *codes, float *red, bool write_hidden) {
  const int t = threadIdx.x;
  const int K = a.K;
  const int nc = K >> 2;
  int xs = 0;
  if (a.pro == PRO_X || a.pro == PRO_GELU) {
    const float4 *src = reinterpret_cast<const float4 *>(a.src + (size_t)c * a.ld_src);
    const float4 *up = a.pro == PRO_GELU
                           ? reinterpret_cast<const float4 *>(a.up + (size_t)c * a.ld_up + a.up_off)
                           : nullptr;
    for (int ch = t; ch < nc; ch += 256) {
      float4 x = src[ch];
      if (a.pro == PRO_GELU) x = f4_gelu_mul(x, up[ch]);
      xs += ChunkPro::store<BITS>(codes, ch, x, in_scale);
    }
    return xs;
  }
  // Norm prologues: K <= 2048, so each thread owns at most two vec4 chunks (t, t + 256).
  const float4 *src = reinterpret_cast<const float4 *>(a.src + (size_t)c * a.ld_src);
  const float4 *g1 = reinterpret_cast<const float4 *>(a.g1);
  float4 sv[2];
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < 2; i++)
    if (t + 256 * i < nc) sv[cnt++] = src[t + 256 * i];
  float inv1 = rms_inv(block_sumsq256_regs<2>(sv, cnt, red), K, a.eps);
  float4 xv[2];
  if (a.pro == PRO_NORM) {
#pragma unroll
    for (int i = 0; i < 2; i++)
      if (i < cnt) xv[i] = f4_norm_apply(sv[i], inv1, g1[t + 256 * i]);
  } else {
    const float4 *res = reinterpret_cast<const float4 *>(a.res + (size_t)c * a.ld_res);
    float4 h[2];
#pragma unroll
    for (int i = 0; i < 2; i++)
      if (i < cnt) {
        h[i] = f4_add(res[t + 256 * i], f4_norm_apply(sv[i], inv1, g1[t + 256 * i]));
        if (a.pro == PRO_JOIN) h[i] = f4_scale(h[i], a.alpha);
        if (write_hidden)
          reinterpret_cast<float4 *>(a.hidden_out + (size_t)c * a.ld_res)[t + 256 * i] = h[i];
      }
    if (a.pro == PRO_NORMRES) {
#pragma unroll
      for (int i = 0; i < 2; i++)
        if (i < cnt) xv[i] = h[i];
    } else {
      float inv2 = rms_inv(block_sumsq256_regs<2>(h, cnt, red), K, a.eps);
      const float4 *g2 = reinterpret_cast<const float4 *>(a.g2);
#pragma unroll
      for (int i = 0; i < 2; i++)
        if (i < cnt) xv[i] = f4_norm_apply(h[i], inv2, g2[t + 256 * i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 2; i++)
    if (i < cnt) xs += ChunkPro::store<BITS>(codes, t + 256 * i, xv[i], in_scale);
  return xs;
}

template <int BITS, int COLS, int RPW, int PPR>
__global__ void __launch_bounds__(256) k_gemv(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int bid = blockIdx.x;
  int s = 0;
  if (a.nseg > 1 && bid >= a.seg[1].block_begin) s = 1;
  if (a.nseg > 2 && bid >= a.seg[2].block_begin) s = 2;
  const GemvSeg sg = a.seg[s];
  const int K = a.K;
  const int row_bytes = K * BITS / 8;
  const int row0 = (bid - sg.block_begin) * (8 * RPW) + warp * RPW;

  uint8_t *codes = smem;                                       // [COLS][K]
  int *xsum = reinterpret_cast<int *>(smem + COLS * K);        // [8]
  float *red = reinterpret_cast<float *>(xsum + 8);            // [8]
  float *cand_v = red + 8;                                     // [8][COLS]
  int *cand_i = reinterpret_cast<int *>(cand_v + 8 * COLS);    // [8][COLS]

  // Weight stream first: it does not depend on the previous kernel.
  uint4 wv[RPW][PPR];
#pragma unroll
  for (int rr = 0; rr < RPW; rr++) {
    const int row = row0 + rr;
#pragma unroll
    for (int i = 0; i < PPR; i++) {
      const int off = lane * 16 + 512 * i;
      if (row < sg.N && off < row_bytes)
        wv[rr][i] = ldg_stream(sg.w + (size_t)row * row_bytes + off);
      else
        wv[rr][i] = make_uint4(0, 0, 0, 0);
    }
  }
  float wscale[RPW];
#pragma unroll
  for (int rr = 0; rr < RPW; rr++)
    wscale[rr] = (row0 + rr < sg.N) ? f16_bits_to_f32(__ldg(sg.s + row0 + rr)) : 0.0f;
  if (t < 8) xsum[t] = 0;
  grid_launch_dependents();
  grid_wait();

  // Prologue: activation codes for every column into shared memory.
  int xs_local[COLS];
#pragma unroll
  for (int c = 0; c < COLS; c++) {
    xs_local[c] = 0;
    if (c < a.cols)
      xs_local[c] = gemv_prologue_col<BITS>(a, c, sg.in_scale, codes + c * K, red,
                                            bid == 0 && a.hidden_out != nullptr);
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < COLS; c++) {
    int v = warp_sum_int(xs_local[c]);
    if (lane == 0 && c < a.cols) atomicAdd(&xsum[c], v);
  }
  __syncthreads();

  // Exact integer code dot.
  int acc[RPW][COLS];
#pragma unroll
  for (int rr = 0; rr < RPW; rr++)
#pragma unroll
    for (int c = 0; c < COLS; c++) acc[rr][c] = 0;
#pragma unroll
  for (int rr = 0; rr < RPW; rr++) {
#pragma unroll
    for (int i = 0; i < PPR; i++) {
      const int off = lane * 16 + 512 * i;
      if (off < row_bytes) {
        const uint4 w = wv[rr][i];
#pragma unroll
        for (int c = 0; c < COLS; c++) {
          if (BITS == 4) {
            const uint4 *xp = reinterpret_cast<const uint4 *>(codes + c * K + 2 * off);
            const uint4 x01 = xp[0], x23 = xp[1];
            const uint32_t M = 0x0F0F0F0Fu;
            int v = acc[rr][c];
            v = dp4a_us(w.x & M, x01.x, v);
            v = dp4a_us((w.x >> 4) & M, x01.y, v);
            v = dp4a_us(w.y & M, x01.z, v);
            v = dp4a_us((w.y >> 4) & M, x01.w, v);
            v = dp4a_us(w.z & M, x23.x, v);
            v = dp4a_us((w.z >> 4) & M, x23.y, v);
            v = dp4a_us(w.w & M, x23.z, v);
            v = dp4a_us((w.w >> 4) & M, x23.w, v);
            acc[rr][c] = v;
          } else {
            const uint4 xv = *reinterpret_cast<const uint4 *>(codes + c * K + off);
            int v = acc[rr][c];
            v = dp4a_ss(w.x, xv.x, v);
            v = dp4a_ss(w.y, xv.y, v);
            v = dp4a_ss(w.z, xv.z, v);
            v = dp4a_ss(w.w, xv.w, v);
            acc[rr][c] = v;
          }
        }
      }
    }
  }

  // Epilogue: one f32 multiply to fold the input scale into the row scale, one against the
  // exact sum, then the output snap (src/kernels/qgemv.ts:681-686, 1168-1172).
  float best_v[COLS];
  int best_i[COLS];
#pragma unroll
  for (int c = 0; c < COLS; c++) {
    best_v[c] = -FLT_MAX;
    best_i[c] = 0x7fffffff;
  }
#pragma unroll
  for (int rr = 0; rr < RPW; rr++) {
    const int row = row0 + rr;
#pragma unroll
    for (int c = 0; c < COLS; c++) {
      int v = warp_sum_int(acc[rr][c]);
      if (lane == 0 && row < sg.N && c < a.cols) {
        int exact = BITS == 4 ? v - 8 * xsum[c] : v;
        float y = __fmul_rn(__fmul_rn(sg.in_scale, wscale[rr]), (float)exact);
        y = srq_out(y, sg.out_scale);
        if (sg.acc_out) sg.acc_out[(size_t)c * sg.N + row] = exact;
        if (a.head) {
          if (a.softcap != 0.0f) y = __fmul_rn(g4_tanh(__fdiv_rn(y, a.softcap)), a.softcap);
          if (a.logits) a.logits[(size_t)c * a.ld_logits + row] = y;
          if (y > best_v[c]) {
            best_v[c] = y;
            best_i[c] = row;
          }
        } else {
          sg.y[(size_t)c * sg.N + row] = y;
        }
      }
    }
  }
  if (a.head) {
    if (lane == 0) {
#pragma unroll
      for (int c = 0; c < COLS; c++) {
        cand_v[warp * COLS + c] = best_v[c];
        cand_i[warp * COLS + c] = best_i[c];
      }
    }
    __syncthreads();
    if (t < COLS && t < a.cols) {
      float bv = -FLT_MAX;
      int bi = 0x7fffffff;
      for (int w = 0; w < 8; w++) {
        float v = cand_v[w * COLS + t];
        int i = cand_i[w * COLS + t];
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

bool gemv_geometry(int bits, int K, int N_total, int *rpw, int *ppr) {
  const int row_bytes = K * bits / 8;
  if (row_bytes % 16 != 0) return false;
  int p = (row_bytes + 511) / 512;
  static const int caps[] = {1, 2, 3, 4, 6, 8};
  int cap = 0;
  for (int c : caps)
    if (c >= p) {
      cap = c;
      break;
    }
  if (!cap) return false;
  int r = 1;
  // Wider rows per warp only where the geometry is instantiated and the launch stays >= 2 waves.
  if (bits == 4 && cap == 2 && N_total / 32 >= 296) r = 4;
  else if (bits == 4 && (cap == 2 || cap == 4) && N_total / 16 >= 296) r = 2;
  else if (bits == 8 && cap == 1 && N_total / 32 >= 296) r = 4;
  else if (bits == 8 && (cap == 1 || cap == 3) && N_total / 16 >= 296) r = 2;
  *rpw = r;
  *ppr = cap;
  return true;
}

template <int BITS, int COLS, int RPW, int PPR>
static cudaError_t launch_gemv_t(const GemvArgs &a, int n_blocks, cudaStream_t st, bool pdl) {
  size_t smem = (size_t)COLS * a.K + 16 * 4 + 8 * COLS * 8;
  auto k = k_gemv<BITS, COLS, RPW, PPR>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    attr_set = true;
  }
  return launch_k(k, dim3(n_blocks), dim3(256), smem, st, pdl, a);
}

template <int BITS, int COLS>
static cudaError_t launch_gemv_c(const GemvArgs &a, int n_blocks, cudaStream_t st, bool pdl) {
  const int r = a.rpw, p = a.ppr;
#define G4_CASE(R, P) \
  if (r == R && p == P) return launch_gemv_t<BITS, COLS, R, P>(a, n_blocks, st, pdl);
  G4_CASE(1, 1) G4_CASE(1, 2) G4_CASE(1, 3) G4_CASE(1, 4) G4_CASE(1, 6) G4_CASE(1, 8)
  if (BITS == 4) {
    G4_CASE(2, 2) G4_CASE(2, 4) G4_CASE(4, 2)
  } else {
    G4_CASE(2, 1) G4_CASE(2, 3) G4_CASE(4, 1)
  }
#undef G4_CASE
  return cudaErrorInvalidConfiguration;
}

cudaError_t launch_gemv(const GemvArgs &a, int bits, int n_blocks, cudaStream_t st, bool pdl) {
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
  const int c = a.cols;
  if (bits == 4) {
    if (c <= 1) return launch_gemv_c<4, 1>(a, n_blocks, st, pdl);
    if (c <= 2) return launch_gemv_c<4, 2>(a, n_blocks, st, pdl);
    if (c <= 4) return launch_gemv_c<4, 4>(a, n_blocks, st, pdl);
    if (c <= 8) return launch_gemv_c<4, 8>(a, n_blocks, st, pdl);
  } else if (bits == 8) {
    if (c <= 1) return launch_gemv_c<8, 1>(a, n_blocks, st, pdl);
    if (c <= 2) return launch_gemv_c<8, 2>(a, n_blocks, st, pdl);
    if (c <= 4) return launch_gemv_c<8, 4>(a, n_blocks, st, pdl);
    if (c <= 8) return launch_gemv_c<8, 8>(a, n_blocks, st, pdl);
  }
  return cudaErrorInvalidConfiguration;
}

// =====================================================================================
// Gathers (embed-gather / ple-gather-4bit(-sliced), src/kernels/embedGather.ts:176-261,
// 547-577): one thread per packed word of 8 int4 codes; the embed scale folds into the row
// scale first, then one multiply per element.
// =====================================================================================

__global__ void __launch_bounds__(256)
k_embed(const int32_t *tokens, const uint8_t *embed_w, const uint16_t *embed_s, float embed_scale,
        const uint8_t *const *ple_slices, int ple_rps, const uint16_t *ple_s, int H, int ple_cols,
        int ple_group, float *residual, float *ple_id) {
  grid_launch_dependents();
  grid_wait();
  const int c = blockIdx.y;
  const int w = blockIdx.x * 256 + threadIdx.x;
  const int hw = H / 8, pw = ple_cols / 8;
  if (w >= hw + pw) return;
  const int row = tokens[c];
  uint32_t word;
  float scale;
  float *dst;
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
                         float *residual, float *ple_id, cudaStream_t st, bool pdl) {
  int words = H / 8 + ple_cols / 8;
  dim3 grid((words + 255) / 256, cols);
  return launch_k(k_embed, grid, dim3(256), 0, st, pdl, tokens, embed_w, embed_s, embed_scale,
                  ple_slices, ple_rps, ple_s, H, ple_cols, ple_group, residual, ple_id);
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
k_dense_bf16(const uint16_t *w, const float *x, int ld_x, float *y, int N, int K, int cols,
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
    if (lane == 0 && c < cols) y[(size_t)c * N + row] = __fmul_rn(alpha, sum);
  }
}

cudaError_t launch_dense_bf16(const uint16_t *w, const float *x, int ld_x, float *y, int N, int K,
                              int cols, float alpha, cudaStream_t st, bool pdl) {
  if (K % 8 != 0 || K > 2048) return cudaErrorInvalidValue;
  cudaError_t e = cudaSuccess;
  for (int c0 = 0; c0 < cols && e == cudaSuccess; c0 += 8) {
    int nc = cols - c0 < 8 ? cols - c0 : 8;
    size_t smem = (size_t)nc * K * 4;
    dim3 grid((N + 7) / 8);
    const float *xc = x + (size_t)c0 * ld_x;
    float *yc = y + (size_t)c0 * N;
    if (nc <= 1) e = launch_k(k_dense_bf16<1>, grid, dim3(256), smem, st, pdl, w, xc, ld_x, yc, N, K, nc, alpha);
    else if (nc <= 2) e = launch_k(k_dense_bf16<2>, grid, dim3(256), smem, st, pdl, w, xc, ld_x, yc, N, K, nc, alpha);
    else if (nc <= 4) e = launch_k(k_dense_bf16<4>, grid, dim3(256), smem, st, pdl, w, xc, ld_x, yc, N, K, nc, alpha);
    else {
      cudaFuncSetAttribute(k_dense_bf16<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
      e = launch_k(k_dense_bf16<8>, grid, dim3(256), smem, st, pdl, w, xc, ld_x, yc, N, K, nc, alpha);
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
                               float *out, int cols, int groups, int group_dim, float eps,
                               float scale, cudaStream_t st, bool pdl) {
  return launch_k(k_ple_combine, dim3(cols, groups), dim3(256), 0, st, pdl, proj, identity, gain,
                  out, groups * group_dim, group_dim, eps, scale);
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

cudaError_t launch_attn_prologue(const AttnPro &a, cudaStream_t st, bool pdl) {
  int roles = a.heads + (a.k ? 2 : 0);
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

#define ATT_BLK 64

__device__ __forceinline__ void attn_range(const AttnArgs &a, int c, int *p_out, int *lo, int *hi) {
  const int p = a.refs.pos ? a.refs.pos[c] : a.refs.pos_base + c;
  int h = p;
  if (a.kv_cap > 0 && a.kv_cap - 1 < h) h = a.kv_cap - 1;
  *p_out = p;
  *lo = a.window > 0 ? max(0, p - a.window + 1) : 0;
  *hi = h;
}

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
    for (int j = j0; j <= j1; j++) {
      const float4 v4 = reinterpret_cast<const float4 *>(V + (size_t)j * HD)[dc];
      const int jl = j - b * ATT_BLK;
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

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st, bool pdl) {
  if (a.heads != 8) return cudaErrorInvalidValue;
  size_t smem = ((size_t)8 * a.hd + 8 * ATT_BLK * 2 + 8) * 4;
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
               int32_t *token_out, float *value_out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  grid_launch_dependents();
  grid_wait();
  const int c = blockIdx.x, t = threadIdx.x, lane = t & 31;
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
                                float *value_out, cudaStream_t st, bool pdl) {
  return launch_k(k_argmax_final, dim3(cols), dim3(256), 0, st, pdl, part_val, part_idx, n_parts,
                  token_dev, token_out, value_out);
}

__global__ void k_advance(int32_t *pos, int cols) {
  grid_launch_dependents();
  grid_wait();
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
