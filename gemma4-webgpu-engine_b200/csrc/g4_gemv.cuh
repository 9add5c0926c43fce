// Device code shared by the GEMV kernels (g4_kernels.cu, g4_gemv2.cu): the linear's prologues
// (activation snap to int8 codes, the fused norms and joins), the weight-ring sizing, the
// attention block range, and the per-head norm + rotation. Same arithmetic everywhere, so every
// path gives the same bits.
#pragma once
#include <float.h>
#include "g4_device.cuh"
#include "g4_kernels.cuh"

namespace g4 {

struct ChunkPro {
  // Snap four activations of column c at chunk ch to codes and store them in the dp4a layout.
  template <int BITS>
  static __device__ __forceinline__ int store(uint8_t *codes, int ch, float4 x, float s, float r) {
    int q0 = srq_code_r(x.x, s, r), q1 = srq_code_r(x.y, s, r), q2 = srq_code_r(x.z, s, r),
        q3 = srq_code_r(x.w, s, r);
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

// Norm gains are weights: a CTA reads its chunks of them before the dependency wait.
struct ProGains {
  float4 g1[2], g2[2];
};
template <int PRO>
__device__ __forceinline__ void prologue_gains(const GemvArgs &a, ProGains &pg) {
  if (PRO != PRO_NORM && PRO != PRO_JOIN && PRO != PRO_NORMRES) return;
  const int t = threadIdx.x, nc = a.K >> 2;
#pragma unroll
  for (int i = 0; i < 2; i++)
    if (t + 256 * i < nc) {
      pg.g1[i] = reinterpret_cast<const float4 *>(a.g1)[t + 256 * i];
      if (PRO == PRO_JOIN) pg.g2[i] = reinterpret_cast<const float4 *>(a.g2)[t + 256 * i];
    }
}

// Compute column c's activation vector through the prologue and store its int8 codes.
// Returns this thread's share of the code sum. Every global load of a prologue is issued
// before any of its results is used, so the prologue costs one round trip to L2.
template <int BITS, int PRO>
__device__ __forceinline__ int gemv_prologue_col(const GemvArgs &a, const ProGains &pg, int c,
                                                 float in_scale, uint8_t *codes, float *red,
                                                 bool write_hidden, float in_scale2 = 0.0f,
                                                 uint8_t *codes2 = nullptr, int *xs2 = nullptr) {
  const int t = threadIdx.x;
  const int K = a.K;
  const int nc = K >> 2;
  int xs = 0;
  if (PRO == PRO_CODES) {
    // K <= 16384: at most four 16-byte pieces per thread.
    const uint4 *src = reinterpret_cast<const uint4 *>(a.src_codes + (size_t)c * a.ld_codes);
    const int n16 = K >> 4;
    uint4 v[4];
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (t + 256 * i < n16) v[i] = src[t + 256 * i];
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (t + 256 * i < n16) {
        if (BITS == 4 && a.codes_plain) {
          // K order -> the dp4a order of each 8-code group (code_pos): even codes, then odd.
          const uint32_t x = v[i].x, y = v[i].y, z = v[i].z, w = v[i].w;
          v[i] = make_uint4(__byte_perm(x, y, 0x6420), __byte_perm(x, y, 0x7531),
                            __byte_perm(z, w, 0x6420), __byte_perm(z, w, 0x7531));
        }
        reinterpret_cast<uint4 *>(codes)[t + 256 * i] = v[i];
        xs = dp4a_ss(v[i].x, 0x01010101, xs);
        xs = dp4a_ss(v[i].y, 0x01010101, xs);
        xs = dp4a_ss(v[i].z, 0x01010101, xs);
        xs = dp4a_ss(v[i].w, 0x01010101, xs);
      }
    return xs;
  }
  const float in_r = __fdiv_rn(1.0f, in_scale);
  if (PRO == PRO_X || PRO == PRO_GELU) {
    // K <= 16384: at most sixteen vec4 chunks per thread, loaded four at a time.
    const float4 *src = reinterpret_cast<const float4 *>(a.src + (size_t)c * a.ld_src);
    const float4 *up = PRO == PRO_GELU
                           ? reinterpret_cast<const float4 *>(a.up + (size_t)c * a.ld_up + a.up_off)
                           : nullptr;
#pragma unroll 1
    for (int i0 = 0; i0 < 16 && t + 256 * i0 < nc; i0 += 4) {
      float4 xv[4], uv[4];
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (t + 256 * (i0 + i) < nc) {
          xv[i] = src[t + 256 * (i0 + i)];
          if (up) uv[i] = up[t + 256 * (i0 + i)];
        }
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (t + 256 * (i0 + i) < nc) {
          const float4 x = up ? f4_gelu_mul(xv[i], uv[i]) : xv[i];
          xs += ChunkPro::store<BITS>(codes, t + 256 * (i0 + i), x, in_scale, in_r);
        }
    }
    return xs;
  }
  // Norm prologues: K <= 2048, so each thread owns at most two vec4 chunks (t, t + 256).
  const float4 *src = reinterpret_cast<const float4 *>(a.src + (size_t)c * a.ld_src);
  const float4 *res = PRO != PRO_NORM ? reinterpret_cast<const float4 *>(a.res + (size_t)c * a.ld_res)
                                        : nullptr;
  float4 sv[2], rv[2];
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < 2; i++)
    if (t + 256 * i < nc) {
      sv[i] = src[t + 256 * i];
      if (res) rv[i] = res[t + 256 * i];
      cnt = i + 1;
    }
  float inv1 = rms_inv(block_sumsq256_regs<2>(sv, cnt, red), K, a.eps);
  float4 xv[2];
  if (PRO == PRO_NORM) {
#pragma unroll
    for (int i = 0; i < 2; i++)
      if (i < cnt) xv[i] = f4_norm_apply(sv[i], inv1, pg.g1[i]);
  } else {
    float4 h[2];
#pragma unroll
    for (int i = 0; i < 2; i++)
      if (i < cnt) {
        h[i] = f4_add(rv[i], f4_norm_apply(sv[i], inv1, pg.g1[i]));
        if (PRO == PRO_JOIN) h[i] = f4_scale(h[i], a.alpha);
        if (write_hidden)
          reinterpret_cast<float4 *>(a.hidden_out + (size_t)c * a.ld_res)[t + 256 * i] = h[i];
      }
    if (PRO == PRO_NORMRES) {
#pragma unroll
      for (int i = 0; i < 2; i++)
        if (i < cnt) xv[i] = h[i];
    } else {
      float inv2 = rms_inv(block_sumsq256_regs<2>(h, cnt, red), K, a.eps);
#pragma unroll
      for (int i = 0; i < 2; i++)
        if (i < cnt) xv[i] = f4_norm_apply(h[i], inv2, pg.g2[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 2; i++)
    if (i < cnt) xs += ChunkPro::store<BITS>(codes, t + 256 * i, xv[i], in_scale, in_r);
  if (codes2) {
    // A second linear on the same input with its own input scale (the gate/up pair).
    const float in_r2 = __fdiv_rn(1.0f, in_scale2);
    int x2 = 0;
#pragma unroll
    for (int i = 0; i < 2; i++)
      if (i < cnt) x2 += ChunkPro::store<BITS>(codes2, t + 256 * i, xv[i], in_scale2, in_r2);
    *xs2 = x2;
  }
  return xs;
}

// The same prologues for an uncalibrated linear (input scale 0.0): column c's activation vector
// is kept in f32 (xf, K floats) instead of being snapped to codes.
template <int PRO>
__device__ __forceinline__ void gemv_prologue_f32(const GemvArgs &a, const ProGains &pg, int c,
                                                  float *xf, float *red, bool write_hidden) {
  const int t = threadIdx.x;
  const int K = a.K;
  const int nc = K >> 2;
  float4 *dst = reinterpret_cast<float4 *>(xf);
  if (PRO == PRO_X || PRO == PRO_GELU) {
    const float4 *src = reinterpret_cast<const float4 *>(a.src + (size_t)c * a.ld_src);
    const float4 *up = PRO == PRO_GELU
                           ? reinterpret_cast<const float4 *>(a.up + (size_t)c * a.ld_up + a.up_off)
                           : nullptr;
    for (int i = t; i < nc; i += 256) dst[i] = up ? f4_gelu_mul(src[i], up[i]) : src[i];
    return;
  }
  const float4 *src = reinterpret_cast<const float4 *>(a.src + (size_t)c * a.ld_src);
  const float4 *res = PRO != PRO_NORM ? reinterpret_cast<const float4 *>(a.res + (size_t)c * a.ld_res)
                                        : nullptr;
  float4 sv[2], rv[2];
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < 2; i++)
    if (t + 256 * i < nc) {
      sv[i] = src[t + 256 * i];
      if (res) rv[i] = res[t + 256 * i];
      cnt = i + 1;
    }
  const float inv1 = rms_inv(block_sumsq256_regs<2>(sv, cnt, red), K, a.eps);
  float4 xv[2];
  if (PRO == PRO_NORM) {
#pragma unroll
    for (int i = 0; i < 2; i++)
      if (i < cnt) xv[i] = f4_norm_apply(sv[i], inv1, pg.g1[i]);
  } else {
    float4 h[2];
#pragma unroll
    for (int i = 0; i < 2; i++)
      if (i < cnt) {
        h[i] = f4_add(rv[i], f4_norm_apply(sv[i], inv1, pg.g1[i]));
        if (PRO == PRO_JOIN) h[i] = f4_scale(h[i], a.alpha);
        if (write_hidden)
          reinterpret_cast<float4 *>(a.hidden_out + (size_t)c * a.ld_res)[t + 256 * i] = h[i];
      }
    if (PRO == PRO_NORMRES) {
#pragma unroll
      for (int i = 0; i < 2; i++)
        if (i < cnt) xv[i] = h[i];
    } else {
      const float inv2 = rms_inv(block_sumsq256_regs<2>(h, cnt, red), K, a.eps);
#pragma unroll
      for (int i = 0; i < 2; i++)
        if (i < cnt) xv[i] = f4_norm_apply(h[i], inv2, pg.g2[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 2; i++)
    if (i < cnt) dst[t + 256 * i] = xv[i];
}

// CTAs for the segments of one launch in proportion to their units (rows or row tiles): at least
// one per segment, at most units[i] each, `target` in total (the launch's resident CTAs: one
// more CTA would run as a second wave that the whole launch waits for). Floors first, then the
// CTAs left over go to the largest remainders (ties: the earlier segment).
inline void split_ctas(const long long *units, int n, int target, long long *nb) {
  long long total = 0, rem[3];
  for (int i = 0; i < n; i++) total += units[i];
  if (target > total) target = (int)total;
  long long used = 0;
  for (int i = 0; i < n; i++) {
    nb[i] = units[i] * target / total;
    rem[i] = units[i] * target % total;
    if (nb[i] < 1) nb[i] = 1;
    used += nb[i];
  }
  for (long long left = target - used; left > 0; left--) {
    int best = -1;
    for (int i = 0; i < n; i++)
      if (nb[i] < units[i] && (best < 0 || rem[i] > rem[best])) best = i;
    if (best < 0) break;
    nb[best]++;
    rem[best] = -1;
  }
}

constexpr int GS_RING = 96 * 1024;   // shared-memory ring per CTA
constexpr int GS_MAX_STAGES = 8;

// A long row is processed as RS "virtual rows" of at most 1 KB (the integer code dot of a row is
// the exact sum of its parts, so the split changes no value).
__host__ __device__ __forceinline__ int gs_row_split(int row_bytes) {
  if (row_bytes <= 1024) return 1;
  if (row_bytes % 2 == 0 && row_bytes / 2 <= 1024 && (row_bytes / 2) % 16 == 0) return 2;
  return 4;
}
// Virtual rows per stage: whole 32-row groups (eight warps x four rows), at most 32 KB.
__host__ __device__ __forceinline__ int gs_stage_vrows(int vrow_bytes) {
  int k = (32 * 1024) / (32 * vrow_bytes);
  return 32 * (k < 1 ? 1 : k);
}

// Split `bytes` at `p` into this CTA's 16-byte-aligned share and prefetch it into L2.
__device__ __forceinline__ void l2_prefetch_share(const void *p, uint64_t bytes, int i, int n) {
  if (!p || bytes == 0) return;
  uint64_t lo = (bytes * (uint64_t)i / n) & ~(uint64_t)15, hi = (bytes * (uint64_t)(i + 1) / n) & ~(uint64_t)15;
  if (i + 1 == n) hi = bytes & ~(uint64_t)15;
  for (uint64_t o = lo; o < hi; o += 65536) {
    uint64_t len = hi - o < 65536 ? hi - o : 65536;
    l2_prefetch((const uint8_t *)p + o, (uint32_t)len);
  }
}


#define ATT_BLK 64

__device__ __forceinline__ void attn_range(const AttnArgs &a, int c, int *p_out, int *lo, int *hi) {
  const int p = a.refs.pos ? a.refs.pos[c] : a.refs.pos_base + c;
  int h = p;
  if (a.kv_cap > 0 && a.kv_cap - 1 < h) h = a.kv_cap - 1;
  *p_out = p;
  *lo = a.window > 0 ? max(0, p - a.window + 1) : 0;
  *hi = h;
}


// Normalise (gain optional) and rotate (cos/sin optional) one head row with one warp. Lane l
// holds vec4 chunks l + 32 g (g < HD / 128), so its loads go out together and it owns whole
// rotation pairs (chunk l + 32 g pairs with chunk l + 32 (g + HD / 256)). The sum of squares
// follows block_sumsq256's order: thread i < HD / 4 squares chunk i, warp g's butterfly sums
// chunks 32 g .. 32 g + 31, and the warp sums are added in ascending order.
template <int HD>
__device__ __forceinline__ void head_norm_rope_warp(const float *src, const float *gain,
                                                    const float *ct, const float *stb, float eps,
                                                    float *dst_s, float *dst_g, int lane) {
  constexpr int NW = HD / 128, NP = NW / 2;
  float4 x[NW], g[NW], cs[NP], sn[NP];
#pragma unroll
  for (int i = 0; i < NW; i++) {
    x[i] = reinterpret_cast<const float4 *>(src)[32 * i + lane];
    if (gain) g[i] = reinterpret_cast<const float4 *>(gain)[32 * i + lane];
  }
  if (ct) {
#pragma unroll
    for (int i = 0; i < NP; i++) {
      cs[i] = reinterpret_cast<const float4 *>(ct)[32 * i + lane];
      sn[i] = reinterpret_cast<const float4 *>(stb)[32 * i + lane];
    }
  }
  float total = 0.0f;
#pragma unroll
  for (int i = 0; i < NW; i++) {
    float acc = 0.0f;
    acc = fmaf(x[i].x, x[i].x, acc);
    acc = fmaf(x[i].y, x[i].y, acc);
    acc = fmaf(x[i].z, x[i].z, acc);
    acc = fmaf(x[i].w, x[i].w, acc);
    acc = warp_sum_bfly(acc);
    total = i == 0 ? acc : __fadd_rn(total, acc);
  }
  const float inv = rms_inv(total, HD, eps);
#pragma unroll
  for (int i = 0; i < NW; i++) {
    x[i].x = __fmul_rn(x[i].x, inv);
    x[i].y = __fmul_rn(x[i].y, inv);
    x[i].z = __fmul_rn(x[i].z, inv);
    x[i].w = __fmul_rn(x[i].w, inv);
    if (gain) {
      x[i].x = __fmul_rn(x[i].x, g[i].x);
      x[i].y = __fmul_rn(x[i].y, g[i].y);
      x[i].z = __fmul_rn(x[i].z, g[i].z);
      x[i].w = __fmul_rn(x[i].w, g[i].w);
    }
  }
  if (ct) {
#pragma unroll
    for (int i = 0; i < NP; i++) {
      const float4 lo = x[i], hi = x[i + NP], cc = cs[i], ss = sn[i];
      float4 r0, r1;
      r0.x = __fsub_rn(__fmul_rn(lo.x, cc.x), __fmul_rn(hi.x, ss.x));
      r0.y = __fsub_rn(__fmul_rn(lo.y, cc.y), __fmul_rn(hi.y, ss.y));
      r0.z = __fsub_rn(__fmul_rn(lo.z, cc.z), __fmul_rn(hi.z, ss.z));
      r0.w = __fsub_rn(__fmul_rn(lo.w, cc.w), __fmul_rn(hi.w, ss.w));
      r1.x = __fadd_rn(__fmul_rn(hi.x, cc.x), __fmul_rn(lo.x, ss.x));
      r1.y = __fadd_rn(__fmul_rn(hi.y, cc.y), __fmul_rn(lo.y, ss.y));
      r1.z = __fadd_rn(__fmul_rn(hi.z, cc.z), __fmul_rn(lo.z, ss.z));
      r1.w = __fadd_rn(__fmul_rn(hi.w, cc.w), __fmul_rn(lo.w, ss.w));
      x[i] = r0;
      x[i + NP] = r1;
    }
  }
#pragma unroll
  for (int i = 0; i < NW; i++) {
    reinterpret_cast<float4 *>(dst_s)[32 * i + lane] = x[i];
    if (dst_g) reinterpret_cast<float4 *>(dst_g)[32 * i + lane] = x[i];
  }
}


}  // namespace g4
