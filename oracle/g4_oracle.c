/*
 * g4_oracle.c -- CPU restatement of the gemma4-webgpu-engine decode/prefill arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (see g4_oracle.h): the parity checker and the timed CPU baseline.
 *
 * Build: -O2 -ffp-contract=off -mfma (oracle/Makefile). Contraction is off so every `a * b + c`
 * written below is two correctly rounded operations; where a fused multiply-add is meant, the
 * code calls fmaf() explicitly. No reassociation flags are used, so every f32 sum happens in the
 * order written. Integer accumulations are exact and therefore order free.
 *
 * Reference citations are `path:line` inside the reference project (src/...).
 */
#include "g4_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ================================================================== scalar arithmetic */

/* f32 -> IEEE half, round to nearest even, subnormals kept. */
uint16_t g4o_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
  int e = (int)exp - 112; /* rebias 127 -> 15 */
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    uint32_t full = man | 0x800000u;
    int shift = 14 - e;
    uint32_t half = full >> shift;
    uint32_t rem = full & ((1u << shift) - 1u);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1u))) half++;
    return (uint16_t)(sign | half);
  }
  uint32_t half = sign | ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++;
  return (uint16_t)half;
}

float g4o_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t x;
  if (exp == 0) {
    if (man == 0) {
      x = sign;
    } else {
      int e = -1;
      do { man <<= 1; e++; } while (!(man & 0x400u));
      man &= 0x3ffu;
      x = sign | ((uint32_t)(112 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    x = sign | 0x7f800000u | (man << 13);
  } else {
    x = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

/* f32 -> bf16 round to nearest even (src/quant.ts:418-428 roundToBf16). */
uint16_t g4o_f32_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t lower = x & 0xffffu;
  uint32_t upper = x >> 16;
  if (lower > 0x8000u || (lower == 0x8000u && (upper & 1u))) upper += 1u;
  return (uint16_t)(upper & 0xffffu);
}

/* bf16 is the top 16 bits of the f32 pattern (src/quant.ts:400-411 bf16ToF32). */
float g4o_bf16_to_f32(uint16_t h) {
  uint32_t x = (uint32_t)h << 16;
  float f;
  memcpy(&f, &x, 4);
  return f;
}

/*
 * e^x in f32: Cody-Waite argument reduction x = n ln2 + r with ln2 split into a 15-bit head and
 * a tail, then the degree-7 Taylor polynomial of e^r on |r| <= ln2/2 in Horner form with fused
 * multiply-adds, then an exact scale by 2^n. Inputs below ln(FLT_MIN) return 0 and above
 * ln(FLT_MAX) return +inf. The CUDA library evaluates the identical operation sequence.
 */
float g4o_exp(float x) {
  if (x < -87.33654f) return 0.0f;
  if (x > 88.72283f) return INFINITY;
  float n = rintf(x * 1.44269504088896341f);
  float r = fmaf(n, -0.693145751953125f, x);
  r = fmaf(n, -1.42860677e-06f, r);
  float p = 1.98412698e-04f;
  p = fmaf(p, r, 1.38888889e-03f);
  p = fmaf(p, r, 8.33333333e-03f);
  p = fmaf(p, r, 4.16666667e-02f);
  p = fmaf(p, r, 1.66666667e-01f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  if (ni > 127) {
    p = p * 2.0f;
    ni = 127;
  }
  uint32_t bits = (uint32_t)(ni + 127) << 23;
  float s;
  memcpy(&s, &bits, 4);
  return p * s;
}

/* tanh(x) = sign(x) (1 - e^{-2|x|}) / (1 + e^{-2|x|}), on the exp above. */
float g4o_tanh(float x) {
  float ax = fabsf(x);
  float t = g4o_exp(-2.0f * ax);
  float r = (1.0f - t) / (1.0f + t);
  return copysignf(r, x);
}

/*
 * gelu_pytorch_tanh with the +/-10 clamp on the tanh argument, in the shader's association:
 * cube = x*x*x; inner = COEF * (x + CUBIC * cube); 0.5 * x * (1 + tanh(inner))
 * (src/kernels/geluMul.ts:101-115; constants 0.7978845608028654, 0.044715, clamp 10 at 67-89).
 */
float g4o_gelu(float x) {
  const float coef = 0.7978845608028654f;
  const float cubic = 0.044715f;
  float cube = (x * x) * x;
  float inner = coef * (x + cubic * cube);
  if (inner < -10.0f) inner = -10.0f;
  if (inner > 10.0f) inner = 10.0f;
  return (0.5f * x) * (1.0f + g4o_tanh(inner));
}

/*
 * SRQ input snap: clamp(roundTiesToEven(f32(x / s)), -128, 127) (src/quant.ts:309-334,
 * srqIn src/kernels/qgemv.ts:624-626). The division is one f32 IEEE divide.
 */
int g4o_srq_code(float x, float s) {
  float q = rintf(x / s);
  if (q < -128.0f) q = -128.0f;
  if (q > 127.0f) q = 127.0f;
  return (int)q;
}

/* SRQ output snap, srqOut src/kernels/qgemv.ts:631-636 and applySrq src/quant.ts:278-288. */
float g4o_srq_out(float v, float s) {
  if (s == 0.0f) return v;
  float q = rintf(v / s);
  if (q < -128.0f) q = -128.0f;
  if (q > 127.0f) q = 127.0f;
  return q * s;
}

static inline uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xBF58476D1CE4E5B9ull;
  z ^= z >> 27;
  z *= 0x94D049BB133111EBull;
  z ^= z >> 31;
  return z;
}

/* The synthetic-model counter hash: a splitmix64 finaliser keyed by (seed, stream). */
uint64_t g4o_hash(uint64_t seed, uint64_t stream, uint64_t i) {
  uint64_t key = mix64(seed ^ (stream * 0x9E3779B97F4A7C15ull));
  return mix64(key + i * 0xD1B54A32D192ED03ull);
}

static inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return mix64(seed ^ (stream * 0x9E3779B97F4A7C15ull));
}

static inline uint64_t keyed(uint64_t key, uint64_t i) {
  return mix64(key + i * 0xD1B54A32D192ED03ull);
}

/* 24-bit uniform in [0, 1), exact in double. */
static inline double unit24(uint64_t h) { return (double)(h >> 40) * (1.0 / 16777216.0); }

/* =========================================================== fixed reduction trees */

/* The 32-lane XOR butterfly, masks 1, 2, 4, 8, 16 (src/kernels/subgroupReduce.ts:49-59):
 * every lane ends with the same balanced pairwise tree; lane 0's value is returned. */
static float butterfly32(const float *v) {
  float a[32], b[32];
  memcpy(a, v, sizeof(a));
  for (int m = 1; m < 32; m <<= 1) {
    for (int i = 0; i < 32; i++) b[i] = a[i] + a[i ^ m];
    memcpy(a, b, sizeof(a));
  }
  return a[0];
}

/* The same butterfly with the masks descending (16, 8, 4, 2, 1): the row reduction of the 2-bit
 * family's f32 path. */
static float butterfly32_desc(const float *v) {
  float a[32], b[32];
  memcpy(a, v, sizeof(a));
  for (int m = 16; m >= 1; m >>= 1) {
    for (int i = 0; i < 32; i++) b[i] = a[i] + a[i ^ m];
    memcpy(a, b, sizeof(a));
  }
  return a[0];
}

/*
 * Sum of squares of v[0..n) in the norm kernels' order (n a multiple of 4): 256 lanes, lane t
 * walks vec4 chunks t, t + 256, ... with an fma per component; each 32-lane group closes with
 * the butterfly; the 8 group sums are added in ascending order. This is the reduction shape of
 * the reference's rms-norm (src/kernels/rmsNorm.ts:110-185: 256 lanes, butterfly, slots summed
 * ascending).
 */
static float sumsq256(const float *v, int n) {
  int nc = n / 4;
  float lanes[256];
  for (int t = 0; t < 256; t++) {
    float acc = 0.0f;
    for (int c = t; c < nc; c += 256) {
      acc = fmaf(v[4 * c + 0], v[4 * c + 0], acc);
      acc = fmaf(v[4 * c + 1], v[4 * c + 1], acc);
      acc = fmaf(v[4 * c + 2], v[4 * c + 2], acc);
      acc = fmaf(v[4 * c + 3], v[4 * c + 3], acc);
    }
    lanes[t] = acc;
  }
  float total = butterfly32(lanes);
  for (int g = 1; g < 8; g++) total = total + butterfly32(lanes + 32 * g);
  return total;
}

/* inv = 1 / sqrt(total / n + eps), each step one IEEE f32 operation. */
float g4o_rms_inv(const float *v, int n, float eps) {
  float total = sumsq256(v, n);
  return 1.0f / sqrtf(total / (float)n + eps);
}

/* ==================================================================== linear layers */

static inline int code4(const uint8_t *row, int k) {
  uint8_t b = row[k >> 1];
  return (int)((k & 1) ? (b >> 4) : (b & 15)) - 8;
}

static inline int code8(const uint8_t *row, int k) { return (int)(int8_t)row[k]; }

/* 2-bit codes in the checkpoint's row layout (src/quant.ts:27-96): 16 per u32 word, code k at
 * bits 2 (k % 16), so byte k / 4 holds codes at bits 2 (k % 4); unsigned 0..3, zero point 2. */
static inline int ucode2(const uint8_t *row, int k) { return (row[k >> 2] >> (2 * (k & 3))) & 3; }

/*
 * qgemvOracle (src/kernels/qgemv.ts:1131-1176) over `cols` columns (qgemmOracle,
 * src/kernels/qgemm.ts:532-552: each column is the GEMV). Calibrated: exact integer code dot,
 * then srqOut((inScale * scale[r]) * f32(acc)). Uncalibrated (in_scale == 0): the f32 code dot in
 * the kernel's lane order (lane l accumulates the row's 16-byte chunks l, l + 32, ... in k order
 * with fused multiply-adds; the lanes close with the butterfly), then (1 * scale[r]) * sum.
 */
void g4o_qgemv(const uint8_t *wq, const uint16_t *scales_f16, const float *x, float in_scale,
               float out_scale, int bits, int N, int K, int cols, float *y, int32_t *acc) {
  const int row_bytes = K * bits / 8;
  const int calibrated = in_scale != 0.0f;
  int16_t *xc = (int16_t *)malloc(sizeof(int16_t) * (size_t)K * (size_t)cols);
  int32_t *xsum = (int32_t *)malloc(sizeof(int32_t) * (size_t)cols);
  if (calibrated) {
    for (int c = 0; c < cols; c++) {
      int32_t s = 0;
      for (int k = 0; k < K; k++) {
        int q = g4o_srq_code(x[(size_t)c * K + k], in_scale);
        xc[(size_t)c * K + k] = (int16_t)q;
        s += q;
      }
      xsum[c] = s;
    }
  }
#pragma omp parallel for schedule(static)
  for (int r = 0; r < N; r++) {
    const uint8_t *row = wq + (size_t)r * row_bytes;
    float scale = g4o_f16_to_f32(scales_f16[r]);
    for (int c = 0; c < cols; c++) {
      float out;
      if (calibrated) {
        const int16_t *xr = xc + (size_t)c * K;
        int32_t a = 0;
        if (bits == 4) {
          /* sum((u - 8) x) = sum(u x) - 8 sum(x), u the unsigned nibble. */
          int32_t s = 0;
          for (int j = 0; j < row_bytes; j++) {
            int lo = row[j] & 15, hi = row[j] >> 4;
            s += lo * xr[2 * j] + hi * xr[2 * j + 1];
          }
          a = s - 8 * xsum[c];
        } else if (bits == 2) {
          /* sum((u - 2) x) = sum(u x) - 2 sum(x) (src/kernels/qgemv.ts:693-868). */
          int32_t s = 0;
          for (int k = 0; k < K; k++) s += ucode2(row, k) * xr[k];
          a = s - 2 * xsum[c];
        } else {
          for (int k = 0; k < K; k++) a += code8(row, k) * xr[k];
        }
        if (acc) acc[(size_t)c * N + r] = a;
        out = (in_scale * scale) * (float)a;
      } else if (bits == 2) {
        /* The 2-bit family's f32 path: lane l takes k = 128 b + 4 l + j (b ascending, then j),
         * one fused multiply-add per code, its own activation sum s_l; lane partial
         * acc_l - 2 s_l; lanes closed by the descending butterfly; then (1 * scale) * sum. */
        const float *xr = x + (size_t)c * K;
        float lanes[32];
        for (int l = 0; l < 32; l++) {
          float a = 0.0f, sx = 0.0f;
          for (int b = 0; b < K / 128; b++)
            for (int j = 0; j < 4; j++) {
              int k = 128 * b + 4 * l + j;
              sx = sx + xr[k];
              a = fmaf((float)ucode2(row, k), xr[k], a);
            }
          lanes[l] = a - 2.0f * sx;
        }
        float sum = butterfly32_desc(lanes);
        if (acc) acc[(size_t)c * N + r] = 0;
        out = (1.0f * scale) * sum;
      } else {
        const float *xr = x + (size_t)c * K;
        int n_chunks = row_bytes / 16;
        int per_chunk = 16 * 8 / bits;
        float lanes[32];
        for (int l = 0; l < 32; l++) {
          float a = 0.0f;
          for (int ch = l; ch < n_chunks; ch += 32) {
            for (int j = 0; j < per_chunk; j++) {
              int k = ch * per_chunk + j;
              int cw = bits == 4 ? code4(row, k) : code8(row, k);
              a = fmaf((float)cw, xr[k], a);
            }
          }
          lanes[l] = a;
        }
        float sum = butterfly32(lanes);
        if (acc) acc[(size_t)c * N + r] = 0;
        out = (1.0f * scale) * sum;
      }
      y[(size_t)c * N + r] = g4o_srq_out(out, out_scale);
    }
  }
  free(xc);
  free(xsum);
}

/* gelu-mul with the SRQ snap as stored values (src/kernels/geluMul.ts:219-240). */
void g4o_gelu_mul(const float *gate, const float *up, float *dst, int n, float srq_scale) {
  for (int i = 0; i < n; i++) {
    float v = g4o_gelu(gate[i]) * up[i];
    if (srq_scale != 0.0f) v = (float)g4o_srq_code(v, srq_scale) * srq_scale;
    dst[i] = v;
  }
}

/* ============================================================================ norms */

/* rms-norm (src/kernels/rmsNorm.ts:131-185): dst = (src * inv) * gain, gain NULL = weightless. */
void g4o_rms_norm(const float *src, const float *gain, float *dst, int rows, int width, float eps) {
  for (int r = 0; r < rows; r++) {
    const float *s = src + (size_t)r * width;
    float inv = g4o_rms_inv(s, width, eps);
    for (int i = 0; i < width; i++) {
      float v = s[i] * inv;
      dst[(size_t)r * width + i] = gain ? v * gain[i] : v;
    }
  }
}

/* norm-residual (src/kernels/mlpEpilogue.ts:145-196): residual + (src * inv) * gain. */
void g4o_norm_residual(const float *src, const float *gain, const float *residual, float *dst,
                       int rows, int width, float eps) {
  for (int r = 0; r < rows; r++) {
    const float *s = src + (size_t)r * width;
    float inv = g4o_rms_inv(s, width, eps);
    for (int i = 0; i < width; i++)
      dst[(size_t)r * width + i] = residual[(size_t)r * width + i] + (s[i] * inv) * gain[i];
  }
}

/* norm-residual-norm (src/kernels/blockJoin.ts:73-160). */
void g4o_norm_residual_norm(const float *src, const float *gain, const float *residual,
                            const float *gain2, float alpha, float *hidden, float *dst,
                            int rows, int width, float eps) {
  for (int r = 0; r < rows; r++) {
    const float *s = src + (size_t)r * width;
    float *h = hidden + (size_t)r * width;
    float inv = g4o_rms_inv(s, width, eps);
    for (int i = 0; i < width; i++)
      h[i] = (residual[(size_t)r * width + i] + (s[i] * inv) * gain[i]) * alpha;
    float inv2 = g4o_rms_inv(h, width, eps);
    for (int i = 0; i < width; i++) dst[(size_t)r * width + i] = (h[i] * inv2) * gain2[i];
  }
}

/* ============================================================================= rope */

/*
 * ropeInverseFrequencies and ropeTables (src/kernels/rope.ts:149-191): invFreq[i] =
 * theta^(-2i / headDim) for the rotating pairs (denominator headDim, not the rotary width), 0
 * for the rest; cos/sin of pos * invFreq in f64, rounded to f32.
 */
void g4o_rope_tables(int head_dim, int rotary_pairs, double theta, int pos0, int npos,
                     float *cos_tab, float *sin_tab) {
  int pairs = head_dim / 2;
  for (int p = 0; p < npos; p++) {
    double pos = (double)(pos0 + p);
    for (int i = 0; i < pairs; i++) {
      double inv = i < rotary_pairs ? pow(theta, (-2.0 * i) / (double)head_dim) : 0.0;
      double angle = pos * inv;
      cos_tab[(size_t)p * pairs + i] = (float)cos(angle);
      sin_tab[(size_t)p * pairs + i] = (float)sin(angle);
    }
  }
}

/* Split-half rotation (src/kernels/rope.ts:213-259): lo' = lo c - hi s; hi' = hi c + lo s. */
static void rope_row(const float *y, const float *c, const float *s, float *out, int width) {
  int p = width / 2;
  for (int i = 0; i < p; i++) {
    float lo = y[i], hi = y[i + p];
    out[i] = (lo * c[i]) - (hi * s[i]);
    out[i + p] = (hi * c[i]) + (lo * s[i]);
  }
}

/* q-norm-rope (src/kernels/attnPrologue.ts:83-170, oracle 268-281). */
void g4o_q_norm_rope(const float *src, const float *gain, const float *cos_tab,
                     const float *sin_tab, float *dst, int rows, int width, int rows_per_pos,
                     float eps) {
  float *y = (float *)malloc(sizeof(float) * (size_t)width);
  int p = width / 2;
  for (int r = 0; r < rows; r++) {
    const float *s = src + (size_t)r * width;
    float inv = g4o_rms_inv(s, width, eps);
    for (int i = 0; i < width; i++) y[i] = (s[i] * inv) * gain[i];
    int tab = r / rows_per_pos;
    rope_row(y, cos_tab + (size_t)tab * p, sin_tab + (size_t)tab * p, dst + (size_t)r * width, width);
  }
  free(y);
}

/* kv-norm-rope-store (src/kernels/attnPrologue.ts:172-260, oracle 318-330; kvStore.ts:89-114):
 * K row normed with the gain and rotated, V row weightless-normed, both stored at start_pos+t. */
void g4o_kv_norm_rope_store(const float *k, const float *v, const float *gain,
                            const float *cos_tab, const float *sin_tab, float *cache,
                            int tokens, int head_dim, int start_pos, int max_context, float eps) {
  float *y = (float *)malloc(sizeof(float) * (size_t)head_dim);
  int p = head_dim / 2;
  size_t vbase = (size_t)max_context * head_dim;
  for (int t = 0; t < tokens; t++) {
    const float *kr = k + (size_t)t * head_dim;
    const float *vr = v + (size_t)t * head_dim;
    float inv = g4o_rms_inv(kr, head_dim, eps);
    for (int i = 0; i < head_dim; i++) y[i] = (kr[i] * inv) * gain[i];
    rope_row(y, cos_tab + (size_t)t * p, sin_tab + (size_t)t * p,
             cache + (size_t)(start_pos + t) * head_dim, head_dim);
    float invv = g4o_rms_inv(vr, head_dim, eps);
    for (int i = 0; i < head_dim; i++) cache[vbase + (size_t)(start_pos + t) * head_dim + i] = vr[i] * invv;
  }
  free(y);
}

/* ======================================================================== attention */

#define ATT_BLOCK 64

/*
 * Multi-query attention for one (query row, head), scale 1.0 (src/kernels/attention.ts:81), no
 * logit softcap, window [p - W + 1, p] or global (src/kernels/attention.ts:482-514).
 *
 * The f32 order the CUDA kernel evaluates: positions in blocks of 64 aligned to absolute
 * position. Per block: the score of position j is a dot over the head with four accumulators
 * (vec4 chunk i feeds accumulator i mod 4, each vec4 an fma chain; s = (a0 + a1) + (a2 + a3),
 * the reference's four-accumulator score, src/kernels/attention.ts:574-588); m = the block max;
 * p_j = exp(s_j - m); l = sum of p_j ascending; o[d] = fma chain of p_j v_j[d] ascending. Blocks
 * merge in ascending order with the flash rescale: M' = max(M, m); a = exp(M - M'); c = exp(m -
 * M'); L = L a + l c; O = O a + o c. out = O / L.
 */
static void attend_row(const float *q, const float *K, const float *V, float *out, int hd, int p,
                       int kv_len, int window) {
  int lo = window > 0 ? (p - window + 1 > 0 ? p - window + 1 : 0) : 0;
  int hi = p < kv_len - 1 ? p : kv_len - 1;
  float M = 0.0f, L = 0.0f;
  float *O = (float *)calloc((size_t)hd, sizeof(float));
  float *o = (float *)malloc(sizeof(float) * (size_t)hd);
  float s[ATT_BLOCK], pr[ATT_BLOCK];
  int first = 1;
  for (int b = lo / ATT_BLOCK; b <= hi / ATT_BLOCK; b++) {
    int j0 = b * ATT_BLOCK > lo ? b * ATT_BLOCK : lo;
    int j1 = (b + 1) * ATT_BLOCK - 1 < hi ? (b + 1) * ATT_BLOCK - 1 : hi;
    float m = -INFINITY;
    for (int j = j0; j <= j1; j++) {
      const float *kr = K + (size_t)j * hd;
      float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int c = 0; c < hd / 4; c++) {
        float *ac = &a[c & 3];
        *ac = fmaf(q[4 * c + 0], kr[4 * c + 0], *ac);
        *ac = fmaf(q[4 * c + 1], kr[4 * c + 1], *ac);
        *ac = fmaf(q[4 * c + 2], kr[4 * c + 2], *ac);
        *ac = fmaf(q[4 * c + 3], kr[4 * c + 3], *ac);
      }
      float sc = (a[0] + a[1]) + (a[2] + a[3]);
      s[j - j0] = sc;
      if (sc > m) m = sc;
    }
    float l = 0.0f;
    for (int j = j0; j <= j1; j++) {
      pr[j - j0] = g4o_exp(s[j - j0] - m);
      l = l + pr[j - j0];
    }
    for (int d = 0; d < hd; d++) {
      float acc = 0.0f;
      for (int j = j0; j <= j1; j++) acc = fmaf(pr[j - j0], V[(size_t)j * hd + d], acc);
      o[d] = acc;
    }
    if (first) {
      M = m;
      L = l;
      memcpy(O, o, sizeof(float) * (size_t)hd);
      first = 0;
    } else {
      float Mn = M > m ? M : m;
      float ea = g4o_exp(M - Mn);
      float ec = g4o_exp(m - Mn);
      L = (L * ea) + (l * ec);
      for (int d = 0; d < hd; d++) O[d] = (O[d] * ea) + (o[d] * ec);
      M = Mn;
    }
  }
  for (int d = 0; d < hd; d++) out[d] = O[d] / L;
  free(O);
  free(o);
}

void g4o_attention(const float *q, const float *cache, float *out, int heads, int head_dim,
                   int q_count, int q_start, int kv_len, int window, int max_context) {
  const float *K = cache;
  const float *V = cache + (size_t)max_context * head_dim;
#pragma omp parallel for collapse(2) schedule(static)
  for (int qi = 0; qi < q_count; qi++)
    for (int h = 0; h < heads; h++) {
      size_t base = ((size_t)qi * heads + h) * head_dim;
      attend_row(q + base, K, V, out + base, head_dim, q_start + qi, kv_len, window);
    }
}

/* ========================================================================= gathers */

/*
 * embed-gather / ple-gather (src/kernels/embedGather.ts:176-261, oracle 319-344): the embed
 * scale folds into the row scale first (one f32 multiply), then one multiply per element:
 * (code - 8) * (out_scale * scale[row, col / group]). A sliced call (slice_rows > 0) writes
 * only slots whose id lies in the slice and reads the slice's own rows; scales stay addressed
 * by the absolute row (src/kernels/embedGather.ts:212-226, src/tableSplit.ts:238-243).
 */
void g4o_embed_gather(const uint8_t *codes, const uint16_t *scales_f16, const int32_t *ids,
                      float *dst, int slots, int cols, int group_size, float out_scale,
                      int slice_start, int slice_rows) {
  int groups = cols / group_size;
  size_t row_bytes = (size_t)cols / 2;
  for (int s = 0; s < slots; s++) {
    int row = ids[s];
    int local = row;
    if (slice_rows > 0) {
      if (row < slice_start || row - slice_start >= slice_rows) continue;
      local = row - slice_start;
    }
    const uint8_t *cr = codes + (size_t)local * row_bytes;
    for (int col = 0; col < cols; col++) {
      float scale = out_scale * g4o_f16_to_f32(scales_f16[(size_t)row * groups + col / group_size]);
      dst[(size_t)s * cols + col] = (float)code4(cr, col) * scale;
    }
  }
}

/*
 * dense-bf16-matmul (src/kernels/denseMatmul.ts:93-222): y[c, r] = alpha * dot(w[r], x[c]),
 * bf16 widened exactly. Order: 32 lanes, lane l walks the row's 8-element chunks l, l + 32, ...
 * with an fma per element, then the butterfly; one multiply by alpha.
 */
void g4o_dense_bf16(const uint16_t *w, const float *x, float *y, int N, int K, int cols,
                    float alpha) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < N; r++) {
    const uint16_t *wr = w + (size_t)r * K;
    for (int c = 0; c < cols; c++) {
      const float *xc = x + (size_t)c * K;
      float lanes[32];
      for (int l = 0; l < 32; l++) {
        float a = 0.0f;
        for (int ch = l; ch < K / 8; ch += 32)
          for (int j = 0; j < 8; j++) a = fmaf(g4o_bf16_to_f32(wr[ch * 8 + j]), xc[ch * 8 + j], a);
        lanes[l] = a;
      }
      y[(size_t)c * N + r] = alpha * butterfly32(lanes);
    }
  }
}

/* ==================================================================== head (K14/K15) */

/* tanh(l / cap) * cap (src/kernels/logitSoftcap.ts:85-120), then argmax with the lowest index
 * among maxima (src/kernels/argmax.ts:267-310). token = {index, value bits}. */
void g4o_softcap_argmax(const float *logits, float *capped, int32_t *token, int n, float cap) {
  int best = -1;
  float bv = -INFINITY;
  for (int i = 0; i < n; i++) {
    float v = cap != 0.0f ? g4o_tanh(logits[i] / cap) * cap : logits[i];
    if (capped) capped[i] = v;
    if (v > bv) {
      bv = v;
      best = i;
    }
  }
  token[0] = best;
  memcpy(&token[1], &bv, 4);
}

/* ==================================================== reference restatements (f64) */

/* rmsNormOracle (src/kernels/rmsNorm.ts:208-245): f64 sum, rounded once. */
void g4o_ref_rms_norm(const float *src, const float *gain, float *dst, int rows, int width,
                      float eps) {
  for (int r = 0; r < rows; r++) {
    double sum = 0.0;
    for (int i = 0; i < width; i++) {
      double v = src[(size_t)r * width + i];
      sum += v * v;
    }
    double inv = 1.0 / sqrt(sum / width + (double)eps);
    for (int i = 0; i < width; i++)
      dst[(size_t)r * width + i] = (float)((double)src[(size_t)r * width + i] * inv * (gain ? (double)gain[i] : 1.0));
  }
}

/* normResidualOracle (src/kernels/mlpEpilogue.ts:196-220). */
void g4o_ref_norm_residual(const float *src, const float *gain, const float *residual,
                           float *dst, int rows, int width, float eps) {
  for (int r = 0; r < rows; r++) {
    double sum = 0.0;
    for (int i = 0; i < width; i++) {
      double v = src[(size_t)r * width + i];
      sum += v * v;
    }
    double inv = 1.0 / sqrt(sum / width + (double)eps);
    for (int i = 0; i < width; i++)
      dst[(size_t)r * width + i] = (float)((double)residual[(size_t)r * width + i] +
                                           (double)src[(size_t)r * width + i] * inv * (double)gain[i]);
  }
}

/* attentionOracle (src/kernels/attention.ts:858-903): f64 scores, max-subtracted softmax, f64
 * weighted V sum, rounded once. k, v are [kv_len, head_dim]. */
void g4o_ref_attention(const float *q, const float *k, const float *v, float *out, int heads,
                       int head_dim, int q_count, int q_start, int kv_len, int window,
                       double scale) {
  double *scores = (double *)malloc(sizeof(double) * (size_t)kv_len);
  for (int qi = 0; qi < q_count; qi++) {
    int p = q_start + qi;
    int lo = window > 0 ? (p - window + 1 > 0 ? p - window + 1 : 0) : 0;
    for (int h = 0; h < heads; h++) {
      size_t qb = ((size_t)qi * heads + h) * head_dim;
      double m = -INFINITY;
      for (int j = lo; j <= p; j++) {
        double d = 0.0;
        for (int i = 0; i < head_dim; i++) d += (double)q[qb + i] * (double)k[(size_t)j * head_dim + i];
        double s = d * scale;
        scores[j] = s;
        if (s > m) m = s;
      }
      double l = 0.0;
      for (int j = lo; j <= p; j++) {
        scores[j] = exp(scores[j] - m);
        l += scores[j];
      }
      for (int i = 0; i < head_dim; i++) {
        double a = 0.0;
        for (int j = lo; j <= p; j++) a += scores[j] * (double)v[(size_t)j * head_dim + i];
        out[qb + i] = (float)(a / l);
      }
    }
  }
  free(scores);
}

/* geluMulOracle (src/kernels/geluMul.ts:172-240): gelu(gate) * up in f64 with the clamp, one
 * rounding to f32, then applySrq. */
void g4o_ref_gelu_mul(const float *gate, const float *up, float *dst, int n, float srq_scale) {
  for (int i = 0; i < n; i++) {
    double x = gate[i];
    double inner0 = 0.7978845608028654 * (x + 0.044715 * x * x * x);
    double inner = inner0 > 10.0 ? 10.0 : (inner0 < -10.0 ? -10.0 : inner0);
    float v = (float)(0.5 * x * (1.0 + tanh(inner)) * (double)up[i]);
    if (srq_scale != 0.0f) v = g4o_srq_out(v, srq_scale);
    dst[i] = v;
  }
}

/* denseMatmulOracle (src/kernels/denseMatmul.ts:222-248): per vec4, four products and three
 * adds in f32, one add into the accumulator, then alpha. w is f32 [N, K]. */
void g4o_ref_dense(const float *w, const float *x, float *y, int N, int K, int cols, float alpha) {
  for (int c = 0; c < cols; c++)
    for (int r = 0; r < N; r++) {
      float sum = 0.0f;
      for (int k = 0; k < K; k += 4) {
        float d = 0.0f;
        for (int j = 0; j < 4; j++) d = d + w[(size_t)r * K + k + j] * x[(size_t)c * K + k + j];
        sum = sum + d;
      }
      y[(size_t)c * N + r] = alpha * sum;
    }
}

/* ====================================================================== table split */

/* planTableSplit (src/tableSplit.ts:125-215): one buffer when the table fits the limit, else
 * slices of floor(cap / rowBytes) rows rounded down to a multiple of 16. Returns 0, or -1 when
 * a single row does not fit. */
int g4o_plan_table_split(uint64_t rows, uint64_t row_bytes, uint64_t limit_bytes,
                         uint64_t slice_bytes, int32_t *n_slices, int32_t *rows_per_slice,
                         int32_t *last_rows) {
  uint64_t total = rows * row_bytes;
  int fits = total > 0 && total <= limit_bytes;
  uint64_t cap = slice_bytes < limit_bytes ? slice_bytes : limit_bytes;
  if (cap < 1) cap = 1;
  uint64_t per = (fits ? limit_bytes : cap) / row_bytes;
  if (per < 1) return -1;
  uint64_t aligned = per >= 16 ? per - (per % 16) : per;
  uint64_t ps = rows < aligned ? rows : aligned;
  uint64_t n = ps ? (rows + ps - 1) / ps : 1;
  if (n == 0) n = 1;
  if (n_slices) *n_slices = (int32_t)n;
  if (rows_per_slice) *rows_per_slice = (int32_t)ps;
  if (last_rows) *last_rows = (int32_t)(rows - (n - 1) * ps);
  return 0;
}

/* ========================================================================= the model */

void g4o_arch_default(g4o_arch *a) {
  a->layer_count = 35;
  a->hidden = 1536;
  a->q_heads = 8;
  a->sliding_hd = 256;
  a->global_hd = 512;
  a->global_mask = (1ull << 4) | (1ull << 9) | (1ull << 14) | (1ull << 19) | (1ull << 24) |
                   (1ull << 29) | (1ull << 34);
  a->window = 512;
  a->producers = 15;
  a->ffn = 6144;
  a->vocab = 262144;
  a->ple_dim = 256;
  a->eps = 1e-6f;
  a->softcap = 30.0f;
  a->theta_sliding = 1e4f;
  a->theta_global = 1e6f;
  a->partial_rotary = 0.25f;
  a->consumer_ffn = 6144;
  a->consumer_mlp_bits = 4;
  a->head_bits = 4;
  a->head_calibrated = 1;
}

/* Synthetic tensor kinds; a layer tensor's hash stream is ((layer + 1) << 8) | kind. */
enum {
  TK_Q_W = 0, TK_Q_S, TK_K_W, TK_K_S, TK_V_W, TK_V_S, TK_O_W, TK_O_S,
  TK_GATE_W, TK_GATE_S, TK_UP_W, TK_UP_S, TK_DOWN_W, TK_DOWN_S,
  TK_PLEG_W, TK_PLEG_S, TK_PLEP_W, TK_PLEP_S,
  TK_LN_IN, TK_LN_POST_ATTN, TK_LN_PRE_FFN, TK_LN_POST_FFN, TK_LN_POST_PLE,
  TK_QNORM, TK_KNORM, TK_LAYER_SCALAR, TK_SRQ,
  TK_EMBED_W = 40, TK_EMBED_S, TK_PLE_W, TK_PLE_S, TK_PLMP_W, TK_PLMP_NORM, TK_FINAL_NORM,
  TK_PROMPT = 50
};

/* Linear sites, in the order of their static activation scale table. */
enum { S_Q = 0, S_K, S_V, S_O, S_GATE, S_UP, S_DOWN, S_PLEG, S_PLEP, S_LM, N_SITES };

/* Base static activation scales per site (in, out); each layer's value is base * (0.9 + 0.2 u)
 * from the hash. lm_head's output scale is 0: the logits are not snapped. */
static const double SRQ_BASE_IN[N_SITES] = {0.04, 0.04, 0.04, 0.04, 0.033, 0.033, 1.0, 0.085, 0.34, 0.024};
static const double SRQ_BASE_OUT[N_SITES] = {0.11, 0.097, 0.092, 0.2, 0.108, 0.11, 3.9, 0.225, 0.085, 0.0};

static uint64_t layer_stream(int layer, int kind) { return ((uint64_t)(layer + 1) << 8) | (uint64_t)kind; }

typedef struct {
  uint8_t *w;
  uint16_t *s;
  int N, K, bits;
  float in_scale, out_scale;
} o_linear;

typedef struct {
  int hd, global, producer;
  o_linear q, k, v, o, gate, up, down, pleg, plep;
  float *ln_in, *ln_post_attn, *ln_pre_ffn, *ln_post_ffn, *ln_post_ple, *q_norm, *k_norm;
  float layer_scalar;
} o_layer;

struct g4o_model {
  g4o_arch a;
  uint64_t seed;
  o_layer *layers;
  uint8_t *embed_w;
  uint16_t *embed_s;
  uint8_t *ple_w;
  uint16_t *ple_s;
  uint16_t *plmp_w;
  float *plmp_norm;
  float *final_norm;
  o_linear lm;
};

static void gen_words(uint8_t *dst, size_t bytes, uint64_t seed, uint64_t stream) {
  uint64_t key = stream_key(seed, stream);
  size_t words = bytes / 4;
  uint32_t *w = (uint32_t *)dst;
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < words; i++) w[i] = (uint32_t)(keyed(key, i) >> 32);
}

/* f16 values lo + (hi - lo) u, computed in f64, rounded to f32 then to f16. */
static void gen_f16(uint16_t *dst, size_t n, uint64_t seed, uint64_t stream, double lo, double hi) {
  uint64_t key = stream_key(seed, stream);
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; i++) {
    double v = lo + (hi - lo) * unit24(keyed(key, i));
    dst[i] = g4o_f32_to_f16((float)v);
  }
}

/* bf16-representable f32 values lo + (hi - lo) u (norm gains, the layer scalar). */
static void gen_bf16_f32(float *dst, size_t n, uint64_t seed, uint64_t stream, double lo, double hi) {
  uint64_t key = stream_key(seed, stream);
  for (size_t i = 0; i < n; i++) {
    double v = lo + (hi - lo) * unit24(keyed(key, i));
    dst[i] = g4o_bf16_to_f32(g4o_f32_to_bf16((float)v));
  }
}

static float srq_scale(uint64_t seed, int layer, int site, int out) {
  double base = out ? SRQ_BASE_OUT[site] : SRQ_BASE_IN[site];
  if (base == 0.0) return 0.0f;
  uint64_t h = g4o_hash(seed, layer_stream(layer, TK_SRQ), (uint64_t)(site * 2 + out));
  return (float)(base * (0.9 + 0.2 * unit24(h)));
}

static void make_linear(o_linear *L, uint64_t seed, int layer, int kw, int ks, int site, int N,
                        int K, int bits) {
  L->N = N;
  L->K = K;
  L->bits = bits;
  size_t bytes = (size_t)N * K * bits / 8;
  L->w = (uint8_t *)malloc(bytes);
  L->s = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)N);
  gen_words(L->w, bytes, seed, layer_stream(layer, kw));
  /* Row scales keep activations O(1): int8 codes are 16x larger than int4, 2-bit ones 4x smaller. */
  double div = bits == 8 ? 16.0 : (bits == 2 ? 0.25 : 1.0);
  gen_f16(L->s, (size_t)N, seed, layer_stream(layer, ks), 1e-3 / div, 1e-2 / div);
  L->in_scale = srq_scale(seed, layer, site, 0);
  L->out_scale = srq_scale(seed, layer, site, 1);
}

static float *make_gain(int n, uint64_t seed, int layer, int kind) {
  float *g = (float *)malloc(sizeof(float) * (size_t)n);
  gen_bf16_f32(g, (size_t)n, seed, layer_stream(layer, kind), 0.5, 1.5);
  return g;
}

g4o_model *g4o_model_synth(const g4o_arch *a, uint64_t seed) {
  g4o_model *m = (g4o_model *)calloc(1, sizeof(g4o_model));
  m->a = *a;
  m->seed = seed;
  int H = a->hidden;
  m->layers = (o_layer *)calloc((size_t)a->layer_count, sizeof(o_layer));
  for (int L = 0; L < a->layer_count; L++) {
    o_layer *ly = &m->layers[L];
    ly->global = (int)((a->global_mask >> L) & 1ull);
    ly->producer = L < a->producers;
    ly->hd = ly->global ? a->global_hd : a->sliding_hd;
    int qrows = a->q_heads * ly->hd;
    make_linear(&ly->q, seed, L, TK_Q_W, TK_Q_S, S_Q, qrows, H, 4);
    if (ly->producer) {
      make_linear(&ly->k, seed, L, TK_K_W, TK_K_S, S_K, ly->hd, H, 4);
      make_linear(&ly->v, seed, L, TK_V_W, TK_V_S, S_V, ly->hd, H, 4);
    }
    make_linear(&ly->o, seed, L, TK_O_W, TK_O_S, S_O, H, qrows, 4);
    const int ffn = ly->producer ? a->ffn : a->consumer_ffn;
    const int mb = ly->producer ? 4 : a->consumer_mlp_bits;
    make_linear(&ly->gate, seed, L, TK_GATE_W, TK_GATE_S, S_GATE, ffn, H, mb);
    make_linear(&ly->up, seed, L, TK_UP_W, TK_UP_S, S_UP, ffn, H, mb);
    make_linear(&ly->down, seed, L, TK_DOWN_W, TK_DOWN_S, S_DOWN, H, ffn, mb);
    make_linear(&ly->pleg, seed, L, TK_PLEG_W, TK_PLEG_S, S_PLEG, a->ple_dim, H, 8);
    make_linear(&ly->plep, seed, L, TK_PLEP_W, TK_PLEP_S, S_PLEP, H, a->ple_dim, 8);
    ly->ln_in = make_gain(H, seed, L, TK_LN_IN);
    ly->ln_post_attn = make_gain(H, seed, L, TK_LN_POST_ATTN);
    ly->ln_pre_ffn = make_gain(H, seed, L, TK_LN_PRE_FFN);
    ly->ln_post_ffn = make_gain(H, seed, L, TK_LN_POST_FFN);
    ly->ln_post_ple = make_gain(H, seed, L, TK_LN_POST_PLE);
    ly->q_norm = make_gain(ly->hd, seed, L, TK_QNORM);
    ly->k_norm = make_gain(ly->hd, seed, L, TK_KNORM);
    float ls;
    gen_bf16_f32(&ls, 1, seed, layer_stream(L, TK_LAYER_SCALAR), 0.03, 0.9);
    ly->layer_scalar = ls;
  }
  size_t V = (size_t)a->vocab;
  const size_t embed_bytes = V * (size_t)H * (size_t)a->head_bits / 8;
  m->embed_w = (uint8_t *)malloc(embed_bytes);
  gen_words(m->embed_w, embed_bytes, seed, layer_stream(-1, TK_EMBED_W));
  m->embed_s = (uint16_t *)malloc(sizeof(uint16_t) * V);
  const double ediv = a->head_bits == 2 ? 0.25 : 1.0;
  gen_f16(m->embed_s, V, seed, layer_stream(-1, TK_EMBED_S), 1e-3 / ediv, 1e-2 / ediv);
  size_t ple_cols = (size_t)a->layer_count * a->ple_dim;
  m->ple_w = (uint8_t *)malloc(V * ple_cols / 2);
  gen_words(m->ple_w, V * ple_cols / 2, seed, layer_stream(-1, TK_PLE_W));
  m->ple_s = (uint16_t *)malloc(sizeof(uint16_t) * V * (size_t)a->layer_count);
  gen_f16(m->ple_s, V * (size_t)a->layer_count, seed, layer_stream(-1, TK_PLE_S), 1e-3, 1e-2);
  m->plmp_w = (uint16_t *)malloc(sizeof(uint16_t) * ple_cols * (size_t)H);
  {
    uint64_t key = stream_key(seed, layer_stream(-1, TK_PLMP_W));
    size_t n = ple_cols * (size_t)H;
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) {
      double v = (2.0 * unit24(keyed(key, i)) - 1.0) * 0.04419417382415922;
      m->plmp_w[i] = g4o_f32_to_bf16((float)v);
    }
  }
  m->plmp_norm = make_gain(a->ple_dim, seed, -1, TK_PLMP_NORM);
  m->final_norm = make_gain(H, seed, -1, TK_FINAL_NORM);
  /* lm_head is tied to embed_tokens (src/execute.ts:207-214): same codes, same row scales. */
  m->lm.w = m->embed_w;
  m->lm.s = m->embed_s;
  m->lm.N = a->vocab;
  m->lm.K = H;
  m->lm.bits = a->head_bits;
  /* An uncalibrated head (the checkpoint's, src/quant.ts:574-585) has both scales 0.0. */
  m->lm.in_scale = a->head_calibrated ? srq_scale(seed, -1, S_LM, 0) : 0.0f;
  m->lm.out_scale = a->head_calibrated ? srq_scale(seed, -1, S_LM, 1) : 0.0f;
  return m;
}

static void free_linear(o_linear *L) {
  free(L->w);
  free(L->s);
}

void g4o_model_free(g4o_model *m) {
  if (!m) return;
  for (int L = 0; L < m->a.layer_count; L++) {
    o_layer *ly = &m->layers[L];
    free_linear(&ly->q);
    if (ly->producer) {
      free_linear(&ly->k);
      free_linear(&ly->v);
    }
    free_linear(&ly->o);
    free_linear(&ly->gate);
    free_linear(&ly->up);
    free_linear(&ly->down);
    free_linear(&ly->pleg);
    free_linear(&ly->plep);
    free(ly->ln_in);
    free(ly->ln_post_attn);
    free(ly->ln_pre_ffn);
    free(ly->ln_post_ffn);
    free(ly->ln_post_ple);
    free(ly->q_norm);
    free(ly->k_norm);
  }
  free(m->layers);
  free(m->embed_w);
  free(m->embed_s);
  free(m->ple_w);
  free(m->ple_s);
  free(m->plmp_w);
  free(m->plmp_norm);
  free(m->final_norm);
  free(m);
}

static const char *LM = "model.language_model.";

static const o_linear *linear_by_module(const g4o_model *m, const char *mod, int *layer_out) {
  if (strcmp(mod, "lm_head") == 0) return &m->lm;
  int L;
  char rest[128];
  if (strncmp(mod, LM, strlen(LM)) != 0) return NULL;
  if (sscanf(mod + strlen(LM), "layers.%d.%127s", &L, rest) != 2) return NULL;
  if (L < 0 || L >= m->a.layer_count) return NULL;
  const o_layer *ly = &m->layers[L];
  if (layer_out) *layer_out = L;
  if (!strcmp(rest, "self_attn.q_proj")) return &ly->q;
  if (!strcmp(rest, "self_attn.k_proj")) return ly->producer ? &ly->k : NULL;
  if (!strcmp(rest, "self_attn.v_proj")) return ly->producer ? &ly->v : NULL;
  if (!strcmp(rest, "self_attn.o_proj")) return &ly->o;
  if (!strcmp(rest, "mlp.gate_proj")) return &ly->gate;
  if (!strcmp(rest, "mlp.up_proj")) return &ly->up;
  if (!strcmp(rest, "mlp.down_proj")) return &ly->down;
  if (!strcmp(rest, "per_layer_input_gate")) return &ly->pleg;
  if (!strcmp(rest, "per_layer_projection")) return &ly->plep;
  return NULL;
}

static int ends_with(const char *s, const char *suf) {
  size_t a = strlen(s), b = strlen(suf);
  return a >= b && strcmp(s + a - b, suf) == 0;
}

const void *g4o_model_tensor(const g4o_model *m, const char *name, uint64_t *bytes) {
  char mod[256];
  size_t H = (size_t)m->a.hidden, V = (size_t)m->a.vocab;
  size_t ple_cols = (size_t)m->a.layer_count * m->a.ple_dim;
  if (!strcmp(name, "model.language_model.embed_tokens.embedding_quantized")) {
    *bytes = V * H * (size_t)m->a.head_bits / 8;
    return m->embed_w;
  }
  if (!strcmp(name, "model.language_model.embed_tokens.embedding_scale")) {
    *bytes = V * 2;
    return m->embed_s;
  }
  if (!strcmp(name, "model.language_model.embed_tokens_per_layer.embedding_quantized")) {
    *bytes = V * ple_cols / 2;
    return m->ple_w;
  }
  if (!strcmp(name, "model.language_model.embed_tokens_per_layer.embedding_scale")) {
    *bytes = V * (size_t)m->a.layer_count * 2;
    return m->ple_s;
  }
  if (!strcmp(name, "model.language_model.per_layer_model_projection.weight")) {
    *bytes = ple_cols * H * 2;
    return m->plmp_w;
  }
  if (!strcmp(name, "model.language_model.per_layer_projection_norm.weight")) {
    *bytes = (size_t)m->a.ple_dim * 4;
    return m->plmp_norm;
  }
  if (!strcmp(name, "model.language_model.norm.weight")) {
    *bytes = H * 4;
    return m->final_norm;
  }
  const char *suffixes[] = {".weight_scale", ".weight"};
  for (int i = 0; i < 2; i++) {
    if (ends_with(name, suffixes[i])) {
      size_t n = strlen(name) - strlen(suffixes[i]);
      if (n >= sizeof(mod)) return NULL;
      memcpy(mod, name, n);
      mod[n] = 0;
      const o_linear *L = linear_by_module(m, mod, NULL);
      if (L) {
        if (i == 0) {
          *bytes = (size_t)L->N * 2;
          return L->s;
        }
        *bytes = (size_t)L->N * L->K * L->bits / 8;
        return L->w;
      }
    }
  }
  int L;
  char rest[128];
  if (strncmp(name, LM, strlen(LM)) == 0 &&
      sscanf(name + strlen(LM), "layers.%d.%127s", &L, rest) == 2 && L >= 0 &&
      L < m->a.layer_count) {
    const o_layer *ly = &m->layers[L];
    struct { const char *n; const float *p; size_t len; } g[] = {
        {"input_layernorm.weight", ly->ln_in, H},
        {"post_attention_layernorm.weight", ly->ln_post_attn, H},
        {"pre_feedforward_layernorm.weight", ly->ln_pre_ffn, H},
        {"post_feedforward_layernorm.weight", ly->ln_post_ffn, H},
        {"post_per_layer_input_norm.weight", ly->ln_post_ple, H},
        {"self_attn.q_norm.weight", ly->q_norm, (size_t)ly->hd},
        {"self_attn.k_norm.weight", ly->k_norm, (size_t)ly->hd},
    };
    for (size_t i = 0; i < sizeof(g) / sizeof(g[0]); i++)
      if (!strcmp(rest, g[i].n)) {
        *bytes = g[i].len * 4;
        return g[i].p;
      }
  }
  *bytes = 0;
  return NULL;
}

float g4o_model_scalar(const g4o_model *m, const char *name) {
  char mod[256];
  const char *sfx[] = {".input_activation_scale", ".output_activation_scale"};
  for (int i = 0; i < 2; i++) {
    if (ends_with(name, sfx[i])) {
      size_t n = strlen(name) - strlen(sfx[i]);
      if (n >= sizeof(mod)) return 0.0f;
      memcpy(mod, name, n);
      mod[n] = 0;
      const o_linear *L = linear_by_module(m, mod, NULL);
      if (!L) return 0.0f;
      return i == 0 ? L->in_scale : L->out_scale;
    }
  }
  int Lr;
  if (strncmp(name, LM, strlen(LM)) == 0 &&
      sscanf(name + strlen(LM), "layers.%d.layer_scalar", &Lr) == 1 && Lr >= 0 &&
      Lr < m->a.layer_count && ends_with(name, "layer_scalar"))
    return m->layers[Lr].layer_scalar;
  return 0.0f;
}

/* --------------------------------------------------------------------- sequences */

struct g4o_seq {
  int max_ctx;
  int n_prod;
  float **cache; /* per producer layer: [2, max_ctx, hd] */
};

g4o_seq *g4o_seq_new(const g4o_model *m, int32_t max_context) {
  g4o_seq *s = (g4o_seq *)calloc(1, sizeof(g4o_seq));
  s->max_ctx = max_context;
  s->n_prod = m->a.producers;
  s->cache = (float **)calloc((size_t)s->n_prod, sizeof(float *));
  for (int L = 0; L < s->n_prod; L++)
    s->cache[L] = (float *)calloc((size_t)2 * max_context * m->layers[L].hd, sizeof(float));
  return s;
}

void g4o_seq_free(g4o_seq *s) {
  if (!s) return;
  for (int L = 0; L < s->n_prod; L++) free(s->cache[L]);
  free(s->cache);
  free(s);
}

static float g_site_in[N_SITES], g_site_out[N_SITES];

static void track(int site, const float *x, int n, int out) {
  float mx = out ? g_site_out[site] : g_site_in[site];
  for (int i = 0; i < n; i++) {
    float v = fabsf(x[i]);
    if (v > mx) mx = v;
  }
  if (out) g_site_out[site] = mx; else g_site_in[site] = mx;
}

void g4o_site_stats(float *max_in, float *max_out, int32_t n_sites) {
  for (int i = 0; i < n_sites && i < N_SITES; i++) {
    max_in[i] = g_site_in[i];
    max_out[i] = g_site_out[i];
  }
  memset(g_site_in, 0, sizeof(g_site_in));
  memset(g_site_out, 0, sizeof(g_site_out));
}

/* A calibrated linear with the raw (pre-snap) output tracked for calibration. */
static void run_linear(const o_linear *L, int site, const float *x, float *y) {
  track(site, x, L->K, 0);
  /* pre-snap output for the statistics */
  float *raw = (float *)malloc(sizeof(float) * (size_t)L->N);
  g4o_qgemv(L->w, L->s, x, L->in_scale, 0.0f, L->bits, L->N, L->K, 1, raw, NULL);
  track(site, raw, L->N, 1);
  for (int i = 0; i < L->N; i++) y[i] = g4o_srq_out(raw[i], L->out_scale);
  free(raw);
}

/* The layer whose cache a layer's attention reads (kvRoleForLayer, src/kv.ts:76-88): its own
 * on a producer, the last producer of the same attention type on a consumer. */
static int cache_layer(const g4o_model *m, int L) {
  if (L < m->a.producers) return L;
  int want = (int)((m->a.global_mask >> L) & 1ull);
  int last = -1;
  for (int p = 0; p < m->a.producers; p++)
    if ((int)((m->a.global_mask >> p) & 1ull) == want) last = p;
  return last;
}

/*
 * One position through the model, following planDecodeStep / planPrefillChunk step order
 * (src/plan.ts:487-824) and resolveStep's slot wiring (src/execute.ts:438-1010).
 */
static void forward_one(const g4o_model *m, g4o_seq *s, int id, int pos, int n_layers,
                        int want_head, int32_t *token, float *logits, float *top2) {
  const g4o_arch *a = &m->a;
  const int H = a->hidden, PD = a->ple_dim, NL = a->layer_count;
  const int ple_cols = NL * PD;
  float *h = (float *)malloc(sizeof(float) * H);
  float *x = (float *)malloc(sizeof(float) * H);
  float *tmp = (float *)malloc(sizeof(float) * H);
  float *ple_id = (float *)malloc(sizeof(float) * ple_cols);
  float *ple_proj = (float *)malloc(sizeof(float) * ple_cols);
  float *ple_in = (float *)malloc(sizeof(float) * ple_cols);
  float *q = (float *)malloc(sizeof(float) * a->q_heads * a->global_hd);
  float *qr = (float *)malloc(sizeof(float) * a->q_heads * a->global_hd);
  float *att = (float *)malloc(sizeof(float) * a->q_heads * a->global_hd);
  float *kk = (float *)malloc(sizeof(float) * a->global_hd);
  float *vv = (float *)malloc(sizeof(float) * a->global_hd);
  const int ffn_max = a->ffn > a->consumer_ffn ? a->ffn : a->consumer_ffn;
  float *gate = (float *)malloc(sizeof(float) * ffn_max);
  float *up = (float *)malloc(sizeof(float) * ffn_max);
  float *act = (float *)malloc(sizeof(float) * ffn_max);
  float *pg = (float *)malloc(sizeof(float) * PD);
  float *pa = (float *)malloc(sizeof(float) * PD);
  float *cs = (float *)malloc(sizeof(float) * a->global_hd);
  float *sn = (float *)malloc(sizeof(float) * a->global_hd);

  /* ---- embed phase (planEmbed, src/plan.ts:727-736) */
  int32_t ids1 = id;
  if (a->head_bits == 2) {
    /* embed-gather-2bit (src/kernels/embedGather.ts:236-256, 319-344): (u - 2) times the row
     * scale with sqrt(H) folded in first. */
    const uint8_t *er = m->embed_w + (size_t)id * H / 4;
    float scale = (float)sqrt((double)H) * g4o_f16_to_f32(m->embed_s[id]);
    for (int k = 0; k < H; k++) h[k] = (float)(ucode2(er, k) - 2) * scale;
  } else {
    g4o_embed_gather(m->embed_w, m->embed_s, &ids1, h, 1, H, H, (float)sqrt((double)H), 0, 0);
  }
  g4o_embed_gather(m->ple_w, m->ple_s, &ids1, ple_id, 1, ple_cols, PD, 16.0f, 0, 0);
  g4o_dense_bf16(m->plmp_w, h, ple_proj, ple_cols, H, 1, (float)pow((double)H, -0.5));
  for (int g = 0; g < NL; g++) {
    const float *pp = ple_proj + (size_t)g * PD;
    float inv = g4o_rms_inv(pp, PD, a->eps);
    for (int i = 0; i < PD; i++) {
      float normed = (pp[i] * inv) * m->plmp_norm[i];
      float sum = normed + ple_id[(size_t)g * PD + i];
      ple_in[(size_t)g * PD + i] = (float)0.7071067811865476 * sum;
    }
  }

  /* ---- layers */
  for (int L = 0; L < n_layers; L++) {
    const o_layer *ly = &m->layers[L];
    const int hd = ly->hd, nh = a->q_heads;
    if (L == 0) g4o_rms_norm(h, ly->ln_in, x, 1, H, a->eps);
    run_linear(&ly->q, S_Q, x, q);
    int rp = ly->global ? (int)(a->partial_rotary * hd / 2) : hd / 2;
    double theta = ly->global ? (double)a->theta_global : (double)a->theta_sliding;
    g4o_rope_tables(hd, rp, theta, pos, 1, cs, sn);
    g4o_q_norm_rope(q, ly->q_norm, cs, sn, qr, nh, hd, nh, a->eps);
    if (ly->producer) {
      run_linear(&ly->k, S_K, x, kk);
      run_linear(&ly->v, S_V, x, vv);
      g4o_kv_norm_rope_store(kk, vv, ly->k_norm, cs, sn, s->cache[L], 1, hd, pos, s->max_ctx, a->eps);
    }
    int cl = cache_layer(m, L);
    g4o_attention(qr, s->cache[cl], att, nh, hd, 1, pos, pos + 1, ly->global ? 0 : a->window, s->max_ctx);
    run_linear(&ly->o, S_O, att, tmp);
    /* join: post_attention_layernorm + residual, then pre_feedforward_layernorm (alpha 1) */
    g4o_norm_residual_norm(tmp, ly->ln_post_attn, h, ly->ln_pre_ffn, 1.0f, h, x, 1, H, a->eps);
    run_linear(&ly->gate, S_GATE, x, gate);
    run_linear(&ly->up, S_UP, x, up);
    for (int i = 0; i < ly->gate.N; i++) act[i] = g4o_gelu(gate[i]) * up[i];
    run_linear(&ly->down, S_DOWN, act, tmp);
    g4o_norm_residual(tmp, ly->ln_post_ffn, h, h, 1, H, a->eps);
    run_linear(&ly->pleg, S_PLEG, h, pg);
    for (int i = 0; i < PD; i++) pa[i] = g4o_gelu(pg[i]) * ple_in[(size_t)L * PD + i];
    run_linear(&ly->plep, S_PLEP, pa, tmp);
    const float *next_gain = L + 1 < NL ? m->layers[L + 1].ln_in : m->final_norm;
    g4o_norm_residual_norm(tmp, ly->ln_post_ple, h, next_gain, ly->layer_scalar, h, x, 1, H, a->eps);
  }

  /* ---- head (planHead, src/plan.ts:761-770) */
  if (want_head) {
    float *lg = (float *)malloc(sizeof(float) * (size_t)a->vocab);
    run_linear(&m->lm, S_LM, x, lg);
    int32_t tk[2];
    g4o_softcap_argmax(lg, lg, tk, a->vocab, a->softcap);
    *token = tk[0];
    if (logits) memcpy(logits, lg, sizeof(float) * (size_t)a->vocab);
    if (top2) {
      float v1 = -INFINITY, v2 = -INFINITY;
      int i1 = -1, i2 = -1;
      for (int i = 0; i < a->vocab; i++) {
        if (lg[i] > v1) {
          v2 = v1; i2 = i1; v1 = lg[i]; i1 = i;
        } else if (lg[i] > v2) {
          v2 = lg[i]; i2 = i;
        }
      }
      top2[0] = v1; top2[1] = (float)i1; top2[2] = v2; top2[3] = (float)i2;
    }
    free(lg);
  }
  free(h); free(x); free(tmp); free(ple_id); free(ple_proj); free(ple_in); free(q); free(qr);
  free(att); free(kk); free(vv); free(gate); free(up); free(act); free(pg); free(pa); free(cs);
  free(sn);
}

int g4o_forward(const g4o_model *m, g4o_seq *s, const int32_t *ids, int32_t n, int32_t start_pos,
                int32_t all_layers, int32_t want_head, int32_t *token, float *logits, float *top2) {
  if (n <= 0 || start_pos < 0 || start_pos + n > s->max_ctx) return -1;
  int nl = all_layers ? m->a.layer_count : m->a.producers;
  for (int t = 0; t < n; t++) {
    if (ids[t] < 0 || ids[t] >= m->a.vocab) return -1;
    int head = want_head && t == n - 1;
    forward_one(m, s, ids[t], start_pos + t, nl, head, token, head ? logits : NULL, head ? top2 : NULL);
  }
  return 0;
}

int g4o_generate(const g4o_model *m, const int32_t *prompt, int32_t n_prompt, int32_t max_new,
                 int32_t max_context, int32_t *tokens, float *gaps) {
  if (n_prompt < 1 || max_new < 1 || n_prompt + max_new > max_context) return -1;
  g4o_seq *s = g4o_seq_new(m, max_context);
  float top2[4];
  int32_t tok = -1;
  if (n_prompt > 1 && g4o_forward(m, s, prompt, n_prompt - 1, 0, 0, 0, NULL, NULL, NULL)) goto fail;
  if (g4o_forward(m, s, prompt + n_prompt - 1, 1, n_prompt - 1, 1, 1, &tok, NULL, top2)) goto fail;
  tokens[0] = tok;
  if (gaps) gaps[0] = top2[0] - top2[2];
  for (int i = 1; i < max_new; i++) {
    int32_t prev = tokens[i - 1];
    if (g4o_forward(m, s, &prev, 1, n_prompt + i - 1, 1, 1, &tok, NULL, top2)) goto fail;
    tokens[i] = tok;
    if (gaps) gaps[i] = top2[0] - top2[2];
  }
  g4o_seq_free(s);
  return 0;
fail:
  g4o_seq_free(s);
  return -1;
}

void g4o_synth_prompt(uint64_t seed, int32_t n, int32_t vocab, int32_t *ids) {
  for (int i = 0; i < n; i++)
    ids[i] = (int32_t)(g4o_hash(seed, (uint64_t)TK_PROMPT, (uint64_t)i) % (uint64_t)vocab);
}

void g4o_threads(int32_t n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
