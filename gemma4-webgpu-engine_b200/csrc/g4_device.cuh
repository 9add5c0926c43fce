// g4_device.cuh -- device arithmetic shared by every kernel of libgemma4_cuda.so.
//
// The library is compiled with --fmad=false, so `a * b + c` is two correctly rounded operations
// and a fused multiply-add appears only where fmaf() is written. Together with IEEE division and
// square root (no fast-math), every f32 value below is a fixed sequence of correctly rounded
// operations in a fixed order: the same numbers for every batch width, grid and stream.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

namespace g4 {

// ------------------------------------------------------------------------------ PDL hooks
// Programmatic dependent launch: a kernel may issue loads of read-only weights before
// `grid_wait()`, which returns once the previous kernel in the stream has completed and its
// memory is visible. Every kernel calls grid_wait() before it reads activations or writes
// anything, so completion of any kernel implies completion of all earlier ones.
__device__ __forceinline__ void grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------------------ hash
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xBF58476D1CE4E5B9ull;
  z ^= z >> 27;
  z *= 0x94D049BB133111EBull;
  z ^= z >> 31;
  return z;
}
__host__ __device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return mix64(seed ^ (stream * 0x9E3779B97F4A7C15ull));
}
__host__ __device__ __forceinline__ uint64_t keyed(uint64_t key, uint64_t i) {
  return mix64(key + i * 0xD1B54A32D192ED03ull);
}
__host__ __device__ __forceinline__ double unit24(uint64_t h) {
  return (double)(h >> 40) * (1.0 / 16777216.0);
}

// ------------------------------------------------------------------------ conversions
__host__ __device__ __forceinline__ uint32_t f32_bits(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t x;
  memcpy(&x, &f, 4);
  return x;
#endif
}
// f32 -> IEEE half, round to nearest even (bit arithmetic, so host and device agree).
__host__ __device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
  uint32_t x = f32_bits(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
  int e = (int)exp - 112;
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
__host__ __device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  uint32_t x = f32_bits(f);
  uint32_t lower = x & 0xffffu, upper = x >> 16;
  if (lower > 0x8000u || (lower == 0x8000u && (upper & 1u))) upper += 1u;
  return (uint16_t)(upper & 0xffffu);
}
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// ------------------------------------------------------------------- scalar arithmetic
// e^x: Cody-Waite reduction x = n ln2 + r (ln2 split into a 15-bit head and a tail), the
// degree-7 Taylor polynomial of e^r in Horner form with fused multiply-adds, and an exact scale
// by 2^n. Below ln(FLT_MIN) returns 0, above ln(FLT_MAX) returns +inf.
__device__ __forceinline__ float g4_exp(float x) {
  if (x < -87.33654f) return 0.0f;
  if (x > 88.72283f) return __int_as_float(0x7f800000);
  float n = rintf(__fmul_rn(x, 1.44269504088896341f));
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
    p = __fmul_rn(p, 2.0f);
    ni = 127;
  }
  return __fmul_rn(p, __uint_as_float((uint32_t)(ni + 127) << 23));
}

// tanh(x) = sign(x) (1 - e^{-2|x|}) / (1 + e^{-2|x|}).
__device__ __forceinline__ float g4_tanh(float x) {
  float ax = fabsf(x);
  float t = g4_exp(__fmul_rn(-2.0f, ax));
  float r = __fdiv_rn(__fsub_rn(1.0f, t), __fadd_rn(1.0f, t));
  return copysignf(r, x);
}

// gelu_pytorch_tanh with the +/-10 clamp: cube = x*x*x; inner = C * (x + K * cube);
// 0.5 * x * (1 + tanh(inner)).
__device__ __forceinline__ float g4_gelu(float x) {
  const float coef = 0.7978845608028654f;
  const float cubic = 0.044715f;
  float cube = __fmul_rn(__fmul_rn(x, x), x);
  float inner = __fmul_rn(coef, __fadd_rn(x, __fmul_rn(cubic, cube)));
  inner = fminf(fmaxf(inner, -10.0f), 10.0f);
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, g4_tanh(inner)));
}

// SRQ snaps: code = clamp(rint(x / s), -128, 127); out = code * s (0 scale: identity).
__device__ __forceinline__ int srq_code(float x, float s) {
  float q = rintf(__fdiv_rn(x, s));
  q = fminf(fmaxf(q, -128.0f), 127.0f);
  return (int)q;
}
__device__ __forceinline__ float srq_out(float v, float s) {
  if (s == 0.0f) return v;
  float q = rintf(__fdiv_rn(v, s));
  q = fminf(fmaxf(q, -128.0f), 127.0f);
  return __fmul_rn(q, s);
}

// The same snaps through a precomputed reciprocal r = RN(1 / s). t = RN(x * r) lies within
// |x / s| * 2^-23 of x / s, and so does RN(x / s); for |x / s| < 130 both are within 1.6e-5 of
// x / s, so whenever t is more than 1e-4 away from a half-integer, rint(t) equals
// rint(RN(x / s)) exactly. Closer to a tie the exact division decides. |t| >= 130 clamps either
// way. Bit-identical to srq_code / srq_out, without a division per element.
__device__ __forceinline__ float srq_q_r(float x, float s, float r) {
  const float t = __fmul_rn(x, r);
  if (fabsf(t) < 130.0f) {
    const float f = __fsub_rn(t, floorf(t));
    if (fabsf(__fsub_rn(f, 0.5f)) > 1e-4f) return fminf(fmaxf(rintf(t), -128.0f), 127.0f);
    return fminf(fmaxf(rintf(__fdiv_rn(x, s)), -128.0f), 127.0f);
  }
  return t > 0.0f ? 127.0f : -128.0f;
}
__device__ __forceinline__ int srq_code_r(float x, float s, float r) { return (int)srq_q_r(x, s, r); }
// The quotient stays a float so a negative value that rounds to zero keeps its sign (-0.0).
__device__ __forceinline__ float srq_out_r(float v, float s, float r) {
  if (s == 0.0f) return v;
  return __fmul_rn(srq_q_r(v, s, r), s);
}

// ---------------------------------------------------------------------- tracing
// Built with -DG4_TRACE (a diagnostic build, never the shipped library): block 0 of each traced
// kernel records (kernel id, %globaltimer) right after its dependency wait, so consecutive
// records give each launch's share of the live critical path. Off: the macro is empty.
#ifdef G4_TRACE
// g4_trace_buf / g4_trace_n are defined in the one translation unit that records (g4_kernels.cu).
#define G4_TRACE_POINT(id)                                                                   \
  do {                                                                                       \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0) {       \
      unsigned long long now;                                                                \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));                                \
      const unsigned int slot = atomicAdd(&g4_trace_n, 1u);                                  \
      if (slot < (1u << 15)) {                                                               \
        g4_trace_buf[2 * slot] = (unsigned long long)(id);                                   \
        g4_trace_buf[2 * slot + 1] = now;                                                    \
      }                                                                                      \
    }                                                                                        \
  } while (0)
// The same record from the thread of block 0 that reaches the call (the call site picks it).
#define G4_TRACE_POINT_T(id)                                                                 \
  do {                                                                                       \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) {                             \
      unsigned long long now;                                                                \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));                                \
      const unsigned int slot = atomicAdd(&g4_trace_n, 1u);                                  \
      if (slot < (1u << 15)) {                                                               \
        g4_trace_buf[2 * slot] = (unsigned long long)(id);                                   \
        g4_trace_buf[2 * slot + 1] = now;                                                    \
      }                                                                                      \
    }                                                                                        \
  } while (0)
// A record with a given time stamp, from whichever thread calls it.
#define G4_TRACE_REC(id, when)                                                               \
  do {                                                                                       \
    const unsigned int slot = atomicAdd(&g4_trace_n, 1u);                                    \
    if (slot < (1u << 15)) {                                                                 \
      g4_trace_buf[2 * slot] = (unsigned long long)(id);                                     \
      g4_trace_buf[2 * slot + 1] = (when);                                                   \
    }                                                                                        \
  } while (0)
#else
#define G4_TRACE_POINT(id) do {} while (0)
#define G4_TRACE_POINT_T(id) do {} while (0)
#endif

// ---------------------------------------------------------------------- mbarriers, bulk copies
#ifdef __CUDACC__
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.b32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on an mbarrier phase: false once `limit` polls have not seen it complete.
__device__ __forceinline__ bool mbar_wait_n(uint64_t *bar, uint32_t parity, int limit) {
  for (int i = 0; i < limit; i++)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// The poll limit of every wait in the library's kernels (build-time option; well under a second).
#ifndef G4_WAIT_POLLS
#define G4_WAIT_POLLS (1 << 22)
#endif
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  return mbar_wait_n(bar, parity, G4_WAIT_POLLS);
}
__device__ __forceinline__ void l2_prefetch(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

#endif

// ---------------------------------------------------------------------- reductions
// The 32-lane XOR butterfly, masks 1, 2, 4, 8, 16: every lane ends with the same balanced
// pairwise tree.
__device__ __forceinline__ float warp_sum_bfly(float v) {
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Sum of squares of v[0..n) (n a multiple of 4) in the 256-lane order: lane t walks vec4
// chunks t, t + 256, ... with one fma per component; each warp closes with the butterfly; the 8
// warp sums are added in ascending order. Must be called by all 256 threads of the block;
// `red` is 8 floats of shared memory. Every thread receives the total.
__device__ __forceinline__ float block_sumsq256(const float *v, int n, float *red) {
  const int t = threadIdx.x;
  const int nc = n >> 2;
  float acc = 0.0f;
  for (int c = t; c < nc; c += 256) {
    float4 x = reinterpret_cast<const float4 *>(v)[c];
    acc = fmaf(x.x, x.x, acc);
    acc = fmaf(x.y, x.y, acc);
    acc = fmaf(x.z, x.z, acc);
    acc = fmaf(x.w, x.w, acc);
  }
  acc = warp_sum_bfly(acc);
  __syncthreads();
  if ((t & 31) == 0) red[t >> 5] = acc;
  __syncthreads();
  float total = red[0];
#pragma unroll
  for (int g = 1; g < 8; g++) total = __fadd_rn(total, red[g]);
  return total;
}

// The same reduction over a vector whose vec4 chunks this thread holds in registers: chunk
// t + 256 i is vals[i] (i < count).
template <int MAXC>
__device__ __forceinline__ float block_sumsq256_regs(const float4 *vals, int count, float *red) {
  const int t = threadIdx.x;
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; i++) {
    if (i < count) {
      float4 x = vals[i];
      acc = fmaf(x.x, x.x, acc);
      acc = fmaf(x.y, x.y, acc);
      acc = fmaf(x.z, x.z, acc);
      acc = fmaf(x.w, x.w, acc);
    }
  }
  acc = warp_sum_bfly(acc);
  __syncthreads();
  if ((t & 31) == 0) red[t >> 5] = acc;
  __syncthreads();
  float total = red[0];
#pragma unroll
  for (int g = 1; g < 8; g++) total = __fadd_rn(total, red[g]);
  return total;
}

__device__ __forceinline__ float rms_inv(float total, int n, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)n), eps)));
}

// Mixed-sign dot product of four u8 by four s8 lanes accumulated into a s32.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace g4
