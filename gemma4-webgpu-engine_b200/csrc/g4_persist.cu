// Persistent B=1 decode step: one cooperative kernel runs every phase of a decode step (embed,
// per-layer inputs, 35 x {q/k/v, attention, o, gate/up, down, per_layer_gate,
// per_layer_projection}, lm_head, argmax), with a grid barrier between dependent phases instead
// of a launch boundary. The step order is planDecodeStep (src/plan.ts:487-859); every phase is
// the arithmetic of its per-launch kernel (shared device code in g4_gemv.cuh, same loops and
// epilogues), so the result is bit-identical to the launch chain.
//
// One CTA per SM (256 threads). The weights of the GEMV phases stream through a shared-memory
// ring of PS_NSLOT slots of PS_SLOT bytes in the order the phases consume them: thread 0 keeps
// the ring full (a slot is refilled with the next chunk, possibly of a later phase, as soon as it
// is consumed), so a phase's weights arrive while earlier phases and barriers run. Every wait is
// bounded: a barrier or copy that gives up raises g4_persist_error, the CTA stops computing, waits
// (bounded) for the copies it issued, and returns.
#include <cuda_runtime.h>
#include <float.h>

#include "g4_device.cuh"
#include "g4_gemv.cuh"
#include "g4_kernels.cuh"
#include "g4_persist.cuh"

namespace g4 {

__device__ int g4_persist_error;
#ifdef G4_TRACE
__device__ unsigned long long g4_ptrace[1 << 16];
__device__ unsigned int g4_ptrace_n;
int persist_trace_take(unsigned long long *out, int max_records) {
  unsigned int n = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&n, g4_ptrace_n, sizeof(n)) != cudaSuccess) return -1;
  if (n > (1u << 15)) n = 1u << 15;
  if ((int)n > max_records) n = (unsigned int)max_records;
  if (n && cudaMemcpyFromSymbol(out, g4_ptrace, (size_t)n * 16) != cudaSuccess) return -1;
  cudaMemcpyToSymbol(g4_ptrace_n, &zero, sizeof(zero));
  return (int)n;
}
#define P_TRACE(id)                                                                 \
  do {                                                                              \
    if (blockIdx.x == 0 && threadIdx.x == 0) {                                      \
      unsigned long long now;                                                       \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));                       \
      const unsigned int slot = atomicAdd(&g4_ptrace_n, 1u);                        \
      if (slot < (1u << 15)) {                                                      \
        g4_ptrace[2 * slot] = (unsigned long long)(id);                             \
        g4_ptrace[2 * slot + 1] = now;                                              \
      }                                                                             \
    }                                                                               \
  } while (0)
#else
#define P_TRACE(id) do {} while (0)
#endif

int persist_error_take() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g4_persist_error, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g4_persist_error, &zero, sizeof(int));
  return v;
}

constexpr int PS_SLOT = 16384;
constexpr int PS_NSLOT = 8;
constexpr int PS_SCRATCH = 64 * 1024;
constexpr int PS_CODES = 12288;        // two code vectors, K <= 6144
constexpr int PS_RSCALE = 2048;        // row scales of a CTA's slice (floats)
constexpr int PS_MISC = 4096;
constexpr int PS_SMEM = PS_NSLOT * PS_SLOT + PS_SCRATCH + PS_CODES + PS_RSCALE * 4 + PS_MISC + 128;

int persist_smem_bytes() { return PS_SMEM; }
int persist_slot_bytes() { return PS_SLOT; }
int persist_max_rows() { return PS_RSCALE; }

// Shared memory, at constant offsets from one base: the ring, the attention / dense scratch, the
// activation codes, the row scales, then the barriers and small arrays.
constexpr int PO_SCRATCH = PS_NSLOT * PS_SLOT;
constexpr int PO_CODES = PO_SCRATCH + PS_SCRATCH;
constexpr int PO_RSCALE = PO_CODES + PS_CODES;
constexpr int PO_FULL = PO_RSCALE + PS_RSCALE * 4;
constexpr int PO_VBAR = PO_FULL + PS_NSLOT * 8;
constexpr int PO_XSUM = PO_VBAR + 8;
constexpr int PO_RED = PO_XSUM + 16 * 4;
constexpr int PO_CANDV = PO_RED + 8 * 4;
constexpr int PO_CANDI = PO_CANDV + 8 * 4;
constexpr int PO_FLAG = PO_CANDI + 8 * 4;
constexpr int PO_YBUF = PO_FLAG + 4 * 4;
constexpr int PO_PROD = PO_YBUF + 2 * 64 * 4;
static_assert(PO_PROD + 256 <= PS_SMEM - 128, "persistent shared-memory layout");

struct PSmem {
  uint8_t *b;
  __device__ __forceinline__ uint8_t *ring() const { return b; }
  __device__ __forceinline__ float *scratch() const { return reinterpret_cast<float *>(b + PO_SCRATCH); }
  __device__ __forceinline__ uint8_t *codes() const { return b + PO_CODES; }
  __device__ __forceinline__ float *rscale() const { return reinterpret_cast<float *>(b + PO_RSCALE); }
  __device__ __forceinline__ uint64_t *full() const { return reinterpret_cast<uint64_t *>(b + PO_FULL); }
  __device__ __forceinline__ uint64_t *vbar() const { return reinterpret_cast<uint64_t *>(b + PO_VBAR); }
  __device__ __forceinline__ int *xsum() const { return reinterpret_cast<int *>(b + PO_XSUM); }
  __device__ __forceinline__ float *red() const { return reinterpret_cast<float *>(b + PO_RED); }
  __device__ __forceinline__ float *cand_v() const { return reinterpret_cast<float *>(b + PO_CANDV); }
  __device__ __forceinline__ int *cand_i() const { return reinterpret_cast<int *>(b + PO_CANDI); }
  __device__ __forceinline__ int *flag() const { return reinterpret_cast<int *>(b + PO_FLAG); }
  __device__ __forceinline__ float *ybuf() const { return reinterpret_cast<float *>(b + PO_YBUF); }
};

// This CTA's row slices of a GEMV phase: a pair owns the same rows of both segments; otherwise
// the CTA sits in one segment's block range (the partition was made for gridDim.x CTAs).
struct PSlices {
  int nsub, seg[2], r0[2], r1[2], row_bytes, srows, nch[2];
};

__device__ __forceinline__ PSlices p_slices(const PPhase &ph, int bid) {
  const GemvArgs &a = ph.g;
  PSlices s;
  s.row_bytes = a.K * ph.bits / 8;
  s.srows = PS_SLOT / s.row_bytes;
  s.nsub = 0;
  if (bid >= a.n_blocks_total) return s;
  if (a.pair) {
    const int nb = a.n_blocks_total;
    const int r0 = (int)(((long long)a.seg[0].N * bid) / nb), r1 = (int)(((long long)a.seg[0].N * (bid + 1)) / nb);
    s.nsub = 2;
    for (int i = 0; i < 2; i++) {
      s.seg[i] = i;
      s.r0[i] = r0;
      s.r1[i] = r1;
    }
  } else {
    int g = 0;
    if (a.nseg > 1 && bid >= a.seg[1].block_begin) g = 1;
    if (a.nseg > 2 && bid >= a.seg[2].block_begin) g = 2;
    const int nb = (g + 1 < a.nseg ? a.seg[g + 1].block_begin : a.n_blocks_total) - a.seg[g].block_begin;
    const int ib = bid - a.seg[g].block_begin;
    s.nsub = 1;
    s.seg[0] = g;
    s.r0[0] = (int)(((long long)a.seg[g].N * ib) / nb);
    s.r1[0] = (int)(((long long)a.seg[g].N * (ib + 1)) / nb);
  }
  for (int i = 0; i < s.nsub; i++) s.nch[i] = (s.r1[i] - s.r0[i] + s.srows - 1) / s.srows;
  return s;
}

// The weight producer (thread 0): walks the GEMV chunks of this CTA in consumption order.
struct PProducer {
  int p;          // phase of the next chunk
  int sub, ci;    // position inside that phase
  PSlices sl;
  bool have;      // sl describes phase p
  uint32_t issued;
};

__device__ __forceinline__ bool producer_next(PProducer &pr, const PPhase *ph, int nph, int bid,
                                              const uint8_t **src, uint32_t *bytes) {
  while (pr.p < nph) {
    if (ph[pr.p].kind != PK_GEMV) {
      pr.p++;
      pr.have = false;
      continue;
    }
    if (!pr.have) {
      pr.sl = p_slices(ph[pr.p], bid);
      pr.sub = 0;
      pr.ci = 0;
      pr.have = true;
    }
    while (pr.sub < pr.sl.nsub && pr.ci >= pr.sl.nch[pr.sub]) {
      pr.sub++;
      pr.ci = 0;
    }
    if (pr.sub >= pr.sl.nsub) {
      pr.p++;
      pr.have = false;
      continue;
    }
    const GemvSeg &sg = ph[pr.p].g.seg[pr.sl.seg[pr.sub]];
    const int cr0 = pr.sl.r0[pr.sub] + pr.ci * pr.sl.srows;
    const int rows = min(pr.sl.srows, pr.sl.r1[pr.sub] - cr0);
    *src = sg.w + (size_t)cr0 * pr.sl.row_bytes;
    *bytes = (uint32_t)(rows * pr.sl.row_bytes);
    pr.ci++;
    return true;
  }
  return false;
}

__device__ __forceinline__ void producer_issue(PProducer &pr, const PPhase *ph, int nph, int bid,
                                               const PSmem &S) {
  const uint8_t *src;
  uint32_t bytes;
  if (!producer_next(pr, ph, nph, bid, &src, &bytes)) return;
  const int slot = pr.issued % PS_NSLOT;
  mbar_expect_tx(&S.full()[slot], bytes);
  bulk_g2s(S.ring() + (size_t)slot * PS_SLOT, src, bytes, &S.full()[slot]);
  pr.issued++;
}

// Grid barrier over the gridDim.x resident CTAs: arrival count plus a generation word, bounded.
__device__ __forceinline__ void grid_sync(unsigned *bar, unsigned &gen, const PSmem &S) {
  __syncthreads();
  if (threadIdx.x == 0 && !S.flag()[0]) {
    __threadfence();
    const unsigned arrived = atomicAdd(bar, 1u);
    if (arrived == gridDim.x - 1) {
      atomicExch(bar, 0u);
      __threadfence();
      atomicAdd(bar + 1, 1u);
    } else {
      unsigned v = gen;
      for (int it = 0; it < (1 << 22) && v == gen; it++)
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar + 1) : "memory");
      if (v == gen) {
        atomicExch(&g4_persist_error, 3);
        S.flag()[0] = 1;
      }
    }
    gen++;
    __threadfence();
  }
  __syncthreads();
}

// ------------------------------------------------------------------ GEMV phase
template <int BITS, int RS, int PRO, int EPI>
__device__ __noinline__ void p_gemv(const PPhase &ph, const PPhase *all, int nph, int bid, const PSmem &S,
                       uint32_t &qc, PProducer &pr) {
  const GemvArgs &a = ph.g;
  constexpr bool pair = EPI == EPI_GELU_CODES && PRO == PRO_JOIN;
  constexpr bool keep_y = EPI == EPI_GELU_CODES;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const PSlices sl = p_slices(ph, bid);
  const int K = a.K;
  const int vb = sl.row_bytes / RS;
  // Row scales of this CTA's rows (independent loads, consumed by the epilogues).
  for (int sub = 0; sub < sl.nsub; sub++)
    for (int i = t; i < sl.r1[sub] - sl.r0[sub]; i += 256)
      S.rscale()[sub * (PS_RSCALE / 2) + i] = f16_bits_to_f32(__ldg(a.seg[sl.seg[sub]].s + sl.r0[sub] + i));
  if (t < 16) S.xsum()[t] = 0;
  ProGains pg;
  prologue_gains<PRO>(a, pg);
  __syncthreads();
  {
    // Codes snapped with this CTA's segment's input scale (q, k and v each have their own).
    const float in0 = sl.nsub ? a.seg[sl.seg[0]].in_scale : a.seg[0].in_scale;
    int x2 = 0;
    const int v = warp_sum_int(gemv_prologue_col<BITS, PRO>(
        a, pg, 0, in0, S.codes(), S.red(), bid == 0 && a.hidden_out != nullptr,
        pair ? a.seg[1].in_scale : 0.0f, pair ? S.codes() + K : nullptr, &x2));
    if (lane == 0) atomicAdd(&S.xsum()[0], v);
    if (pair) {
      x2 = warp_sum_int(x2);
      if (lane == 0) atomicAdd(&S.xsum()[8], x2);
    }
  }
  __syncthreads();
  float best_v = -FLT_MAX;
  int best_i = 0x7fffffff;
  for (int sub = 0; sub < sl.nsub; sub++) {
    const GemvSeg &sg = a.seg[sl.seg[sub]];
    const float out_r = sg.out_scale != 0.0f ? __fdiv_rn(1.0f, sg.out_scale) : 0.0f;
    const uint8_t *ccodes = S.codes() + (pair ? sub * K : 0);
    const int xs = S.xsum()[sub * 8];
    for (int ci = 0; ci < sl.nch[sub]; ci++) {
      const int slot = qc % PS_NSLOT;
      if (!S.flag()[0] && !mbar_wait(&S.full()[slot], (qc / PS_NSLOT) & 1)) {
        if (t == 0) atomicExch(&g4_persist_error, 1);
        S.flag()[0] = 1;
      }
      const int cr0 = sl.r0[sub] + ci * sl.srows;
      const int vrows = min(sl.srows, sl.r1[sub] - cr0) * RS;
      const uint8_t *sw = S.ring() + (size_t)slot * PS_SLOT;
      for (int g0 = warp * 4; g0 < vrows; g0 += 32) {
        int acc[4] = {0, 0, 0, 0};
        for (int off = lane * 16; off < vb; off += 512) {
          uint4 w[4];
          int koff[4];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const int vr = g0 + q;
            koff[q] = (vr % RS) * vb + off;
            w[q] = vr < vrows ? *reinterpret_cast<const uint4 *>(sw + (size_t)vr * vb + off)
                              : make_uint4(0, 0, 0, 0);
          }
          constexpr int NX = RS == 1 ? 1 : (RS == 2 ? 2 : 4);
          uint4 xa[NX], xb[NX];
#pragma unroll
          for (int j = 0; j < NX; j++) {
            if (BITS == 4) {
              const uint4 *xp = reinterpret_cast<const uint4 *>(ccodes + 2 * koff[j]);
              xa[j] = xp[0];
              xb[j] = xp[1];
            } else {
              xa[j] = *reinterpret_cast<const uint4 *>(ccodes + koff[j]);
            }
          }
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const uint4 x01 = xa[q % NX];
            int v = acc[q];
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
            acc[q] = v;
          }
        }
        // The transposed reduction of k_qgemv_stream (integer adds: order free).
        const bool hi16 = lane >= 16, hi8 = (lane & 8) != 0;
        const int my_vrow = (hi16 ? 2 : 0) + (hi8 ? 1 : 0);
        int b0 = (hi16 ? acc[2] : acc[0]) + __shfl_xor_sync(0xffffffffu, hi16 ? acc[0] : acc[2], 16);
        int b1 = (hi16 ? acc[3] : acc[1]) + __shfl_xor_sync(0xffffffffu, hi16 ? acc[1] : acc[3], 16);
        int v = (hi8 ? b1 : b0) + __shfl_xor_sync(0xffffffffu, hi8 ? b0 : b1, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        if (RS >= 2) v += __shfl_xor_sync(0xffffffffu, v, 8);
        if (RS >= 4) v += __shfl_xor_sync(0xffffffffu, v, 16);
        const int vr = g0 + my_vrow;
        if ((lane & (8 * RS - 1)) == 0 && vr < vrows) {
          const int row = cr0 + vr / RS;
          const float wscale = S.rscale()[sub * (PS_RSCALE / 2) + row - sl.r0[sub]];
          const int exact = BITS == 4 ? v - 8 * xs : v;
          float y = __fmul_rn(__fmul_rn(sg.in_scale, wscale), (float)exact);
          y = srq_out_r(y, sg.out_scale, out_r);
          if (keep_y) {
            S.ybuf()[sub * 64 + row - sl.r0[sub]] = y;
          } else if (EPI == EPI_HEAD) {
            if (a.softcap != 0.0f) y = __fmul_rn(g4_tanh(__fdiv_rn(y, a.softcap)), a.softcap);
            if (a.logits) a.logits[row] = y;
            if (y > best_v || (y == best_v && row < best_i)) {
              best_v = y;
              best_i = row;
            }
          } else {
            sg.y[row] = y;
          }
        }
      }
      __syncthreads();
      if (t == 0 && !S.flag()[0]) producer_issue(pr, all, nph, bid, S);
      qc++;
    }
  }
  if (keep_y && sl.nsub > 0) {
    const int rows = sl.r1[0] - sl.r0[0];
    const float cr = __fdiv_rn(1.0f, a.codes_scale);
    for (int i = t; i < rows; i += 256) {
      const float g = S.ybuf()[i];
      const float u = pair ? S.ybuf()[64 + i] : a.epi_up[a.epi_up_off + sl.r0[0] + i];
      const float h = __fmul_rn(g4_gelu(g), u);
      a.codes_out[code_pos(sl.r0[0] + i, a.codes_bits)] = (uint8_t)(srq_code_r(h, a.codes_scale, cr) & 255);
    }
  }
  if (EPI == EPI_HEAD) {
#pragma unroll
    for (int o = 8; o < 32; o <<= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ov > best_v || (ov == best_v && oi < best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    if (lane == 0) {
      S.cand_v()[warp] = best_v;
      S.cand_i()[warp] = best_i;
    }
    __syncthreads();
    if (t == 0 && bid < a.n_blocks_total) {
      float bv = -FLT_MAX;
      int bi = 0x7fffffff;
      for (int w = 0; w < 8; w++)
        if (S.cand_v()[w] > bv || (S.cand_v()[w] == bv && S.cand_i()[w] < bi)) {
          bv = S.cand_v()[w];
          bi = S.cand_i()[w];
        }
      a.part_val[bid] = bv;
      a.part_idx[bid] = bi;
    }
  }
}

// ------------------------------------------------------------------ attention phase
// Work items (block, head) of the one column; item i runs on CTA i mod gridDim.x. Per item the
// arithmetic of k_attn_decode<HD, 1>: the new position's K/V rows (stored by head 0's item), the
// four-accumulator scores, block max, exp, the ascending l and o chains (V staged in shared
// memory PS_SCRATCH bytes at a time), the partial, and the merge by the last item of the head.
template <int HD>
__device__ __noinline__ void p_attn(const AttnDec &a, int bid, const PSmem &S, uint32_t &vuse) {
  constexpr int NH = 8, NC = HD / 4;
  constexpr int VROWS = PS_SCRATCH / (HD * 4) < ATT_BLK ? PS_SCRATCH / (HD * 4) : ATT_BLK;
  float *vs = S.scratch();                          // [VROWS][HD]
  float *qs = S.rscale();                           // [HD]   (free during attention)
  float *kc = qs + HD;                            // [HD]
  float *vc = kc + HD;                            // [HD]   V row of the new position
  float *ss = vc + HD;                            // [64]   scores, then probabilities
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  int p, lo, hi;
  {
    AttnArgs r;
    r.refs = a.refs;
    r.window = a.window;
    r.kv_cap = 0;
    attn_range(r, 0, &p, &lo, &hi);
  }
  const int nb = hi / ATT_BLK - lo / ATT_BLK + 1;
  const int seq = a.refs.seq ? a.refs.seq[0] : 0;
  float *K = a.cache + (size_t)seq * a.seq_stride;
  float *V = K + (size_t)a.max_ctx * HD;
  for (int item = bid; item < nb * NH; item += gridDim.x) {
    const int bi = item / NH, h = item % NH;
    const int b = lo / ATT_BLK + bi;
    const int j0 = max(b * ATT_BLK, lo), j1 = min(b * ATT_BLK + ATT_BLK - 1, hi);
    const bool cur = a.k != nullptr && j1 == p;
    const float *ct = a.cos_tab + (size_t)p * (HD / 2);
    const float *stb = a.sin_tab + (size_t)p * (HD / 2);
    if (w == 0)
      head_norm_rope_warp<HD>(a.q + (size_t)h * HD, a.qgain, ct, stb, a.eps, qs, nullptr, lane);
    if (cur && w == 1)
      head_norm_rope_warp<HD>(a.k, a.kgain, ct, stb, a.eps, kc, h == 0 ? K + (size_t)p * HD : nullptr, lane);
    if (cur && w == 2)
      head_norm_rope_warp<HD>(a.v, nullptr, nullptr, nullptr, a.eps, vc, h == 0 ? V + (size_t)p * HD : nullptr, lane);
    __syncthreads();
    // Scores: thread (jl, m), accumulator m of position jl.
    {
      const int jl = t >> 2, m = t & 3;
      const int j = b * ATT_BLK + jl;
      const bool valid = j >= j0 && j <= j1;
      float acc = 0.0f;
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
            const float4 q4 = reinterpret_cast<const float4 *>(qs)[m + 4 * (i0 + i)];
            acc = fmaf(q4.x, k4[i].x, acc);
            acc = fmaf(q4.y, k4[i].y, acc);
            acc = fmaf(q4.z, k4[i].z, acc);
            acc = fmaf(q4.w, k4[i].w, acc);
          }
        }
      }
      const float v1 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
      const float v2 = __fadd_rn(v1, __shfl_xor_sync(0xffffffffu, v1, 2));
      if (m == 0) ss[jl] = valid ? v2 : -FLT_MAX;
    }
    __syncthreads();
    float mx;
    {
      const float s0 = ss[lane], s1 = ss[lane + 32];
      mx = fmaxf(s0, s1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      __syncthreads();
      if (w == 0) {
        const int ja = b * ATT_BLK + lane, jb = ja + 32;
        ss[lane] = (ja >= j0 && ja <= j1) ? g4_exp(__fsub_rn(s0, mx)) : 0.0f;
        ss[lane + 32] = (jb >= j0 && jb <= j1) ? g4_exp(__fsub_rn(s1, mx)) : 0.0f;
      }
    }
    // Weighted V, ascending j, V staged VROWS rows at a time (thread dc < NC).
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    float l = 0.0f;
    const int dc = t;
    for (int s0 = b * ATT_BLK; s0 < b * ATT_BLK + ATT_BLK; s0 += VROWS) {
      const int sj0 = max(s0, j0), sj1 = min(s0 + VROWS - 1, cur ? p - 1 : j1);
      __syncthreads();   // the previous stage's V rows are no longer read
      if (sj1 >= sj0 && t == 0) {
        mbar_expect_tx(S.vbar(), (uint32_t)(sj1 - sj0 + 1) * HD * 4);
        bulk_g2s(vs + (size_t)(sj0 - s0) * HD, V + (size_t)sj0 * HD, (uint32_t)(sj1 - sj0 + 1) * HD * 4, S.vbar());
      }
      if (sj1 >= sj0) {
        if (!mbar_wait(S.vbar(), vuse & 1)) {
          if (t == 0) atomicExch(&g4_persist_error, 2);
          mbar_wait(S.vbar(), vuse & 1);
        }
        vuse++;
      }
      __syncthreads();
      if (dc < NC) {
        const int e1 = min(s0 + VROWS - 1, j1);
        for (int j = max(s0, j0); j <= e1; j++) {
          const float4 v4 = (cur && j == p) ? reinterpret_cast<const float4 *>(vc)[dc]
                                            : reinterpret_cast<const float4 *>(vs + (size_t)(j - s0) * HD)[dc];
          const float pj = ss[j - b * ATT_BLK];
          o.x = fmaf(pj, v4.x, o.x);
          o.y = fmaf(pj, v4.y, o.y);
          o.z = fmaf(pj, v4.z, o.z);
          o.w = fmaf(pj, v4.w, o.w);
          l = __fadd_rn(l, pj);
        }
      }
    }
    if (nb == 1) {
      if (dc < NC) {
        float4 r;
        r.x = __fdiv_rn(o.x, l);
        r.y = __fdiv_rn(o.y, l);
        r.z = __fdiv_rn(o.z, l);
        r.w = __fdiv_rn(o.w, l);
        reinterpret_cast<float4 *>(a.out + (size_t)h * HD)[dc] = r;
      }
      __syncthreads();
      continue;
    }
    const size_t slot = (size_t)bi * NH + h;
    if (dc < NC) {
      reinterpret_cast<float4 *>(a.part_o + slot * HD)[dc] = o;
      if (dc == 0) {
        a.part_m[slot] = mx;
        a.part_l[slot] = l;
      }
    }
    __threadfence();
    __syncthreads();
    int *cnt = a.counter + h;
    if (t == 0) S.flag()[1] = atomicAdd(cnt, 1) == nb - 1;
    __syncthreads();
    if (S.flag()[1]) {
      __threadfence();
      // k_attn_merge's fold for head h, blocks 0..nb-1 in ascending order.
      if (t < NC) {
        float M = __ldcg(a.part_m + h), L = __ldcg(a.part_l + h);
        float4 O = __ldcg(reinterpret_cast<const float4 *>(a.part_o + (size_t)h * HD) + t);
        for (int k2 = 1; k2 < nb; k2++) {
          const size_t sk = (size_t)k2 * NH + h;
          const float mm = __ldcg(a.part_m + sk), ll = __ldcg(a.part_l + sk);
          const float4 ok = __ldcg(reinterpret_cast<const float4 *>(a.part_o + sk * HD) + t);
          const float Mn = fmaxf(M, mm);
          const float e1 = g4_exp(__fsub_rn(M, Mn)), e2 = g4_exp(__fsub_rn(mm, Mn));
          L = __fadd_rn(__fmul_rn(L, e1), __fmul_rn(ll, e2));
          O.x = __fadd_rn(__fmul_rn(O.x, e1), __fmul_rn(ok.x, e2));
          O.y = __fadd_rn(__fmul_rn(O.y, e1), __fmul_rn(ok.y, e2));
          O.z = __fadd_rn(__fmul_rn(O.z, e1), __fmul_rn(ok.z, e2));
          O.w = __fadd_rn(__fmul_rn(O.w, e1), __fmul_rn(ok.w, e2));
          M = Mn;
        }
        float4 r;
        r.x = __fdiv_rn(O.x, L);
        r.y = __fdiv_rn(O.y, L);
        r.z = __fdiv_rn(O.z, L);
        r.w = __fdiv_rn(O.w, L);
        reinterpret_cast<float4 *>(a.out + (size_t)h * HD)[t] = r;
      }
      if (t == 0) *cnt = 0;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ small phases
__device__ __noinline__ void p_embed(const PEmbed &e, int bid) {
  const int hw = e.H / 8, pw = e.ple_cols / 8;
  const int row = e.tokens[0];
  for (int w = bid * 256 + threadIdx.x; w < hw + pw; w += gridDim.x * 256) {
    uint32_t word;
    float scale;
    float *dst;
    if (w < hw) {
      word = reinterpret_cast<const uint32_t *>(e.embed_w)[(size_t)row * hw + w];
      scale = __fmul_rn(e.embed_scale, f16_bits_to_f32(e.embed_s[row]));
      dst = e.residual + 8 * w;
    } else {
      const int wp = w - hw;
      const int slice = row / e.ple_rps, local = row - slice * e.ple_rps;
      word = reinterpret_cast<const uint32_t *>(e.ple_slices[slice])[(size_t)local * pw + wp];
      const int groups = e.ple_cols / e.ple_group;
      scale = __fmul_rn(16.0f, f16_bits_to_f32(e.ple_s[(size_t)row * groups + (8 * wp) / e.ple_group]));
      dst = e.ple_id + 8 * wp;
    }
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __fmul_rn((float)((int)((word >> (4 * j)) & 15u) - 8), scale);
    reinterpret_cast<float4 *>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4 *>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// k_dense_bf16<1>: warp per row, lane l walks chunks l, l + 32, ..., butterfly, alpha.
__device__ __noinline__ void p_dense(const PDense &d, int bid, const PSmem &S) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float *xs = S.scratch();
  for (int i = t; i < d.K / 4; i += 256) reinterpret_cast<float4 *>(xs)[i] = reinterpret_cast<const float4 *>(d.x)[i];
  __syncthreads();
  const int nch = d.K / 8;
  for (int row = bid * 8 + warp; row < d.N; row += gridDim.x * 8) {
    float acc = 0.0f;
    constexpr int MAXCH = 8;
    uint4 wv[MAXCH];
#pragma unroll
    for (int i = 0; i < MAXCH; i++) {
      const int ch = lane + 32 * i;
      wv[i] = ch < nch ? ldg_stream(d.w + (size_t)row * d.K + 8 * ch) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < MAXCH; i++) {
      const int ch = lane + 32 * i;
      if (ch < nch) {
        const uint32_t ww[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
        const float4 xa = reinterpret_cast<const float4 *>(xs + 8 * ch)[0];
        const float4 xb = reinterpret_cast<const float4 *>(xs + 8 * ch)[1];
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float wf = (j & 1) ? __uint_as_float(ww[j >> 1] & 0xffff0000u) : __uint_as_float(ww[j >> 1] << 16);
          acc = fmaf(wf, xv[j], acc);
        }
      }
    }
    const float sum = warp_sum_bfly(acc);
    if (lane == 0) d.y[row] = __fmul_rn(d.alpha, sum);
  }
}

// k_ple_combine: group g on CTA g.
__device__ __noinline__ void p_combine(const PCombine &c, int bid, const PSmem &S) {
  for (int g = bid; g < c.groups; g += gridDim.x) {
    const size_t base = (size_t)g * c.group_dim;
    const float inv = rms_inv(block_sumsq256(c.proj + base, c.group_dim, S.red()), c.group_dim, c.eps);
    for (int ch = threadIdx.x; ch < c.group_dim / 4; ch += 256) {
      const float4 p = reinterpret_cast<const float4 *>(c.proj + base)[ch];
      const float4 id = reinterpret_cast<const float4 *>(c.identity + base)[ch];
      const float4 gg = reinterpret_cast<const float4 *>(c.gain)[ch];
      reinterpret_cast<float4 *>(c.out + base)[ch] = f4_scale(f4_add(f4_norm_apply(p, inv, gg), id), c.scale);
    }
    __syncthreads();
  }
}

// k_argmax_final on CTA 0 (greatest value, lowest index), then the position advance.
__device__ __noinline__ void p_argmax(const PArgmax &m, int bid, const PSmem &S) {
  if (bid != 0) return;
  const int t = threadIdx.x, lane = t & 31;
  float bv = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = t; i < m.n_parts; i += 256) {
    const float v = m.part_val[i];
    const int ix = m.part_idx[i];
    if (v > bv || (v == bv && ix < bi)) {
      bv = v;
      bi = ix;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    S.cand_v()[t >> 5] = bv;
    S.cand_i()[t >> 5] = bi;
  }
  __syncthreads();
  if (t == 0) {
    for (int w = 1; w < 8; w++)
      if (S.cand_v()[w] > bv || (S.cand_v()[w] == bv && S.cand_i()[w] < bi)) {
        bv = S.cand_v()[w];
        bi = S.cand_i()[w];
      }
    if (m.token_dev) m.token_dev[0] = bi;
    if (m.token_out) m.token_out[0] = bi;
    if (m.value_out) m.value_out[0] = bv;
    if (m.advance) m.pos[0] += 1;
  }
}

template <int BITS, int PRO, int EPI>
__device__ __forceinline__ void p_gemv_rs(const PPhase &P, const PPhase *ph, int nph, int bid,
                                          const PSmem &S, uint32_t &qc, PProducer &pr) {
  if (P.rs == 1) p_gemv<BITS, 1, PRO, EPI>(P, ph, nph, bid, S, qc, pr);
  else if (P.rs == 2) p_gemv<BITS, 2, PRO, EPI>(P, ph, nph, bid, S, qc, pr);
  else p_gemv<BITS, 4, PRO, EPI>(P, ph, nph, bid, S, qc, pr);
}

__device__ __forceinline__ void p_gemv_dispatch(const PPhase &P, const PPhase *ph, int nph, int bid,
                                                const PSmem &S, uint32_t &qc, PProducer &pr) {
  switch (P.variant) {
    case PV_Q0: p_gemv_rs<4, PRO_NORM, EPI_Y>(P, ph, nph, bid, S, qc, pr); break;
    case PV_QKV: p_gemv_rs<4, PRO_JOIN, EPI_Y>(P, ph, nph, bid, S, qc, pr); break;
    case PV_O1:
    case PV_O2: p_gemv_rs<4, PRO_X, EPI_Y>(P, ph, nph, bid, S, qc, pr); break;
    case PV_GATEUP: p_gemv_rs<4, PRO_JOIN, EPI_GELU_CODES>(P, ph, nph, bid, S, qc, pr); break;
    case PV_DOWN: p_gemv_rs<4, PRO_CODES, EPI_Y>(P, ph, nph, bid, S, qc, pr); break;
    case PV_PLEG: p_gemv_rs<8, PRO_NORMRES, EPI_GELU_CODES>(P, ph, nph, bid, S, qc, pr); break;
    case PV_PLEP: p_gemv_rs<8, PRO_CODES, EPI_Y>(P, ph, nph, bid, S, qc, pr); break;
    case PV_HEAD: p_gemv_rs<4, PRO_JOIN, EPI_HEAD>(P, ph, nph, bid, S, qc, pr); break;
    default:
      if (threadIdx.x == 0) atomicExch(&g4_persist_error, 4);
      S.flag()[0] = 1;
      break;
  }
}

// ------------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(256, 1) k_decode_persist(const PPhase *ph, int nph, unsigned *bar) {
  extern __shared__ __align__(1024) uint8_t psm_raw[];
  uint8_t *base = psm_raw + ((128 - (smem_u32(psm_raw) & 127)) & 127);
  PSmem S;
  S.b = base;
  const int bid = blockIdx.x, t = threadIdx.x;
  unsigned gen = 0;
  PProducer &pr = *reinterpret_cast<PProducer *>(base + PO_PROD);   // thread 0's state
  if (t == 0) {
    pr.p = 0;
    pr.have = false;
    pr.issued = 0;
  }
  if (t == 0) {
    for (int i = 0; i < PS_NSLOT; i++) mbar_init(&S.full()[i], 1);
    mbar_init(S.vbar(), 1);
    mbar_fence_init();
    S.flag()[0] = 0;
    S.flag()[1] = 0;
  }
  __syncthreads();
  grid_launch_dependents();
  if (t == 0) {
    // Weights do not depend on the step: fill the ring before waiting for the previous kernel.
    for (int i = 0; i < PS_NSLOT; i++) producer_issue(pr, ph, nph, bid, S);
  }
  grid_wait();
  if (t == 0) asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(gen) : "l"(bar + 1) : "memory");
  uint32_t qc = 0, vuse = 0;
  for (int i = 0; i < nph && !S.flag()[0]; i++) {
    const PPhase &P = ph[i];
    P_TRACE(P.kind * 100 + P.variant);
    switch (P.kind) {
      case PK_EMBED: p_embed(P.em, bid); break;
      case PK_DENSE: p_dense(P.de, bid, S); break;
      case PK_COMBINE: p_combine(P.co, bid, S); break;
      case PK_ATTN:
        if (P.at.hd == 256) p_attn<256>(P.at, bid, S, vuse);
        else p_attn<512>(P.at, bid, S, vuse);
        break;
      case PK_ARGMAX: p_argmax(P.am, bid, S); break;
      case PK_GEMV:
        p_gemv_dispatch(P, ph, nph, bid, S, qc, pr);
        break;
      default: break;
    }
    P_TRACE(10000 + P.kind * 100 + P.variant);
    if (P.sync_after) grid_sync(bar, gen, S);
  }
  // Copies issued and not consumed (only after an abort) land before the CTA leaves.
  if (t == 0)
    for (uint32_t q = qc; q < pr.issued; q++) mbar_wait(&S.full()[q % PS_NSLOT], (q / PS_NSLOT) & 1);
  __syncthreads();
}

cudaError_t launch_decode_persist(const PPhase *ph, int nph, unsigned *bar, int grid,
                                  cudaStream_t st) {
  static DeviceOnce attr;
  attr([&] {
    cudaFuncSetAttribute(k_decode_persist, cudaFuncAttributeMaxDynamicSharedMemorySize, PS_SMEM);
  });
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = PS_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_decode_persist, ph, nph, bar);
}

int persist_max_grid(int device) {
  int per_sm = 0, sms = 0;
  cudaFuncSetAttribute(k_decode_persist, cudaFuncAttributeMaxDynamicSharedMemorySize, PS_SMEM);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_persist, 256, PS_SMEM) != cudaSuccess)
    return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  return per_sm >= 1 ? sms : 0;
}

}  // namespace g4
