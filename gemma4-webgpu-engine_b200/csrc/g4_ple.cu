// The per-layer-input tail of a decode step (src/plan.ts:669-754) as ONE launch on one
// thread-block cluster: the post-FFN norm-residual (the residual stream, and the gate's int8
// input codes), per_layer_input_gate (int8 [PD x H]), gelu(gate) * the layer's per-layer input
// snapped to per_layer_projection's codes, and per_layer_projection (int8 [H x PD])
// (src/kernels/pleMatmul.ts, src/kernels/geluMul.ts:67-115).
//
// As two streaming-GEMV launches this tail pays two launch links and two prologues for under a
// megabyte of weights. Here a cluster of 16 CTAs runs it: CTA r requests its 16 gate rows and
// its H / 16 projection rows by bulk copy before the dependency wait; after the wait each CTA
// runs the norm-residual prologue (as each GEMV CTA does), then its gate rows over all H codes,
// and writes their 16 codes per column into every CTA's shared memory (distributed shared
// memory); after one cluster barrier each CTA runs its projection rows over all PD codes.
// The launch reads `src` before the barrier and writes `y` after it, so the two may alias (the
// decode chain passes the same buffer).
//
// Arithmetic: the prologue is the GEMV's own (gemv_prologue_col), the dots are exact int32
// dp4a sums (any order), and the epilogues are the GEMV's (y = srqOut(in_scale * row_scale *
// acc); h = gelu(y) * u; code = srq_code(h)), so the launch gives the two GEMVs' bits.
//
// Sized for decode columns: 1..16 per launch. Batches of 16 and more go through the tensor-core
// GEMMs; on the CUDA cores this form's dp4a work grows with the columns and, at 16 to 64
// columns, took longer than the two GEMMs and the quantize between them.
#include <float.h>
#include "g4_device.cuh"
#include "g4_kernels.cuh"
#include "g4_gemv.cuh"

namespace g4 {

__device__ int g4_ple_error;   // 1: the weight copies never completed (bounded wait gave up)

#ifdef G4_TRACE
// Diagnostic build: this unit's record buffer (device variables are per unit).
__device__ unsigned long long g4_trace_buf[1 << 16];
__device__ unsigned int g4_trace_n;
int ple_trace_take(unsigned long long *out, int max_records) {
  unsigned int n = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&n, g4_trace_n, sizeof(n)) != cudaSuccess) return -1;
  if (n > (1u << 15)) n = 1u << 15;
  if ((int)n > max_records) n = (unsigned int)max_records;
  if (n && cudaMemcpyFromSymbol(out, g4_trace_buf, (size_t)n * 16) != cudaSuccess) return -1;
  cudaMemcpyToSymbol(g4_trace_n, &zero, sizeof(zero));
  return (int)n;
}
#endif

int *ple_error_addr() {
  void *p = nullptr;
  return cudaGetSymbolAddress(&p, g4_ple_error) == cudaSuccess ? (int *)p : nullptr;
}

int ple_error_take() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g4_ple_error, sizeof(int)) != cudaSuccess) return 0;
  if (v) cudaMemcpyToSymbol(g4_ple_error, &z, sizeof(int));
  return v;
}

constexpr int PB_CS = 16;       // CTAs in the cluster
constexpr int PB_R1 = 16;       // gate rows per CTA (PD = 256)
constexpr int PB_PD = PB_CS * PB_R1;
constexpr int PB_NC = 4;        // columns per register group
constexpr int PB_MAXC = 16;     // columns per launch

__device__ __forceinline__ uint32_t pb_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t pb_mapa(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ int dp4a_x4(uint4 w, uint4 x, int v) {
  v = dp4a_ss(w.x, x.x, v);
  v = dp4a_ss(w.y, x.y, v);
  v = dp4a_ss(w.z, x.z, v);
  return dp4a_ss(w.w, x.w, v);
}

struct PbLayout {
  size_t w1, w2, s1, s2, cin, c2, own, red, bar, total;
};
__host__ __device__ inline size_t pb_align(size_t x) { return (x + 127) & ~(size_t)127; }
__host__ __device__ inline PbLayout pb_layout(int H, int cols) {
  PbLayout L;
  const int R2 = H / PB_CS;
  size_t o = 0;
  L.w1 = o; o = pb_align(o + (size_t)PB_R1 * H);       // this CTA's gate rows
  L.w2 = o; o = pb_align(o + (size_t)R2 * PB_PD);      // this CTA's projection rows
  L.s1 = o; o = pb_align(o + PB_R1 * 4);
  L.s2 = o; o = pb_align(o + (size_t)R2 * 4);
  L.cin = o; o = pb_align(o + (size_t)cols * H);       // the gate's input codes (K order)
  L.c2 = o; o = pb_align(o + (size_t)cols * PB_PD);    // the projection's input codes (all CTAs')
  L.own = o; o = pb_align(o + (size_t)cols * PB_R1);   // this CTA's 16 codes per column
  L.red = o; o = pb_align(o + 32 * 4);
  L.bar = o; o = pb_align(o + 8);
  L.total = o;
  return L;
}

__global__ void __launch_bounds__(256, 2) k_ple_block(const PleArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int H = a.H, cols = a.cols, R2 = H / PB_CS;
  const PbLayout L = pb_layout(H, cols);
  uint8_t *w1s = sm + L.w1, *w2s = sm + L.w2, *cin = sm + L.cin, *c2 = sm + L.c2, *own = sm + L.own;
  float *s1f = reinterpret_cast<float *>(sm + L.s1), *s2f = reinterpret_cast<float *>(sm + L.s2);
  float *red = reinterpret_cast<float *>(sm + L.red);
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm + L.bar);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int r = (int)pb_rank();
  if (t == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  // Weights (both slices), row scales and the norm gain before the dependency wait.
  if (t == 0) {
    mbar_expect_tx(bar, (uint32_t)(PB_R1 * H + R2 * PB_PD));
    bulk_g2s(w1s, a.w1 + (size_t)r * PB_R1 * H, (uint32_t)(PB_R1 * H), bar);
    bulk_g2s(w2s, a.w2 + (size_t)r * R2 * PB_PD, (uint32_t)(R2 * PB_PD), bar);
  }
  if (t == 32)
    for (int i = 0; i < 4; i++) l2_prefetch_share(a.prefetch[i], a.prefetch_bytes[i], r, PB_CS);
  for (int i = t; i < PB_R1; i += 256) s1f[i] = f16_bits_to_f32(__ldg(a.s1 + r * PB_R1 + i));
  for (int i = t; i < R2; i += 256) s2f[i] = f16_bits_to_f32(__ldg(a.s2 + r * R2 + i));
  GemvArgs g = {};
  g.pro = PRO_NORMRES;
  g.K = H;
  g.src = a.src;
  g.ld_src = a.ld_src;
  g.res = a.res;
  g.ld_res = a.ld_res;
  g.g1 = a.g1;
  g.eps = a.eps;
  g.alpha = 1.0f;
  g.hidden_out = a.hidden_out;
  ProGains pg;
  prologue_gains<PRO_NORMRES>(g, pg);
  grid_launch_dependents();
  grid_wait();
  G4_TRACE_POINT(3010);

  // The norm-residual of every column, snapped to the gate's codes (CTA 0 writes the residual).
#pragma unroll 1
  for (int c = 0; c < cols; c++)
    gemv_prologue_col<8, PRO_NORMRES>(g, pg, c, a.in1, cin + (size_t)c * H, red,
                                      r == 0 && a.hidden_out != nullptr);
  if (!mbar_wait(bar, 0) && t == 0) {
    // Record it and give the copy a second bounded wait before going on (the cluster barrier
    // below needs every CTA; the step's result is void and the host reads the flag).
    atomicExch(&g4_ple_error, 1);
    mbar_wait(bar, 0);
  }
  __syncthreads();
  G4_TRACE_POINT(3011);

  // ---- the gate: warp w owns rows 2w and 2w + 1; lanes split K into 16-byte pieces.
  {
    const float o1r = a.out1 != 0.0f ? __fdiv_rn(1.0f, a.out1) : 0.0f;
    const float i2r = __fdiv_rn(1.0f, a.in2);
    const int nq = H >> 4;
    const uint4 *wa = reinterpret_cast<const uint4 *>(w1s + (size_t)(2 * warp) * H);
    const uint4 *wb = reinterpret_cast<const uint4 *>(w1s + (size_t)(2 * warp + 1) * H);
#pragma unroll 1
    for (int c0 = 0; c0 < cols; c0 += PB_NC) {
      // The lane that finishes (row rr, column c0 + c) is lane rr * PB_NC + c: its per-layer
      // input goes out before the dots.
      const int my_rr = lane / PB_NC, my_c = c0 + lane % PB_NC;
      const bool finisher = lane < 2 * PB_NC && my_c < cols;
      const int my_row = r * PB_R1 + 2 * warp + my_rr;
      const float u = finisher ? a.ple_in[(size_t)my_c * a.ld_ple + a.ple_off + my_row] : 0.0f;
      int acc[2][PB_NC];
#pragma unroll
      for (int c = 0; c < PB_NC; c++) acc[0][c] = acc[1][c] = 0;
      for (int k = lane; k < nq; k += 32) {
        const uint4 w0 = wa[k], w1 = wb[k];
#pragma unroll
        for (int c = 0; c < PB_NC; c++)
          if (c0 + c < cols) {
            const uint4 x = reinterpret_cast<const uint4 *>(cin + (size_t)(c0 + c) * H)[k];
            acc[0][c] = dp4a_x4(w0, x, acc[0][c]);
            acc[1][c] = dp4a_x4(w1, x, acc[1][c]);
          }
      }
      int mine = 0;
#pragma unroll
      for (int rr = 0; rr < 2; rr++)
#pragma unroll
        for (int c = 0; c < PB_NC; c++) {
          const int v = warp_sum_int(acc[rr][c]);
          if (lane == rr * PB_NC + c) mine = v;
        }
      if (finisher) {
        const int i = 2 * warp + my_rr;
        float y = __fmul_rn(__fmul_rn(a.in1, s1f[i]), (float)mine);
        y = srq_out_r(y, a.out1, o1r);
        const float h = __fmul_rn(g4_gelu(y), u);
        own[my_c * PB_R1 + i] = (uint8_t)(srq_code_r(h, a.in2, i2r) & 255);
      }
    }
  }
  __syncthreads();
  // This CTA's 16 codes of each column go to every CTA of the cluster (one 16-byte store each).
  for (int i = t; i < cols * PB_CS; i += 256) {
    const int c = i / PB_CS, d = i - c * PB_CS;
    const uint4 q = *reinterpret_cast<const uint4 *>(own + c * PB_R1);
    asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(
                     pb_mapa(c2 + (size_t)c * PB_PD + r * PB_R1, (uint32_t)d)),
                 "r"(q.x), "r"(q.y), "r"(q.z), "r"(q.w)
                 : "memory");
  }
  // Every CTA's codes in place (and no shared memory is read remotely afterwards).
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
  G4_TRACE_POINT(3012);

  // ---- the projection: thread pair (2j, 2j + 1) owns row j, one 128-byte half of PD each;
  // pieces are visited in a rotated order so the eight loads of a quarter warp hit eight
  // different bank groups. R2 is a multiple of 16, so a warp's rows are all in range or all out.
  {
    const float o2r = a.out2 != 0.0f ? __fdiv_rn(1.0f, a.out2) : 0.0f;
    const int h = t & 1;
    for (int j = t >> 1; j < R2; j += 128) {
      const uint8_t *wr = w2s + (size_t)j * PB_PD + h * 128;
#pragma unroll 1
      for (int c0 = 0; c0 < cols; c0 += PB_NC) {
        int acc[PB_NC];
#pragma unroll
        for (int c = 0; c < PB_NC; c++) acc[c] = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const int m = (i + 2 * j + h) & 7;
          const uint4 w = *reinterpret_cast<const uint4 *>(wr + m * 16);
#pragma unroll
          for (int c = 0; c < PB_NC; c++)
            if (c0 + c < cols)
              acc[c] = dp4a_x4(w, *reinterpret_cast<const uint4 *>(c2 + (size_t)(c0 + c) * PB_PD + h * 128 + m * 16),
                               acc[c]);
        }
#pragma unroll
        for (int c = 0; c < PB_NC; c++) acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 1);
        if (h == 0) {
          const float sc = __fmul_rn(a.in2, s2f[j]);
#pragma unroll
          for (int c = 0; c < PB_NC; c++)
            if (c0 + c < cols)
              a.y[(size_t)(c0 + c) * a.ld_y + r * R2 + j] = srq_out_r(__fmul_rn(sc, (float)acc[c]), a.out2, o2r);
        }
      }
    }
  }
}

size_t ple_block_smem(int H, int cols) { return pb_layout(H, cols).total; }

static cudaLaunchConfig_t pb_config(const PleArgs &a, cudaStream_t st, cudaLaunchAttribute *attr, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(PB_CS);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = ple_block_smem(a.H, a.cols);
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PB_CS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cfg;
}

static cudaError_t pb_set_attrs() {
  cudaError_t e = cudaFuncSetAttribute(k_ple_block, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)ple_block_smem(2048, PB_MAXC));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_ple_block, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}

bool ple_block_fits(int H, int PD, int cols) {
  // H a multiple of 256: whole 16-byte pieces, and H / 16 projection rows a multiple of 16;
  // H <= 2048: the norm prologue's two vec4 chunks per thread.
  if (PD != PB_PD || H % 256 != 0 || H > 2048 || cols < 1 || cols > PB_MAXC) return false;
  if (pb_set_attrs() != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  PleArgs a;
  memset(&a, 0, sizeof(a));
  a.H = H;
  a.cols = cols;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = pb_config(a, nullptr, attr, false);
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k_ple_block, &cfg) == cudaSuccess && n >= 1) return true;
  cudaGetLastError();
  return false;
}

cudaError_t launch_ple_block(const PleArgs &a, cudaStream_t st, bool pdl) {
  if (a.cols < 1 || a.cols > PB_MAXC || a.H % 256 != 0 || a.H > 2048) return cudaErrorInvalidValue;
  static DeviceOnce attr_set;
  attr_set([&] { pb_set_attrs(); });
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = pb_config(a, st, attr, pdl);
  return cudaLaunchKernelEx(&cfg, k_ple_block, a);
}

}  // namespace g4
