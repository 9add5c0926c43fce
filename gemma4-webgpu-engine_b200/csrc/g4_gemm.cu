// Tensor-core quantized linear for many columns (prefill chunks, batched decode): the qgemm
// column contract of src/kernels/qgemm.ts:76-110, 490-552 (every token column is exactly the
// qgemv of src/kernels/qgemv.ts:1131-1176) computed with tcgen05 int8 MMA.
//
// D[128 weight rows][BN tokens] = A[128][K] * B[BN][K]^T, int8 x int8 -> int32 in TMEM.
//   A: weight codes as signed int8. int8 weights arrive by TMA straight into the 128-byte
//      swizzled K-major layout the MMA reads; int4 weights arrive packed (TMA, no swizzle) and
//      four unpack warps write them as (u - 8) into that layout.
//   B: the activation codes of BN tokens (k_quantize wrote them, plain K order), TMA, swizzled.
// The int32 accumulators are exact, so the epilogue y = srqOut((inScale * scale[r]) * f32(acc))
// gives the GEMV's bits.
//
// Warps: 0 issues TMA, 1 owns TMEM and issues the MMAs (one thread), 2-5 unpack and then run the
// epilogue (warp w reads TMEM lanes 32 (w % 4) .. + 31). Every mbarrier wait is bounded; a wait
// that gives up raises g4_gemm_error, the copies and MMAs already issued are waited for (bounded),
// and the TMEM is released on every path.
#include <cuda.h>
#include <cuda_runtime.h>
#include <float.h>
#include <string.h>
#include <mutex>

#include "g4_device.cuh"
#include "g4_kernels.cuh"

namespace g4 {

__device__ int g4_gemm_error;
#ifdef G4_TRACE
__device__ unsigned long long g4_trace_buf[1 << 16];
__device__ unsigned int g4_trace_n;
// Per launch: the latest accumulator-complete time over the CTAs, and the CTAs finished so far
// (the last one records both, then clears them for the next launch).
__device__ unsigned long long g4_gemm_accmax;
__device__ unsigned int g4_gemm_done;
// The latest CTA start and the latest return from the dependency wait over the launch's CTAs.
__device__ unsigned long long g4_gemm_entrymax, g4_gemm_waitmax;
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long now;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
  return now;
}
int gemm_trace_take(unsigned long long *out, int max_records) {
  unsigned int n = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&n, g4_trace_n, sizeof(n)) != cudaSuccess) return -1;
  if (n > (1u << 15)) n = 1u << 15;
  if ((int)n > max_records) n = (unsigned int)max_records;
  if (n && cudaMemcpyFromSymbol(out, g4_trace_buf, (size_t)n * 16) != cudaSuccess) return -1;
  cudaMemcpyToSymbol(g4_trace_n, &zero, sizeof(zero));
  return (int)n;
}
#endif

int *gemm_error_addr() {
  void *p = nullptr;
  return cudaGetSymbolAddress(&p, g4_gemm_error) == cudaSuccess ? (int *)p : nullptr;
}

int gemm_error_take() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g4_gemm_error, sizeof(int)) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g4_gemm_error, &zero, sizeof(int));
  return v;
}

// ------------------------------------------------------------------ tensor maps (host)
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_u8(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer,
                 uint64_t row_stride, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  if (((uintptr_t)base & 15) || (row_stride & 15) || box_inner * 1u > 256 || box_outer > 256) return -2;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box,
                  elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

// 32-bit elements (the 2-bit family's interleaved tiles: inner = K words, outer = tiles).
int make_tmap_u32(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer,
                  uint64_t row_stride, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  if (((uintptr_t)base & 15) || (row_stride & 15) || box_inner > 256 || box_outer > 256) return -2;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(base), dims, strides, box,
                  elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

// ------------------------------------------------------------------ device helpers
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart
// (start >> 4, leading offset 1, stride offset 1024 >> 4, descriptor version 1, layout 2).
__device__ __forceinline__ uint64_t sw128_desc(const void *p) {
  const uint32_t a = smem_u32(p);
  return (uint64_t)((a >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::i8: D s32, A s8, B s8, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t ad, uint64_t bd, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(ad), "l"(bd), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Every thread of every CTA in the cluster (the warp-divergent form: the role branches rejoin here).
__device__ __forceinline__ void cluster_sync_all() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// This CTA's shared address `p` mapped to cluster CTA `rank`'s copy, and a 32-bit load from it.
__device__ __forceinline__ uint32_t map_dsmem(const void *p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
  return remote;
}
__device__ __forceinline__ int4 ld_dsmem_v4(uint32_t remote) {
  int4 v;
  asm volatile("ld.shared::cluster.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(remote));
  return v;
}

// Eight packed int4 weights (code i at bits 4i) to eight signed int8 (u - 8), in K order.
__device__ __forceinline__ uint2 unpack8(uint32_t w) {
  const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  uint32_t a = __byte_perm(lo, hi, 0x5140), b = __byte_perm(lo, hi, 0x7362);
  // u - 8 in two's complement: flip bit 3, then copy bit 3 into the high nibble.
  a ^= 0x08080808u;
  b ^= 0x08080808u;
  a |= (a & 0x08080808u) * 0x1Eu;
  b |= (b & 0x08080808u) * 0x1Eu;
  return make_uint2(a, b);
}

constexpr int GM_BM = 128;       // weight rows per tile (MMA M)
constexpr int GM_BK = 128;       // K per stage: one 128-byte swizzle atom of int8

// NSTAGE 0: the default depth (3 at BN 256, 6 at BN 64, else 4, one CTA per SM); 2 (BN 128) or
// 3 (BN 64): two CTAs share an SM (their epilogues overlap each other's main loops). Int8
// weights land in the MMA tile directly, so their stages carry no packed staging buffer.
template <int BN, int NSTAGE = 0, int BITS = 4>
struct GemmShape {
  static constexpr int STAGES = NSTAGE ? NSTAGE : (BN >= 256 ? 3 : (BN <= 64 ? 6 : 4));
  static constexpr int A_BYTES = GM_BM * GM_BK;          // 16 KB
  static constexpr int B_BYTES = BN * GM_BK;
  static constexpr int P_BYTES = BITS == 8 ? 0 : GM_BM * GM_BK / 2;   // packed staging, 8 KB
  static constexpr int P2_BYTES = GM_BM * GM_BK / 4;     // 2-bit tiles: 8 x 128 words, 4 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + P_BYTES;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int SMEM = 1024 + BAR_OFF + (3 * STAGES + 2) * 8 + 64 + 4 * 32 * 8;
};

// CLU > 1: K split over a thread-block cluster of CLU CTAs along z (gridDim.z == CLU). Every CTA
// accumulates its K range in TMEM and parks the int32 partial in its own shared memory; after a
// cluster barrier each CTA sums all partials of its share of the tile's token columns through
// distributed shared memory (exact integer adds, fixed rank order) and runs the epilogue on it.
template <int BITS, int BN, int EPI, int NSTAGE, int CLU>
__global__ void __launch_bounds__(192, (NSTAGE == 2 || NSTAGE == 3) ? 2 : 1)
    k_qgemm_tc(const __grid_constant__ GemmMaps maps, const GemmArgs a) {
  using S = GemmShape<BN, NSTAGE, BITS>;
  constexpr int NS = S::STAGES;
  extern __shared__ __align__(1024) uint8_t gsm_raw[];
  uint8_t *gsm = gsm_raw + ((1024 - (smem_u32(gsm_raw) & 1023)) & 1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(gsm + S::BAR_OFF);
  uint64_t *aready = full + NS;
  uint64_t *empty = aready + NS;
  uint64_t *accf = empty + NS;
  uint32_t *tslot = reinterpret_cast<uint32_t *>(accf + 2);
  int *flags = reinterpret_cast<int *>(tslot + 2);         // [0]: error seen
  auto A = [&](int s) { return gsm + s * S::STAGE_BYTES; };
  auto B = [&](int s) { return gsm + s * S::STAGE_BYTES + S::A_BYTES; };
  auto P = [&](int s) { return gsm + s * S::STAGE_BYTES + S::A_BYTES + S::B_BYTES; };

#ifdef G4_TRACE
  const unsigned long long t_entry = gtimer();
#endif
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  // This CTA's segment (a multi-segment launch) and its tile within it.
  int sg = 0;
  for (int i = 1; i < a.nseg; i++)
    if ((int)blockIdx.x >= a.tile_begin[i]) sg = i;
  const int gN = sg ? a.more[sg - 1].N : a.N;
  const uint16_t *gS = sg ? a.more[sg - 1].s : a.s;
  const float gIn = sg ? a.more[sg - 1].in_scale : a.in_scale;
  const float gOut = sg ? a.more[sg - 1].out_scale : a.out_scale;
  float *const gY = sg ? a.more[sg - 1].y : a.y;
  const int gLdY = sg ? a.more[sg - 1].ld_y : a.ld_y;
  const CUtensorMap *tmW = &maps.w[sg], *tmX = &maps.x[sg];
  const int n0 = ((int)blockIdx.x - (sg ? a.tile_begin[sg] : 0)) * GM_BM, m0 = blockIdx.y * BN;
  // This CTA's K tiles: split blockIdx.z of a.splits (an even share, at least one tile).
  const int KTALL = a.K / GM_BK;
  const int kt_begin = (int)(((long long)KTALL * blockIdx.z) / gridDim.z);
  const int KT = (int)(((long long)KTALL * (blockIdx.z + 1)) / gridDim.z) - kt_begin;

  if (t == 0) {
    for (int s = 0; s < NS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&aready[s], 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    mbar_fence_init();
    flags[0] = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  grid_launch_dependents();
  // The producer requests the first stages' weights before the dependency wait (weights never
  // depend on the previous kernel), so their fetch overlaps that kernel's tail.
  const uint32_t wbytes = BITS == 4 ? S::P_BYTES : (BITS == 2 ? S::P2_BYTES : S::A_BYTES);
  const int npre = KT < NS ? KT : NS;
  auto load_w = [&](int kt) {
    const int s = kt % NS, kg = kt_begin + kt;
    if (BITS == 4)
      tma_load_2d(P(s), tmW, kg * (GM_BK / 2), n0, &full[s]);
    else if (BITS == 2)
      tma_load_2d(P(s), tmW, kg * GM_BK, n0 / 16, &full[s]);
    else
      tma_load_2d(A(s), tmW, kg * GM_BK, n0, &full[s]);
  };
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmW)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmX)) : "memory");
    for (int kt = 0; kt < npre; kt++) {
      mbar_expect_tx(&full[kt], wbytes + S::B_BYTES);
      load_w(kt);
    }
  }
  grid_wait();
  G4_TRACE_POINT(5000 + BITS * 100 + (BN == 64 ? 1 : 2) + (CLU > 1 ? 10 : 0));
#ifdef G4_TRACE
  if (t == 64) {
    atomicMax(&g4_gemm_entrymax, t_entry);
    atomicMax(&g4_gemm_waitmax, gtimer());
  }
#endif

  if (warp == 0) {
    if (lane == 0) {
      // Producer: codes of the prefetched stages, then weights and codes of stage kt once the
      // MMAs of kt - NS have read the slot.
      int issued = 0;
      for (int kt = 0; kt < KT; kt++) {
        const int s = kt % NS;
        if (kt >= NS && !mbar_wait(&empty[s], (uint32_t)((kt / NS - 1) & 1))) {
          atomicExch(&g4_gemm_error, 1);
          flags[0] = 1;
          break;
        }
        if (kt >= npre) {
          mbar_expect_tx(&full[s], wbytes + S::B_BYTES);
          load_w(kt);
        }
        tma_load_2d(B(s), tmX, (kt_begin + kt) * GM_BK, m0, &full[s]);
        issued = kt + 1;
      }
      // Every copy issued lands before the CTA can leave (the last NS are the ones not yet
      // known to be consumed).
      for (int kt = issued - NS < 0 ? 0 : issued - NS; kt < issued; kt++)
        mbar_wait(&full[kt % NS], (uint32_t)((kt / NS) & 1));
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_i8(BN);
      for (int kt = 0; kt < KT; kt++) {
        const int s = kt % NS;
        uint64_t *ready = BITS != 8 ? &aready[s] : &full[s];
        if (!mbar_wait(ready, (uint32_t)((kt / NS) & 1))) {
          atomicExch(&g4_gemm_error, 1);
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint64_t ad = sw128_desc(A(s)), bd = sw128_desc(B(s));
#pragma unroll
        for (int kk = 0; kk < GM_BK / 32; kk++)
          mma_i8(tmem, ad + 2 * kk, bd + 2 * kk, IDESC, (kt | kk) != 0 ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      mma_commit(accf);   // after the last MMA issued (or at once, if none was)
    }
  } else {
    const int tu = t - 64;   // 0..127
    if (BITS == 2) {
      // Thread tu: tile tu / 16 of the stage's eight, 16-column chunk (tu / 2) % 8, rows
      // 8 (tu % 2) .. + 7 of the tile; 16 words in, 8 rows x 16 signed codes (u - 2) out.
      const int lt = tu >> 4, ch = (tu >> 1) & 7, half = tu & 1;
      for (int kt = 0; kt < KT; kt++) {
        const int s = kt % NS;
        if (!mbar_wait(&full[s], (uint32_t)((kt / NS) & 1))) {
          atomicExch(&g4_gemm_error, 1);
          flags[0] = 1;
          break;
        }
        const uint4 *src = reinterpret_cast<const uint4 *>(P(s) + lt * 512 + ch * 64);
        uint32_t w[16];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const uint4 v = src[q];
          w[4 * q] = v.x;
          w[4 * q + 1] = v.y;
          w[4 * q + 2] = v.z;
          w[4 * q + 3] = v.w;
        }
        uint8_t *dst = A(s);
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const int rr = 8 * half + i, row = 16 * lt + rr;
          uint32_t o[4];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const uint32_t lo = __byte_perm(w[4 * q] >> (2 * rr), w[4 * q + 1] >> (2 * rr), 0x0040);
            const uint32_t hi = __byte_perm(w[4 * q + 2] >> (2 * rr), w[4 * q + 3] >> (2 * rr), 0x0040);
            uint32_t v = __byte_perm(lo, hi, 0x5410) & 0x03030303u;
            // u - 2 as signed bytes: flip bit 1; where it is then set (u < 2), set bits 2..7.
            v ^= 0x02020202u;
            v |= (v & 0x02020202u) * 0x7Fu;
            o[q] = v;
          }
          *reinterpret_cast<uint4 *>(dst + (row >> 3) * 1024 + (row & 7) * 128 + ((ch ^ (row & 7)) << 4)) =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&aready[s]);
      }
    }
    if (BITS == 4) {
      for (int kt = 0; kt < KT; kt++) {
        const int s = kt % NS;
        if (!mbar_wait(&full[s], (uint32_t)((kt / NS) & 1))) {
          atomicExch(&g4_gemm_error, 1);
          flags[0] = 1;
          break;
        }
        const uint8_t *p = P(s);
        uint8_t *dst = A(s);
#pragma unroll
        for (int it = 0; it < 8; it++) {
          const int idx = tu + 128 * it;   // (row, 16-element chunk)
          const int row = idx >> 3, ch = idx & 7;
          const uint2 pk = *reinterpret_cast<const uint2 *>(p + row * 64 + ch * 8);
          const uint2 lo = unpack8(pk.x), hi = unpack8(pk.y);
          *reinterpret_cast<uint4 *>(dst + (row >> 3) * 1024 + (row & 7) * 128 + ((ch ^ (row & 7)) << 4)) =
              make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&aready[s]);
      }
    }
    // ---- epilogue
    const bool ok = mbar_wait(accf, 0);
    if (!ok) {
      atomicExch(&g4_gemm_error, 1);
      mbar_wait(accf, 0);
    }
    tc_fence_after();
#ifdef G4_TRACE
    if (t == 64) {
      G4_TRACE_POINT_T(205000 + BITS * 100 + (BN == 64 ? 1 : 2) + (CLU > 1 ? 10 : 0));
      atomicMax(&g4_gemm_accmax, gtimer());
    }
#endif
    const int q = warp & 3;
    const int row = n0 + 32 * q + lane;
    const bool row_ok = row < gN;
    const float wscale = row_ok ? f16_bits_to_f32(gS[row]) : 0.0f;
    const float sc = __fmul_rn(gIn, wscale);
    const float out_r = gOut != 0.0f ? __fdiv_rn(1.0f, gOut) : 0.0f;
    bool last = true;
    if (CLU > 1) {
      // Park the partial, int32 [BN tokens][128 rows], over the stage buffers (every MMA that
      // read them has completed).
      int32_t *pbuf = reinterpret_cast<int32_t *>(gsm);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t acc[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, acc);
#pragma unroll
        for (int j = 0; j < 32; j++) pbuf[(c0 + j) * GM_BM + 32 * q + lane] = (int)acc[j];
      }
      last = false;   // reduced and stored after the cluster barrier below
    } else if (gridDim.z > 1) {
      // Split K: add this CTA's partial into the workspace; the tile's last split finishes.
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t acc[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, acc);
        if (ok && !flags[0] && row_ok) {
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int tok = m0 + c0 + j;
            if (tok < a.M) atomicAdd(a.acc_ws + (size_t)tok * a.ld_ws + row, (int)acc[j]);
          }
        }
      }
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      int *cnt = a.tile_cnt + blockIdx.y * gridDim.x + blockIdx.x;
      if (t == 64) flags[1] = atomicAdd(cnt, 1) == (int)gridDim.z - 1;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      last = flags[1] != 0;
      if (last) {
        __threadfence();
        if (t == 64) *cnt = 0;
      }
    }
    if constexpr (EPI == EPI_HEAD) {
      // Through shared memory (the stage buffers, free once every MMA completed): the int32 sums
      // parked as [BN tokens][128 rows], then each thread's row of logits for every token (a
      // short loop, 8 tokens in flight), then per token the greatest value over the tile's rows,
      // lowest row on ties, scanned by 128 / BN threads per token in bank-rotated order.
      int32_t *ab = reinterpret_cast<int32_t *>(gsm);
      float *yb = reinterpret_cast<float *>(gsm);
      const bool store = ok && !flags[0];
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t acc[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, acc);
#pragma unroll
        for (int j = 0; j < 32; j++) ab[(c0 + j) * GM_BM + 32 * q + lane] = (int)acc[j];
      }
#pragma unroll 8
      for (int j = 0; j < BN; j++) {
        const int slot = j * GM_BM + 32 * q + lane;
        float y = __fmul_rn(sc, (float)ab[slot]);
        y = srq_out_r(y, gOut, out_r);
        if (a.softcap != 0.0f) y = __fmul_rn(g4_tanh(__fdiv_rn(y, a.softcap)), a.softcap);
        const int tok = m0 + j;
        if (store && a.logits && row_ok && tok < a.M) a.logits[(size_t)tok * a.ld_logits + row] = y;
        yb[slot] = y;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      constexpr int TPT = BN <= GM_BM ? GM_BM / BN : 1;   // threads per token
      constexpr int R = GM_BM / TPT;                       // rows each scans
      const int u = t - 64;
#pragma unroll 1
      for (int j = TPT > 1 ? u / TPT : u; j < BN; j += 128 / TPT) {
        const int h = TPT > 1 ? u % TPT : 0;
        float bv = -FLT_MAX;
        int bi = 0x7fffffff;
#pragma unroll 8
        for (int i = 0; i < R; i++) {
          const int r = h * R + ((i + u) & (R - 1));
          const float v = yb[j * GM_BM + r];
          if (n0 + r < gN && (v > bv || (v == bv && n0 + r < bi))) {
            bv = v;
            bi = n0 + r;
          }
        }
        if (TPT == 2) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, 1);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, 1);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        const int tok = m0 + j;
        if (h == 0 && store && tok < a.M) {
          a.part_val[(size_t)tok * a.n_parts + blockIdx.x] = bv;
          a.part_idx[(size_t)tok * a.n_parts + blockIdx.x] = bi;
        }
      }
      last = false;
    }
#pragma unroll 1
    for (int c0 = 0; c0 < BN && last; c0 += 32) {
      uint32_t acc[32];
      if (gridDim.z > 1) {
        // The tile's full sums, read back (all 32 loads in flight together), then the workspace
        // is cleared for the next launch.
        int32_t *wp = a.acc_ws + (size_t)(m0 + c0) * a.ld_ws + row;
        const int nt = min(32, a.M - (m0 + c0));
#pragma unroll
        for (int j = 0; j < 32; j++) acc[j] = (row_ok && j < nt) ? (uint32_t)__ldcg(wp + (size_t)j * a.ld_ws) : 0u;
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (row_ok && j < nt) wp[(size_t)j * a.ld_ws] = 0;
      } else {
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, acc);
      }
      // After a failed wait nothing is stored.
      const bool store = ok && !flags[0];
#pragma unroll
      for (int j = 0; j < 32; j++) {
        const int tok = m0 + c0 + j;
        float y = __fmul_rn(sc, (float)(int)acc[j]);
        y = srq_out_r(y, gOut, out_r);
        if (store && row_ok && tok < a.M) gY[(size_t)tok * gLdY + row] = y;
      }
    }
  }
  if constexpr (CLU > 1) {
    cluster_sync_all();   // every CTA of the cluster has parked its partial
    if (warp >= 2) {
      // This CTA's share: PER token columns. Thread u takes rows 4g..4g+3 (g = u % 32) of the
      // tokens u / 32 + 4i, 16-byte loads from every rank's partial, all in flight together.
      constexpr int PER = BN / CLU;
      constexpr int ITEMS = PER / 4;
      const int u = t - 64, g = u & 31, jb = u >> 5;
      const int t0 = (int)cluster_rank() * PER;
      const float out_r = gOut != 0.0f ? __fdiv_rn(1.0f, gOut) : 0.0f;
      float sc[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int row = n0 + 4 * g + e;
        sc[e] = row < gN ? __fmul_rn(gIn, f16_bits_to_f32(gS[row])) : 0.0f;
      }
      const int32_t *mine = reinterpret_cast<const int32_t *>(gsm) + t0 * GM_BM + 4 * g;
      const bool store = !flags[0] && g4_gemm_error == 0;
      int4 v[CLU][ITEMS];
#pragma unroll
      for (int r = 0; r < CLU; r++) {
        const uint32_t base = map_dsmem(mine, (uint32_t)r);
#pragma unroll
        for (int it = 0; it < ITEMS; it++) v[r][it] = ld_dsmem_v4(base + (uint32_t)((jb + 4 * it) * GM_BM * 4));
      }
#pragma unroll
      for (int it = 0; it < ITEMS; it++) {
        int4 sum = v[0][it];
#pragma unroll
        for (int r = 1; r < CLU; r++) {
          sum.x += v[r][it].x;
          sum.y += v[r][it].y;
          sum.z += v[r][it].z;
          sum.w += v[r][it].w;
        }
        const int tok = m0 + t0 + jb + 4 * it;
        const int sv[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int row = n0 + 4 * g + e;
          float y = __fmul_rn(sc[e], (float)sv[e]);
          y = srq_out_r(y, gOut, out_r);
          if (store && row < gN && tok < a.M) gY[(size_t)tok * gLdY + row] = y;
        }
      }
    }
    cluster_sync_all();   // no CTA leaves while another still reads its partial
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
  }
#ifdef G4_TRACE
  if (t == 64) {
    const int id = 5000 + BITS * 100 + (BN == 64 ? 1 : 2) + (CLU > 1 ? 10 : 0);
    G4_TRACE_POINT_T(300000 + id);
    __threadfence();
    const unsigned int total = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(&g4_gemm_done, 1u) == total - 1) {
      G4_TRACE_REC(500000 + id, atomicExch(&g4_gemm_accmax, 0ull));
      G4_TRACE_REC(600000 + id, atomicExch(&g4_gemm_entrymax, 0ull));
      G4_TRACE_REC(700000 + id, atomicExch(&g4_gemm_waitmax, 0ull));
      G4_TRACE_REC(400000 + id, gtimer());
      g4_gemm_done = 0;
    }
  }
#endif
}

// Persistent form for many tiles (prefill): one CTA per SM loops over tiles (m-major order, so
// the CTAs running at once share a token tile in L2). Warps: 0 TMA, 1 MMA + TMEM owner, 2-5 int4
// unpack, 6-9 epilogue. Two TMEM accumulators of BN columns: the MMAs of tile i + 1 run while the
// epilogue warps read tile i. Stage and accumulator barriers use running counters for their
// phases; every wait is bounded.
template <int BITS, int BN, int EPI>
__global__ void __launch_bounds__(320, 1)
    k_qgemm_persist(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                    const GemmArgs a) {
  using S = GemmShape<BN, 4>;
  constexpr int NS = S::STAGES;
  extern __shared__ __align__(1024) uint8_t gsm_raw[];
  uint8_t *gsm = gsm_raw + ((1024 - (smem_u32(gsm_raw) & 1023)) & 1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(gsm + S::BAR_OFF);
  uint64_t *aready = full + NS;
  uint64_t *empty = aready + NS;
  uint64_t *acc_full = empty + NS;      // [2]
  uint64_t *acc_empty = acc_full + 2;   // [2]
  uint32_t *tslot = reinterpret_cast<uint32_t *>(acc_empty + 2);
  int *flags = reinterpret_cast<int *>(tslot + 2);
  float *cand_v = reinterpret_cast<float *>(flags + 14);
  int *cand_i = reinterpret_cast<int *>(cand_v + 4 * 32);
  auto A = [&](int s) { return gsm + s * S::STAGE_BYTES; };
  auto B = [&](int s) { return gsm + s * S::STAGE_BYTES + S::A_BYTES; };
  auto P = [&](int s) { return gsm + s * S::STAGE_BYTES + S::A_BYTES + S::B_BYTES; };
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int KT = a.K / GM_BK;
  const int n_tiles = (a.N + GM_BM - 1) / GM_BM, m_tiles = (a.M + BN - 1) / BN;
  const int tiles = n_tiles * m_tiles;

  if (t == 0) {
    for (int s = 0; s < NS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&aready[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_fence_init();
    flags[0] = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(2 * BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  grid_launch_dependents();
  grid_wait();

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t wbytes = BITS == 4 ? S::P_BYTES : S::A_BYTES;
      uint32_t g = 0;
      for (int tile = blockIdx.x; tile < tiles && !flags[0]; tile += gridDim.x) {
        const int n0 = (tile % n_tiles) * GM_BM, m0 = (tile / n_tiles) * BN;
        for (int kt = 0; kt < KT; kt++, g++) {
          const int s = g % NS;
          if (g >= (uint32_t)NS && !mbar_wait(&empty[s], ((g / NS) - 1) & 1)) {
            atomicExch(&g4_gemm_error, 1);
            flags[0] = 1;
            break;
          }
          mbar_expect_tx(&full[s], wbytes + S::B_BYTES);
          if (BITS == 4)
            tma_load_2d(P(s), &tmW, kt * (GM_BK / 2), n0, &full[s]);
          else
            tma_load_2d(A(s), &tmW, kt * GM_BK, n0, &full[s]);
          tma_load_2d(B(s), &tmX, kt * GM_BK, m0, &full[s]);
        }
      }
      for (uint32_t q = g > (uint32_t)NS ? g - NS : 0; q < g; q++) mbar_wait(&full[q % NS], (q / NS) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_i8(BN);
      uint32_t g = 0, lt = 0;
      for (int tile = blockIdx.x; tile < tiles && !flags[0]; tile += gridDim.x, lt++) {
        const int b = lt & 1;
        const uint32_t u = lt >> 1;
        if (u >= 1 && !mbar_wait(&acc_empty[b], (u - 1) & 1)) {
          atomicExch(&g4_gemm_error, 1);
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BN);
        for (int kt = 0; kt < KT; kt++, g++) {
          const int s = g % NS;
          uint64_t *ready = BITS == 4 ? &aready[s] : &full[s];
          if (!mbar_wait(ready, (g / NS) & 1)) {
            atomicExch(&g4_gemm_error, 1);
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(A(s)), bd = sw128_desc(B(s));
#pragma unroll
          for (int kk = 0; kk < GM_BK / 32; kk++)
            mma_i8(d, ad + 2 * kk, bd + 2 * kk, IDESC, (kt | kk) != 0 ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        mma_commit(&acc_full[b]);
      }
    }
  } else if (warp < 6) {
    if (BITS == 4) {
      const int tu = t - 64;   // 0..127
      const uint32_t total = (uint32_t)((tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * KT;
      for (uint32_t g = 0; g < total && !flags[0]; g++) {
        const int s = g % NS;
        if (!mbar_wait(&full[s], (g / NS) & 1)) {
          atomicExch(&g4_gemm_error, 1);
          flags[0] = 1;
          break;
        }
        const uint8_t *p = P(s);
        uint8_t *dst = A(s);
#pragma unroll
        for (int it = 0; it < 8; it++) {
          const int idx = tu + 128 * it;
          const int row = idx >> 3, ch = idx & 7;
          const uint2 pk = *reinterpret_cast<const uint2 *>(p + row * 64 + ch * 8);
          const uint2 lo = unpack8(pk.x), hi = unpack8(pk.y);
          *reinterpret_cast<uint4 *>(dst + (row >> 3) * 1024 + (row & 7) * 128 + ((ch ^ (row & 7)) << 4)) =
              make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&aready[s]);
      }
    }
  } else {
    // ---- epilogue warps 6-9: warp w reads TMEM lanes 32 (w % 4) .. + 31
    const int q = warp & 3;
    uint32_t lt = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, lt++) {
      const int b = lt & 1;
      const bool ok = !flags[0] && mbar_wait(&acc_full[b], (lt >> 1) & 1);
      if (!ok) {
        atomicExch(&g4_gemm_error, 1);
        flags[0] = 1;
        break;
      }
      tc_fence_after();
      const int nt = tile % n_tiles, n0 = nt * GM_BM, m0 = (tile / n_tiles) * BN;
      const int row = n0 + 32 * q + lane;
      const bool row_ok = row < a.N;
      const float wscale = row_ok ? f16_bits_to_f32(a.s[row]) : 0.0f;
      const float sc = __fmul_rn(a.in_scale, wscale);
      const float out_r = a.out_scale != 0.0f ? __fdiv_rn(1.0f, a.out_scale) : 0.0f;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t acc[32];
        tmem_ld32(tmem + (uint32_t)(b * BN) + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, acc);
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const int tok = m0 + c0 + j;
          float y = __fmul_rn(sc, (float)(int)acc[j]);
          y = srq_out_r(y, a.out_scale, out_r);
          if (EPI == EPI_HEAD) {
            if (a.softcap != 0.0f) y = __fmul_rn(g4_tanh(__fdiv_rn(y, a.softcap)), a.softcap);
            if (a.logits && row_ok && tok < a.M) a.logits[(size_t)tok * a.ld_logits + row] = y;
            float bv = row_ok ? y : -FLT_MAX;
            int bi = row_ok ? row : 0x7fffffff;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
              const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
              if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
              }
            }
            if (lane == j) {
              cand_v[q * 32 + j] = bv;
              cand_i[q * 32 + j] = bi;
            }
          } else {
            if (row_ok && tok < a.M) a.y[(size_t)tok * a.ld_y + row] = y;
          }
        }
        if (EPI == EPI_HEAD) {
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (q == 0) {
            float bv = cand_v[lane];
            int bi = cand_i[lane];
#pragma unroll
            for (int w2 = 1; w2 < 4; w2++) {
              const float ov = cand_v[w2 * 32 + lane];
              const int oi = cand_i[w2 * 32 + lane];
              if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
              }
            }
            const int tok = m0 + c0 + lane;
            if (tok < a.M) {
              a.part_val[(size_t)tok * a.n_parts + nt] = bv;
              a.part_idx[(size_t)tok * a.n_parts + nt] = bi;
            }
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
      }
      // This accumulator may take the next tile's MMAs.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN) : "memory");
  }
}

template <int BITS, int BN, int EPI>
static cudaError_t launch_gemm_persist(const CUtensorMap &tmW, const CUtensorMap &tmX, const GemmArgs &a,
                                       int grid, cudaStream_t st, bool pdl) {
  auto k = k_qgemm_persist<BITS, BN, EPI>;
  const int smem = GemmShape<BN, 4>::SMEM + 64;
  static DeviceOnce attr;
  attr([&] {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(320);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr1[1];
  attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr1[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr1;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, tmW, tmX, a);
}

// Tiles along x: the segments' 128-row tiles end to end.
static int gemm_x_tiles(const GemmArgs &a) {
  return a.nseg > 1 ? a.tile_begin[a.nseg] : (a.N + GM_BM - 1) / GM_BM;
}
static GemmMaps one_map(const CUtensorMap &tmW, const CUtensorMap &tmX) {
  GemmMaps m;
  memset(&m, 0, sizeof(m));
  m.w[0] = tmW;
  m.x[0] = tmX;
  return m;
}

template <int BITS, int BN, int EPI, int NSTAGE = 0>
static cudaError_t launch_gemm_t(const GemmMaps &maps, const GemmArgs &a, cudaStream_t st, bool pdl) {
  auto k = k_qgemm_tc<BITS, BN, EPI, NSTAGE, 0>;
  const int smem = GemmShape<BN, NSTAGE, BITS>::SMEM;
  static DeviceOnce attr;
  attr([&] {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gemm_x_tiles(a), (a.M + BN - 1) / BN, a.splits > 1 ? a.splits : 1);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr1[1];
  attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr1[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr1;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, maps, a);
}

// NSTAGE 0: six stages, one CTA per SM; 3: three stages, two CTAs per SM (launches of more CTAs
// than SMs).
template <int BITS, int CLU, int NSTAGE>
static cudaError_t launch_gemm_cluster_t(const GemmMaps &maps, const GemmArgs &a, cudaStream_t st, bool pdl) {
  auto k = k_qgemm_tc<BITS, 64, EPI_Y, NSTAGE, CLU>;
  const int smem = GemmShape<64, NSTAGE, BITS>::SMEM;
  static DeviceOnce attr;
  attr([&] {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
  });
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gemm_x_tiles(a), (a.M + 63) / 64, CLU);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = CLU;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, k, maps, a);
}

static cudaError_t launch_cluster_maps(const GemmMaps &m, const GemmArgs &a, int bits, cudaStream_t st, bool pdl) {
  if (a.K % GM_BK != 0 || a.N < 1 || a.M < 1 || a.head || a.splits > a.K / GM_BK ||
      (bits != 2 && bits != 4 && bits != 8))
    return cudaErrorInvalidValue;
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Three stages (two CTAs per SM) when the launch has more CTAs than SMs; else six, so a CTA's
  // whole K range (at most six 128-deep tiles at these splits) is requested before the wait.
  const bool two = gemm_x_tiles(a) * ((a.M + 63) / 64) * a.splits > sms;
  switch (a.splits * 100 + bits * 10 + (two ? 1 : 0)) {
    case 240: return launch_gemm_cluster_t<4, 2, 0>(m, a, st, pdl);
    case 440: return launch_gemm_cluster_t<4, 4, 0>(m, a, st, pdl);
    case 840: return launch_gemm_cluster_t<4, 8, 0>(m, a, st, pdl);
    case 280: return launch_gemm_cluster_t<8, 2, 0>(m, a, st, pdl);
    case 480: return launch_gemm_cluster_t<8, 4, 0>(m, a, st, pdl);
    case 880: return launch_gemm_cluster_t<8, 8, 0>(m, a, st, pdl);
    case 241: return launch_gemm_cluster_t<4, 2, 3>(m, a, st, pdl);
    case 441: return launch_gemm_cluster_t<4, 4, 3>(m, a, st, pdl);
    case 841: return launch_gemm_cluster_t<4, 8, 3>(m, a, st, pdl);
    case 281: return launch_gemm_cluster_t<8, 2, 3>(m, a, st, pdl);
    case 481: return launch_gemm_cluster_t<8, 4, 3>(m, a, st, pdl);
    case 881: return launch_gemm_cluster_t<8, 8, 3>(m, a, st, pdl);
    case 220: return launch_gemm_cluster_t<2, 2, 0>(m, a, st, pdl);
    case 420: return launch_gemm_cluster_t<2, 4, 0>(m, a, st, pdl);
    case 820: return launch_gemm_cluster_t<2, 8, 0>(m, a, st, pdl);
    case 221: return launch_gemm_cluster_t<2, 2, 3>(m, a, st, pdl);
    case 421: return launch_gemm_cluster_t<2, 4, 3>(m, a, st, pdl);
    case 821: return launch_gemm_cluster_t<2, 8, 3>(m, a, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_qgemm_cluster(const CUtensorMap &tmW, const CUtensorMap &tmX, const GemmArgs &a,
                                 int bits, cudaStream_t st, bool pdl) {
  if (a.nseg > 1) return cudaErrorInvalidValue;
  return launch_cluster_maps(one_map(tmW, tmX), a, bits, st, pdl);
}

cudaError_t launch_qgemm_multi(const GemmMaps &m, const GemmArgs &a, int bits, int bn, cudaStream_t st, bool pdl) {
  if (a.nseg < 2 || a.nseg > 3 || a.head || a.tile_begin[0] != 0) return cudaErrorInvalidValue;
  for (int i = 0; i < a.nseg; i++) {
    const int n = i ? a.more[i - 1].N : a.N;
    if (n < 1 || a.tile_begin[i + 1] - a.tile_begin[i] != (n + GM_BM - 1) / GM_BM) return cudaErrorInvalidValue;
  }
  if (bn != 64 && bn != -128) return cudaErrorInvalidValue;
  if (a.splits > 1) return bn == 64 ? launch_cluster_maps(m, a, bits, st, pdl) : cudaErrorInvalidValue;
  if (a.K % GM_BK != 0 || a.K < GM_BK) return cudaErrorInvalidValue;
  if (bn == -128) {
    if (bits == 4) return launch_gemm_t<4, 128, EPI_Y, 2>(m, a, st, pdl);
    if (bits == 8) return launch_gemm_t<8, 128, EPI_Y, 2>(m, a, st, pdl);
    if (bits == 2) return launch_gemm_t<2, 128, EPI_Y, 2>(m, a, st, pdl);
    return cudaErrorInvalidValue;
  }
  // More CTAs than SMs: three stages, two CTAs per SM.
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool two = gemm_x_tiles(a) * ((a.M + 63) / 64) > sms;
  if (bits == 4) return two ? launch_gemm_t<4, 64, EPI_Y, 3>(m, a, st, pdl) : launch_gemm_t<4, 64, EPI_Y>(m, a, st, pdl);
  if (bits == 8) return two ? launch_gemm_t<8, 64, EPI_Y, 3>(m, a, st, pdl) : launch_gemm_t<8, 64, EPI_Y>(m, a, st, pdl);
  if (bits == 2) return two ? launch_gemm_t<2, 64, EPI_Y, 3>(m, a, st, pdl) : launch_gemm_t<2, 64, EPI_Y>(m, a, st, pdl);
  return cudaErrorInvalidValue;
}

template <int BITS, int EPI>
static cudaError_t launch_gemm_b(const CUtensorMap &tmW, const CUtensorMap &tmX, const GemmArgs &a,
                                 int bn, cudaStream_t st, bool pdl) {
  const GemmMaps m = one_map(tmW, tmX);
  if (bn == 64) return launch_gemm_t<BITS, 64, EPI>(m, a, st, pdl);
  if (bn == 128) return launch_gemm_t<BITS, 128, EPI>(m, a, st, pdl);
  if (bn == 256) return launch_gemm_t<BITS, 256, EPI>(m, a, st, pdl);
  if (bn == -128) return launch_gemm_t<BITS, 128, EPI, 2>(m, a, st, pdl);
  if (bn == -64) return launch_gemm_t<BITS, 64, EPI, 3>(m, a, st, pdl);
  return cudaErrorInvalidValue;
}

cudaError_t launch_qgemm_persist(const CUtensorMap &tmW, const CUtensorMap &tmX, const GemmArgs &a,
                                 int bits, int grid, cudaStream_t st, bool pdl) {
  if (a.K % GM_BK != 0 || a.K < GM_BK || a.N < 1 || a.M < 1 || a.splits > 1 || grid < 1)
    return cudaErrorInvalidValue;
  if (bits == 4)
    return a.head ? launch_gemm_persist<4, 128, EPI_HEAD>(tmW, tmX, a, grid, st, pdl)
                  : launch_gemm_persist<4, 128, EPI_Y>(tmW, tmX, a, grid, st, pdl);
  if (bits == 8)
    return a.head ? launch_gemm_persist<8, 128, EPI_HEAD>(tmW, tmX, a, grid, st, pdl)
                  : launch_gemm_persist<8, 128, EPI_Y>(tmW, tmX, a, grid, st, pdl);
  return cudaErrorInvalidValue;
}

cudaError_t launch_qgemm(const CUtensorMap &tmW, const CUtensorMap &tmX, const GemmArgs &a, int bits,
                         int bn, cudaStream_t st, bool pdl) {
  if (a.K % GM_BK != 0 || a.K < GM_BK || a.N < 1 || a.M < 1 || a.nseg > 1) return cudaErrorInvalidValue;
  if (a.splits > 1 && (a.head || !a.acc_ws || !a.tile_cnt || a.splits > a.K / GM_BK || a.ld_ws < a.N))
    return cudaErrorInvalidValue;
  if (bits == 4) {
    if (a.head) return launch_gemm_b<4, EPI_HEAD>(tmW, tmX, a, bn, st, pdl);
    return launch_gemm_b<4, EPI_Y>(tmW, tmX, a, bn, st, pdl);
  }
  if (bits == 8) {
    if (a.head) return launch_gemm_b<8, EPI_HEAD>(tmW, tmX, a, bn, st, pdl);
    return launch_gemm_b<8, EPI_Y>(tmW, tmX, a, bn, st, pdl);
  }
  if (bits == 2) {
    if (a.head) return launch_gemm_b<2, EPI_HEAD>(tmW, tmX, a, bn, st, pdl);
    return launch_gemm_b<2, EPI_Y>(tmW, tmX, a, bn, st, pdl);
  }
  return cudaErrorInvalidValue;
}

int gemm_tile_rows() { return GM_BM; }

}  // namespace g4
