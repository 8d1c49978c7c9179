// Tensor-core GEMM for sm_100a (tcgen05 + TMA + tensor memory), written for this
// library's contractions: the weight gradients, the per-lag correlation stack of the
// synaptic layers, the feedforward projections and the chunked delay contraction of
// the reverse scan.
//
//   D[z][m, n]  (=, +=, or masked =)  sum_seg sum_p sum_k
//        A_pa(p)(m + seg*a_mn_seg + z*a_mn_z,  k + seg*a_k_seg + z*a_k_z) *
//        B_pb(p)(n + seg*b_mn_seg + z*b_mn_z,  k + seg*b_k_seg + z*b_k_z)
//
// Operands are bf16 "pieces" (an fp32 value split into hi + lo bf16 parts; a product
// list such as {hi.hi, hi.lo, lo.hi} then gives fp32-level accuracy with an fp32
// accumulator), each either K-major (the reduction index contiguous) or MN-major (the
// row index contiguous, e.g. a (T*B, N) activation reduced over T*B).  One CTA
// computes one 128 x BN output tile: thread 0 streams 128x64 / BNx64 operand tiles with
// cp.async.bulk.tensor (128-byte swizzle, per-CTA loads, no multicast) into a ring of
// shared-memory stages, thread 32 issues tcgen05.mma (M=128, N=BN, K=16) into a tensor-
// memory accumulator and frees each stage with tcgen05.commit, and all four warps read
// the accumulator back with tcgen05.ld for the epilogue.  Rows / columns / reduction
// entries outside the tensors are zero-filled by the tensor map, so ragged shapes and
// time shifts past the end of a sequence need no padding.  Every wait is bounded: on
// expiry the CTA records ST_TIMEOUT in the status word, drains and returns.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace delrec {

// GEMM_PARTIALS (gemm_run only): the ksplit fp32 partials stay in `part` (split-major,
// each M x N with row stride N, also for ksplit == 1) for the caller to sum
enum : int { GEMM_STORE = 0, GEMM_ACCUM = 1, GEMM_MASKED = 2, GEMM_PARTIALS = 3 };

constexpr int kGemmBM = 128, kGemmBK = 64, kGemmThreads = 128, kGemmMaxProd = 6;

struct GemmArgs {
  int M, N, K;                 // output rows and columns; reduction length per product
  int nprod;                   // products (<= kGemmMaxProd)
  int pa[kGemmMaxProd], pb[kGemmMaxProd];   // A / B piece (tensor map 0..2) of each product
  int nseg;                    // reduction segments, each with its own operand shifts
  // operand shifts (in elements) of the row (mn) and reduction (k) coordinates, per
  // segment (_seg) and per batch index z (_z).  The coordinate that is contiguous in
  // memory (k of a K-major operand, mn of an MN-major one) must shift by multiples of 8.
  int a_mn_seg, a_k_seg, b_mn_seg, b_k_seg;
  int a_mn_z, a_k_z, b_mn_z, b_k_z;
  int ksplit;                  // reduction split over gridDim.y (partials -> k_gemm_reduce)
  float* D;
  long long ldd, d_z, d_split; // row stride; stride per z; stride per split partial
  int mode;                    // GEMM_STORE / GEMM_ACCUM / GEMM_MASKED (ksplit == 1 only)
  const uint8_t* mask;         // GEMM_MASKED: write D[m,n] where mask[m*ldmask + n*mask_cs] == z
  long long ldmask, mask_cs;
  int z0;                      // batch index of gridDim.z slice 0 (z = z0 + blockIdx.z)
  long long spin_ns;           // wait limit in nanoseconds
};

__host__ __device__ constexpr int gemm_stages(int BN) { return BN >= 256 ? 4 : 6; }
__host__ __device__ constexpr size_t gemm_smem_bytes(int BN) {
  return (size_t)gemm_stages(BN) * (kGemmBM * kGemmBK * 2 + (size_t)BN * kGemmBK * 2) + 1024;
}

// ---- PTX wrappers --------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for the phase of `parity` to complete, at most limit_ns; on expiry raise the CTA's
// abort flag and the status word.  Returns false when aborted (here or elsewhere).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long limit_ns, volatile int* abort) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (unsigned it = 1;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (*abort) return false;
      if ((long long)(global_ns() - t0) > limit_ns) {
        *abort = 1;
        flag_status(ST_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"((unsigned long long)map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Shared-memory matrix descriptors of tiles written by TMA with the 128-byte swizzle
// (tile base 1024-aligned):
//  * K-major: rows of 128 bytes (64 reduction elements), 8-row groups 1024 bytes apart;
//    the next K=16 slice starts 32 bytes further;
//  * MN-major: 64-element (128-byte) rows along M/N, one per reduction index, 8-row
//    groups 1024 bytes apart, 64-wide M/N blocks LBO = 8192 bytes apart (boxes of 64
//    rows placed back to back); the next K=16 slice starts 2048 bytes further.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, bool mn_major) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);                  // start address
  d |= (uint64_t)(mn_major ? (8192 >> 4) : 1) << 16;          // leading byte offset
  d |= (uint64_t)(1024 >> 4) << 32;                           // stride byte offset
  d |= (uint64_t)1 << 46;                                     // descriptor version
  d |= (uint64_t)2 << 61;                                     // 128-byte swizzle
  return d;
}
// instruction descriptor: fp32 accumulate, bf16 A and B, M=128, N=BN, operand majors
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int BN, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kGemmBM >> 4) << 24);
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(
          tmem),
      "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of the warp's 32 tensor-memory lanes (thread = row)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- the GEMM kernel -----------------------------------------------------------------
// grid: x = output tiles (row-tile major), y = reduction splits, z = batch index.
// AMN / BMN: the operand is MN-major (its M / N index contiguous in memory, e.g. a
// (T*B, N) activation reduced over its rows) instead of K-major.
template <int BN, bool AMN, bool BMN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap a0, const __grid_constant__ CUtensorMap a1,
              const __grid_constant__ CUtensorMap a2, const __grid_constant__ CUtensorMap b0,
              const __grid_constant__ CUtensorMap b1, const __grid_constant__ CUtensorMap b2, const GemmArgs g) {
  constexpr int STAGES = gemm_stages(BN);
  constexpr uint32_t A_BYTES = kGemmBM * kGemmBK * 2, B_BYTES = BN * kGemmBK * 2;
  extern __shared__ unsigned char dsm[];
  __shared__ __align__(8) uint64_t bars[2 * STAGES + 1];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t base = (smem_u32(dsm) + 1023u) & ~1023u;
  const uint32_t sA = base, sB = base + STAGES * A_BYTES;
  const uint32_t full0 = smem_u32(&bars[0]), empty0 = smem_u32(&bars[STAGES]), done = smem_u32(&bars[2 * STAGES]);
  const int ntn = (g.N + BN - 1) / BN;
  const int m0 = (int)(blockIdx.x / ntn) * kGemmBM, n0 = (int)(blockIdx.x % ntn) * BN;
  const int z = g.z0 + (int)blockIdx.z, split = blockIdx.y;
  const int kb = (g.K + kGemmBK - 1) / kGemmBK;
  const int S = g.nseg * g.nprod * kb;
  const int j0 = (int)((long long)S * split / g.ksplit), j1 = (int)((long long)S * (split + 1) / g.ksplit);

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(done, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&a0) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&b0) : "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"((uint32_t)BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  volatile int* abort = &s_abort;
  // Launched as a programmatic dependent (the step-by-step scans), the set-up above overlaps
  // the previous kernel's tail; operands are read only below.  Without the launch
  // attribute both instructions do nothing.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (j1 > j0) {
    if (warp == 0 && lane == 0) {
      // ---- producer: TMA loads of the A / B tiles of each reduction step
      for (int j = j0; j < j1; ++j) {
        const int it = j - j0, s = it % STAGES;
        const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
        if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, g.spin_ns, abort)) break;
        const int kblk = j % kb, pj = j / kb, prod = pj % g.nprod, seg = pj / g.nprod;
        const int ia = g.pa[prod], ib = g.pb[prod];
        const CUtensorMap* ma = ia == 0 ? &a0 : (ia == 1 ? &a1 : &a2);
        const CUtensorMap* mb = ib == 0 ? &b0 : (ib == 1 ? &b1 : &b2);
        const int ak = kblk * kGemmBK + seg * g.a_k_seg + z * g.a_k_z;
        const int am = m0 + seg * g.a_mn_seg + z * g.a_mn_z;
        const int bk = kblk * kGemmBK + seg * g.b_k_seg + z * g.b_k_z;
        const int bm = n0 + seg * g.b_mn_seg + z * g.b_mn_z;
        mbar_expect_tx(full0 + 8 * s, A_BYTES + B_BYTES);
        if (AMN) {
#pragma unroll
          for (int q = 0; q < kGemmBM / 64; ++q)
            tma_load_2d(sA + s * A_BYTES + q * 8192, ma, am + 64 * q, ak, full0 + 8 * s);
        } else {
          tma_load_2d(sA + s * A_BYTES, ma, ak, am, full0 + 8 * s);
        }
        if (BMN) {
#pragma unroll
          for (int q = 0; q < BN / 64; ++q) tma_load_2d(sB + s * B_BYTES + q * 8192, mb, bm + 64 * q, bk, full0 + 8 * s);
        } else {
          tma_load_2d(sB + s * B_BYTES, mb, bk, bm, full0 + 8 * s);
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ---- MMA issuer: 4 MMAs of K=16 per 64-wide stage
      constexpr uint32_t idesc = umma_idesc_bf16(BN, AMN, BMN);
      constexpr uint64_t astep = AMN ? (2048 >> 4) : (32 >> 4), bstep = BMN ? (2048 >> 4) : (32 >> 4);
      for (int j = j0; j < j1; ++j) {
        const int it = j - j0, s = it % STAGES;
        const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
        if (!mbar_wait(full0 + 8 * s, ph, g.spin_ns, abort)) break;
        tc_fence_after();
        const uint64_t ad = umma_desc_sw128(sA + s * A_BYTES, AMN), bd = umma_desc_sw128(sB + s * B_BYTES, BMN);
#pragma unroll
        for (int kk = 0; kk < kGemmBK / 16; ++kk)
          umma_bf16(tmem, ad + astep * kk, bd + bstep * kk, idesc, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(empty0 + 8 * s);
      }
      umma_commit(done);   // arrives once every MMA issued above has completed
    }
  }
  __syncwarp();

  // ---- epilogue: warp w holds rows m0 + 32 w + lane of the tile
  const bool have = j1 > j0;
  bool ok = true;
  if (have) ok = mbar_wait(done, 0, g.spin_ns, abort);
  __syncwarp();
  tc_fence_after();
  const int m = m0 + warp * 32 + lane;
  float* drow = g.D + (size_t)blockIdx.z * g.d_z + (size_t)split * g.d_split + (size_t)m * g.ldd;
  const bool vec = (g.ldd % 4 == 0) && ((((uintptr_t)g.D) & 15) == 0) && (g.d_z % 4 == 0) && (g.d_split % 4 == 0);
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    float v[32];
    if (have && ok) {
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), v);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0.f;
    }
    if (!ok || m >= g.M) continue;
    const int nb = n0 + c * 32;
    if (nb >= g.N) continue;
    if (g.mode == GEMM_MASKED) {
      const uint8_t* mrow = g.mask + (size_t)m * g.ldmask;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (nb + i < g.N && mrow[(size_t)(nb + i) * g.mask_cs] == (uint8_t)z) drow[nb + i] = v[i];
    } else if (vec && nb + 32 <= g.N) {
      float4* d4 = (float4*)(drow + nb);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 w = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        if (g.mode == GEMM_ACCUM) {
          const float4 o = d4[q];
          w.x += o.x; w.y += o.y; w.z += o.z; w.w += o.w;
        }
        d4[q] = w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (nb + i < g.N) drow[nb + i] = g.mode == GEMM_ACCUM ? drow[nb + i] + v[i] : v[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN)
                              : "memory");
}

// Sum of the split partials in split order (deterministic), then the output mode.
__global__ void k_gemm_reduce(int M, int N, int ksplit, const float* __restrict__ part, long long p_split,
                              long long p_z, long long ldp, float* __restrict__ D, long long ldd, long long d_z,
                              int mode, const uint8_t* __restrict__ mask, long long ldmask, long long mask_cs,
                              int z0) {
  asm volatile("griddepcontrol.wait;" ::: "memory");   // no-op unless launched as a dependent
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int zi = blockIdx.y, z = z0 + zi;
  const size_t total = (size_t)M * N;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(e / N), n = (int)(e % N);
    const float* p = part + (size_t)zi * p_z + (size_t)m * ldp + n;
    float s = 0.f;
    for (int k = 0; k < ksplit; ++k) s += p[(size_t)k * p_split];
    float* d = D + (size_t)zi * d_z + (size_t)m * ldd + n;
    if (mode == GEMM_MASKED) {
      if (mask[(size_t)m * ldmask + (size_t)n * mask_cs] == (uint8_t)z) *d = s;
    } else if (mode == GEMM_ACCUM) {
      *d += s;
    } else {
      *d = s;
    }
  }
}


// ---- host side -------------------------------------------------------------------------
typedef CUresult (*TmapEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver (looked up once; no link-time libcuda dependency)
static TmapEncodeFn tmap_encoder() {
  static TmapEncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (TmapEncodeFn)p;
  }
  return fn;
}

// A bf16 matrix of `rows` x `cols` (row stride ld elements) read as 64-column x box_rows
// boxes with the 128-byte swizzle; reads outside [0,cols) x [0,rows) return zeros.
static bool tmap_bf16(CUtensorMap* m, const void* base, long long cols, long long rows, long long ld, int box_rows) {
  TmapEncodeFn fn = tmap_encoder();
  if (!fn || !base || cols < 1 || rows < 1 || ((uintptr_t)base & 15) || ((ld * 2) & 15) || ld < cols) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)kGemmBK, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Operand pieces of one side: up to 3 bf16 matrices of the same shape and stride.
//  K-major (mn_major = 0): rows = the M (or N) index, cols = the reduction index;
//  MN-major (mn_major = 1): rows = the reduction index, cols = the M (or N) index.
struct GemmSide {
  const void* p[3];
  int n;               // pieces
  long long rows, cols, ld;
  int mn_major;
};

// Reduction split: long reductions are cut into parts of at most ~24K products-times-
// elements, whose fp32 partials are summed outside the tensor core (its accumulator
// loses accuracy over very long sums), and grids of fewer tiles than SMs are split
// further, to the count that costs the fewest waves per unit of work (one CTA per SM:
// 144 CTAs of 16 tiles x 9 parts run in one wave where 16 x 10 would take two).
// At most max_ks parts and at least min_stages stages of 64 per part.
static int gemm_pick_ksplit(int M, int N, int K, int nprod, int nseg, int nz, int BN, int max_ks = 32,
                            int min_stages = 8) {
  const long long tiles = (long long)((M + kGemmBM - 1) / kGemmBM) * ((N + BN - 1) / BN) * nz;
  const long long steps = (long long)nseg * nprod * ((K + kGemmBK - 1) / kGemmBK);
  const long long cap = std::max<long long>(1, std::min<long long>(max_ks, steps / min_stages));
  long long ks = std::min<long long>(cap, std::max<long long>(1, (steps * kGemmBK + 24575) / 24576));
  if (tiles < 148) {
    long long best = ks;
    double best_cost = (double)((tiles * ks + 147) / 148) / (double)ks;
    for (long long k = ks + 1; k <= cap; ++k) {
      const double cost = (double)((tiles * k + 147) / 148) / (double)k;
      if (cost < best_cost - 1e-9) {
        best = k;
        best_cost = cost;
      }
    }
    ks = best;
  }
  return (int)ks;
}
// output columns per tile: the widest of 64 / 128 / 256 that the output needs
static int gemm_pick_bn(int N) { return N <= 64 ? 64 : (N <= 128 ? 128 : 256); }

// bytes of split-K partials a gemm_run call with these sizes needs from its workspace
static size_t gemm_partial_bytes(int M, int N, int ksplit, int nz, bool keep_parts = false) {
  return (ksplit > 1 || keep_parts) ? align256((size_t)M * N * ksplit * nz * sizeof(float)) : 0;
}

template <int BN, bool AMN, bool BMN>
static int gemm_launch_t(const CUtensorMap* ma, const CUtensorMap* mb, const GemmArgs& g, int nz, cudaStream_t st,
                         bool pdl) {
  static bool attr_set[64] = {false};   // per device
  const size_t smem = gemm_smem_bytes(BN);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DELREC_ERR_CUDA;
  auto kern = k_gemm_tc<BN, AMN, BMN>;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return DELREC_ERR_CUDA;
    attr_set[dev] = true;
  }
  const int tiles = ((g.M + kGemmBM - 1) / kGemmBM) * ((g.N + BN - 1) / BN);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles, g.ksplit, nz);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, ma[0], ma[1], ma[2], mb[0], mb[1], mb[2], g) != cudaSuccess) return DELREC_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? DELREC_OK : DELREC_ERR_CUDA;
}
template <bool AMN, bool BMN>
static int gemm_launch_bn(int BN, const CUtensorMap* ma, const CUtensorMap* mb, const GemmArgs& g, int nz,
                          cudaStream_t st, bool pdl = false) {
  return BN == 64 ? gemm_launch_t<64, AMN, BMN>(ma, mb, g, nz, st, pdl)
                  : (BN == 128 ? gemm_launch_t<128, AMN, BMN>(ma, mb, g, nz, st, pdl)
                               : gemm_launch_t<256, AMN, BMN>(ma, mb, g, nz, st, pdl));
}

// A GEMM with its tensor maps encoded once, for loops that launch the same product many
// times (the step-by-step scans): gemm_prepare validates and encodes, gemm_exec launches,
// optionally into another destination D of the same shape.
struct GemmLaunch {
  CUtensorMap ma[3], mb[3];
  GemmArgs g;                 // as launched (D = the partials when the reduction is split)
  int nz, BN;
  bool amn, bmn;
  bool split;                 // partials summed by k_gemm_reduce into D
  float* D;                   // final destination and its layout / mode
  long long ldd, d_z;
  int mode;
  float* part;
};

static int gemm_prepare(const GemmSide& A, const GemmSide& B, GemmArgs g, int nz, int BN, float* part,
                        GemmLaunch* L) {
  if (g.M < 1 || g.N < 1 || g.K < 1 || nz < 1 || g.nprod < 1 || g.nprod > kGemmMaxProd || g.nseg < 1)
    return DELREC_ERR_ARG;
  if (g.ksplit < 1) g.ksplit = 1;
  if (BN != 64 && BN != 128 && BN != 256) return DELREC_ERR_ARG;
  // the contiguous coordinate of a tensor-map box must stay 16-byte aligned
  const int a_contig = (A.mn_major ? (g.a_mn_seg | g.a_mn_z) : (g.a_k_seg | g.a_k_z));
  const int b_contig = (B.mn_major ? (g.b_mn_seg | g.b_mn_z) : (g.b_k_seg | g.b_k_z));
  if ((a_contig & 7) || (b_contig & 7)) return DELREC_ERR_ARG;
  for (int p = 0; p < g.nprod; ++p)
    if (g.pa[p] < 0 || g.pa[p] >= A.n || g.pb[p] < 0 || g.pb[p] >= B.n) return DELREC_ERR_ARG;
  for (int i = 0; i < 3; ++i) {
    const int ia = i < A.n ? i : 0, ib = i < B.n ? i : 0;
    if (!tmap_bf16(&L->ma[i], A.p[ia], A.cols, A.rows, A.ld, A.mn_major ? 64 : kGemmBM)) return DELREC_ERR_ARG;
    if (!tmap_bf16(&L->mb[i], B.p[ib], B.cols, B.rows, B.ld, B.mn_major ? 64 : BN)) return DELREC_ERR_ARG;
  }
  if (g.spin_ns <= 0) g.spin_ns = 2000000000ll;
  L->D = g.D;
  L->ldd = g.ldd;
  L->d_z = g.d_z;
  L->mode = g.mode;
  L->part = part;
  const bool keep_parts = g.mode == GEMM_PARTIALS;
  L->split = g.ksplit > 1 && !keep_parts;
  if (g.ksplit > 1 || keep_parts) {
    if (!part) return DELREC_ERR_WORKSPACE;
    g.D = part;
    g.ldd = g.N;
    g.d_split = (long long)g.M * g.N;
    g.d_z = g.d_split * g.ksplit;
    g.mode = GEMM_STORE;
  }
  L->g = g;
  L->nz = nz;
  L->BN = BN;
  L->amn = A.mn_major != 0;
  L->bmn = B.mn_major != 0;
  return DELREC_OK;
}

// pdl: the GEMM (and its reduce) are launched as programmatic dependents of the work
// before them on the stream (both wait for it before reading anything)
static int gemm_exec(const GemmLaunch& L, float* D, cudaStream_t st, unsigned long long* launches,
                     bool pdl = false) {
  GemmArgs g = L.g;
  float* dst = D ? D : L.D;
  if (!L.split && L.mode != GEMM_PARTIALS) g.D = dst;
  int rc;
  if (L.amn)
    rc = L.bmn ? gemm_launch_bn<true, true>(L.BN, L.ma, L.mb, g, L.nz, st, pdl)
               : gemm_launch_bn<true, false>(L.BN, L.ma, L.mb, g, L.nz, st, pdl);
  else
    rc = L.bmn ? gemm_launch_bn<false, true>(L.BN, L.ma, L.mb, g, L.nz, st, pdl)
               : gemm_launch_bn<false, false>(L.BN, L.ma, L.mb, g, L.nz, st, pdl);
  if (rc) return rc;
  ++*launches;
  if (L.split) {
    const size_t total = (size_t)g.M * g.N;
    int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 8);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(blocks, L.nz);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_gemm_reduce, g.M, g.N, g.ksplit, (const float*)L.part, (long long)g.d_split,
                           (long long)g.d_z, (long long)g.N, dst, (long long)L.ldd, (long long)L.d_z, L.mode,
                           g.mask, (long long)g.ldmask, (long long)g.mask_cs, g.z0) != cudaSuccess)
      return DELREC_ERR_CUDA;
    ++*launches;
  }
  return DELREC_OK;
}

// D (mode) = sum over products of A-pieces x B-pieces^T, see GemmArgs.  `g` carries the
// sizes, products, shifts, output and mode; ksplit > 1 runs the reduction in that many
// parts whose fp32 partials (in `part`, gemm_partial_bytes) are summed in a fixed order.
static int gemm_run(const GemmSide& A, const GemmSide& B, GemmArgs g, int nz, int BN, float* part, cudaStream_t st,
                    unsigned long long* launches) {
  GemmLaunch L;
  const int rc = gemm_prepare(A, B, g, nz, BN, part, &L);
  return rc ? rc : gemm_exec(L, nullptr, st, launches);
}

}  // namespace delrec
