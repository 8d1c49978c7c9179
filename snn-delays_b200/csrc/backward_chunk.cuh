// Chunked reverse scan of a hybrid (or axonal) delay layer: the delay contraction of the
// synapses whose lag reaches past the current chunk of time steps runs as a tensor-core
// GEMM once per chunk; only the short-lag synapses stay in the step-by-step SIMT loop.
//
// Notation (hybrid layer, integer offsets k_io in [0, K], base taps of source o at lags
// l0_o + j >= 1 with weights w_oj):
//   G_k(tau)[b,o] = sum_i W[i,o] [k_io == k] gr(tau)[b,i]       (per-offset masked product)
//   gz(s)[b,o]    = sum_k G_k(s + k)[b,o]                         (the delayed gradient)
//   gfut(t)[b,o]  = sum_j w_oj gz(t + l0_o + j)[b,o]              (input of the LIF backward)
//
// Time is cut into chunks of C = 8 steps, processed from the last one down.  For chunk
// [t0, t0 + C):
//   1. k_bwd_chunk runs the C reverse LIF steps (one cooperative launch).  gfut(t) reads
//      gz(s) from global memory -- which already holds every contribution of gr(tau) for
//      tau >= t0 + C (the later chunks' GEMMs) -- plus a per-source ring in shared memory
//      with the contributions of this chunk's own gr(tau), tau in (t, t0 + C).  Such a
//      contribution can reach a step of this chunk only through a synapse with
//      l0_o + k_io <= tau - t0 <= C - 1; those short synapses are the only ones summed on
//      the CUDA cores (12 % of them at BASELINE config 4, 0.45 % on the critical path).
//      The step also writes gr(t) as bf16 hi/lo pieces in a sample-major (B, T, N) layout.
//   2. k_chunk_gz computes G_k(tau) for every tau of the chunk, every sample, source and
//      offset on the tensor cores (tcgen05, M = 128 rows = 16 samples x 8 steps, N = 256
//      columns = (source, offset) pairs, reduction over the N targets with the products
//      hi.hi + hi.lo + lo.hi of the bf16 pieces, fp32 accumulation) and adds the shifted
//      sums sum_k G_k(s + k) into gz(s) for s in [t0 - 8, t0 + 7].
// Every gz element receives at most one add per launch and the launches are ordered on
// the stream, so the result does not depend on scheduling.  gz is complete for s once the
// GEMMs of all chunks holding s .. s + K have run, i.e. before the source pass reads it.
#pragma once

#include <cuda_bf16.h>

#include "backward_hybrid64.cuh"
#include "gemm_tc.cuh"

namespace delrec {

constexpr int kChunk = 8;   // time steps per chunk; also the ring slots of the SIMT scan

struct ChunkArgs {
  int T, B, N, K, CS, NT, TAPS, CAPS, CAP, boff_stride;
  int t0, t_hi;            // this launch runs steps t_hi .. t0 (reverse); t_hi < t0 + kChunk
  const float* gy;
  const float* u;
  const float* keep;
  const int* tap_l0;
  const int* tap_nt;
  const float* tap_w;
  const int2* ent;         // (N, CAP) bucket entries (i, weight bits), buckets padded to 8
  const int* boff;         // bucket k of source o starts at boff[o*boff_stride + k]
  float* dx;
  float* gr;
  const float* gz;         // (T,B,N): all contributions of gr(tau), tau >= t0 + kChunk
  __nv_bfloat16* ga_hi;    // (B, T, Np) bf16 pieces of gr for the chunk GEMM
  __nv_bfloat16* ga_lo;
  int Np;
  float* lam;              // (B, N) LIF gradient carried from step t0 to step t0 - 1
  LifK lif;
  float* grx;              // [2][tiles][N][64] exchange of gr(t)
  unsigned int* arrive;    // [tiles] arrival counters, zeroed once before the first chunk
  unsigned int arr_base;   // arrivals per tile published by the earlier chunks of this scan
  long long spin_limit;
};

template <int TPF>
__global__ void __launch_bounds__(512, 1) k_bwd_chunk(ChunkArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_abort;
  constexpr int BT = kH64BT, NTH = kH64Threads, PPT = 2, RING = kChunk;
  const int NT = a.NT;
  const int rank = (int)(blockIdx.x % a.CS), tile = (int)(blockIdx.x / a.CS);
  const int tiles = (int)(gridDim.x / a.CS);
  const int N = a.N, T = a.T, B = a.B, K = a.K, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int o0 = rank * NT;
  const int nts = max(0, min(NT, N - o0));
  const int b0 = tile * BT;
  const int nb = max(0, min(BT, B - b0));
  const size_t BN = (size_t)B * N;
  const int t0 = a.t0, t_hi = a.t_hi;

  const Hyb64Smem P = hyb64_smem_plan(N, NT, a.CAPS, K, a.TAPS, RING);
  const int RS = P.ring_stride;
  float* grc = (float*)smem;                                                   // [N][64]
  uint16_t* sidx = (uint16_t*)(smem + P.grc);                                  // [NT][CAPS]
  float* sw = (float*)(smem + P.grc + P.idx);                                  // [NT][CAPS]
  int* sbo = (int*)(smem + P.grc + P.idx + P.w);                               // [NT][K+2]
  int* surg = sbo + NT * (K + 2);                                              // [NT]
  int* tl0 = (int*)(smem + P.grc + P.idx + P.w + P.boff);                      // [NT]
  int* tnt = tl0 + NT;
  float* tw = (float*)(tnt + NT);                                              // [NT][TAPS]
  float* ring = (float*)(smem + P.grc + P.idx + P.w + P.boff + P.taps);        // [NT][RS]

  // ---- init: taps and bucket offsets first (small), then only the short buckets
  // (k <= C - 1 - l0) of the block's sources, one warp per source, and the ring
  for (int ol = tid; ol < NT; ol += NTH) {
    const bool ok = ol < nts;
    tl0[ol] = ok ? a.tap_l0[o0 + ol] : RING;
    tnt[ol] = ok ? a.tap_nt[o0 + ol] : 0;
    surg[ol] = ok && a.tap_l0[o0 + ol] <= 1;
  }
  for (int e = tid; e < NT * (K + 2); e += NTH) {
    const int ol = e / (K + 2);
    int off = ol < nts ? a.boff[(size_t)(o0 + ol) * a.boff_stride + e % (K + 2)] : 0;
    if (off > a.CAPS) {
      flag_status(ST_INDEX_RANGE);
      off = a.CAPS;
    }
    sbo[e] = off;
  }
  for (int e = tid; e < NT * a.TAPS; e += NTH) {
    const int ol = e / a.TAPS;
    tw[e] = ol < nts ? a.tap_w[(size_t)(o0 + ol) * a.TAPS + (e % a.TAPS)] : 0.f;
  }
  for (int e = tid; e < NT * RS; e += NTH) ring[e] = 0.f;
  if (tid == 0) s_abort = 0;
  __syncthreads();
  // entries past a source's short prefix are never read, so they are not loaded
  for (int ol = warp; ol < nts; ol += NTH / 32) {
    const int kl = min(K, RING - 1 - tl0[ol]);
    const int tot = kl >= 0 ? sbo[ol * (K + 2) + kl + 1] : 0;
    const int2* src = a.ent + (size_t)(o0 + ol) * a.CAP;
    for (int pos = lane; pos < tot; pos += 32) {
      const int2 en = src[pos];
      sidx[(size_t)ol * a.CAPS + pos] = (uint16_t)en.x;
      sw[(size_t)ol * a.CAPS + pos] = __int_as_float(en.y);
    }
  }
  __syncthreads();

  int pol[PPT], pbl[PPT];
  bool pin[PPT], pok[PPT];
  float lam[PPT], kp[PPT];
  float pf_gy[PPT], pf_u[PPT], pf_tap[PPT][TPF];
  LifPre pf_pre[PPT];
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    const int p = tid + k * NTH;
    pol[k] = p % NT;
    pbl[k] = p / NT;
    pin[k] = pol[k] < nts && pbl[k] < BT;
    pok[k] = pin[k] && pbl[k] < nb;
    const size_t pe = (size_t)(b0 + pbl[k]) * N + o0 + pol[k];
    lam[k] = (pok[k] && t_hi < T - 1) ? a.lam[pe] : 0.f;
    kp[k] = (pok[k] && a.keep) ? a.keep[pe] : 1.f;
  }
  auto prefetch_lif = [&](int t) {
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      pf_gy[k] = 0.f;
      pf_u[k] = 0.f;
      if (pok[k] && t >= t0) {
        const size_t idx = ((size_t)t * B + b0 + pbl[k]) * N + o0 + pol[k];
        pf_gy[k] = __ldcs(a.gy + idx);
        pf_u[k] = __ldcs(a.u + idx);
      }
    }
  };
  // gz(t + l) for every tap: the part of the later chunks (read-only during this launch)
  auto prefetch_taps = [&](int t) {
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
#pragma unroll
      for (int j = 0; j < TPF; ++j) pf_tap[k][j] = 0.f;
      if (pok[k] && t >= t0) {
        const size_t idx = ((size_t)t * B + b0 + pbl[k]) * N + o0 + pol[k];
        const int lo = tl0[pol[k]], n = tnt[pol[k]];
#pragma unroll
        for (int j = 0; j < TPF; ++j) {
          const int l = lo + j;
          if (j < n && t + l < T && tw[pol[k] * a.TAPS + j] != 0.f)
            pf_tap[k][j] = __ldcg(a.gz + idx + (size_t)l * BN);
        }
      }
    }
  };
  prefetch_lif(t_hi);
  prefetch_taps(t_hi);
#pragma unroll
  for (int k = 0; k < PPT; ++k) pf_pre[k] = lif_bwd_prep(pf_u[k], a.lif);

  const uint32_t gbase = (uint32_t)__cvta_generic_to_shared(grc) + lane * 8;
  const int ol_w = warp;   // the warp's source
  const uint16_t* wix = sidx + (size_t)ol_w * a.CAPS;
  const float* wwv = sw + (size_t)ol_w * a.CAPS;
  const int* wbo = sbo + ol_w * (K + 2);
  float* wring = ring + (size_t)ol_w * RS + 2 * lane;
  const bool w_ok = ol_w < nts;
  const bool w_urg = w_ok && surg[ol_w];
  const int w_l0 = w_ok ? tl0[ol_w] : RING;
  unsigned int arrivals = a.arr_base;
  const size_t xtile = (size_t)N * BT;

  for (int t = t_hi; t >= t0; --t) {
    float cur_gy[PPT], cur_tap[PPT][TPF];
    LifPre cur_pre[PPT];
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      cur_gy[k] = pf_gy[k];
      cur_pre[k] = pf_pre[k];
#pragma unroll
      for (int j = 0; j < TPF; ++j) cur_tap[k][j] = pf_tap[k][j];
    }
    prefetch_lif(t - 1);
    float* xb = a.grx + ((size_t)(t & 1) * tiles + tile) * xtile;
    // ===== A: LIF backward of the block's pairs
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int ol = pol[k], bl = pbl[k];
      if (!pin[k]) continue;
      float grv = 0.f;
      const float* rrow = ring + (size_t)ol * RS + bl;
      if (pok[k]) {
        const int lo = tl0[ol], n = tnt[ol];   // n <= TAPS <= TPF (checked by the planner)
        float gfut = 0.f;
#pragma unroll
        for (int j = 0; j < TPF; ++j) {
          const int l = lo + j;
          if (j < n && t + l < T) {
            float g = cur_tap[k][j];
            if (t + l <= t_hi) g += rrow[((t + l) % RING) * 64];
            gfut = fmaf(tw[ol * a.TAPS + j], g, gfut);
          }
        }
        const float gY = __fadd_rn(cur_gy[k], gfut);
        const float du = lif_backward_pre(gY, lam[k], cur_pre[k], a.lif);
        lam[k] = lif_carry(du, a.lif);
        grv = __fmul_rn(du, kp[k]);
        const int o = o0 + ol, b = b0 + bl;
        const size_t idx = ((size_t)t * B + b) * N + o;
        a.dx[idx] = du;
        if (a.gr != a.dx) a.gr[idx] = grv;   // (gr is dx itself without dropout)
        const __nv_bfloat16 h = __float2bfloat16_rn(grv);
        const size_t ai = ((size_t)b * T + t) * a.Np + o;
        a.ga_hi[ai] = h;
        a.ga_lo[ai] = __float2bfloat16_rn(grv - __bfloat162float(h));
      }
      __stcg(xb + (size_t)(o0 + ol) * BT + bl, grv);
    }
    __syncthreads();
    if (tid == 0) {   // release: the block's exchange writes (ordered by the barrier) first
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      atomicAdd(a.arrive + tile, 1u);
    }
    arrivals += a.CS;
    // ===== C1: the short synapses of gr(t+1) (staged at step t+1) into slots t+1-k.
    // A contribution to slot s is read at step s - l0 - j, inside this chunk only when
    // s >= t0 + l0, i.e. k <= (t + 1 - t0) - l0.
    if (w_ok && t + 1 <= t_hi) {
      const int kmax = min(K, t + 1 - t0 - w_l0);
      for (int k = kmax; k >= 0; --k) {
        if (k == 0 && w_urg) continue;
        const int tau = t + 1 - k;
        const int beg = wbo[k], end = wbo[k + 1];
        if (((beg | end) & 7) != 0) { flag_status(ST_INDEX_RANGE); continue; }
        const float2 s = h64_bucket(wix, wwv, beg, end, gbase);
        float2* cell = (float2*)(wring + (tau % RING) * 64);
        float2 c = *cell;
        c.x += s.x;
        c.y += s.y;
        *cell = c;
      }
    }
    prefetch_taps(t - 1);
#pragma unroll
    for (int k = 0; k < PPT; ++k) pf_pre[k] = lif_bwd_prep(pf_u[k], a.lif);
    // gr(t0) reaches no step of this chunk: the last step neither waits nor stages
    if (t > t0) {
      __syncthreads();   // C1 done reading the staged gr(t+1)
      // ===== W: the tile's gr(t)
      if (tid == 0) {
        long long polls = 0;
        unsigned int seen;
        do {
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(a.arrive + tile) : "memory");
          if (++polls > a.spin_limit) { flag_status(ST_TIMEOUT); s_abort = 1; break; }
        } while (seen < arrivals);
      }
      __syncthreads();
      if (s_abort) return;
      {
        const int n4 = N * BT / 4;
        const float4* xs = (const float4*)xb;
        float4* gd = (float4*)grc;
        for (int v = tid; v < n4; v += NTH) gd[v] = __ldcg(xs + v);
      }
      __syncthreads();
      // ===== C2: offset 0 of a source with a lag-1 tap (read at step t - 1)
      if (w_urg) {
        const int beg = wbo[0], end = wbo[1];
        if (((beg | end) & 7) != 0) {
          flag_status(ST_INDEX_RANGE);
        } else {
          const float2 s = h64_bucket(wix, wwv, beg, end, gbase);
          float2* cell = (float2*)(wring + (t % RING) * 64);
          float2 c = *cell;
          c.x += s.x;
          c.y += s.y;
          *cell = c;
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int k = 0; k < PPT; ++k)
    if (pok[k]) a.lam[(size_t)(b0 + pbl[k]) * N + o0 + pol[k]] = lam[k];
}

// The latency floor of the step-by-step part of the reverse scans: the same grid, block
// size, shared memory and per-tile exchange as k_bwd_chunk / k_bwd_hybrid64, but nothing
// else -- per step each block publishes its slice of the tile's gr row block to L2,
// release-arrives at the tile counter, waits for the tile and restages the tile's N x 64
// values into shared memory.  T steps of it bound any scan that exchanges gr every step.
__global__ void __launch_bounds__(512, 1) k_exchange_floor(int T, int N, int CS, int NT, float* grx,
                                                           unsigned int* arrive, long long spin_limit) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_abort;
  float* grc = (float*)smem;   // [N][64]
  constexpr int BT = kH64BT, NTH = kH64Threads;
  const int tid = threadIdx.x;
  const int rank = (int)(blockIdx.x % CS), tile = (int)(blockIdx.x / CS), tiles = (int)(gridDim.x / CS);
  const int o0 = rank * NT, nts = max(0, min(NT, N - o0));
  const size_t xtile = (size_t)N * BT;
  for (int e = tid; e < N * BT; e += NTH) grc[e] = 0.f;
  if (tid == 0) s_abort = 0;
  __syncthreads();
  unsigned int arrivals = 0;
  for (int t = T - 1; t >= 0; --t) {
    float* xb = grx + ((size_t)(t & 1) * tiles + tile) * xtile;
    for (int e = tid; e < nts * BT; e += NTH) __stcg(xb + (size_t)o0 * BT + e, grc[(size_t)o0 * BT + e]);
    __syncthreads();
    if (tid == 0) {
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      atomicAdd(arrive + tile, 1u);
    }
    arrivals += CS;
    if (tid == 0) {
      long long polls = 0;
      unsigned int seen;
      do {
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(arrive + tile) : "memory");
        if (++polls > spin_limit) { flag_status(ST_TIMEOUT); s_abort = 1; break; }
      } while (seen < arrivals);
    }
    __syncthreads();
    if (s_abort) return;
    const float4* xs = (const float4*)xb;
    float4* gd = (float4*)grc;
    for (int v = tid; v < N * BT / 4; v += NTH) gd[v] = __ldcg(xs + v);
    __syncthreads();
  }
}

// ---- the chunk GEMM ---------------------------------------------------------------------
// Reduction blocks of 32 (64-byte rows, 64-byte swizzle) in a four-stage ring: a stage is
// 48 KB (both pieces of A and B), so three stages are in flight while the MMAs read one.
constexpr int kGzRows = 128, kGzCols = 256, kGzSamples = kGzRows / kChunk, kGzK = 32, kGzStages = 4;
// sources per column tile: as many as 256 columns hold, rounded down to a multiple of 4 (the
// epilogue adds groups of 4 consecutive sources with one vector reduction)
__host__ __device__ constexpr int gz_ntg(int KP1) { return (kGzCols / KP1) & ~3; }
constexpr uint32_t kGzABytes = kGzRows * kGzK * 2, kGzBBytes = kGzCols * kGzK * 2;
constexpr uint32_t kGzStageBytes = 2 * kGzABytes + 2 * kGzBBytes;
constexpr size_t kGzSmem = (size_t)kGzStages * kGzStageBytes + 1024;

constexpr int kGzEpiWarps = 4, kGzThreads = 64 + 32 * kGzEpiWarps;

// The last column tile holds the sources left over (N - (ntiles-1) * gz_ntg); its MMAs
// are `ncl` columns wide (the used columns rounded up to 16) and its B boxes `ncl` rows.
struct GzArgs {
  int T, B, N, t0, ntiles, ncl;
  float* gz;
  long long spin_ns;
};

// Work items of one launch: tile n * tiles_m + m of each full column block (n < ntiles-1),
// then the last column block's sample tiles, two per item (m = 2r, 2r+1) when that block
// is at most 128 columns wide: both tiles share the item's B stage and one accumulator
// (columns 0.. and 128..), so a launch has fewer items to spread over the SMs.
struct GzItem {
  int n, m;
  bool two;
};
__host__ __device__ inline int gz_items(int tiles_m, int ntiles, int ncl) {
  return (ntiles - 1) * tiles_m + (ncl <= kGzCols / 2 ? (tiles_m + 1) / 2 : tiles_m);
}
__device__ __forceinline__ GzItem gz_item(int it, int tiles_m, int ntiles, int ncl) {
  const int nfull = (ntiles - 1) * tiles_m;
  GzItem w;
  if (it < nfull) {
    w.n = it / tiles_m;
    w.m = it % tiles_m;
    w.two = false;
  } else if (ncl <= kGzCols / 2) {
    w.n = ntiles - 1;
    w.m = 2 * (it - nfull);
    w.two = w.m + 1 < tiles_m;
  } else {
    w.n = ntiles - 1;
    w.m = it - nfull;
    w.two = false;
  }
  return w;
}

// Shared-memory descriptor of a K-major tile written by TMA with the 64-byte swizzle (tile
// base 512-aligned): rows of 64 bytes (32 reduction elements), 8-row groups 512 bytes
// apart; the next K=16 slice starts 32 bytes further.
__device__ __forceinline__ uint64_t umma_desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);   // start address
  d |= (uint64_t)1 << 16;                      // leading byte offset (unused when swizzled)
  d |= (uint64_t)(512 >> 4) << 32;             // stride byte offset
  d |= (uint64_t)1 << 46;                      // descriptor version
  d |= (uint64_t)4 << 61;                      // 64-byte swizzle
  return d;
}

// gz[0..3] += v (one vector reduction; gz 16-byte aligned)
__device__ __forceinline__ void red_add_v4(float* gz, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(gz), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"((unsigned long long)map), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// Persistent chunk GEMM: one CTA per SM walks the work items (gz_item: tile n * tiles_m + m
// of the full column blocks, so the CTAs of a wave share the masked-W tile of their column
// block through L2; then the last block's tiles, in pairs when it is narrow).
// A tile is 16 samples x the chunk's 8 steps (rows b*8 + q) against 256 (source, offset)
// columns (source-major, KP1 = K+1 offsets per source, gz_ntg(KP1) sources per tile);
// A = gr pieces from the (B, T, Np) layout through a 3-D tensor map (box 32 x 8 x 16),
// B = the offset-masked W pieces (tile rows of 256, K-major; the last column tile's maps
// have boxes of ncl rows).
// Warp roles: warp 0 streams the pieces of each 32-wide reduction block (A of the item's
// one or two sample tiles, B) through a four-stage ring (TMA, per-CTA loads); warp 1 issues
// 6 MMAs per block and sample tile (3 products x 2 K-steps) into one of two tensor-memory
// accumulators (256 columns each; a paired item's second tile at column 128), so the MMAs
// of the next item run while warps 2..5 drain the previous one; the epilogue warps read
// their 32-lane quarter of the accumulator (thread = row (b, q)), form the shift sums over
// the offsets with shuffles inside each sample's 8-lane group, and add them into gz.
template <int KP1>
__global__ void __launch_bounds__(kGzThreads, 1)
    k_chunk_gz(const __grid_constant__ CUtensorMap mahi, const __grid_constant__ CUtensorMap malo,
               const __grid_constant__ CUtensorMap mbhi, const __grid_constant__ CUtensorMap mblo,
               const __grid_constant__ CUtensorMap mlhi, const __grid_constant__ CUtensorMap mllo, const GzArgs g) {
  static_assert(KP1 >= 1 && KP1 <= kChunk + 1, "offset window wider than two chunks");
  constexpr int NTG = gz_ntg(KP1), USED = NTG * KP1;
  extern __shared__ unsigned char dsm[];
  __shared__ __align__(8) uint64_t bars[2 * kGzStages + 4];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t base = (smem_u32(dsm) + 1023u) & ~1023u;
  const uint32_t full0 = smem_u32(&bars[0]), empty0 = smem_u32(&bars[kGzStages]);
  const uint32_t accf0 = smem_u32(&bars[2 * kGzStages]), acce0 = smem_u32(&bars[2 * kGzStages + 2]);
  const int t0 = g.t0, kb = (g.N + kGzK - 1) / kGzK;
  const int tiles_m = (g.B + kGzSamples - 1) / kGzSamples, total = gz_items(tiles_m, g.ntiles, g.ncl);
  const int last_n = g.ntiles - 1;

  if (tid == 0) {
    for (int s = 0; s < kGzStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int q = 0; q < 2; ++q) {
      mbar_init(accf0 + 8 * q, 1);
      mbar_init(acce0 + 8 * q, kGzEpiWarps);
    }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&mahi) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&mbhi) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((unsigned long long)&mlhi) : "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"((uint32_t)(2 * kGzCols))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  volatile int* abort = &s_abort;
  // Launched as a programmatic dependent of the chunk's step kernel, the set-up above
  // overlaps that kernel's tail; the gr pieces and gz are read and added only below.
  // Without the launch attribute both instructions do nothing.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int item = blockIdx.x; item < total && !*abort; item += gridDim.x) {
        const GzItem w = gz_item(item, tiles_m, g.ntiles, g.ncl);
        const int b0 = w.m * kGzSamples, n0 = w.n * kGzCols;
        const bool narrow = w.n == last_n;
        const CUtensorMap* bh = narrow ? &mlhi : &mbhi;
        const CUtensorMap* bl = narrow ? &mllo : &mblo;
        const uint32_t bbytes = narrow ? (uint32_t)g.ncl * kGzK * 2 : kGzBBytes;
        for (int j = 0; j < kb; ++j, ++it) {
          const int s = it % kGzStages;
          const uint32_t ph = (uint32_t)(it / kGzStages) & 1u;
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, g.spin_ns, abort)) break;
          const uint32_t st = base + s * kGzStageBytes, fb = full0 + 8 * s;
          mbar_expect_tx(fb, (w.two ? 4u : 2u) * kGzABytes + 2u * bbytes);
          tma_load_3d(st, &mahi, j * kGzK, t0, b0, fb);
          tma_load_3d(st + kGzABytes, &malo, j * kGzK, t0, b0, fb);
          tma_load_2d(st + 2 * kGzABytes, bh, j * kGzK, n0, fb);
          tma_load_2d(st + 2 * kGzABytes + kGzBBytes, bl, j * kGzK, n0, fb);
          if (w.two) {   // the second tile's A pieces in the upper halves of the B regions
            tma_load_3d(st + 2 * kGzABytes + kGzBBytes / 2, &mahi, j * kGzK, t0, b0 + kGzSamples, fb);
            tma_load_3d(st + 2 * kGzABytes + kGzBBytes + kGzBBytes / 2, &malo, j * kGzK, t0, b0 + kGzSamples, fb);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_full = umma_idesc_bf16(kGzCols, false, false);
      const uint32_t idesc_narrow = (idesc_full & ~(0x3Fu << 17)) | ((uint32_t)(g.ncl >> 3) << 17);
      int it = 0, lt = 0;
      for (int item = blockIdx.x; item < total && !*abort; item += gridDim.x, ++lt) {
        const GzItem w = gz_item(item, tiles_m, g.ntiles, g.ncl);
        const uint32_t idesc = w.n == last_n ? idesc_narrow : idesc_full;
        const int acc = lt & 1;
        const uint32_t u = (uint32_t)(lt >> 1);
        // the epilogue has drained this accumulator's previous tile
        if (!mbar_wait(acce0 + 8 * acc, (u & 1u) ^ 1u, g.spin_ns, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * kGzCols);
        bool ok = true;
        for (int j = 0; j < kb; ++j, ++it) {
          const int s = it % kGzStages;
          const uint32_t ph = (uint32_t)(it / kGzStages) & 1u;
          if (!mbar_wait(full0 + 8 * s, ph, g.spin_ns, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t st = base + s * kGzStageBytes;
          const uint64_t ahi = umma_desc_sw64(st), alo = umma_desc_sw64(st + kGzABytes);
          const uint64_t bhi = umma_desc_sw64(st + 2 * kGzABytes);
          const uint64_t blo = umma_desc_sw64(st + 2 * kGzABytes + kGzBBytes);
#pragma unroll
          for (int kk = 0; kk < kGzK / 16; ++kk) {
            umma_bf16(d, ahi + 2 * kk, bhi + 2 * kk, idesc, (j > 0 || kk > 0) ? 1u : 0u);
            umma_bf16(d, ahi + 2 * kk, blo + 2 * kk, idesc, 1u);
            umma_bf16(d, alo + 2 * kk, bhi + 2 * kk, idesc, 1u);
          }
          if (w.two) {   // second sample tile into accumulator columns 128..
            const uint64_t a1hi = umma_desc_sw64(st + 2 * kGzABytes + kGzBBytes / 2);
            const uint64_t a1lo = umma_desc_sw64(st + 2 * kGzABytes + kGzBBytes + kGzBBytes / 2);
            const uint32_t d1 = d + (uint32_t)(kGzCols / 2);
#pragma unroll
            for (int kk = 0; kk < kGzK / 16; ++kk) {
              umma_bf16(d1, a1hi + 2 * kk, bhi + 2 * kk, idesc, (j > 0 || kk > 0) ? 1u : 0u);
              umma_bf16(d1, a1hi + 2 * kk, blo + 2 * kk, idesc, 1u);
              umma_bf16(d1, a1lo + 2 * kk, bhi + 2 * kk, idesc, 1u);
            }
          }
          umma_commit(empty0 + 8 * s);
        }
        if (!ok) break;
        umma_commit(accf0 + 8 * acc);   // arrives once this tile's MMAs have completed
      }
    }
  } else {
    // ---- epilogue warps 2..5: TMEM lane quarter qd = warp % 4 holds rows 32 qd + lane
    const int qd = warp & 3;
    const int q = lane & 7, grp = lane & 24;
    const size_t BN = (size_t)g.B * g.N;
    const bool vec = (g.N & 3) == 0;
    const int s0 = t0 + q, s1 = t0 + q - kChunk;
    int lt = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x, ++lt) {
      const GzItem w = gz_item(item, tiles_m, g.ntiles, g.ncl);
      const int acc = lt & 1;
      const uint32_t u = (uint32_t)(lt >> 1);
      const int ob = w.n * NTG;
      // columns the MMAs wrote (the narrow tile's columns past ncl hold an older tile's
      // values; they belong to sources >= N, whose sums are never added)
      const int wcols = w.n == last_n ? g.ncl : kGzCols;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(accf0 + 8 * acc, u & 1u, g.spin_ns, abort));
      if (!ok) break;
      tc_fence_after();
      for (int h = 0; h < (w.two ? 2 : 1); ++h) {   // sample tile m + h at accumulator column 128 h
        const int b = (w.m + h) * kGzSamples + qd * 4 + (lane >> 3);
        const bool brow = b < g.B;
        float* row0 = (brow && s0 < g.T) ? g.gz + (size_t)s0 * BN + (size_t)b * g.N : nullptr;
        float* row1 = (brow && s1 >= 0) ? g.gz + (size_t)s1 * BN + (size_t)b * g.N : nullptr;
        const uint32_t taddr = tmem + ((uint32_t)(qd * 32) << 16) + (uint32_t)(acc * kGzCols + h * (kGzCols / 2));
        float a0[4], a1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a0[i] = a1[i] = 0.f;
#pragma unroll
        for (int cc = 0; cc < kGzCols / 32; ++cc) {
          if (cc * 32 >= USED || cc * 32 >= wcols) break;
          float v[32];
          tmem_ld32(taddr + (uint32_t)(cc * 32), v);
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int c = cc * 32 + jj;
            if (c < USED) {
              const int k = c % KP1, ol = c / KP1, g4 = ol & 3;
              const int src = q + k;   // lane of row tau = t0 + src (window 0) or t0 + src - 8
              const float x = __shfl_sync(0xffffffffu, v[jj], grp | (src & 7));
              if (src < kChunk) a0[g4] += x;
              else a1[g4] += x;
              if (k == KP1 - 1 && g4 == 3) {   // sources ol-3 .. ol complete
                const int o = ob + ol - 3;
                if (vec) {
                  if (row0 && o < g.N) red_add_v4(row0 + o, a0[0], a0[1], a0[2], a0[3]);
                  if (row1 && o < g.N) red_add_v4(row1 + o, a1[0], a1[1], a1[2], a1[3]);
                } else {
#pragma unroll
                  for (int i = 0; i < 4; ++i) {
                    if (row0 && o + i < g.N) atomicAdd(row0 + o + i, a0[i]);
                    if (row1 && o + i < g.N) atomicAdd(row1 + o + i, a1[i]);
                  }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) a0[i] = a1[i] = 0.f;
              }
            }
          }
        }
      }
      // the accumulator's reads are complete: hand it back to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(acce0 + 8 * acc) : "memory");
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 2)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * kGzCols))
                 : "memory");
}

// Offset-masked W as the GEMM's B operand: row r = tile * 256 + c, c = ol * KP1 + k
// (source o = tile * gz_ntg(KP1) + ol, offset k), column i (target):
// value W[i, o] if offsets[i, o] == k, else 0; written as bf16 hi + lo pieces with row
// stride Np (columns >= N and unused rows are zero).
__global__ void k_mask_w(int N, int Np, int KP1, int rows, const float* __restrict__ W,
                         const uint8_t* __restrict__ offT, __nv_bfloat16* __restrict__ hi,
                         __nv_bfloat16* __restrict__ lo) {
  const int NTG = gz_ntg(KP1);
  const size_t total = (size_t)rows * Np;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / Np), i = (int)(e % Np);
    const int tile = r / kGzCols, c = r % kGzCols;
    const int ol = c / KP1, k = c % KP1, o = tile * NTG + ol;
    float v = 0.f;
    if (c < NTG * KP1 && o < N && i < N && (offT ? (int)offT[(size_t)o * N + i] : 0) == k) v = W[(size_t)i * N + o];
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[e] = h;
    lo[e] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

}  // namespace delrec
