// Reverse-time BPTT scan of an axonal delay layer with the per-step contraction on the
// tensor cores (mma.sync m16n8k16 bf16, fp32 accumulate).
//
// Same block layout and step structure as k_bwd_hybrid64 (16 sources x 64 samples per
// block, cooperative single wave, deferred sums overlapping the gr exchange), but the
// axonal contraction has no per-synapse offset, so each step's
//   gz(t+1)[o, b] = sum_i W[i, o] gr(t+1)[i, b]      (o in the block's 16 sources)
// is one dense 16 x 64 x N product.  fp32 accuracy from bf16: every operand is split
// into hi + lo pieces (hi = x rounded to bf16; lo = x - hi, exact in fp32, rounded to
// bf16: |x - hi - lo| <= 2^-17 |x|) and the product is hi.hi + hi.lo + lo.hi
// (the dropped lo.lo term is below 2^-16 relative).  The split is integer arithmetic:
// float <-> bf16 conversions run at a quarter of the ALU rate.
//   W^T slice: Wp[piece][source][target], resident for the whole scan
//   gr(t):     Gp[piece][sample][target], restaged every step from the L2 exchange
//              (the exchange is sample-major: one float4 of targets -> 4 + 4 bf16)
// Warp w computes n-tile (w & 7) (8 samples) over half of the targets (w >> 3); the two
// halves meet in shared memory.  Urgent sources (first tap at lag 1) take the product
// of gr(t) after the exchange (C2), all others the product of gr(t+1) before it (C1).
#pragma once

#include <cuda_bf16.h>

#include "prep.cuh"

namespace delrec {

struct AxMmaArgs {
  int T, B, N, CS, TAPS;
  const float* gy;
  const float* u;
  const float* keep;
  const float* W;         // (N, N) W[i, o]
  const int* tap_l0;
  const int* tap_nt;
  const float* tap_w;
  float* dx;
  float* gr;
  float* gz;              // (T,B,N)
  LifK lif;
  float* grx;             // [2][tiles][64][N] exchange of gr(t), sample-major
  unsigned int* arrive;   // [tiles] arrival counters, zero at launch
  long long spin_limit;
};

constexpr int kAxNT = 16, kAxBT = 64, kAxThreads = 512, kAxKMAX = 4;
// A block with at most kAxUrgMax urgent sources takes their product of gr(t) in fp32 on
// the CUDA cores while restaging gr(t) (W columns of those sources kept in fp32).
constexpr int kAxUrgMax = 4;

struct AxMmaSmem {
  size_t gp, wp, ring, cred, taps, wu, total;
  int ldk;                // bf16 per row: N + 8 (4-word bank offset between rows)
  int ring_stride;
};
__host__ __device__ inline AxMmaSmem axmma_smem_plan(int N, int TAPS) {
  AxMmaSmem p;
  p.ldk = ((N + 15) / 16) * 16 + 8;
  p.ring_stride = kAxKMAX * 64 + 2;
  p.gp = align256((size_t)2 * kAxBT * p.ldk * 2);
  p.wp = align256((size_t)2 * kAxNT * p.ldk * 2);
  p.ring = align256((size_t)kAxNT * p.ring_stride * 4);
  p.cred = align256((size_t)8 * 32 * 4 * 4);
  p.taps = align256((size_t)kAxNT * (TAPS + 3) * 4);
  p.wu = align256((size_t)kAxUrgMax * N * 4 + 16 * 4);
  p.total = p.gp + p.wp + p.ring + p.cred + p.taps + p.wu;
  return p;
}

// hi/lo bf16 bit patterns of x in the upper halves of the returned words
__device__ __forceinline__ void split_bits(float x, uint32_t& hi, uint32_t& lo) {
  hi = (__float_as_uint(x) + 0x8000u) & 0xffff0000u;   // nearest bf16 (ties away from zero)
  const float r = __fsub_rn(x, __uint_as_float(hi));      // exact: hi/2 <= x <= 2 hi
  lo = (__float_as_uint(r) + 0x8000u) & 0xffff0000u;
}
// two bf16 (upper halves of a, b) packed as {a, b}
__device__ __forceinline__ uint32_t pack_hi16(uint32_t a, uint32_t b) { return __byte_perm(a, b, 0x7632); }

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// C fragment (16 sources x 8 samples of n-tile nt) of the product W-slice^T . gr over the
// targets of k-half kh; returns the lane's 4 values: rows g, g+8, columns 2c, 2c+1.
__device__ __forceinline__ void ax_mma_pass(const __nv_bfloat16* __restrict__ Gp, const __nv_bfloat16* __restrict__ Wp,
                                            int ldk, int nk16, int nt, int kh, int lane, float (&out)[4]) {
  const int g = lane >> 2, c = lane & 3;
  float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
  const size_t gpiece = (size_t)kAxBT * ldk, wpiece = (size_t)kAxNT * ldk;
  const __nv_bfloat16* grow = Gp + (size_t)(nt * 8 + g) * ldk + 2 * c;
  const __nv_bfloat16* wrow0 = Wp + (size_t)g * ldk + 2 * c;
  const __nv_bfloat16* wrow1 = Wp + (size_t)(g + 8) * ldk + 2 * c;
  const int kt0 = kh * ((nk16 + 1) / 2), kt1 = min(nk16, kt0 + (nk16 + 1) / 2);
#pragma unroll 2
  for (int kt = kt0; kt < kt1; ++kt) {
    const int k0 = kt * 16;
    uint32_t ah[4], al[4], bh[2], bl[2];
    ah[0] = *(const uint32_t*)(wrow0 + k0);
    ah[1] = *(const uint32_t*)(wrow1 + k0);
    ah[2] = *(const uint32_t*)(wrow0 + k0 + 8);
    ah[3] = *(const uint32_t*)(wrow1 + k0 + 8);
    al[0] = *(const uint32_t*)(wrow0 + wpiece + k0);
    al[1] = *(const uint32_t*)(wrow1 + wpiece + k0);
    al[2] = *(const uint32_t*)(wrow0 + wpiece + k0 + 8);
    al[3] = *(const uint32_t*)(wrow1 + wpiece + k0 + 8);
    bh[0] = *(const uint32_t*)(grow + k0);
    bh[1] = *(const uint32_t*)(grow + k0 + 8);
    bl[0] = *(const uint32_t*)(grow + gpiece + k0);
    bl[1] = *(const uint32_t*)(grow + gpiece + k0 + 8);
    float(&acc)[4] = (kt & 1) ? acc1 : acc0;
    mma_bf16_16816(acc, ah[0], ah[1], ah[2], ah[3], bh[0], bh[1]);
    mma_bf16_16816(acc, ah[0], ah[1], ah[2], ah[3], bl[0], bl[1]);
    mma_bf16_16816(acc, al[0], al[1], al[2], al[3], bh[0], bh[1]);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) out[q] = acc0[q] + acc1[q];
}

// Restage of gr(t) (sample-major exchange rows of N = 128 MI floats) as bf16 hi/lo pieces:
// warp w takes samples w + 16 j (j < 4), a lane float4 i4 = lane + 32 m of each row; all
// 4 MI loads are issued before the first split.  With `fuse`, the urgent sources'
//   gz(t)[u, b] = sum_i W[i, u] gr(t)[i, b]
// is summed in fp32 from the same registers (lane partials, then a warp tree) into the
// ring cell `slot` of each urgent source.
template <int MI>
__device__ __forceinline__ void ax_restage(const float* __restrict__ xb, int N, __nv_bfloat16* __restrict__ Gp,
                                           int ldk, int warp, int lane, bool fuse, int nurg,
                                           const float* __restrict__ wu, const int* __restrict__ ulist,
                                           float* __restrict__ ring, int RS, int slot, int nb) {
  constexpr int J = kAxBT / 16;
  float4 xr[J][MI];
#pragma unroll
  for (int j = 0; j < J; ++j)
#pragma unroll
    for (int m = 0; m < MI; ++m) xr[j][m] = __ldcg((const float4*)(xb + (size_t)(warp + 16 * j) * N) + lane + 32 * m);
#pragma unroll
  for (int j = 0; j < J; ++j)
#pragma unroll
    for (int m = 0; m < MI; ++m) {
      __nv_bfloat16* dh = Gp + (size_t)(warp + 16 * j) * ldk + 4 * (lane + 32 * m);
      uint32_t h0, l0, h1, l1, h2, l2, h3, l3;
      split_bits(xr[j][m].x, h0, l0);
      split_bits(xr[j][m].y, h1, l1);
      split_bits(xr[j][m].z, h2, l2);
      split_bits(xr[j][m].w, h3, l3);
      *(uint2*)dh = make_uint2(pack_hi16(h0, h1), pack_hi16(h2, h3));
      *(uint2*)(dh + (size_t)kAxBT * ldk) = make_uint2(pack_hi16(l0, l1), pack_hi16(l2, l3));
    }
  if (!fuse) return;
  for (int q = 0; q < nurg; ++q) {
    const float4* w4 = (const float4*)(wu + (size_t)q * N);
    float v[J];
#pragma unroll
    for (int j = 0; j < J; ++j) v[j] = 0.f;
#pragma unroll
    for (int m = 0; m < MI; ++m) {
      const float4 w = w4[lane + 32 * m];
#pragma unroll
      for (int j = 0; j < J; ++j) {
        v[j] = fmaf(w.x, xr[j][m].x, v[j]);
        v[j] = fmaf(w.y, xr[j][m].y, v[j]);
        v[j] = fmaf(w.z, xr[j][m].z, v[j]);
        v[j] = fmaf(w.w, xr[j][m].w, v[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < J; ++j) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v[j] += __shfl_xor_sync(0xffffffffu, v[j], off);
      const int smp = warp + 16 * j;
      if (lane == 0 && smp < nb) ring[(size_t)ulist[q] * RS + slot + smp] += v[j];
    }
  }
}

template <int TPF>
__global__ void __launch_bounds__(512, 1) k_bwd_axonal_mma(AxMmaArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_abort, s_any_urg;
  constexpr int NT = kAxNT, BT = kAxBT, NTH = kAxThreads, PPT = 2, KMAX = kAxKMAX;
  const int rank = (int)(blockIdx.x % a.CS), tile = (int)(blockIdx.x / a.CS);
  const int tiles = (int)(gridDim.x / a.CS);
  const int N = a.N, T = a.T, B = a.B, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int o0 = rank * NT;
  const int nts = max(0, min(NT, N - o0));
  const int b0 = tile * BT;
  const int nb = max(0, min(BT, B - b0));
  const size_t BN = (size_t)B * N;

  const AxMmaSmem P = axmma_smem_plan(N, a.TAPS);
  const int ldk = P.ldk, RS = P.ring_stride, nk16 = (N + 15) / 16;
  __nv_bfloat16* Gp = (__nv_bfloat16*)smem;                                      // [2][64][ldk]
  __nv_bfloat16* Wp = (__nv_bfloat16*)(smem + P.gp);                             // [2][16][ldk]
  float* ring = (float*)(smem + P.gp + P.wp);                                    // [16][RS]
  float* cred = (float*)(smem + P.gp + P.wp + P.ring);                           // [8][32][4]
  int* tl0 = (int*)(smem + P.gp + P.wp + P.ring + P.cred);                       // [16]
  int* tnt = tl0 + NT;
  int* surg = tnt + NT;
  float* tw = (float*)(surg + NT);                                               // [16][TAPS]
  float* wu = (float*)(smem + P.gp + P.wp + P.ring + P.cred + P.taps);          // [kAxUrgMax][N]
  int* ulist = (int*)(wu + (size_t)kAxUrgMax * N);                               // [kAxUrgMax]

  // ---- init: W pieces of the block's sources, taps, ring, staged gr = 0
  for (int e = tid; e < NT * ldk; e += NTH) {
    const int ol = e / ldk, i = e % ldk;
    const float wv = (ol < nts && i < N) ? a.W[(size_t)i * N + o0 + ol] : 0.f;
    uint32_t hb, lb;
    split_bits(wv, hb, lb);
    Wp[e] = __ushort_as_bfloat16((unsigned short)(hb >> 16));
    Wp[(size_t)NT * ldk + e] = __ushort_as_bfloat16((unsigned short)(lb >> 16));
  }
  for (int e = tid; e < 2 * BT * ldk; e += NTH) Gp[e] = __float2bfloat16_rn(0.f);
  for (int ol = tid; ol < NT; ol += NTH) {
    const bool ok = ol < nts;
    tl0[ol] = ok ? a.tap_l0[o0 + ol] : 2;
    tnt[ol] = ok ? a.tap_nt[o0 + ol] : 0;
    surg[ol] = ok && a.tap_l0[o0 + ol] <= 1;
  }
  for (int e = tid; e < NT * a.TAPS; e += NTH) {
    const int ol = e / a.TAPS;
    tw[e] = ol < nts ? a.tap_w[(size_t)(o0 + ol) * a.TAPS + (e % a.TAPS)] : 0.f;
  }
  for (int e = tid; e < NT * RS; e += NTH) ring[e] = 0.f;
  if (tid == 0) {
    s_abort = 0;
    int nu = 0;
    for (int ol = 0; ol < nts; ++ol)
      if (a.tap_l0[o0 + ol] <= 1) {
        if (nu < kAxUrgMax) ulist[nu] = ol;
        ++nu;
      }
    s_any_urg = nu;
  }
  __syncthreads();
  const int nurg = s_any_urg;
  const bool any_urg = nurg != 0;
  // fused urgent product: whole float4 rows per lane (N % 128 == 0) and few urgent sources
  const bool fuse_urg = any_urg && nurg <= kAxUrgMax && (N & 127) == 0 && N <= 512;
  if (fuse_urg)
    for (int e = tid; e < nurg * N; e += NTH) wu[e] = a.W[(size_t)(e % N) * N + o0 + ulist[e / N]];
  __syncthreads();

  // ---- per-thread (source, sample) pairs p = tid + k*NTH: ol = p % NT, bl = p / NT
  int pol[PPT], pbl[PPT];
  bool pin[PPT], pok[PPT];
  float lam[PPT], kp[PPT];
  float pf_gy[PPT], pf_u[PPT], pf_tap[PPT][TPF];
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    const int p = tid + k * NTH;
    pol[k] = p % NT;
    pbl[k] = p / NT;
    pin[k] = pol[k] < nts && pbl[k] < BT;
    pok[k] = pin[k] && pbl[k] < nb;
    lam[k] = 0.f;
    kp[k] = (pok[k] && a.keep) ? a.keep[(size_t)(b0 + pbl[k]) * N + o0 + pol[k]] : 1.f;
  }
  // loads for step t: gy, u (issued at the start of step t+1) and the taps at lags >= 3
  // with nonzero weight (issued after the deferred sums of step t+1: gz(t+l) was written at
  // step t+l-1 >= t+2).  Split so that the load queue never holds a whole step's loads.
  auto prefetch_lif = [&](int t) {
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      pf_gy[k] = 0.f;
      pf_u[k] = 0.f;
      if (pok[k] && t >= 0) {
        const size_t idx = ((size_t)t * B + b0 + pbl[k]) * N + o0 + pol[k];
        pf_gy[k] = __ldcs(a.gy + idx);
        pf_u[k] = __ldcs(a.u + idx);
      }
    }
  };
  auto prefetch_taps = [&](int t) {
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
#pragma unroll
      for (int j = 0; j < TPF; ++j) pf_tap[k][j] = 0.f;
      if (pok[k] && t >= 0) {
        const size_t idx = ((size_t)t * B + b0 + pbl[k]) * N + o0 + pol[k];
        const int lo = tl0[pol[k]], n = tnt[pol[k]];
#pragma unroll
        for (int j = 0; j < TPF; ++j) {
          const int l = lo + j;
          if (j < n && l >= 3 && t + l < T && tw[pol[k] * a.TAPS + j] != 0.f)
            pf_tap[k][j] = __ldcg(a.gz + idx + (size_t)l * BN);
        }
      }
    }
  };
  prefetch_lif(T - 1);
  prefetch_taps(T - 1);

  const int nt8 = warp & 7, kh = warp >> 3, g = lane >> 2, c = lane & 3;
  // ring cells of this lane's C values: sources g and g+8, samples nt8*8 + 2c (+1)
  float* rc0 = ring + (size_t)g * RS + nt8 * 8 + 2 * c;
  float* rc1 = ring + (size_t)(g + 8) * RS + nt8 * 8 + 2 * c;
  const bool u0 = g < nts && surg[g], u1 = g + 8 < nts && surg[g + 8];
  float* cr = cred + ((size_t)nt8 * 32 + lane) * 4;
  unsigned int arrivals = 0;
  const size_t xtile = (size_t)N * BT;

  // one pass of the product into ring slot `slot`, rows selected by `urgent`
  auto contract = [&](int slot, bool urgent) {
    float v[4];
    ax_mma_pass(Gp, Wp, ldk, nk16, nt8, kh, lane, v);
    if (kh == 1) {
#pragma unroll
      for (int q = 0; q < 4; ++q) cr[q] = v[q];
    }
    __syncthreads();
    if (kh == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] += cr[q];
      if (g < nts && u0 == urgent) {
        float2* cell = (float2*)(rc0 + (slot % KMAX) * 64);
        float2 x = *cell;
        x.x += v[0];
        x.y += v[1];
        *cell = x;
      }
      if (g + 8 < nts && u1 == urgent) {
        float2* cell = (float2*)(rc1 + (slot % KMAX) * 64);
        float2 x = *cell;
        x.x += v[2];
        x.y += v[3];
        *cell = x;
      }
    }
  };

  for (int t = T - 1; t >= 0; --t) {
    float cur_gy[PPT], cur_u[PPT], cur_tap[PPT][TPF];
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      cur_gy[k] = pf_gy[k];
      cur_u[k] = pf_u[k];
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
      float* rrow = ring + (size_t)ol * RS + bl;
      if (pok[k]) {
        const int lo = tl0[ol], n = tnt[ol];   // n <= TAPS <= TPF
        float gfut = 0.f;
#pragma unroll
        for (int j = 0; j < TPF; ++j) {
          const int l = lo + j;
          if (j < n && t + l < T) {
            const float gv = l <= 2 ? rrow[((t + l) % KMAX) * 64] : cur_tap[k][j];
            gfut = fmaf(tw[ol * a.TAPS + j], gv, gfut);
          }
        }
        const float gY = __fadd_rn(cur_gy[k], gfut);
        const float du = lif_backward(gY, cur_u[k], lam[k], a.lif);
        lam[k] = lif_carry(du, a.lif);
        grv = __fmul_rn(du, kp[k]);
        const size_t idx = ((size_t)t * B + b0 + bl) * N + o0 + ol;
        a.dx[idx] = du;
        if (a.gr != a.dx) a.gr[idx] = grv;   // (gr is dx itself without dropout)
      }
      rrow[((t + 2) % KMAX) * 64] = 0.f;   // last read of slot t+2 was above
      __stcg(xb + (size_t)bl * N + o0 + ol, grv);
    }
    __syncthreads();
    if (tid == 0) {   // release: the block's exchange writes (ordered by the barrier) first
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      atomicAdd(a.arrive + tile, 1u);
    }
    arrivals += a.CS;
    // ===== C1: product of gr(t+1) (staged) for the non-urgent sources -> slot t+1
    if (t + 1 < T) contract(t + 1, false);
    __syncthreads();
    // ===== F: gz(t+1) is complete
    if (t + 1 < T) {
#pragma unroll
      for (int k = 0; k < PPT; ++k)
        if (pok[k]) {
          const size_t idx = ((size_t)(t + 1) * B + b0 + pbl[k]) * N + o0 + pol[k];
          a.gz[idx] = ring[(size_t)pol[k] * RS + ((t + 1) % KMAX) * 64 + pbl[k]];
        }
    }
    prefetch_taps(t - 1);
    // ===== W: the tile's gr(t), staged as bf16 pieces
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
    if ((N & 127) == 0 && N <= 512) {
      const int MI = N >> 7;
      if (MI == 1) ax_restage<1>(xb, N, Gp, ldk, warp, lane, fuse_urg, nurg, wu, ulist, ring, RS, (t % KMAX) * 64, nb);
      else if (MI == 2) ax_restage<2>(xb, N, Gp, ldk, warp, lane, fuse_urg, nurg, wu, ulist, ring, RS, (t % KMAX) * 64, nb);
      else if (MI == 3) ax_restage<3>(xb, N, Gp, ldk, warp, lane, fuse_urg, nurg, wu, ulist, ring, RS, (t % KMAX) * 64, nb);
      else ax_restage<4>(xb, N, Gp, ldk, warp, lane, fuse_urg, nurg, wu, ulist, ring, RS, (t % KMAX) * 64, nb);
    } else {
      const int n4 = N / 4;   // N % 4 == 0 (planner)
      for (int smp = warp; smp < BT; smp += NTH / 32) {
        const float4* xs = (const float4*)(xb + (size_t)smp * N);
        __nv_bfloat16* dh = Gp + (size_t)smp * ldk;
        for (int i4 = lane; i4 < n4; i4 += 32) {
          const float4 x = __ldcg(xs + i4);
          uint32_t h0, l0, h1, l1, h2, l2, h3, l3;
          split_bits(x.x, h0, l0);
          split_bits(x.y, h1, l1);
          split_bits(x.z, h2, l2);
          split_bits(x.w, h3, l3);
          *(uint2*)(dh + 4 * i4) = make_uint2(pack_hi16(h0, h1), pack_hi16(h2, h3));
          *(uint2*)(dh + (size_t)BT * ldk + 4 * i4) = make_uint2(pack_hi16(l0, l1), pack_hi16(l2, l3));
        }
      }
    }
    __syncthreads();
    // ===== C2: product of gr(t) for the urgent sources -> slot t (tensor cores when the
    // restage did not take it)
    if (any_urg && !fuse_urg) contract(t, true);
    __syncthreads();
  }
  // ---- gz(0): its deferred product of gr(0) (staged)
  contract(0, false);
  __syncthreads();
#pragma unroll
  for (int k = 0; k < PPT; ++k)
    if (pok[k]) a.gz[((size_t)b0 + pbl[k]) * N + o0 + pol[k]] = ring[(size_t)pol[k] * RS + pbl[k]];
}

}  // namespace delrec
