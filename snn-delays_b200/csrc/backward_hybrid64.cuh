// Reverse-time BPTT scan of the hybrid delay layer: cooperative single-wave form with
// 64-sample tiles (two samples per lane) and the synapse sums moved off the step-to-step
// critical path.
//
// Layout: a block owns NT <= 16 source neurons o (one per warp) and a tile of 64 samples;
// the blocks of a tile together cover all N neurons and exchange gr(t) through L2.
// gr(t) of the tile (all N targets x 64 samples) is staged in shared memory as rows
// grc[i][0..63]; lane l handles samples 2l and 2l+1 (one 8-byte load per synapse).
//
// Identity used (integer offsets k_io in [0, K], base lags l >= 1):
//   gz(tau)[o] = sum_i W[i,o] gr(tau + k_io)[i],   gfut(t)[o] = sum_j h_o(l_j) gz(t + l_j)[o].
// A contribution of gr(t')[i] reaches gfut at t = t' - k_io - l_j <= t' - (k_io + l0_o).
// Only the synapses with k_io + l0_o = 1 (offset 0 into a source whose first tap is lag
// 1) are needed by the very next step ("urgent"); every other contribution of gr(t+1)
// can be summed one step later.  So step t runs
//   A.  LIF backward of the block's (o, b) pairs -> gr(t); gfut(t) reads the ring slots
//       t+1 and t+2 in shared memory and the older gz values prefetched from global
//       memory during the previous step; gr(t) goes to the tile's L2 exchange buffer;
//   C1. the deferred sums of gr(t+1) (still staged) for all non-urgent buckets into the
//       ring slots t+1-k  -- while the other blocks' gr(t) travels;
//   F.  gz(t+1) is complete: written out to global memory (dmask, later taps);
//   W.  wait for the tile's arrivals of step t, stage gr(t);
//   C2. the urgent buckets of gr(t) into ring slot t.
// The ring has K+2 slots per source: slot tau is live from the first contribution to
// gz(tau) (gr(tau+K), step tau+K-1) to its last read (tap l=2 at step tau-2), and is
// cleared right after that read.
#pragma once

#include "prep.cuh"

namespace delrec {

struct Hyb64Args {
  int T, B, N, K, CS, NT, TAPS, CAPS, CAP;   // NT <= 16 sources per block (one per warp)
  const float* gy;
  const float* u;
  const float* keep;
  const int* tap_l0;
  const int* tap_nt;
  const float* tap_w;
  const int2* ent;        // (N, CAP) bucket entries (i, weight bits), buckets padded to 8
  const int* boff;        // bucket k of source o starts at boff[o*boff_stride + k], k <= K+1
  int boff_stride;
  float* dx;
  float* gr;
  float* gz;              // (T,B,N), or null when nothing downstream reads it (then no tap
                          // may sit at lag >= 3)
  LifK lif;
  float* grx;             // [2][tiles][N][64] exchange of gr(t)
  unsigned int* arrive;   // [tiles] arrival counters, zero at launch
  long long spin_limit;   // polls before a wait gives up (sets ST_TIMEOUT)
};

constexpr int kH64NTMax = 16, kH64BT = 64, kH64Threads = 512;

struct Hyb64Smem {
  size_t grc, idx, w, boff, taps, ring, total;
  int ring_stride;        // floats per source: KMAX*64 + 2 (bank offset between sources)
};
__host__ __device__ inline Hyb64Smem hyb64_smem_plan(int N, int NT, int CAPS, int K, int TAPS, int KMAX) {
  Hyb64Smem p;
  p.ring_stride = KMAX * 64 + 2;
  p.grc = align256((size_t)N * 64 * 4);
  p.idx = align256((size_t)NT * CAPS * 2);
  p.w = align256((size_t)NT * CAPS * 4);
  p.boff = align256((size_t)NT * (K + 2) * 4 + NT * 4);
  p.taps = align256((size_t)NT * (TAPS + 2) * 4);
  p.ring = align256((size_t)NT * p.ring_stride * 4);
  p.total = p.grc + p.idx + p.w + p.boff + p.taps + p.ring;
  return p;
}

// acc2 += sum over the bucket [beg, end) of w_e * grc[i_e][2 lane .. 2 lane + 1]
__device__ __forceinline__ float2 h64_bucket(const uint16_t* __restrict__ ix, const float* __restrict__ wv, int beg,
                                             int end, uint32_t gbase) {
  float2 a0 = make_float2(0.f, 0.f), a1 = a0, a2 = a0, a3 = a0;
#pragma unroll 2
  for (int e = beg; e < end; e += 8) {
    const uint4 i8 = *(const uint4*)(ix + e);   // 8 x u16 target rows
    const float4 wa = *(const float4*)(wv + e);
    const float4 wb = *(const float4*)(wv + e + 4);
    float2 g[8];
    const uint32_t r[8] = {i8.x & 0xffffu, i8.x >> 16, i8.y & 0xffffu, i8.y >> 16,
                           i8.z & 0xffffu, i8.z >> 16, i8.w & 0xffffu, i8.w >> 16};
#pragma unroll
    for (int q = 0; q < 8; ++q)
      asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(g[q].x), "=f"(g[q].y) : "r"(gbase + (r[q] << 8)));
    a0.x = fmaf(wa.x, g[0].x, a0.x); a0.y = fmaf(wa.x, g[0].y, a0.y);
    a1.x = fmaf(wa.y, g[1].x, a1.x); a1.y = fmaf(wa.y, g[1].y, a1.y);
    a2.x = fmaf(wa.z, g[2].x, a2.x); a2.y = fmaf(wa.z, g[2].y, a2.y);
    a3.x = fmaf(wa.w, g[3].x, a3.x); a3.y = fmaf(wa.w, g[3].y, a3.y);
    a0.x = fmaf(wb.x, g[4].x, a0.x); a0.y = fmaf(wb.x, g[4].y, a0.y);
    a1.x = fmaf(wb.y, g[5].x, a1.x); a1.y = fmaf(wb.y, g[5].y, a1.y);
    a2.x = fmaf(wb.z, g[6].x, a2.x); a2.y = fmaf(wb.z, g[6].y, a2.y);
    a3.x = fmaf(wb.w, g[7].x, a3.x); a3.y = fmaf(wb.w, g[7].y, a3.y);
  }
  return make_float2((a0.x + a1.x) + (a2.x + a3.x), (a0.y + a1.y) + (a2.y + a3.y));
}

template <int KMAX, int TPF>
__global__ void __launch_bounds__(512, 1) k_bwd_hybrid64(Hyb64Args a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_abort;
  constexpr int BT = kH64BT, NTH = kH64Threads, PPT = 2;   // NT * 64 <= PPT * NTH
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

  const Hyb64Smem P = hyb64_smem_plan(N, NT, a.CAPS, K, a.TAPS, KMAX);
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

  // ---- init: resident bucket lists, taps, ring, staged gr
  for (int e = tid; e < NT * a.CAPS; e += NTH) {
    const int ol = e / a.CAPS, pos = e % a.CAPS;
    int2 en = make_int2(0, 0);
    if (ol < nts) {
      const int tot = a.boff[(size_t)(o0 + ol) * a.boff_stride + K + 1];
      if (pos < tot) en = a.ent[(size_t)(o0 + ol) * a.CAP + pos];
    }
    sidx[e] = (uint16_t)en.x;
    sw[e] = __int_as_float(en.y);
  }
  for (int e = tid; e < NT * (K + 2); e += NTH) {
    const int ol = e / (K + 2);
    int off = ol < nts ? a.boff[(size_t)(o0 + ol) * a.boff_stride + e % (K + 2)] : 0;
    if (off > a.CAPS) {   // the resident row holds CAPS entries (8-aligned)
      flag_status(ST_INDEX_RANGE);
      off = a.CAPS;
    }
    sbo[e] = off;
  }
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
  for (int e = tid; e < N * BT; e += NTH) grc[e] = 0.f;
  for (int e = tid; e < NT * RS; e += NTH) ring[e] = 0.f;
  if (tid == 0) s_abort = 0;
  __syncthreads();

  // ---- per-thread pairs p = tid + k*NTH: ol = p % NT, bl = p / NT
  int pol[PPT], pbl[PPT];
  bool pin[PPT], pok[PPT];   // pair inside the block's slice x tile; and a real sample
  float lam[PPT], kp[PPT];
  float pf_gy[PPT], pf_u[PPT], pf_tap[PPT][TPF];
  LifPre pf_pre[PPT];   // u-only part of the LIF backward of the prefetched step
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
  // loads for step t: gy, u and the taps l >= 3 (gz(t+l) was written at step t+l-1 >= t+2)
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
          if (j < n && l >= 3 && t + l < T && a.gz && tw[pol[k] * a.TAPS + j] != 0.f)
            pf_tap[k][j] = __ldcg(a.gz + idx + (size_t)l * BN);
        }
      }
    }
  };
  prefetch_lif(T - 1);
  prefetch_taps(T - 1);
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
  unsigned int arrivals = 0;
  const size_t xtile = (size_t)N * BT;

  for (int t = T - 1; t >= 0; --t) {
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
      float* rrow = ring + (size_t)ol * RS + bl;
      if (pok[k]) {
        const int lo = tl0[ol], n = tnt[ol];   // n <= TAPS <= TPF (checked by the planner)
        float gfut = 0.f;
#pragma unroll
        for (int j = 0; j < TPF; ++j) {
          const int l = lo + j;
          if (j < n && t + l < T) {
            const float g = l <= 2 ? rrow[((t + l) % KMAX) * 64] : cur_tap[k][j];
            gfut = fmaf(tw[ol * a.TAPS + j], g, gfut);
          }
        }
        const float gY = __fadd_rn(cur_gy[k], gfut);
        const float du = lif_backward_pre(gY, lam[k], cur_pre[k], a.lif);
        lam[k] = lif_carry(du, a.lif);
        grv = __fmul_rn(du, kp[k]);
        const size_t idx = ((size_t)t * B + b0 + bl) * N + o0 + ol;
        a.dx[idx] = du;
        if (a.gr != a.dx) a.gr[idx] = grv;   // (gr is dx itself without dropout)
      }
      // slot t+2 (== t-K mod KMAX) had its last read above; it next receives gz(t-K)
      rrow[((t + 2) % KMAX) * 64] = 0.f;
      __stcg(xb + (size_t)(o0 + ol) * BT + bl, grv);
    }
    __syncthreads();
    if (tid == 0) {   // release: the block's exchange writes (ordered by the barrier) first
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      atomicAdd(a.arrive + tile, 1u);
    }
    arrivals += a.CS;
    // ===== C1: deferred sums of gr(t+1) into slots t+1-k
    if (w_ok && t + 1 < T) {
      for (int k = K; k >= 0; --k) {
        const int tau = t + 1 - k;
        if (tau < 0) continue;
        if (k == 0 && w_urg) continue;
        const int beg = wbo[k], end = wbo[k + 1];
        if (((beg | end) & 7) != 0) { flag_status(ST_INDEX_RANGE); continue; }
        const float2 s = h64_bucket(wix, wwv, beg, end, gbase);
        float2* cell = (float2*)(wring + (tau % KMAX) * 64);
        float2 c = *cell;
        c.x += s.x;
        c.y += s.y;
        *cell = c;
      }
    }
    __syncthreads();
    // ===== F: gz(t+1) is complete
    if (t + 1 < T && a.gz) {
#pragma unroll
      for (int k = 0; k < PPT; ++k)
        if (pok[k]) {
          const size_t idx = ((size_t)(t + 1) * B + b0 + pbl[k]) * N + o0 + pol[k];
          a.gz[idx] = ring[(size_t)pol[k] * RS + ((t + 1) % KMAX) * 64 + pbl[k]];
        }
    }
    prefetch_taps(t - 1);
    // the u-only part of step t-1's LIF backward (its u arrived during this step)
#pragma unroll
    for (int k = 0; k < PPT; ++k) pf_pre[k] = lif_bwd_prep(pf_u[k], a.lif);
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
    // ===== C2: urgent bucket (offset 0 of a source with a lag-1 tap) of gr(t)
    if (w_urg) {
      const int beg = wbo[0], end = wbo[1];
      if (((beg | end) & 7) != 0) {
        flag_status(ST_INDEX_RANGE);
      } else {
        const float2 s = h64_bucket(wix, wwv, beg, end, gbase);
        float2* cell = (float2*)(wring + (t % KMAX) * 64);
        float2 c = *cell;
        c.x += s.x;
        c.y += s.y;
        *cell = c;
      }
    }
    __syncthreads();
  }
  // ---- gz(0): its deferred offset-0 sums of gr(0)
  if (w_ok && !w_urg) {
    const int beg = wbo[0], end = wbo[1];
    if (((beg | end) & 7) == 0) {
      const float2 s = h64_bucket(wix, wwv, beg, end, gbase);
      float2* cell = (float2*)wring;
      float2 c = *cell;
      c.x += s.x;
      c.y += s.y;
      *cell = c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < PPT; ++k)
    if (pok[k] && a.gz) a.gz[((size_t)b0 + pbl[k]) * N + o0 + pol[k]] = ring[(size_t)pol[k] * RS + pbl[k]];
}

}  // namespace delrec
