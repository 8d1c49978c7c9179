// Reverse-time BPTT scan of the hybrid delay layer (learned axonal base + frozen integer
// offsets), specialised for the common shapes: batch tile of 32 samples (lane = sample),
// 32 source neurons per block (2 per warp, 16 warps), offsets K <= KMAX-1.
//
// Per reverse step t each block of the cluster
//   A. runs the LIF backward for its (b, o) pairs: dL/dy(t) = gy + sum_j h_o(l_j) gz_{m_j}(t+l_j),
//      m_j = max(0, 1 - l_j), giving gr(t) = du * keep;
//   B. refreshes its own slice of its shared copy of gr(t), cluster barrier (every peer
//      finished reading step t+1), pushes the slice into every peer's copy (16-byte DSMEM
//      stores), cluster barrier (the copy of step t is complete);
//   C. for each of the warp's sources o and each offset k, sums the bucket
//      sum_{i: off[i,o] = k} W[i,o] gr(t)[i,b] over the source's bucket list, which stays
//      resident in shared memory for the whole scan (16-bit target index + fp32 weight),
//      into slot (t-k) mod KMAX of the source's ring.  Slot tau accumulates the offsets in
//      decreasing order, so at step tau+m it holds gz_m(tau) = sum over offsets >= m
//      (the part of gz a base lag <= 0 can reach); gz_m(t-m) is read out after the sweep
//      and slot t is cleared once gz_0(t) is out.
// The per-step work is one FMA per (synapse, sample); its shared-memory traffic is one
// conflict-free 128-byte row of gr per (synapse, warp) plus the broadcast list entries.
#pragma once

#include <cooperative_groups.h>

#include "prep.cuh"

namespace cg = cooperative_groups;

namespace delrec {

struct HybArgs {
  int T, B, N, K, CS, NT, TAPS, MM, CAPS;
  const float* gy;
  const float* u;
  const float* keep;
  const int* tap_l0;
  const int* tap_nt;
  const float* tap_w;
  const int2* ent;        // (N, CAP) bucket entries (i, weight bits), buckets padded to 8
  const int* boff;        // (N, K+2)
  int CAP;
  float* dx;
  float* gr;
  float* gz;              // gz_m at gz + m*T*B*N, m = 0..MM
  LifK lif;
  // cooperative mode: gr exchange through L2 instead of distributed shared memory
  float* grx;             // [2][tiles][N][32]
  unsigned int* arrive;   // [tiles] arrival counters, zero at launch
  long long spin_limit;   // polls before a barrier gives up (sets ST_TIMEOUT)
};

struct HybSmem {
  size_t gr_cur, idx, w, boff, taps, ring, total;
};
__host__ __device__ inline HybSmem hyb_smem_plan(int N, int NT, int CAPS, int K, int TAPS, int KMAX) {
  HybSmem p;
  p.gr_cur = align256((size_t)N * 32 * 4);
  p.idx = align256((size_t)NT * CAPS * 2);
  p.w = align256((size_t)NT * CAPS * 4);
  p.boff = align256((size_t)NT * (K + 2) * 4);
  p.taps = align256((size_t)NT * (TAPS + 2) * 4);
  p.ring = align256((size_t)NT * KMAX * 32 * 4);
  p.total = p.gr_cur + p.idx + p.w + p.boff + p.taps + p.ring;
  return p;
}

// COOP = false: the blocks of a batch tile form a thread-block cluster and share gr
//   through distributed shared memory (at most 16 blocks per cluster; a GPC hosts one
//   16-block cluster, so at most 7 such clusters are co-resident on a B200).
// COOP = true: a cooperative launch (every block co-resident, or the launch fails); the
//   blocks of a tile publish their gr slices to a double-buffered L2 buffer and meet at
//   an arrival counter per tile.  The wait polls with an iteration limit; on expiry the
//   block records ST_TIMEOUT and leaves (its peers then expire at their next wait).
template <int KMAX, bool COOP>
__global__ void __launch_bounds__(512, 1) k_bwd_hybrid(HybArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_abort;
  constexpr int BT = 32, NTH = 512, SPW = 2, PPT = 2;
  const int rank = COOP ? (int)(blockIdx.x % a.CS) : (int)cg::this_cluster().block_rank();
  const int N = a.N, T = a.T, B = a.B, NT = a.NT, K = a.K, MM = a.MM, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int tile = blockIdx.x / a.CS;
  const int o0 = rank * NT;
  const int nts = max(0, min(NT, N - o0));
  const int b0 = tile * BT;
  const int nb = max(0, min(BT, B - b0));
  const size_t TBN = (size_t)T * B * N;

  const HybSmem P = hyb_smem_plan(N, NT, a.CAPS, K, a.TAPS, KMAX);
  float* grc = (float*)smem;                                            // [N][32]
  uint16_t* sidx = (uint16_t*)(smem + P.gr_cur);                        // [NT][CAPS]
  float* sw = (float*)(smem + P.gr_cur + P.idx);                        // [NT][CAPS]
  int* sbo = (int*)(smem + P.gr_cur + P.idx + P.w);                     // [NT][K+2]
  int* tl0 = (int*)(smem + P.gr_cur + P.idx + P.w + P.boff);            // [NT]
  int* tnt = tl0 + NT;
  float* tw = (float*)(tnt + NT);                                        // [NT][TAPS]
  float* ring = (float*)(smem + P.gr_cur + P.idx + P.w + P.boff + P.taps);  // [NT][KMAX][32]

  // ---- init: resident bucket lists, taps, rings, zero tails of gz_m (m >= 1)
  for (int e = tid; e < NT * a.CAPS; e += NTH) {
    const int ol = e / a.CAPS, pos = e % a.CAPS;
    int2 en = make_int2(0, 0);
    if (ol < nts) {
      const int tot = a.boff[(size_t)(o0 + ol) * (K + 2) + K + 1];
      if (pos < tot) en = a.ent[(size_t)(o0 + ol) * a.CAP + pos];
    }
    sidx[e] = (uint16_t)(en.x * (BT * 4));   // byte offset of gr row i (N <= 512)
    sw[e] = __int_as_float(en.y);
  }
  for (int e = tid; e < NT * (K + 2); e += NTH) {
    const int ol = e / (K + 2);
    sbo[e] = ol < nts ? a.boff[(size_t)(o0 + ol) * (K + 2) + e % (K + 2)] : 0;
  }
  for (int ol = tid; ol < NT; ol += NTH) {
    const bool ok = ol < nts;
    tl0[ol] = ok ? a.tap_l0[o0 + ol] : 1;
    tnt[ol] = ok ? a.tap_nt[o0 + ol] : 0;
  }
  for (int e = tid; e < NT * a.TAPS; e += NTH) {
    const int ol = e / a.TAPS;
    tw[e] = ol < nts ? a.tap_w[(size_t)(o0 + ol) * a.TAPS + (e % a.TAPS)] : 0.f;
  }
  for (int e = tid; e < N * BT; e += NTH) grc[e] = 0.f;
  for (int e = tid; e < NT * KMAX * 32; e += NTH) ring[e] = 0.f;
  // gz_m(tau) for tau >= T - m never receives a contribution
  for (int m = 1; m <= MM; ++m)
    for (int tau = max(0, T - m); tau < T; ++tau)
      for (int p = tid; p < NT * BT; p += NTH) {
        const int bl = p / NT, ol = p % NT;
        if (ol < nts && bl < nb) a.gz[(size_t)m * TBN + ((size_t)tau * B + b0 + bl) * N + o0 + ol] = 0.f;
      }
  float lam[PPT];
#pragma unroll
  for (int k = 0; k < PPT; ++k) lam[k] = 0.f;
  if (tid == 0) s_abort = 0;
  __syncthreads();
  if (!COOP) cg::this_cluster().sync();
  const size_t xtile = (size_t)N * BT;
  unsigned int arrivals = 0;

  for (int t = T - 1; t >= 0; --t) {
    // ===== A: LIF backward of own pairs (p = tid + NTH k -> b = p / NT, o = p % NT)
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int p = tid + k * NTH;
      const int bl = p / NT, ol = p % NT;
      float grv = 0.f;
      if (bl < BT && ol < nts && bl < nb) {
        const int o = o0 + ol, b = b0 + bl;
        const size_t idx = ((size_t)t * B + b) * N + o;
        const float gyv = a.gy[idx], uv = a.u[idx];
        float gfut = 0.f;
        const int lo = tl0[ol], n = tnt[ol];
        for (int j = 0; j < n; ++j) {
          const int l = lo + j;
          const int m = l < 1 ? 1 - l : 0;
          const int tt = t + l;
          if (m <= MM && tt >= 0 && tt + m < T)
            gfut = fmaf(tw[ol * a.TAPS + j], __ldcg(a.gz + (size_t)m * TBN + (size_t)((long long)idx + (long long)l * B * N)), gfut);
        }
        const float gY = __fadd_rn(gyv, gfut);
        const float du = lif_backward(gY, uv, lam[k], a.lif);
        lam[k] = lif_carry(du, a.lif);
        const float kp = a.keep ? a.keep[(size_t)b * N + o] : 1.f;
        grv = __fmul_rn(du, kp);
        a.dx[idx] = du;
        if (a.gr != a.dx) a.gr[idx] = grv;   // (gr is dx itself without dropout)
      }
      if (bl < BT && ol < nts) grc[(size_t)(o0 + ol) * BT + bl] = grv;
    }
    // ===== B: publish the own slice of gr(t) to every block of the tile
    __syncthreads();
    if (!COOP) {
      cg::cluster_group cl = cg::this_cluster();
      cl.sync();  // the peers finished reading their copies of step t+1
      if (a.CS > 1 && nts > 0) {
        const int n4 = nts * BT / 4;
        const float4* src = (const float4*)(grc + (size_t)o0 * BT);
        for (int v = tid; v < n4 * (a.CS - 1); v += NTH) {
          int r = v / n4;
          r += (r >= rank);
          float4* dst = (float4*)cl.map_shared_rank(grc + (size_t)o0 * BT, r);
          dst[v % n4] = src[v % n4];
        }
      }
      cl.sync();
    } else if (a.CS > 1) {
      float* xb = a.grx + ((size_t)(t & 1) * (gridDim.x / a.CS) + tile) * xtile;
      const int n4 = nts * BT / 4;
      const float4* src = (const float4*)(grc + (size_t)o0 * BT);
      float4* dst = (float4*)(xb + (size_t)o0 * BT);
      for (int v = tid; v < n4; v += NTH) __stcg(dst + v, src[v]);
      __syncthreads();
      arrivals += a.CS;
      if (tid == 0) {
        __threadfence();
        atomicAdd(a.arrive + tile, 1u);
        long long polls = 0;
        unsigned int seen;
        do {
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(a.arrive + tile) : "memory");
          if (++polls > a.spin_limit) { flag_status(ST_TIMEOUT); s_abort = 1; break; }
        } while (seen < arrivals);
      }
      __syncthreads();
      if (s_abort) return;
      // gather the peers' slices (L2; the own slice is already local)
      const int rows4 = N * BT / 4;
      const float4* xs = (const float4*)xb;
      float4* gd = (float4*)grc;
      const int own0 = o0 * BT / 4, own1 = (o0 + nts) * BT / 4;
      for (int v = tid; v < rows4; v += NTH)
        if (v < own0 || v >= own1) gd[v] = __ldcg(xs + v);
      __syncthreads();
    }
    // ===== C: bucket sums of the warp's sources into their rings.  The gather uses
    // 32-bit shared-memory addresses: lane base + the entry's precomputed row offset.
    const uint32_t gbase = (uint32_t)__cvta_generic_to_shared(grc) + lane * 4;
    for (int s = 0; s < SPW; ++s) {
      const int ol = warp * SPW + s;
      if (ol >= nts) continue;
      const uint16_t* ix = sidx + (size_t)ol * a.CAPS;
      const float* wv = sw + (size_t)ol * a.CAPS;
      const int* bo = sbo + ol * (K + 2);
      float* rg = ring + (size_t)ol * KMAX * 32 + lane;
      for (int k = K; k >= 0; --k) {
        const int beg = bo[k], end = bo[k + 1];
        float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
        // buckets start and end on multiples of 8 entries (16-byte aligned index loads)
        if (((beg | end) & 7) != 0) { flag_status(ST_INDEX_RANGE); continue; }
#pragma unroll 2
        for (int e = beg; e < end; e += 8) {
          const uint4 i8 = *(const uint4*)(ix + e);               // 8 x u16 byte offsets
          const float4 wa = *(const float4*)(wv + e);
          const float4 wb = *(const float4*)(wv + e + 4);
          float g0, g1, g2, g3, g4, g5, g6, g7;
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(g0) : "r"(gbase + (i8.x & 0xffffu)));
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(g1) : "r"(gbase + (i8.x >> 16)));
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(g2) : "r"(gbase + (i8.y & 0xffffu)));
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(g3) : "r"(gbase + (i8.y >> 16)));
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(g4) : "r"(gbase + (i8.z & 0xffffu)));
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(g5) : "r"(gbase + (i8.z >> 16)));
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(g6) : "r"(gbase + (i8.w & 0xffffu)));
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(g7) : "r"(gbase + (i8.w >> 16)));
          acc0 = fmaf(wa.x, g0, acc0);
          acc1 = fmaf(wa.y, g1, acc1);
          acc2 = fmaf(wa.z, g2, acc2);
          acc3 = fmaf(wa.w, g3, acc3);
          acc0 = fmaf(wb.x, g4, acc0);
          acc1 = fmaf(wb.y, g5, acc1);
          acc2 = fmaf(wb.z, g6, acc2);
          acc3 = fmaf(wb.w, g7, acc3);
        }
        if (t - k >= 0) {
          float* cell = rg + ((t - k) % KMAX) * 32;
          *cell += (acc0 + acc1) + (acc2 + acc3);
        }
      }
      if (lane < nb) {
        const int o = o0 + ol;
        for (int m = 0; m <= MM; ++m) {
          const int tau = t - m;
          if (tau < 0) break;
          a.gz[(size_t)m * TBN + ((size_t)tau * B + b0 + lane) * N + o] = rg[(tau % KMAX) * 32];
        }
      }
      rg[(t % KMAX) * 32] = 0.f;
    }
    __syncthreads();  // gz written this step is read by other threads in A of step t-1
  }
  if (!COOP) cg::this_cluster().sync();
}

}  // namespace delrec
