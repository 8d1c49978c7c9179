// Reverse-time BPTT scan on thread-block clusters.
//
// A cluster of CS blocks owns a batch tile of BT samples; block `rank` owns the source
// neurons [rank*NT, rank*NT + NT).  Per reverse step t every block
//   A. finishes dL/dy for its (b, o) pairs from the recurrent future gradient, runs the
//      LIF backward step (surrogate gradient, reset algebra) and produces
//      gr = dL/drec = du * keep for its neurons;
//   B. pushes its gr slice into every cluster peer's shared-memory copy of gr(t)
//      (distributed shared memory, 16-byte stores) and joins the cluster barrier
//      (release/acquire), so each block holds the full gr(t) of its batch tile;
//   C. accumulates the contribution of gr(t) to its sources:
//      MODE 0 axonal   gz[b,o] = sum_i W[i,o] gr[b,i]          register-tiled GEMV, W slice
//                      resident in shared memory
//      MODE 1 hybrid   gz[b,o](t-k) += sum_{i: off[i,o]=k} W[i,o] gr[b,i]   per-source
//                      bucket lists, a (K+1)-slot ring of partial gz in shared memory
//      MODE 2 synaptic gfut[b,o](t-l) += sum_{i,l} W[i,o] h_io(l) gr[b,i]   per-source lag
//                      buckets, an L-slot ring of future gradients in shared memory
//   For MODE 0/1 the recurrent gradient of the spike is the axonal interpolation
//   gfut[b,o](t) = sum_l h_o(l) gz[b,o](t+l) (h of the learned base for the hybrid),
//   read back from the gz written at later steps.
// The double-buffered gr copy makes one cluster barrier per step sufficient.
// Matches the autograd of delrec/delay_layers_pytorch.py:121-194 / 271-325 and the
// reference kernels recdel_base.py:189-285, synaptic_eventdriven.py:323-364.
#pragma once

#include <cooperative_groups.h>

#include "prep.cuh"

namespace cg = cooperative_groups;

namespace delrec {

struct BwdArgs {
  int T, B, N, L, KH, CS, NT, TAPS, NKEY, CAP, KS;
  int MM;                 // hybrid: partial sums gz_m (offsets >= m) kept for m = 0..MM
  const float* gy;
  const float* u;
  const float* keep;
  const float* W;         // (N,N) row-major W[i][o]
  const int* tap_l0;
  const int* tap_nt;
  const float* tap_w;
  const int2* ent;        // bucket entries, CAP per source
  const int* boff;        // (N, NKEY+1)
  float* dx;
  float* gr;
  float* gz;
  int w_smem;
  LifK lif;
};

// shared memory plan (bytes), shared by host and device
struct BwdSmem {
  size_t gr_cur, ws, red, ring, taps, stage, total;
};
__host__ __device__ inline BwdSmem bwd_smem_plan(int mode, int N, int NT, int BT, int KS, int KH, int L,
                                                 int TAPS, int w_smem, int MM) {
  BwdSmem p;
  p.gr_cur = align256((size_t)2 * N * BT * 4);
  p.ws = (mode == 0 && w_smem) ? align256((size_t)N * NT * 4) : 0;
  p.red = (mode == 0) ? align256((size_t)KS * BT * NT * 4) : 0;
  p.ring = mode == 1 ? align256((size_t)(MM + 1) * KH * NT * BT * 4)
                      : (mode == 2 ? align256((size_t)L * NT * BT * 4) : 0);
  p.taps = (mode != 2) ? align256((size_t)NT * (TAPS + 2) * 4) : 0;
  p.stage = mode != 0 ? align256((size_t)8 * 32 * 8) : 0;
  p.total = p.gr_cur + p.ws + p.red + p.ring + p.taps + p.stage;
  return p;
}

template <int MODE, int BT, int PPT>
__global__ void __launch_bounds__(256) k_bwd(BwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int N = a.N, T = a.T, B = a.B, NT = a.NT, NTH = blockDim.x, tid = threadIdx.x;
  const int tile = blockIdx.x / a.CS;
  const int o0 = rank * NT;
  const int nts = max(0, min(NT, N - o0));
  const int b0 = tile * BT;
  const int nb = max(0, min(BT, B - b0));

  const BwdSmem P = bwd_smem_plan(MODE, N, NT, BT, a.KS, a.KH, a.L, a.TAPS, a.w_smem, a.MM);
  const size_t TBN = (size_t)T * B * N;
  float* gr_cur = (float*)smem;                                  // [2][N][BT]
  float* Ws = (float*)(smem + P.gr_cur);                         // [N][NT]
  float* red = (float*)(smem + P.gr_cur + P.ws);                 // [KS][BT][NT]
  float* ring = (float*)(smem + P.gr_cur + P.ws + P.red);        // [slots][NT][BT]
  int* tl0 = (int*)(smem + P.gr_cur + P.ws + P.red + P.ring);    // [NT]
  int* tnt = tl0 + NT;
  float* tw = (float*)(tnt + NT);                                 // [NT][TAPS]
  int2* stage = (int2*)(smem + P.gr_cur + P.ws + P.red + P.ring + P.taps);  // [8 warps][32]

  // ---- init
  for (size_t e = tid; e < (size_t)2 * N * BT; e += NTH) gr_cur[e] = 0.f;
  if (MODE == 0 && a.w_smem) {
    for (size_t e = tid; e < (size_t)N * NT; e += NTH) {
      const int i = (int)(e / NT), ol = (int)(e % NT);
      Ws[e] = ol < nts ? a.W[(size_t)i * N + o0 + ol] : 0.f;
    }
  }
  const int slots = MODE == 1 ? a.KH * (a.MM + 1) : (MODE == 2 ? a.L : 0);
  for (size_t e = tid; e < (size_t)slots * NT * BT; e += NTH) ring[e] = 0.f;
  if (MODE == 1) {
    // gz_m(tau) for tau >= T - m never receives a contribution: store its zeros up front
    for (int m = 1; m <= a.MM; ++m)
      for (int tau = max(0, T - m); tau < T; ++tau)
        for (int p = tid; p < NT * BT; p += NTH) {
          const int bl = p / NT, ol = p % NT;
          if (ol < nts && bl < nb) a.gz[(size_t)m * TBN + ((size_t)tau * B + b0 + bl) * N + o0 + ol] = 0.f;
        }
  }
  if (MODE != 2) {
    for (int ol = tid; ol < NT; ol += NTH) {
      const bool ok = ol < nts;
      tl0[ol] = ok ? a.tap_l0[o0 + ol] : 1;
      tnt[ol] = ok ? a.tap_nt[o0 + ol] : 0;
    }
    for (int e = tid; e < NT * a.TAPS; e += NTH) {
      const int ol = e / a.TAPS;
      tw[e] = ol < nts ? a.tap_w[(size_t)(o0 + ol) * a.TAPS + (e % a.TAPS)] : 0.f;
    }
  }
  float lam[PPT];
#pragma unroll
  for (int k = 0; k < PPT; ++k) lam[k] = 0.f;
  cl.sync();

  const int lane = tid & 31, warp = tid >> 5, nwarp = NTH >> 5;
  constexpr int G = 32 / BT;  // entry groups per warp in the sparse accumulation
  const int bl_lane = lane % BT, g_lane = lane / BT;

  for (int t = T - 1; t >= 0; --t) {
    float* grc = gr_cur + (size_t)(t & 1) * N * BT;
    // ===== A: LIF backward for own (b, o) pairs
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int p = tid + k * NTH;
      const int bl = p / NT, ol = p % NT;
      if (bl >= BT) continue;
      float grv = 0.f;
      if (ol < nts && bl < nb) {
        const int o = o0 + ol, b = b0 + bl;
        const size_t idx = ((size_t)t * B + b) * N + o;
        float gfut = 0.f;
        if (MODE == 2) {
          float* cell = ring + ((size_t)(t % a.L) * NT + ol) * BT + bl;
          gfut = *cell;
          *cell = 0.f;
        } else {
          // gfut = sum_j h(l_j) gz_{m_j}(t + l_j), m_j = max(0, 1 - l_j): a base lag
          // l <= 0 only reaches synapses whose offset is >= 1 - l (their total lag >= 1)
          const int lo = tl0[ol], n = tnt[ol];
          for (int j = 0; j < n; ++j) {
            const int l = lo + j;
            const int m = l < 1 ? 1 - l : 0;
            if (m > a.MM) { flag_status(ST_LAG_RANGE); continue; }
            const int tt = t + l;
            if (tt >= 0 && tt + m < T)
              gfut = fmaf(tw[ol * a.TAPS + j], a.gz[(size_t)m * TBN + (size_t)((long long)idx + (long long)l * B * N)], gfut);
          }
        }
        const float gY = __fadd_rn(a.gy[idx], gfut);
        const float du = lif_backward(gY, a.u[idx], lam[k], a.lif);
        lam[k] = lif_carry(du, a.lif);
        const float kp = a.keep ? a.keep[(size_t)b * N + o] : 1.f;
        grv = __fmul_rn(du, kp);
        a.dx[idx] = du;
        if (a.gr != a.dx) a.gr[idx] = grv;   // (gr is dx itself without dropout)
      }
      if (ol < nts) grc[(size_t)(o0 + ol) * BT + bl] = grv;
    }
    __syncthreads();
    // ===== B: share own slice with the peers, cluster barrier
    if (a.CS > 1 && nts > 0) {
      const int n4 = nts * BT / 4;
      const float4* src = (const float4*)(grc + (size_t)o0 * BT);
      for (int r = 0; r < a.CS; ++r) {
        if (r == rank) continue;
        float4* dst = (float4*)cl.map_shared_rank(grc + (size_t)o0 * BT, r);
        for (int v = tid; v < n4; v += NTH) dst[v] = src[v];
      }
    }
    cl.sync();
    // ===== C: accumulate the contribution of gr(t)
    if (MODE == 0) {
      const int nbt = BT / 4, not4 = NT / 4, tiles = nbt * not4;
      const int tl = tid % tiles, ks = tid / tiles;
      if (ks < a.KS) {
        const int bt = tl / not4, ot = tl % not4;
        const int i0 = (int)(((long long)N * ks) / a.KS), i1 = (int)(((long long)N * (ks + 1)) / a.KS);
        float acc[4][4];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
          for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
        for (int i = i0; i < i1; ++i) {
          const float4 g = *(const float4*)(grc + (size_t)i * BT + bt * 4);
          float4 w;
          if (a.w_smem) {
            w = *(const float4*)(Ws + (size_t)i * NT + ot * 4);
          } else {
            const float* wr = a.W + (size_t)i * N + o0 + ot * 4;
            const int oo = o0 + ot * 4;
            w.x = oo + 0 < N ? __ldg(wr + 0) : 0.f;
            w.y = oo + 1 < N ? __ldg(wr + 1) : 0.f;
            w.z = oo + 2 < N ? __ldg(wr + 2) : 0.f;
            w.w = oo + 3 < N ? __ldg(wr + 3) : 0.f;
          }
          const float gg[4] = {g.x, g.y, g.z, g.w};
          const float ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(gg[x], ww[y], acc[x][y]);
        }
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
          for (int y = 0; y < 4; ++y) red[((size_t)ks * BT + bt * 4 + x) * NT + ot * 4 + y] = acc[x][y];
      }
      __syncthreads();
      for (int p = tid; p < BT * NT; p += NTH) {
        const int bl = p / NT, ol = p % NT;
        if (bl < nb && ol < nts) {
          float sacc = 0.f;
          for (int k = 0; k < a.KS; ++k) sacc = __fadd_rn(sacc, red[((size_t)k * BT + bl) * NT + ol]);
          a.gz[((size_t)t * B + b0 + bl) * N + o0 + ol] = sacc;
        }
      }
    } else {
      // sparse accumulation over the per-source bucket lists; one warp per source.
      // Entries (i, w) are sorted by key and every bucket is padded with (0, 0) to a
      // multiple of 4*G, so key boundaries fall on the warp-uniform loop index.  The
      // warp loads 32 entries at a time (coalesced), stages them in shared memory and
      // prefetches the next chunk while it accumulates the current one; lane b reads
      // gr[i][b] (conflict-free rows).
      int2* sbuf = stage + warp * 32;
      for (int ol = warp; ol < nts; ol += nwarp) {
        const int o = o0 + ol;
        const int* bo = a.boff + (size_t)o * (a.NKEY + 1);
        const int2* E = a.ent + (size_t)o * a.CAP;
        const int total = __ldg(bo + a.NKEY);
        int key = 0;
        int kend = __ldg(bo + 1);
        float acc = 0.f;
        auto flush = [&](int k) {
#pragma unroll
          for (int off = BT; off < 32; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
          const int tau = t - k;
          if (g_lane == 0 && bl_lane < nb && tau >= 0) {
            if (MODE == 1) {
              // bucket k feeds the partial sums of every threshold m <= k
              const int mtop = k < a.MM ? k : a.MM;
              for (int m = 0; m <= mtop; ++m) {
                float* cell = ring + (((size_t)m * a.KH + tau % a.KH) * NT + ol) * BT + bl_lane;
                *cell = __fadd_rn(*cell, acc);
              }
            } else {
              float* cell = ring + ((size_t)(tau % a.L) * NT + ol) * BT + bl_lane;
              *cell = __fadd_rn(*cell, acc);
            }
          }
          acc = 0.f;
        };
        int2 nxt = lane < total ? __ldg(E + lane) : make_int2(0, 0);
        for (int base = 0; base < total; base += 32) {
          __syncwarp();
          sbuf[lane] = nxt;
          __syncwarp();
          nxt = (base + 32 + lane < total) ? __ldg(E + base + 32 + lane) : make_int2(0, 0);
          const int lim = min(32, total - base);
          for (int jj = 0; jj < lim; jj += 4 * G) {
            while (base + jj >= kend) {
              flush(key);
              ++key;
              kend = __ldg(bo + key + 1);
            }
#pragma unroll
            for (int uu = 0; uu < 4; ++uu) {
              const int2 en = sbuf[jj + uu * G + g_lane];
              acc = fmaf(__int_as_float(en.y), grc[(size_t)en.x * BT + bl_lane], acc);
            }
          }
        }
        flush(key);
        if (MODE == 1 && g_lane == 0 && bl_lane < nb) {
          // gz_m(t - m) received its last contribution (offset m) at this step
          for (int m = 0; m <= a.MM; ++m) {
            const int tau = t - m;
            if (tau < 0) break;
            float* cell = ring + (((size_t)m * a.KH + tau % a.KH) * NT + ol) * BT + bl_lane;
            a.gz[(size_t)m * TBN + ((size_t)tau * B + b0 + bl_lane) * N + o] = *cell;
            *cell = 0.f;
          }
        }
      }
    }
    __syncthreads();
  }
  cl.sync();
}

}  // namespace delrec
