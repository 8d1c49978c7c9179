// Parameter-gradient reductions over the T*B rows, run after the reverse scan.
//
// k_syn_cstack_combine  synaptic dW, dd, ds from the per-lag correlation stack
//   C_l[i,o] = sum_{t,b} gr[t,b,i] y[t-l,b,o] (tensor-core GEMMs on the host side), over
//   the lags of each synapse's triangle window (the reference's Cstack,
//   synaptic_eventdriven.py:453-468).
// k_source_pass / k_source_reduce  per-neuron sums: db[n] = sum gr[.,.,n] and, for
//   axonal/hybrid, dmask_n[j] = sum gz[t,b,n] y[t-l0-j,b,n] mapped to dd_n, ds_n through
//   the closed-form triangle derivatives (recdel_base.py:337-342 +
//   AxonalRecdelTriton.backward :421-435).
#pragma once

#include <cuda_bf16.h>

#include "prep.cuh"

namespace delrec {

// Synaptic parameter gradients from the per-lag correlation stack (the reference's Cstack,
// synaptic_eventdriven.py:453-468), computed for all lags on the tensor cores:
//   C_l[i, o] = sum_{t,b} gr[t, b, i] y[t - l, b, o],   l = 0..L-1,
// combined over each synapse's lag window (TW lags from max(1, floor(1+d-s) - 1)):
//   dW = sum_l h(l) C_l,  dd = W sum_l dh/dd(l) C_l,  dsm = W sum_l dh/ds(l) C_l.
template <int TW>
__global__ void k_syn_cstack_combine(int N, int Lm1, const float* __restrict__ dT, const float* __restrict__ s,
                                     const float* __restrict__ W, const float* __restrict__ C,
                                     float* __restrict__ dW, float* __restrict__ dd, float* __restrict__ dsm) {
  const size_t nn = (size_t)N * N;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < nn; e += (size_t)gridDim.x * blockDim.x) {
    const int i = (int)(e / N), o = (int)(e % N);
    const Tri tr = make_tri(dT[(size_t)o * N + i], s[o]);
    const int lo = (int)floorf(__fsub_rn(tr.onepd, tr.s)) - 1;
    const int lag = lo < 1 ? 1 : lo;
    float dw = 0.f, gdd = 0.f, gds = 0.f;
#pragma unroll
    for (int j = 0; j < TW; ++j) {
      const int l = lag + j;
      if (l > Lm1) break;
      const float c = C[(size_t)l * nn + e];
      dw = fmaf(tri_h(tr, l), c, dw);
      gdd = fmaf(tri_dh_dd(tr, l), c, gdd);
      gds = fmaf(tri_dh_ds(tr, l), c, gds);
    }
    if (dW) dW[e] = dw;
    const float w = W[e];
    if (dd) dd[e] = __fmul_rn(w, gdd);
    if (dsm) dsm[e] = __fmul_rn(w, gds);
  }
}

// out[e] = sum_s part[s*n + e]  (fixed order)
__global__ void k_sum_splits(const float* __restrict__ part, int splits, size_t n, float* __restrict__ out) {
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int s2 = 0; s2 < splits; ++s2) v += part[(size_t)s2 * n + e];
    out[e] = v;
  }
}

// ds[o] = sum_i dsm[i,o]  (column sums of a (N,N) matrix, fixed order)
__global__ void k_colsum(const float* __restrict__ m, int R, int C, float* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float v = 0.f;
  for (int r = 0; r < R; ++r) v += m[(size_t)r * C + c];
  out[c] = v;
}

// Per-neuron reductions.  Block = 32 neurons (lanes) x 8 samples (warps); grid.y runs
// over chunks of 8 samples and each block writes one partial row per neuron.
// part layout per chunk: [N][TAPS + 1]  (TAPS dmask sums, then the gr sum)
// Each thread walks its (sample, neuron) through time once: gr and y are read once,
// coalesced over neurons.  y holds the layer's spikes, so
//   dmask[n][j] = sum_{t,b} gz_m[t,b,n] y[t-l_j,b,n] = sum_{(t',b): y != 0} y[t',b,n] gz_m[t'+l_j,b,n]
// reads gz only at the spike times (a few percent of the elements).
struct SrcArgs {
  int T, B, N, TAPS;
  int MM;               // hybrid: a tap at base lag l <= 0 pairs with gz_{1-l}
  const float* gr;
  const float* gz;      // null: only db
  const float* y;
  const int* tap_l0;
  const int* tap_nt;
  const float* tap_w;   // k_source_pass: the taps' weights (z pieces)
  float* part;
  int Np;               // k_source_pass: row stride of the z pieces (N rounded up to 8)
};

template <int TAPSMAX>
__global__ void __launch_bounds__(256) k_source_reduce(SrcArgs a) {
  __shared__ float sred[8][32][TAPSMAX + 1];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int n = blockIdx.x * 32 + lane;
  const int b = blockIdx.y * 8 + w;
  const int N = a.N, B = a.B, T = a.T;
  float dm[TAPSMAX];
  float sg = 0.f;
#pragma unroll
  for (int j = 0; j < TAPSMAX; ++j) dm[j] = 0.f;
  int lo = 1, nt = 0;
  if (n < N && a.gz) { lo = a.tap_l0[n]; nt = a.tap_nt[n]; }
  if (n < N && b < B) {
    const size_t step = (size_t)B * N;
    const size_t TBN = (size_t)T * step;
    const size_t base = (size_t)b * N + n;
    const float* gp = a.gr + base;
    const float* yp = a.y + base;
    const bool want_y = a.gz != nullptr;
    auto spike = [&](int tp, float yv) {
#pragma unroll
      for (int j = 0; j < TAPSMAX; ++j) {
        const int l = lo + j;
        const int tt = tp + l;
        const int m = l < 1 ? 1 - l : 0;
        if (j < nt && m <= a.MM && tt >= 0 && tt < T)
          dm[j] = fmaf(__ldg(a.gz + (size_t)m * TBN + (size_t)tt * step + base), yv, dm[j]);
      }
    };
    int t = 0;
    for (; t + 4 <= T; t += 4) {
      float g[4], yv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        g[q] = __ldcs(gp + (size_t)(t + q) * step);
        yv[q] = want_y ? __ldcs(yp + (size_t)(t + q) * step) : 0.f;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        sg += g[q];
        if (yv[q] != 0.f) spike(t + q, yv[q]);
      }
    }
    for (; t < T; ++t) {
      sg += __ldcs(gp + (size_t)t * step);
      const float yv = want_y ? __ldcs(yp + (size_t)t * step) : 0.f;
      if (yv != 0.f) spike(t, yv);
    }
  }
#pragma unroll
  for (int j = 0; j < TAPSMAX; ++j) sred[w][lane][j] = dm[j];
  sred[w][lane][TAPSMAX] = sg;
  __syncthreads();
  if (w == 0 && n < N) {
    float* out = a.part + ((size_t)blockIdx.y * N + n) * (a.TAPS + 1);
    for (int j = 0; j < a.TAPS; ++j) {
      float v = 0.f;
      for (int g = 0; g < 8; ++g) v += j < TAPSMAX ? sred[g][lane][j] : 0.f;
      out[j] = v;
    }
    float v = 0.f;
    for (int g = 0; g < 8; ++g) v += sred[g][lane][TAPSMAX];
    out[a.TAPS] = v;
  }
}

// One time-major pass per (sample, neuron) for the axonal / hybrid layers, fusing
//   * the per-neuron sums: db partials (sum of gr) and the dmask partials
//     dmask[n][j] = sum_{t,b} gz_m(t)[b,n] y[t - l_j, b, n]  (m = max(0, 1 - l_j)), and
//   * the bf16 pieces (hi, lo) of the interpolated delayed spikes
//     z_m[t,b,o] = sum_{j: l_j >= 1-m} w_o[j] y[t - l_j, b, o]  (the weight-gradient GEMM
//     operand, variant m for synapses whose offset reaches base lags <= 0).
// Block = 32 neurons (lanes) x 8 samples (warps); grid.y over chunks of 8 samples, grid.z
// over time chunks (each first replays the preceding L-1+MM steps of spikes).  gr, y and
// gz_m are streamed once, coalesced, four steps per batch of independent loads.  y holds
// spikes (0/1): the thread keeps its own spike history as a 128-bit shift register (bit
// p = spike at t_in - p), so every lagged spike is a bit test.  Outputs for time te trail
// the input time t_in by MM steps (base lags down to 1-MM look ahead).
// Requires L - 1 + MM <= 127 and MM <= MMX.
// bits [p0, p0 + 32) of the 128-bit history (h1:h0); positions below 0 read as 0
__device__ __forceinline__ uint32_t hist_window(uint64_t h0, uint64_t h1, int p0) {
  if (p0 < 0) return (uint32_t)(h0 << (-p0));
  if (p0 >= 64) return (uint32_t)(h1 >> (p0 - 64));
  if (p0 == 0) return (uint32_t)h0;
  return (uint32_t)((h0 >> p0) | (h1 << (64 - p0)));
}
template <int TAPSMAX, int MMX>
__global__ void __launch_bounds__(256, 2) k_source_pass(SrcArgs a, int want_z, int warm, __nv_bfloat16* __restrict__ zh) {
  __shared__ float sred[8][32][TAPSMAX + 1];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int n = blockIdx.x * 32 + lane;
  const int b = blockIdx.y * 8 + w;
  const int N = a.N, B = a.B, T = a.T, MM = a.MM;
  const int tch = (T + gridDim.z - 1) / gridDim.z;
  const int c0 = blockIdx.z * tch, c1 = min(T, c0 + tch);   // this block's output times
  float dm[TAPSMAX], tw[TAPSMAX];
  float sg = 0.f;
#pragma unroll
  for (int j = 0; j < TAPSMAX; ++j) dm[j] = 0.f;
  int lo = 1, nt = 0;
  if (n < N) {
    lo = a.tap_l0[n];
    nt = a.tap_nt[n];
  }
  // taps j < nt with lag l_j = lo + j; a tap needing offset threshold m_j = max(0, 1-l_j)
  // above MM never contributes.  zmask[m]: taps counted in z variant m (l_j >= 1 - m)
  uint32_t tmask = 0u, zmask[MMX + 1];
#pragma unroll
  for (int m = 0; m <= MMX; ++m) zmask[m] = 0u;
#pragma unroll
  for (int j = 0; j < TAPSMAX; ++j) {
    const int l = lo + j;
    tw[j] = (n < N && j < nt) ? a.tap_w[(size_t)n * a.TAPS + j] : 0.f;
    if (j < nt && 1 - l <= MM) tmask |= 1u << j;
#pragma unroll
    for (int m = 0; m <= MMX; ++m)
      if (j < nt && m <= MM && l >= 1 - m) zmask[m] |= 1u << j;
  }
  if (n < N && b < B && c0 < c1) {
    const size_t step = (size_t)B * N;
    const size_t TBN = (size_t)T * step;
    const size_t ZP = (size_t)T * B * a.Np;   // one z piece (T*B rows of Np)
    const size_t base = (size_t)b * N + n;
    uint64_t h0 = 0ull, h1 = 0ull;
    // warm-up: spikes of the steps before the chunk (8 independent loads per batch)
    const int w0 = max(0, c0 + MM - warm), w1 = min(T, c0 + MM);
    for (int t0 = w0; t0 < w1; t0 += 8) {
      float yw[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) yw[q] = t0 + q < w1 ? __ldcs(a.y + (size_t)(t0 + q) * step + base) : 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (t0 + q >= w1) break;
        h1 = (h1 << 1) | (h0 >> 63);
        h0 = (h0 << 1) | (yw[q] != 0.f ? 1ull : 0ull);
      }
    }
    // outputs te in [c0, c1), inputs t_in = te + MM; the loads of batch k+1 are issued
    // before batch k is processed (two batches in flight per thread)
    constexpr int U = 8;
    float ng[U], nyv[U], ngzv[U][MMX + 1];
    auto load_batch = [&](int t0) {
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int te = t0 + q, tin = te + MM;
        ng[q] = te < c1 ? __ldcs(a.gr + (size_t)te * step + base) : 0.f;
        nyv[q] = (te < c1 && tin < T) ? __ldcs(a.y + (size_t)tin * step + base) : 0.f;
#pragma unroll
        for (int m = 0; m <= MMX; ++m)
          ngzv[q][m] = (a.gz && m <= MM && te < c1) ? __ldcs(a.gz + (size_t)m * TBN + (size_t)te * step + base) : 0.f;
      }
    };
    load_batch(c0);
    for (int t0 = c0; t0 < c1; t0 += U) {
      float g[U], yv[U], gzv[U][MMX + 1];
#pragma unroll
      for (int q = 0; q < U; ++q) {
        g[q] = ng[q];
        yv[q] = nyv[q];
#pragma unroll
        for (int m = 0; m <= MMX; ++m) gzv[q][m] = ngzv[q][m];
      }
      if (t0 + U < c1) load_batch(t0 + U);
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int te = t0 + q;
        if (te >= c1) break;
        sg += g[q];
        h1 = (h1 << 1) | (h0 >> 63);
        h0 = (h0 << 1) | (yv[q] != 0.f ? 1ull : 0ull);
        // bit j: spike at te - l_j  (history bit l_j + MM); spikes before t=0 read as 0
        const uint32_t bits = hist_window(h0, h1, lo + MM) & tmask;
        const size_t zidx = ((size_t)te * B + b) * a.Np + n;
        if (bits == 0u) {
          if (want_z) {
            const __nv_bfloat16 zero = __float2bfloat16_rn(0.f);
            for (int m = 0; m <= MM; ++m) {
              zh[(size_t)m * 2 * ZP + zidx] = zero;
              zh[(size_t)m * 2 * ZP + ZP + zidx] = zero;
            }
          }
          continue;
        }
        if (a.gz) {
#pragma unroll
          for (int j = 0; j < TAPSMAX; ++j) {
            const int mj = lo + j < 1 ? 1 - lo - j : 0;
            float gsel = gzv[q][0];
#pragma unroll
            for (int m = 1; m <= MMX; ++m) gsel = m == mj ? gzv[q][m] : gsel;
            if ((bits >> j) & 1u) dm[j] = __fadd_rn(dm[j], gsel);
          }
        }
        if (want_z) {
#pragma unroll
          for (int m = 0; m <= MMX; ++m) {
            if (m > MM) break;
            const uint32_t zb = bits & zmask[m];
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < TAPSMAX; ++j)
              if ((zb >> j) & 1u) acc = __fadd_rn(acc, tw[j]);
            const __nv_bfloat16 h = __float2bfloat16_rn(acc);
            zh[(size_t)m * 2 * ZP + zidx] = h;
            zh[(size_t)m * 2 * ZP + ZP + zidx] = __float2bfloat16_rn(acc - __bfloat162float(h));
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < TAPSMAX; ++j) sred[w][lane][j] = dm[j];
  sred[w][lane][TAPSMAX] = sg;
  __syncthreads();
  if (w == 0 && n < N) {
    float* out = a.part + (((size_t)blockIdx.z * gridDim.y + blockIdx.y) * N + n) * (a.TAPS + 1);
    for (int j = 0; j < a.TAPS; ++j) {
      float v = 0.f;
      for (int g = 0; g < 8; ++g) v += j < TAPSMAX ? sred[g][lane][j] : 0.f;
      out[j] = v;
    }
    float v = 0.f;
    for (int g = 0; g < 8; ++g) v += sred[g][lane][TAPSMAX];
    out[a.TAPS] = v;
  }
}

// Combine the row splits: db[n], and dd[n], ds[n] from dmask via the triangle derivatives.
// st_dd != 0 (single-tap forward at the integer lag l = 1 + d, recdel_base.py:265-278):
// dd[n] = dmask[l + 1] - dmask[l] straight-through instead, ds untouched.
__global__ void k_source_finalize(int N, int TAPS, int splits, const float* __restrict__ part,
                                  const float* __restrict__ d, const float* __restrict__ s,
                                  const int* __restrict__ l0, const int* __restrict__ nt,
                                  float* db, float* dd, float* ds, int st_dd) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float gsum = 0.f;
  for (int sp = 0; sp < splits; ++sp) gsum += part[((size_t)sp * N + n) * (TAPS + 1) + TAPS];
  if (db) db[n] = gsum;
  if (!dd && !ds) return;
  const Tri tr = make_tri(d[n], s[n]);
  const int lo = l0[n], cnt = nt[n];
  if (st_dd) {
    const int j0 = (int)floorf(tr.onepd + 0.5f) - lo;
    float m0 = 0.f, m1 = 0.f;
    for (int sp = 0; sp < splits; ++sp) {
      const float* pr = part + ((size_t)sp * N + n) * (TAPS + 1);
      if (j0 >= 0 && j0 < cnt) m0 += pr[j0];
      if (j0 + 1 >= 0 && j0 + 1 < cnt) m1 += pr[j0 + 1];
    }
    if (dd) dd[n] = m1 - m0;
    return;
  }
  float gd = 0.f, gs = 0.f;
  for (int j = 0; j < cnt; ++j) {
    float m = 0.f;
    for (int sp = 0; sp < splits; ++sp) m += part[((size_t)sp * N + n) * (TAPS + 1) + j];
    gd = fmaf(m, tri_dh_dd(tr, lo + j), gd);
    gs = fmaf(m, tri_dh_ds(tr, lo + j), gs);
  }
  if (dd) dd[n] = gd;
  if (ds) ds[n] = gs;
}

// closed-form hybrid delay gradient (synaptic_hybrid.py:83-113):
// dd[i,o] = W[i,o] * sum_{l=1}^{LM-1} C[i,o,l] * g(l - 1 - d[i,o]),  g = sign/s^2 on |.|<=s
__global__ void k_hybrid_delay_grad(int N, int LM, const float* __restrict__ C, const float* __restrict__ W,
                                    const float* __restrict__ d, float s, float* __restrict__ dd) {
  const size_t n2 = (size_t)N * N;
  const float inv_s2 = 1.f / (s * s);
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n2; e += (size_t)gridDim.x * blockDim.x) {
    const float dv = d[e];
    float tap = 0.f;
    for (int l = 1; l < LM; ++l) {
      const float aa = (float)l - 1.f - dv;
      float g = aa > 0.f ? inv_s2 : (aa < 0.f ? -inv_s2 : 0.f);
      if (!(fabsf(aa) <= s)) g = 0.f;
      tap = fmaf(g, C[e * LM + l], tap);
    }
    dd[e] = W[e] * tap;
  }
}

}  // namespace delrec
