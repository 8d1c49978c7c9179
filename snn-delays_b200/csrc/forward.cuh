// Forward time scans.  One thread block owns one sample for all T steps and all N
// neurons, so the recurrence never leaves the block; per step it
//   * axonal:  gathers z_o = sum_l h_o(l) y[t-l,o] from a bit-packed spike history in
//              shared memory, compacts the nonzero z into an event list, and accumulates
//              rec_i = sum_events W[i,o] z_o in registers (spike-sparse: only sources with
//              a spike inside their delay window cost anything);
//   * synaptic / hybrid: reads rec from a delay ring (shared memory when it fits),
//              runs the LIF update, compacts the neurons that fired, and scatters each
//              fired source's W[:,o] * h(l; d_io) into the ring slots t+l of its targets.
// Matches delrec/delay_layers_pytorch.py:121-194 (axonal v2) and :271-325 (synaptic
// v2); the hybrid delay d[i,o] = base[o] + offsets[i,o] (networks.py:823-829) is formed
// on the fly from a uint8 offset table.
#pragma once

#include "prep.cuh"

namespace delrec {

struct FwdArgs {
  int T, B, N, L, R, NW, TAPS;
  const float* x;
  const float* WT;        // W transposed: WT[o*N + i] = W[i,o]
  const int4* rec;        // per-synapse scatter records (k_syn_records / k_syn_records_syn)
  const float* bias;      // (N) or null
  const float* keep;      // (B,N) or null
  const float* s;         // (N) half-widths
  const float* dT;        // synaptic: d transposed (N,N)
  const uint8_t* offT;    // hybrid: offsets transposed (N,N)
  const float* base;      // hybrid base (N)
  const int* tap_l0;
  const int* tap_nt;
  const float* tap_w;
  float* y;
  float* u;
  float* ring_g;          // global ring (B, L, N) when it does not fit in shared memory
  int ring_smem;
  LifK lif;
};

// --------------------------------------------------------------------------------
// axonal: z-gather + register accumulation.   dynamic smem:
//   hist  R*NW u32 | l0 N int | nt N int | w N*TAPS f32 | ev_o N int | ev_z N f32
// --------------------------------------------------------------------------------
template <int IPT>
__global__ void __launch_bounds__(512, 2) k_fwd_axonal(FwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_warp[33];
  const int N = a.N, T = a.T, B = a.B, NTH = blockDim.x, tid = threadIdx.x;
  const int b = blockIdx.x;
  uint32_t* hist = (uint32_t*)smem;
  int* sl0 = (int*)(hist + (size_t)a.R * a.NW);
  int* snt = sl0 + N;
  float* sw = (float*)(snt + N);
  int* ev_o = (int*)(sw + (size_t)N * a.TAPS);
  float* ev_z = (float*)(ev_o + N);

  for (int e = tid; e < a.R * a.NW; e += NTH) hist[e] = 0u;
  for (int o = tid; o < N; o += NTH) { sl0[o] = a.tap_l0[o]; snt[o] = a.tap_nt[o]; }
  for (int e = tid; e < N * a.TAPS; e += NTH) sw[e] = a.tap_w[e];

  float v[IPT], kp[IPT], bs[IPT];
#pragma unroll
  for (int q = 0; q < IPT; ++q) {
    const int i = q * NTH + tid;
    v[q] = a.lif.v0;
    kp[q] = (a.keep && i < N) ? a.keep[(size_t)b * N + i] : 1.f;
    bs[q] = (a.bias && i < N) ? a.bias[i] : 0.f;
  }
  __syncthreads();

  const int rounds = cdiv(N, NTH);
  for (int t = 0; t < T; ++t) {
    // ---- z gather + compaction of the nonzero delayed inputs
    int nev = 0;
    for (int r = 0; r < rounds; ++r) {
      const int o = r * NTH + tid;
      float z = 0.f;
      if (o < N) {
        const int lo = sl0[o], n = snt[o];
        const int word = o >> 5;
        const uint32_t bit = 1u << (o & 31);
        for (int j = 0; j < n; ++j) {
          const int tt = t - lo - j;
          if (tt >= 0 && (hist[(size_t)(tt & (a.R - 1)) * a.NW + word] & bit))
            z = __fadd_rn(z, sw[(size_t)o * a.TAPS + j]);
        }
      }
      nev += block_compact(z != 0.f, o, z, ev_o, ev_z, nev, s_warp);
    }
    // ---- rec_i = sum over events of W[i,o] * z_o
    // The W rows of EV events are loaded together (the loads depend only on the
    // compacted event list), then accumulated in event order.
    constexpr int EV = IPT >= 8 ? 2 : 16 / IPT;
    float acc[IPT];
#pragma unroll
    for (int q = 0; q < IPT; ++q) acc[q] = 0.f;
    for (int e0 = 0; e0 < nev; e0 += EV) {
      const int cnt = min(EV, nev - e0);
      float wv[EV][IPT], zv[EV];
#pragma unroll
      for (int k = 0; k < EV; ++k) {
        zv[k] = 0.f;
#pragma unroll
        for (int q = 0; q < IPT; ++q) wv[k][q] = 0.f;
        if (k < cnt) {
          const float* wrow = a.WT + (size_t)ev_o[e0 + k] * N;
          zv[k] = ev_z[e0 + k];
#pragma unroll
          for (int q = 0; q < IPT; ++q) {
            const int i = q * NTH + tid;
            if (i < N) wv[k][q] = __ldg(wrow + i);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < EV; ++k)
        if (k < cnt) {
#pragma unroll
          for (int q = 0; q < IPT; ++q) acc[q] = fmaf(wv[k][q], zv[k], acc[q]);
        }
    }
    // ---- LIF, outputs, spike bits
    const size_t rowoff = ((size_t)t * B + b) * N;
#pragma unroll
    for (int q = 0; q < IPT; ++q) {
      const int i = q * NTH + tid;
      bool sp = false;
      if (i < N) {
        const float rec = __fmul_rn(__fadd_rn(acc[q], bs[q]), kp[q]);
        const float av = __fadd_rn(a.x[rowoff + i], rec);
        const float uu = lif_charge(v[q], av, a.lif);
        sp = lif_fire(uu, a.lif);
        v[q] = lif_reset(uu, sp, a.lif);
        a.y[rowoff + i] = sp ? 1.f : 0.f;
        a.u[rowoff + i] = uu;
      }
      const unsigned m = __ballot_sync(0xffffffffu, sp);
      const int word = (q * NTH + (tid & ~31)) >> 5;
      if ((tid & 31) == 0 && word < a.NW) hist[(size_t)(t & (a.R - 1)) * a.NW + word] = m;
    }
    __syncthreads();
  }
}

// --------------------------------------------------------------------------------
// axonal, 4 neurons per thread (N % 4 == 0, 16-byte aligned x / y / u / WT rows): the
// same step as k_fwd_axonal with every event costing one 16-byte W load and four FMAs
// per thread instead of one load and one FMA, so the per-event bookkeeping (event
// read, address) is shared by four targets.  The events are compacted in ascending
// source order and accumulated in that order, so the result equals k_fwd_axonal's
// bit for bit.   dynamic smem: hist R*NW u32 | l0 N int | nt N int | w N*TAPS f32 | ev N int2
// --------------------------------------------------------------------------------
template <int EV>
__global__ void __launch_bounds__(256) k_fwd_axonal4(FwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_warp[8];
  const int N = a.N, T = a.T, B = a.B, NTH = blockDim.x, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, nw = NTH >> 5;
  const int b = blockIdx.x;
  uint32_t* hist = (uint32_t*)smem;
  int* sl0 = (int*)(hist + (size_t)a.R * a.NW);
  int* snt = sl0 + N;
  float* sw = (float*)(snt + N);
  int2* ev = (int2*)(sw + (size_t)N * a.TAPS);

  for (int e = tid; e < a.R * a.NW; e += NTH) hist[e] = 0u;
  for (int o = tid; o < N; o += NTH) { sl0[o] = a.tap_l0[o]; snt[o] = a.tap_nt[o]; }
  for (int e = tid; e < N * a.TAPS; e += NTH) sw[e] = a.tap_w[e];

  const int i0 = 4 * tid;       // the thread's neurons i0 .. i0+3 (targets, and sources of the gather)
  const bool act = i0 < N;
  float v[4], kp[4], bs[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[q] = a.lif.v0;
    kp[q] = (a.keep && act) ? a.keep[(size_t)b * N + i0 + q] : 1.f;
    bs[q] = (a.bias && act) ? a.bias[i0 + q] : 0.f;
  }
  float4 xn = make_float4(0.f, 0.f, 0.f, 0.f);   // x of the next step, loaded a step ahead
  if (act && T > 0) xn = __ldcs((const float4*)(a.x + (size_t)b * N + i0));
  __syncthreads();

  for (int t = 0; t < T; ++t) {
    const float4 x4 = xn;
    if (act && t + 1 < T) xn = __ldcs((const float4*)(a.x + ((size_t)(t + 1) * B + b) * N + i0));
    // ---- z gather of the thread's 4 sources
    float z[4];
    int c = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      z[q] = 0.f;
      if (act) {
        const int o = i0 + q;
        const int lo = sl0[o], n = snt[o];
        const uint32_t bit = 1u << (o & 31);
        for (int j = 0; j < n; ++j) {
          const int tt = t - lo - j;
          if (tt >= 0 && (hist[(size_t)(tt & (a.R - 1)) * a.NW + (o >> 5)] & bit))
            z[q] = __fadd_rn(z[q], sw[(size_t)o * a.TAPS + j]);
        }
        c += z[q] != 0.f;
      }
    }
    // ---- compaction in ascending source order (block scan of the per-thread counts)
    int inc = c;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += n;
    }
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    int pos = inc - c, nev = 0;
    for (int w2 = 0; w2 < nw; ++w2) {
      const int cw = s_warp[w2];
      if (w2 < warp) pos += cw;
      nev += cw;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (z[q] != 0.f) ev[pos++] = make_int2(i0 + q, __float_as_int(z[q]));
    __syncthreads();
    // ---- rec_i = sum over events of W[i,o] z_o: the W rows of EV events loaded together
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int e0 = 0; e0 < nev; e0 += EV) {
      const int cnt = min(EV, nev - e0);
      float4 wv[EV];
      float zv[EV];
#pragma unroll
      for (int k = 0; k < EV; ++k) {
        zv[k] = 0.f;
        wv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k < cnt) {
          const int2 e = ev[e0 + k];
          zv[k] = __int_as_float(e.y);
          if (act) wv[k] = __ldg((const float4*)(a.WT + (size_t)e.x * N + i0));
        }
      }
#pragma unroll
      for (int k = 0; k < EV; ++k)
        if (k < cnt) {
          acc.x = fmaf(wv[k].x, zv[k], acc.x);
          acc.y = fmaf(wv[k].y, zv[k], acc.y);
          acc.z = fmaf(wv[k].z, zv[k], acc.z);
          acc.w = fmaf(wv[k].w, zv[k], acc.w);
        }
    }
    // ---- LIF, outputs, spike bits (8 threads fill one 32-neuron history word)
    unsigned nib = 0;
    if (act) {
      const size_t rowoff = ((size_t)t * B + b) * N + i0;
      const float xa[4] = {x4.x, x4.y, x4.z, x4.w};
      const float ra[4] = {acc.x, acc.y, acc.z, acc.w};
      float ya[4], ua[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float rec = __fmul_rn(__fadd_rn(ra[q], bs[q]), kp[q]);
        const float av = __fadd_rn(xa[q], rec);
        const float uu = lif_charge(v[q], av, a.lif);
        const bool sp = lif_fire(uu, a.lif);
        v[q] = lif_reset(uu, sp, a.lif);
        ya[q] = sp ? 1.f : 0.f;
        ua[q] = uu;
        nib |= (sp ? 1u : 0u) << q;
      }
      __stcs((float4*)(a.y + rowoff), make_float4(ya[0], ya[1], ya[2], ya[3]));
      __stcs((float4*)(a.u + rowoff), make_float4(ua[0], ua[1], ua[2], ua[3]));
    }
    unsigned wd = nib << (4 * (lane & 7));
    wd |= __shfl_xor_sync(0xffffffffu, wd, 1);
    wd |= __shfl_xor_sync(0xffffffffu, wd, 2);
    wd |= __shfl_xor_sync(0xffffffffu, wd, 4);
    if ((lane & 7) == 0 && act) hist[(size_t)(t & (a.R - 1)) * a.NW + (i0 >> 5)] = wd;
    __syncthreads();
  }
}

// --------------------------------------------------------------------------------
// synaptic / hybrid: delay ring + spike-event scatter.   dynamic smem:
//   ring L*N f32 (if ring_smem) | ev_o N int | s N f32 | base N f32
//   | hybrid: tap l0 N int | tap count N int | tap weights N*TAPS f32
// The global loads of up to 8 events (W row element, delay or offset) are issued
// together before their ring updates, so a step waits on about one L2 round trip
// instead of one per fired source; the ring cells still receive the events in order.
// Hybrid synapses use the integer-offset identity h(l; base_o + k) = h(l - k; base_o):
// the source's base taps (lags l0_o + j, weights h(l0_o + j; base_o)) land k slots
// later, so the per-synapse work is one offset byte, one weight and a few adds.
// --------------------------------------------------------------------------------
template <int IPT, bool HYB>
__global__ void __launch_bounds__(512) k_fwd_synaptic(FwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_warp[33];
  constexpr int EB = 8;
  const int N = a.N, T = a.T, B = a.B, L = a.L, NTH = blockDim.x, tid = threadIdx.x;
  const int b = blockIdx.x;
  float* ring;
  int* ev_o;
  if (a.ring_smem) {
    ring = (float*)smem;
    ev_o = (int*)(ring + (size_t)L * N);
  } else {
    ring = a.ring_g + (size_t)b * L * N;
    ev_o = (int*)smem;
  }
  float* s_s = (float*)(ev_o + N);
  float* s_base = s_s + N;
  int* s_l0 = (int*)(s_base + N);
  int* s_nt = s_l0 + N;
  float* s_tw = (float*)(s_nt + N);
  for (size_t e = tid; e < (size_t)L * N; e += NTH) ring[e] = 0.f;
  for (int o = tid; o < N; o += NTH) {
    s_s[o] = a.s[o];
    s_base[o] = HYB ? a.base[o] : 0.f;
    if (HYB) {
      s_l0[o] = a.tap_l0[o];
      s_nt[o] = a.tap_nt[o];
    }
  }
  if (HYB)
    for (int e = tid; e < N * a.TAPS; e += NTH) s_tw[e] = a.tap_w[e];

  float v[IPT], kp[IPT], bs[IPT], xn[IPT];
#pragma unroll
  for (int q = 0; q < IPT; ++q) {
    const int i = q * NTH + tid;
    v[q] = a.lif.v0;
    kp[q] = (a.keep && i < N) ? a.keep[(size_t)b * N + i] : 1.f;
    bs[q] = (a.bias && i < N) ? a.bias[i] : 0.f;
    xn[q] = (i < N && T > 0) ? __ldcs(a.x + (size_t)b * N + i) : 0.f;
  }
  __syncthreads();

  int slot = 0;  // t mod L
  for (int t = 0; t < T; ++t) {
    const size_t rowoff = ((size_t)t * B + b) * N;
    float xc[IPT];
#pragma unroll
    for (int q = 0; q < IPT; ++q) {
      const int i = q * NTH + tid;
      xc[q] = xn[q];
      xn[q] = (i < N && t + 1 < T) ? __ldcs(a.x + rowoff + (size_t)B * N + i) : 0.f;
    }
    int nev = 0;
#pragma unroll
    for (int q = 0; q < IPT; ++q) {
      const int i = q * NTH + tid;
      bool sp = false;
      if (i < N) {
        float* cell = ring + (size_t)slot * N + i;
        const float rsum = *cell;
        *cell = 0.f;
        const float rec = __fmul_rn(__fadd_rn(rsum, bs[q]), kp[q]);
        const float av = __fadd_rn(xc[q], rec);
        const float uu = lif_charge(v[q], av, a.lif);
        sp = lif_fire(uu, a.lif);
        v[q] = lif_reset(uu, sp, a.lif);
        __stcs(a.y + rowoff + i, sp ? 1.f : 0.f);
        __stcs(a.u + rowoff + i, uu);
      }
      nev += block_compact(sp, i, 0.f, ev_o, nullptr, nev, s_warp);
    }
    // ---- scatter the fired sources into the ring (lags 1..L-1)
    for (int e0 = 0; e0 < nev; e0 += EB) {
      const int ne = min(EB, nev - e0);
      int oo[EB];
#pragma unroll
      for (int j = 0; j < EB; ++j) oo[j] = j < ne ? ev_o[e0 + j] : 0;
#pragma unroll
      for (int q = 0; q < IPT; ++q) {
        const int i = q * NTH + tid;
        if (i >= N) continue;
        // 16-byte records, four in flight (the kernel runs two blocks per SM: 64 registers)
        constexpr int RB = 4;
#pragma unroll
        for (int j0 = 0; j0 < EB; j0 += RB) {   // static: the event ids stay in registers
          if (j0 >= ne) break;
          int4 rv[RB];
#pragma unroll
          for (int jj = 0; jj < RB; ++jj)
            if (j0 + jj < ne) rv[jj] = __ldg(a.rec + (size_t)oo[j0 + jj] * N + i);
#pragma unroll
          for (int jj = 0; jj < RB; ++jj) {
            const int j = j0 + jj;
            if (j >= ne) break;
            const int4 r = rv[jj];
            if (r.x != kRecGeneric) {
              const float wq[3] = {__int_as_float(r.y), __int_as_float(r.z), __int_as_float(r.w)};
#pragma unroll
              for (int q2 = 0; q2 < 3; ++q2) {
                if (wq[q2] != 0.f) {
                  int sl = slot + r.x + q2;   // lag in [1, L-1]
                  if (sl >= L) sl -= L;
                  float* cell = ring + (size_t)sl * N + i;
                  *cell = __fadd_rn(*cell, wq[q2]);
                }
              }
              continue;
            }
            // a synapse with a wide window: walk it
            const int o = oo[j];
            const size_t off = (size_t)o * N + i;
            const float wj = __ldg(a.WT + off);
            if (HYB) {   // every tap of the base, shifted by the offset
              const int lo = s_l0[o] + (int)a.offT[off], n = s_nt[o];
              const float* hw = s_tw + (size_t)o * a.TAPS;
              for (int q2 = 0; q2 < n; ++q2) {
                const float h = hw[q2];
                const int l = lo + q2;
                if (!(h > 0.f) || l < 1) continue;
                if (l > L - 1) { flag_status(ST_LAG_RANGE); continue; }
                int sl = slot + l;
                if (sl >= L) sl -= L;
                float* cell = ring + (size_t)sl * N + i;
                *cell = __fadd_rn(*cell, __fmul_rn(wj, h));
              }
            } else {     // the synapse's own triangle
              const Tri tr = make_tri(__ldg(a.dT + off), s_s[o]);
              int lo = (int)floorf(__fsub_rn(tr.onepd, tr.s));
              int hi = (int)ceilf(__fadd_rn(tr.onepd, tr.s));
              lo = lo < 1 ? 1 : lo;
              if (hi > L - 1) {
                if (tri_clamped(tr, L) > 0.f) flag_status(ST_LAG_RANGE);
                hi = L - 1;
              }
              for (int l = lo; l <= hi; ++l) {
                const float c = tri_clamped(tr, l);
                if (c > 0.f) {
                  int sl = slot + l;
                  if (sl >= L) sl -= L;
                  float* cell = ring + (size_t)sl * N + i;
                  *cell = __fadd_rn(*cell, __fmul_rn(wj, __fdiv_rn(c, tr.s2)));
                }
              }
            }
          }
        }
      }
    }
    __syncthreads();
    slot = (slot + 1 == L) ? 0 : slot + 1;
  }
}

}  // namespace delrec
