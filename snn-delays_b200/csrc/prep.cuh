// Per-call preparation kernels (run once per layer forward/backward, O(N^2) work):
// transposed weight/delay copies for coalesced per-event loads, the per-source tap
// tables of the axonal interpolation, and the per-source bucket lists that drive the
// backward's sparse accumulation.  Also the block-wide ordered compaction helper.
#pragma once

#include "common.cuh"

namespace delrec {

// ---------------------------------------------------------------------------------
// ordered block-wide compaction: appends `key` (and `val`) of every thread whose
// `pred` is set, in thread order, at out[base + ...]; returns the number appended.
// Must be called by every thread of the block (blockDim.x a multiple of 32, <= 1024).
// s_warp needs 33 ints.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ int block_compact(bool pred, int key, float val, int* out_k,
                                             float* out_v, int base, int* s_warp) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const unsigned m = __ballot_sync(0xffffffffu, pred);
  if (lane == 0) s_warp[w] = __popc(m);
  __syncthreads();
  if (w == 0) {
    const int v = lane < nw ? s_warp[lane] : 0;
    int inc = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += n;
    }
    if (lane < nw) s_warp[lane] = inc - v;
    if (lane == 31) s_warp[32] = inc;
  }
  __syncthreads();
  if (pred) {
    const int pos = base + s_warp[w] + __popc(m & ((1u << lane) - 1u));
    out_k[pos] = key;
    if (out_v) out_v[pos] = val;
  }
  const int total = s_warp[32];
  __syncthreads();
  return total;
}

// out[c*R + r] = in[r*C + c]   (tiled transpose, 32x32 tiles, 32x8 threads)
__global__ void k_transpose(const float* __restrict__ in, float* __restrict__ out, int R, int C) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int r = r0 + k, c = c0 + threadIdx.x;
    tile[k][threadIdx.x] = (r < R && c < C) ? in[(size_t)r * C + c] : 0.f;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int c = c0 + k, r = r0 + threadIdx.x;
    if (r < R && c < C) out[(size_t)c * R + r] = tile[threadIdx.x][k];
  }
}

// hybrid offsets (N,N) fp32 [i][o] -> uint8 transposed [o][i]; flags values outside [0,K]
__global__ void k_offsets_u8T(const float* __restrict__ off, uint8_t* __restrict__ offT, int N, int K) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int r = r0 + k, c = c0 + threadIdx.x;
    tile[k][threadIdx.x] = (r < N && c < N) ? off[(size_t)r * N + c] : 0.f;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += 8) {
    const int c = c0 + k, r = r0 + threadIdx.x;
    if (r < N && c < N) {
      float v = tile[threadIdx.x][k];
      int iv = (int)v;
      if (!(v >= 0.f) || (float)iv != v || iv > K) { flag_status(ST_INDEX_RANGE); iv = iv < 0 ? 0 : (iv > K ? K : iv); }
      offT[(size_t)c * N + r] = (uint8_t)iv;
    }
  }
}

// Per-source taps of the axonal triangle: for source o, lags l0[o] .. l0[o]+nt[o]-1
// (inside [lmin, L-1]) with weights w[o*TAPS + j] = h(l0 + j; d_o, s_o).  The window
// covers every lag whose clamp input s - |l - (1+d)| is >= 0 (h = 0 at the boundary
// but dh/dd != 0 there), trimmed to it.  lmin = 1 for axonal delays; for the hybrid
// base lmin = 1 - K: a lag l' <= 0 of the base reaches the synapses whose integer
// offset k satisfies l' + k >= 1.
__global__ void k_taps(const float* __restrict__ d, const float* __restrict__ s, int N, int Lm1,
                       int TAPS, int lmin, int* __restrict__ l0, int* __restrict__ nt, float* __restrict__ w) {
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= N) return;
  const Tri tr = make_tri(d[o], s[o]);
  int lo = (int)floorf(__fsub_rn(tr.onepd, tr.s)) - 1;
  int hi = (int)ceilf(__fadd_rn(tr.onepd, tr.s)) + 1;
  lo = lo < lmin ? lmin : lo;
  hi = hi > Lm1 ? Lm1 : hi;
  while (lo <= hi && !(tri_clamped(tr, lo) >= 0.f)) ++lo;
  while (hi >= lo && !(tri_clamped(tr, hi) >= 0.f)) --hi;
  int n = hi - lo + 1;
  if (n < 0) n = 0;
  if (n > TAPS) { flag_status(ST_LAG_RANGE); n = TAPS; }
  l0[o] = lo;
  nt[o] = n;
  for (int j = 0; j < TAPS; ++j) w[(size_t)o * TAPS + j] = j < n ? tri_h(tr, lo + j) : 0.f;
}

// A single tap at lag 1 with weight 1 per neuron (synaptic layers in the hybrid scan:
// gfut(t) = gz(t+1) with the per-synapse lags carried by the bucket keys)
__global__ void k_unit_taps(int N, int* __restrict__ l0, int* __restrict__ nt, float* __restrict__ w) {
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= N) return;
  l0[o] = 1;
  nt[o] = 1;
  w[o] = 1.f;
}

// Scatter records of a hybrid layer's forward, one per synapse (o-major, like WT): the
// positive base taps of source o shifted by the synapse's integer offset k,
//   rec = {lag of the first positive tap + k, fl(W h_0), fl(W h_1), fl(W h_2)},
// with the taps that land below lag 1 zeroed (they never enter the ring).  Sources with
// more than 3 positive taps get lag = INT_MIN: the forward walks their full window.
constexpr int kRecGeneric = -2147483647 - 1;
__global__ void k_syn_records(int N, int L, const uint8_t* __restrict__ offT, const float* __restrict__ WT,
                              const int* __restrict__ l0, const int* __restrict__ nt,
                              const float* __restrict__ tw, int TAPS, int4* __restrict__ rec) {
  const size_t nn = (size_t)N * N;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < nn; e += (size_t)gridDim.x * blockDim.x) {
    const int o = (int)(e / N);
    const float* h = tw + (size_t)o * TAPS;
    const int n = nt[o];
    int first = -1, cnt = 0;
    for (int j = 0; j < n; ++j)
      if (h[j] > 0.f) {
        if (first < 0) first = j;
        cnt = j - first + 1;
      }
    int4 r = make_int4(1, 0, 0, 0);
    if (cnt > 3) {
      r.x = kRecGeneric;
    } else if (first >= 0) {
      const int lag0 = l0[o] + first + (int)offT[e];
      const float w = WT[e];
      float ws[3];
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int l = lag0 + q;
        ws[q] = (q < cnt && l >= 1) ? __fmul_rn(w, h[first + q]) : 0.f;
        if (q < cnt && l > L - 1) {
          flag_status(ST_LAG_RANGE);
          ws[q] = 0.f;
        }
      }
      r = make_int4(lag0, __float_as_int(ws[0]), __float_as_int(ws[1]), __float_as_int(ws[2]));
    }
    rec[e] = r;
  }
}

// Scatter records of a synaptic layer's forward (o-major): the positive lags of the
// synapse's own triangle, rec = {first lag, fl(W fl(c_l / s^2)) for the next three lags}
// (exactly the products the per-event loop forms), INT_MIN for wider triangles.
__global__ void k_syn_records_syn(int N, int L, const float* __restrict__ dT, const float* __restrict__ s,
                                  const float* __restrict__ WT, int4* __restrict__ rec) {
  const size_t nn = (size_t)N * N;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < nn; e += (size_t)gridDim.x * blockDim.x) {
    const int o = (int)(e / N);
    const Tri tr = make_tri(dT[e], s[o]);
    int lo = (int)floorf(__fsub_rn(tr.onepd, tr.s));
    int hi = (int)ceilf(__fadd_rn(tr.onepd, tr.s));
    lo = lo < 1 ? 1 : lo;
    if (hi > L - 1) {
      if (tri_clamped(tr, L) > 0.f) flag_status(ST_LAG_RANGE);
      hi = L - 1;
    }
    int first = -1, cnt = 0;
    for (int l = lo; l <= hi; ++l)
      if (tri_clamped(tr, l) > 0.f) {
        if (first < 0) first = l;
        cnt = l - first + 1;
      }
    int4 r = make_int4(1, 0, 0, 0);
    if (cnt > 3) {
      r.x = kRecGeneric;
    } else if (first >= 0) {
      const float w = WT[e];
      float ws[3];
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const float c = q < cnt ? tri_clamped(tr, first + q) : 0.f;
        ws[q] = c > 0.f ? __fmul_rn(w, __fdiv_rn(c, tr.s2)) : 0.f;
      }
      r = make_int4(first, __float_as_int(ws[0]), __float_as_int(ws[1]), __float_as_int(ws[2]));
    }
    rec[e] = r;
  }
}

// Dense triangle mask out[r*L + l] (build_mask / build_syn_mask)
__global__ void k_build_mask(int R, int L, const float* __restrict__ d, const float* __restrict__ s,
                             int s_period, float* __restrict__ out) {
  const size_t n = (size_t)R * L;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / L), l = (int)(e % L);
    const Tri tr = make_tri(d[r], s[r % s_period]);
    out[e] = tri_h(tr, l);
  }
}

// Backward bucket lists.  For each source o, the targets i are listed grouped by an
// integer key and in increasing i within a key:
//   hybrid   key = offset k_io in [0, NKEY-1], weight W[i,o]            (one entry per synapse)
//   synaptic key = lag l in [1, NKEY-1] of every nonzero tap, weight fl(W[i,o] * h_io(l))
// ent[o*CAP + e] = (i, weight bits); boff[o*(NKEY+1) + key] = first entry of the key.
// One block per source.
// Every bucket is padded with (0, 0.0f) entries to a multiple of PADM.
template <int MODE>  // 1 hybrid, 2 synaptic
__global__ void k_buckets(int N, int NKEY, int CAP, int PADM, const float* __restrict__ W,
                          const uint8_t* __restrict__ offT, const float* __restrict__ dT,
                          const float* __restrict__ s, int2* __restrict__ ent, int* __restrict__ boff) {
  __shared__ int s_warp[33];
  extern __shared__ int s_dyn[];
  int* s_k = s_dyn;                                 // keys of the current round (compaction)
  float* s_v = (float*)(s_dyn + blockDim.x);
  const int o = blockIdx.x;
  int2* E = ent + (size_t)o * CAP;
  int* bo = boff + (size_t)o * (NKEY + 1);
  int cnt = 0;
  for (int key = 0; key < NKEY; ++key) {
    if (threadIdx.x == 0) bo[key] = cnt;
    for (int r0 = 0; r0 < N; r0 += blockDim.x) {
      const int i = r0 + threadIdx.x;
      bool pred = false;
      float wv = 0.f;
      if (i < N) {
        const float wio = W[(size_t)i * N + o];
        if (MODE == 1) {
          pred = (int)offT[(size_t)o * N + i] == key;
          wv = wio;
        } else {
          const Tri tr = make_tri(dT[(size_t)o * N + i], s[o]);
          if (key >= 1) {
            const float c = tri_clamped(tr, key);
            if (c > 0.f) {
              pred = true;
              wv = __fmul_rn(wio, __fdiv_rn(c, tr.s2));
            }
          }
        }
      }
      const int n = block_compact(pred, i, wv, s_k, s_v, 0, s_warp);
      for (int e = threadIdx.x; e < n; e += blockDim.x) {
        if (cnt + e < CAP) E[cnt + e] = make_int2(s_k[e], __float_as_int(s_v[e]));
        else flag_status(ST_INDEX_RANGE);
      }
      cnt += n;
      __syncthreads();
    }
    const int padded = ((cnt + PADM - 1) / PADM) * PADM;
    for (int e = cnt + threadIdx.x; e < padded; e += blockDim.x) {
      if (e < CAP) E[e] = make_int2(0, 0);
      else flag_status(ST_INDEX_RANGE);
    }
    cnt = padded;
    __syncthreads();
  }
  if (threadIdx.x == 0) bo[NKEY] = cnt < CAP ? cnt : CAP;
}

}  // namespace delrec
