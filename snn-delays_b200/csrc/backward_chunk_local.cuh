// Sample-local form of the chunked reverse scan's step part (see backward_chunk.cuh for
// the chunking): a block owns S samples (1 or 2) and every source neuron of the layer, so the
// step needs no exchange of gr between blocks and no grid-wide wait.  This is possible
// because, with the long-lag synapses contracted by the chunk GEMM, a step only sums the
// short-lag synapses (l0_o + k_io <= 7, 12 % at BASELINE config 4): their bucket lists
// (16-bit target, fp32 weight; about 195 KB at N = 512) are shared by every block and
// stay in L1 / L2, while the per-sample state -- the LIF carry, gr(t) of the block's
// samples and the per-source ring of this chunk's short contributions -- is in shared
// memory.  Per step t (position q = t - t0 in the chunk):
//   A. LIF backward of the block's (sample, source) pairs: gfut from gz (later chunks,
//      prefetched a step ahead) plus the ring; gr(t) to shared memory and global memory
//      (fp32 and the bf16 pieces of the chunk GEMM);
//   C. for every source o with a short bucket k <= q - l0_o, the bucket sum of gr(t) over
//      its targets into ring slot t - k (read by a later step of this chunk): one warp
//      per source, lanes over the bucket's entries, a shuffle reduction per sample.
// The blocks are independent (a plain launch, no co-residency needed).
#pragma once

#include "backward_chunk.cuh"

namespace delrec {

constexpr int kLocSMax = 2, kLocThreads = 512, kLocGroup = 8;   // lanes per (source, bucket) pair
constexpr int kLocPairCache = 1024;   // pairs staged in shared memory (the rest read from global)

// The short prefix of every source's bucket list (buckets k <= min(K, 7 - l0)) split into
// 16-bit targets and fp32 weights (6 bytes per entry, same row layout as `ent`).
__global__ void k_short_entries(int N, int K, int CAP, int boff_stride, const int2* __restrict__ ent,
                                const int* __restrict__ boff, const int* __restrict__ tap_l0,
                                uint16_t* __restrict__ sidx, float* __restrict__ sw) {
  const int o = blockIdx.x;
  if (o >= N) return;
  const int kl = min(K, kChunk - 1 - tap_l0[o]);
  const int tot = kl >= 0 ? min(boff[(size_t)o * boff_stride + kl + 1], CAP) : 0;
  for (int pos = threadIdx.x; pos < tot; pos += blockDim.x) {
    const int2 e = ent[(size_t)o * CAP + pos];
    sidx[(size_t)o * CAP + pos] = (uint16_t)e.x;
    sw[(size_t)o * CAP + pos] = __int_as_float(e.y);
  }
}

// Shared memory of the step kernel: taps, the per-source ring of this chunk's short
// contributions, gr(t) of the block's samples, the pair counts per chunk position; the
// rest caches the short entries of the smallest lags.
struct LocSmem {
  size_t taps, ring, grs, cnt, pairs, fixed;
};
__host__ __device__ inline LocSmem loc_smem_plan(int N, int TAPS, int S) {
  LocSmem p;
  p.taps = align256((size_t)N * (2 + TAPS) * 4);                // l0, n, weights
  p.ring = align256((size_t)N * kChunk * S * 4);                // [N][8][S]
  p.grs = align256((size_t)S * N * 4);                          // gr(t) [S][N]
  p.cnt = 256;                                                  // pairs with lag <= q
  p.pairs = (size_t)kLocPairCache * 16;                        // the first (source, bucket) pairs
  p.fixed = p.taps + p.ring + p.grs + p.cnt + p.pairs;
  return p;
}
// entries (6 bytes each) the shared-memory cache of a block with `smem` bytes holds
__host__ __device__ inline int loc_entry_cap(size_t smem, const LocSmem& p) {
  if (smem <= p.fixed + 512) return 0;
  const size_t room = smem - p.fixed - 512;   // two 256-byte alignment pads
  return (int)(room / 6) & ~7;
}

// Exclusive prefix sum of one value per thread over a block of kLocThreads threads
// (scratch: 17 ints of shared memory); returns the thread's prefix, *total the sum.
__device__ __forceinline__ int loc_block_exscan(int v, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, inc, m);
    if (lane >= m) inc += u;
  }
  if (lane == 31) scratch[warp] = inc;
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int w = 0; w < kLocThreads / 32; ++w) {
      const int x = scratch[w];
      scratch[w] = run;
      run += x;
    }
    scratch[16] = run;
  }
  __syncthreads();
  const int r = scratch[warp] + inc - v;
  *total = scratch[16];
  __syncthreads();
  return r;
}

// Once per layer backward (one block of kLocThreads threads): the short buckets (k <=
// min(K, 7 - l0)) as (source, bucket) pairs sorted by their total lag lambda = l0 + k,
// and a compact copy of the entries of the smallest lags, 1..lam_s, that fit a step
// kernel's shared-memory cache of `ecap` entries.
//   pairs[j] = {o | k << 16, begin, end, cached}: entries [begin, end) of the compact
//   cache (cached) or of the (N, CAP) short-entry rows;  cnt[q] = pairs with lambda <= q;
//   meta = {lam_s, cached entries}.
__global__ void __launch_bounds__(kLocThreads, 1)
    k_short_pairs(int N, int K, int CAP, int boff_stride, const int* __restrict__ boff,
                  const int* __restrict__ tap_l0, const uint16_t* __restrict__ sidx,
                  const float* __restrict__ sw, int ecap, uint16_t* __restrict__ cidx, float* __restrict__ cw,
                  int4* __restrict__ pairs, int* __restrict__ cnt, int* __restrict__ meta) {
  __shared__ int s_ent[kChunk], s_pair[kChunk], s_scan[17], s_lam;
  __shared__ int s_cum[1024 + 1];   // cache offset of each source (N <= 1024)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < kChunk) s_ent[tid] = s_pair[tid] = 0;
  __syncthreads();
  for (int o = tid; o < N; o += kLocThreads) {
    const int l0 = tap_l0[o], kl = min(K, kChunk - 1 - l0);
    for (int k = 0; k <= kl; ++k) {
      const int n = boff[(size_t)o * boff_stride + k + 1] - boff[(size_t)o * boff_stride + k];
      atomicAdd(&s_ent[l0 + k], n);
      atomicAdd(&s_pair[l0 + k], 1);
    }
  }
  __syncthreads();
  if (tid == 0) {
    int tot = 0, lam = 0;
    for (int l = 1; l < kChunk; ++l) {
      tot += s_ent[l];
      if (tot > ecap) break;
      lam = l;
    }
    s_lam = lam;
  }
  __syncthreads();
  const int lam_s = s_lam;
  // compact cache: each source's entries of lags <= lam_s, sources in order
  int carry = 0;
  for (int o0 = 0; o0 < N; o0 += kLocThreads) {
    const int o = o0 + tid;
    int len = 0;
    if (o < N) {
      const int kc = min(min(K, kChunk - 1 - tap_l0[o]), lam_s - tap_l0[o]);
      len = kc >= 0 ? min(boff[(size_t)o * boff_stride + kc + 1], CAP) : 0;
    }
    int total;
    const int at = carry + loc_block_exscan(len, s_scan, &total);
    if (o < N) s_cum[o] = at;
    carry += total;
  }
  if (tid == 0) s_cum[min(N, 1024)] = carry;
  __syncthreads();
  // the cached prefixes, copied as one flat range: entry e belongs to the last source o
  // with s_cum[o] <= e; eight independent loads in flight per thread, coalesced over e
  {
    const int Nc = min(N, 1024);
    for (int e0 = 0; e0 < carry; e0 += 8 * kLocThreads) {
      uint16_t iv[8];
      float wv[8];
      int ev[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int e = e0 + j * kLocThreads + tid;
        ev[j] = e;
        if (e < carry) {
          int lo = 0, hi = Nc;   // s_cum[lo] <= e < s_cum[hi]
          while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (s_cum[mid] <= e) lo = mid;
            else hi = mid;
          }
          const size_t src = (size_t)lo * CAP + (e - s_cum[lo]);
          iv[j] = sidx[src];
          wv[j] = sw[src];
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (ev[j] < carry) {
          cidx[ev[j]] = iv[j];
          cw[ev[j]] = wv[j];
        }
    }
  }
  if (tid == 0) {
    meta[0] = lam_s;
    meta[1] = carry;
    int run = 0;
    cnt[0] = 0;
    for (int q = 1; q < kChunk; ++q) {
      run += s_pair[q];
      cnt[q] = run;
    }
  }
  __syncthreads();
  // pairs: for each lambda, the sources with a bucket of that lag, in source order
  int pbase = 0;
  for (int lam = 1; lam < kChunk; ++lam) {
    int cache_run = 0;
    for (int o0 = 0; o0 < N; o0 += kLocThreads) {
      const int o = o0 + tid;
      int has = 0, k = 0, len = 0;
      if (o < N) {
        const int l0 = tap_l0[o], kl = min(K, kChunk - 1 - l0);
        k = lam - l0;
        has = (k >= 0 && k <= kl) ? 1 : 0;
        const int kc = min(kl, lam_s - l0);
        len = kc >= 0 ? min(boff[(size_t)o * boff_stride + kc + 1], CAP) : 0;
      }
      int tp, tl;
      const int pp = loc_block_exscan(has, s_scan, &tp);
      const int cp = cache_run + loc_block_exscan(len, s_scan, &tl);
      if (has) {
        const int beg = boff[(size_t)o * boff_stride + k], end = boff[(size_t)o * boff_stride + k + 1];
        const bool cached = lam <= lam_s;
        int4 pr;
        pr.x = o | (k << 16);
        pr.y = cached ? cp + beg : (int)((size_t)o * CAP + beg);
        pr.z = cached ? cp + end : (int)((size_t)o * CAP + end);
        pr.w = cached ? 1 : 0;
        pairs[pbase + pp] = pr;
      }
      pbase += tp;
      cache_run += tl;
    }
  }
}

struct LocArgs {
  ChunkArgs c;             // shapes, tensors, taps, chunk bounds (the exchange fields unused)
  const uint16_t* sidx;    // short entries (N, CAP): target
  const float* sw;         //                         weight
  const uint16_t* cidx;    // compact cache of the lags <= lam_s (k_short_pairs)
  const float* cw;
  const int4* pairs;       // (source, bucket) pairs sorted by lag
  const int* cnt;          // [8] pairs with lag <= q
  const int* meta;         // {lam_s, cached entries}
  int ecap;                // entries the block's shared-memory cache holds
};

template <int TPF, int PPT, int NTH, int S>
__global__ void __launch_bounds__(NTH, 1) k_bwd_chunk_local(LocArgs la) {
  extern __shared__ __align__(16) unsigned char smem[];
  const ChunkArgs& a = la.c;
  constexpr int RING = kChunk, G = kLocGroup;
  const int N = a.N, T = a.T, B = a.B, TAPS = a.TAPS, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int b0 = (int)blockIdx.x * S;
  const int nb = max(0, min(S, B - b0));
  const size_t BN = (size_t)B * N;
  const int t0 = a.t0, t_hi = a.t_hi;

  const LocSmem P = loc_smem_plan(N, TAPS, S);
  int* tl0 = (int*)smem;                                   // [N]
  int* tnt = tl0 + N;                                      // [N]
  float* tw = (float*)(tnt + N);                           // [N][TAPS]
  float* ring = (float*)(smem + P.taps);                   // [N][RING][S]
  float* grs = (float*)(smem + P.taps + P.ring);           // [S][N]
  int* scnt = (int*)(smem + P.taps + P.ring + P.grs);      // [RING]
  int4* spairs = (int4*)(smem + P.taps + P.ring + P.grs + P.cnt);   // [cnt[RING-1]]
  uint16_t* cidx = (uint16_t*)(smem + P.fixed);            // [ecap] cached targets
  float* cw = (float*)(smem + P.fixed + align256((size_t)la.ecap * 2));   // [ecap] cached weights

  for (int o = tid; o < N; o += NTH) {
    tl0[o] = a.tap_l0[o];
    tnt[o] = a.tap_nt[o];
  }
  for (int e = tid; e < N * TAPS; e += NTH) tw[e] = a.tap_w[e];
  for (int e = tid; e < N * RING * S; e += NTH) ring[e] = 0.f;
  if (tid < RING) scnt[tid] = la.cnt[tid];
  for (int j = tid; j < min(la.cnt[RING - 1], kLocPairCache); j += NTH) spairs[j] = la.pairs[j];
  {
    // the compact cache (16-byte pieces; its size is a multiple of 8 entries)
    const int ncached = min(la.meta[1], la.ecap);
    const int n16 = (ncached + 7) / 8;
    const uint4* gi = (const uint4*)la.cidx;
    uint4* si = (uint4*)cidx;
    for (int v = tid; v < n16; v += NTH) si[v] = gi[v];
    const float4* gw = (const float4*)la.cw;
    float4* sw4 = (float4*)cw;
    for (int v = tid; v < n16 * 2; v += NTH) sw4[v] = gw[v];
  }
  __syncthreads();
  // Launched as a programmatic dependent of the previous chunk's GEMM, the set-up above
  // (static tables written before the first chunk) overlaps that GEMM's last tiles; lam
  // and gz below are what the previous kernels wrote.  Without the launch attribute both
  // instructions do nothing.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // pairs p = tid + k * NTH: sample bl = p / N, source o = p % N
  int po[PPT], pb[PPT];
  bool pok[PPT];
  float lam[PPT], kp[PPT];
  float pf_gy[PPT], pf_u[PPT], pf_tap[PPT][TPF];
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    const int p = tid + k * NTH;
    po[k] = p % N;
    pb[k] = p / N;
    pok[k] = pb[k] < nb;
    const size_t pe = (size_t)(b0 + pb[k]) * N + po[k];
    lam[k] = (pok[k] && t_hi < T - 1) ? a.lam[pe] : 0.f;
    kp[k] = (pok[k] && a.keep) ? a.keep[pe] : 1.f;
  }
  auto prefetch_lif = [&](int t) {
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      pf_gy[k] = 0.f;
      pf_u[k] = 0.f;
      if (pok[k] && t >= t0) {
        const size_t idx = ((size_t)t * B + b0 + pb[k]) * N + po[k];
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
      if (pok[k] && t >= t0) {
        const size_t idx = ((size_t)t * B + b0 + pb[k]) * N + po[k];
        const int lo = tl0[po[k]], n = tnt[po[k]];
#pragma unroll
        for (int j = 0; j < TPF; ++j) {
          const int l = lo + j;
          if (j < n && t + l < T && tw[po[k] * TAPS + j] != 0.f) pf_tap[k][j] = __ldcg(a.gz + idx + (size_t)l * BN);
        }
      }
    }
  };
  prefetch_lif(t_hi);
  prefetch_taps(t_hi);

  const int g = lane / G, gl = lane % G;   // 8-lane group of the warp, lane in the group
  for (int t = t_hi; t >= t0; --t) {
    float cur_gy[PPT], cur_u[PPT], cur_tap[PPT][TPF];
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      cur_gy[k] = pf_gy[k];
      cur_u[k] = pf_u[k];
#pragma unroll
      for (int j = 0; j < TPF; ++j) cur_tap[k][j] = pf_tap[k][j];
    }
    prefetch_lif(t - 1);
    // ===== A: LIF backward of the block's pairs
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int o = po[k], bl = pb[k];
      if (bl >= S) continue;
      float grv = 0.f;
      if (pok[k]) {
        const int lo = tl0[o], n = tnt[o];   // n <= 2*ceil(s_max)+1 <= TPF (checked by the planner)
        const float* rrow = ring + (size_t)o * RING * S + bl;
        float gfut = 0.f;
#pragma unroll
        for (int j = 0; j < TPF; ++j) {
          const int l = lo + j;
          if (j < n && t + l < T) {
            float gv = cur_tap[k][j];
            if (t + l <= t_hi) gv += rrow[((t + l) % RING) * S];
            gfut = fmaf(tw[o * TAPS + j], gv, gfut);
          }
        }
        const float gY = __fadd_rn(cur_gy[k], gfut);
        const float du = lif_backward_pre(gY, lam[k], lif_bwd_prep(cur_u[k], a.lif), a.lif);
        lam[k] = lif_carry(du, a.lif);
        grv = __fmul_rn(du, kp[k]);
        const int b = b0 + bl;
        const size_t idx = ((size_t)t * B + b) * N + o;
        a.dx[idx] = du;
        if (a.gr != a.dx) a.gr[idx] = grv;   // (gr is dx itself without dropout)
        const __nv_bfloat16 h = __float2bfloat16_rn(grv);
        const size_t ai = ((size_t)b * T + t) * a.Np + o;
        a.ga_hi[ai] = h;
        a.ga_lo[ai] = __float2bfloat16_rn(grv - __bfloat162float(h));
      }
      grs[bl * N + o] = grv;
    }
    prefetch_taps(t - 1);
    __syncthreads();
    // ===== C: the pairs of lag <= q (a prefix of the sorted list) into ring slots t - k;
    // an 8-lane group per pair, the block's 64 groups round-robin over the pairs
    const int q = t - t0;
    const int np = q > 0 ? scnt[q] : 0;
    for (int base = warp * (32 / G); base < np; base += NTH / G) {
      const int j = base + g;
      const bool act = j < np;
      int4 pr = make_int4(0, 0, 0, 0);
      if (act) pr = j < kLocPairCache ? spairs[j] : la.pairs[j];
      const uint16_t* ix = pr.w ? cidx : la.sidx;
      const float* wv = pr.w ? cw : la.sw;
      float acc[S];
#pragma unroll
      for (int s2 = 0; s2 < S; ++s2) acc[s2] = 0.f;
      // 4 consecutive entries per lane (bucket bounds and cache offsets are multiples of 8)
      for (int e = pr.y + 4 * gl; e < pr.z; e += 4 * G) {
        const ushort4 i4 = *(const ushort4*)(ix + e);
        const float4 w4 = *(const float4*)(wv + e);
#pragma unroll
        for (int s2 = 0; s2 < S; ++s2) {
          const float* gs = grs + s2 * N;
          acc[s2] = fmaf(w4.x, gs[i4.x], acc[s2]);
          acc[s2] = fmaf(w4.y, gs[i4.y], acc[s2]);
          acc[s2] = fmaf(w4.z, gs[i4.z], acc[s2]);
          acc[s2] = fmaf(w4.w, gs[i4.w], acc[s2]);
        }
      }
#pragma unroll
      for (int s2 = 0; s2 < S; ++s2) {
#pragma unroll
        for (int m = G / 2; m >= 1; m >>= 1) acc[s2] += __shfl_xor_sync(0xffffffffu, acc[s2], m);
      }
      if (act && gl == 0) {
        const int o = pr.x & 0xffff, k = pr.x >> 16;
        float* cell = ring + ((size_t)o * RING + (t - k) % RING) * S;
#pragma unroll
        for (int s2 = 0; s2 < S; ++s2) cell[s2] += acc[s2];
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int k = 0; k < PPT; ++k)
    if (pok[k]) a.lam[(size_t)(b0 + pb[k]) * N + po[k]] = lam[k];
}

}  // namespace delrec
