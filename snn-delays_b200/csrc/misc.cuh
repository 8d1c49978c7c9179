// Plain multi-step LIF layer (the SpikingJelly LIFNode the model zoo places between
// projections, networks.py:84-96) and the DCLS feedforward delay layer
// (networks.py:22-50: Gaussian-interpolated learnable positions, causal conv over time).
// DCLS 0.1.1 is a third-party package that is not part of the reference tree; the
// construction below restates its published Gaussian method:
//   c = P + K//2, sg = |SIG| + eps, g_k = exp(-0.5 ((k - c)/sg)^2), ker_k = w g_k / (sum g + eps)
#pragma once

#include "common.cuh"

namespace delrec {

__global__ void k_lif_fwd(int T, int M, LifK p, const float* __restrict__ x, float* __restrict__ y,
                          float* __restrict__ u) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  float v = p.v0;
  for (int t = 0; t < T; ++t) {
    const size_t idx = (size_t)t * M + m;
    const float uu = lif_charge(v, x[idx], p);
    const bool s = lif_fire(uu, p);
    v = lif_reset(uu, s, p);
    y[idx] = s ? 1.f : 0.f;
    if (u) u[idx] = uu;
  }
}

__global__ void k_lif_bwd(int T, int M, LifK p, const float* __restrict__ gy, const float* __restrict__ u,
                          float* __restrict__ dx) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  float lam = 0.f;
  for (int t = T - 1; t >= 0; --t) {
    const size_t idx = (size_t)t * M + m;
    const float du = lif_backward(gy[idx], u[idx], lam, p);
    lam = lif_carry(du, p);
    dx[idx] = du;
  }
}

// ---- DCLS ---------------------------------------------------------------------------
// normalized Gaussian weights of one (co, ci) kernel row
__device__ __forceinline__ void dcls_gauss(int K, float P, float SIG, float* g, float* S, float* c_out,
                                           float* sg_out) {
  const float c = P + (float)(K / 2);
  const float sg = fabsf(SIG) + 1e-7f;
  float sum = 0.f;
  for (int k = 0; k < K; ++k) {
    const float z = ((float)k - c) / sg;
    g[k] = expf(-0.5f * z * z);
    sum += g[k];
  }
  *S = sum + 1e-7f;
  *c_out = c;
  *sg_out = sg;
}

// ker[(co*cin_g + ci)*K + k]
__global__ void k_dcls_build(int rows, int K, const float* __restrict__ w, const float* __restrict__ P,
                             const float* __restrict__ SIG, float* __restrict__ ker) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float g[64];
  float S, c, sg;
  dcls_gauss(K, P[r], SIG[r], g, &S, &c, &sg);
  for (int k = 0; k < K; ++k) ker[(size_t)r * K + k] = w[r] * (g[k] / S);
}

// out[t,b,co] = bias[co] + sum_{ci in group(co)} sum_k ker[co,ci,k] * x[t + k - lpad, b, cin0 + ci]
__global__ void k_dcls_conv(int T, int B, int Cin, int Cout, int groups, int K, int lpad,
                            const float* __restrict__ x, const float* __restrict__ ker,
                            const float* __restrict__ bias, float* __restrict__ out) {
  const size_t total = (size_t)T * B * Cout;
  const int cin_g = Cin / groups, cout_g = Cout / groups;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int co = (int)(e % Cout);
    const size_t tb = e / Cout;
    const int b = (int)(tb % B), t = (int)(tb / B);
    const int g = co / cout_g;
    float acc = bias ? bias[co] : 0.f;
    for (int ci = 0; ci < cin_g; ++ci) {
      const float* kr = ker + ((size_t)co * cin_g + ci) * K;
      const int cin = g * cin_g + ci;
      for (int k = 0; k < K; ++k) {
        const int ts = t + k - lpad;
        if (ts >= 0 && ts < T) acc = fmaf(kr[k], x[((size_t)ts * B + b) * Cin + cin], acc);
      }
    }
    out[e] = acc;
  }
}

// dx[t,b,cin] = sum_{co in group} sum_k gout[t - k + lpad, b, co] * ker[co, ci, k]
__global__ void k_dcls_dx(int T, int B, int Cin, int Cout, int groups, int K, int lpad,
                          const float* __restrict__ gout, const float* __restrict__ ker, float* __restrict__ dx) {
  const size_t total = (size_t)T * B * Cin;
  const int cin_g = Cin / groups, cout_g = Cout / groups;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int cin = (int)(e % Cin);
    const size_t tb = e / Cin;
    const int b = (int)(tb % B), t = (int)(tb / B);
    const int g = cin / cin_g, ci = cin % cin_g;
    float acc = 0.f;
    for (int cog = 0; cog < cout_g; ++cog) {
      const int co = g * cout_g + cog;
      const float* kr = ker + ((size_t)co * cin_g + ci) * K;
      for (int k = 0; k < K; ++k) {
        const int to = t - k + lpad;
        if (to >= 0 && to < T) acc = fmaf(kr[k], gout[((size_t)to * B + b) * Cout + co], acc);
      }
    }
    dx[e] = acc;
  }
}

// dker[co,ci,k] = sum_{t,b} gout[t,b,co] * x[t + k - lpad, b, cin]   (one block per (co,ci,k))
__global__ void k_dcls_dker(int T, int B, int Cin, int Cout, int groups, int K, int lpad,
                            const float* __restrict__ x, const float* __restrict__ gout, float* __restrict__ dker) {
  __shared__ float red[256];
  const int cin_g = Cin / groups, cout_g = Cout / groups;
  const int r = blockIdx.x;  // (co*cin_g + ci)*K + k
  const int k = r % K, ci = (r / K) % cin_g, co = r / (K * cin_g);
  const int cin = (co / cout_g) * cin_g + ci;
  float acc = 0.f;
  const int TB = T * B;
  for (int e = threadIdx.x; e < TB; e += blockDim.x) {
    const int t = e / B, b = e % B;
    const int ts = t + k - lpad;
    if (ts >= 0 && ts < T) acc = fmaf(gout[(size_t)e * Cout + co], x[((size_t)ts * B + b) * Cin + cin], acc);
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) dker[r] = red[0];
}

// chain rule through the kernel construction: dw, dP, dSIG per (co, ci)
__global__ void k_dcls_params(int rows, int K, const float* __restrict__ w, const float* __restrict__ P,
                              const float* __restrict__ SIG, const float* __restrict__ dker,
                              float* dw, float* dP, float* dSIG) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float g[64];
  float S, c, sg;
  dcls_gauss(K, P[r], SIG[r], g, &S, &c, &sg);
  const float* dk = dker + (size_t)r * K;
  // a_k = g_k / S;  ker_k = w a_k
  float dws = 0.f, dot_a = 0.f, dc = 0.f, dsg = 0.f, sum_gc = 0.f, sum_gs = 0.f;
  for (int k = 0; k < K; ++k) {
    const float a = g[k] / S;
    dws += dk[k] * a;
    dot_a += dk[k] * g[k];
    const float z = ((float)k - c) / sg;
    sum_gc += g[k] * z / sg;          // d g_k / d c = g_k (k-c)/sg^2
    sum_gs += g[k] * z * z / sg;      // d g_k / d sg = g_k (k-c)^2/sg^3
  }
  // d(g_k/S)/dc = g_k' / S - g_k sum(g') / S^2
  for (int k = 0; k < K; ++k) {
    const float z = ((float)k - c) / sg;
    const float gc = g[k] * z / sg, gs = g[k] * z * z / sg;
    dc += dk[k] * (gc / S - g[k] * sum_gc / (S * S));
    dsg += dk[k] * (gs / S - g[k] * sum_gs / (S * S));
  }
  (void)dot_a;
  if (dw) dw[r] = dws;
  if (dP) dP[r] = w[r] * dc;
  if (dSIG) dSIG[r] = w[r] * dsg * (SIG[r] > 0.f ? 1.f : (SIG[r] < 0.f ? -1.f : 0.f));
}

// db[co] = sum_{t,b} gout[t,b,co]: a block of 32 warps per 32 output columns (lane =
// column, coalesced rows); warp w sums rows w, w+32, ...; the 32 warp partials are added
// in a fixed order (deterministic)
__global__ void __launch_bounds__(1024) k_dcls_dbias(int TB, int Cout, const float* __restrict__ gout,
                                                     float* __restrict__ db) {
  __shared__ float part[32][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int co = blockIdx.x * 32 + lane;
  float v = 0.f;
  if (co < Cout) {
#pragma unroll 8
    for (int e = w; e < TB; e += 32) v += gout[(size_t)e * Cout + co];
  }
  part[w][lane] = v;
  __syncthreads();
  if (w == 0) {
    float sum = 0.f;
    for (int k = 0; k < 32; ++k) sum += part[k][lane];
    if (co < Cout) db[co] = sum;
  }
}

}  // namespace delrec
