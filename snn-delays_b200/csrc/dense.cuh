// Tensor-core weight gradient of the axonal and hybrid layers.
//
// dW[i,o] = sum_{t,b} gr[t,b,i] * z_{v(k)}[t-k, b, o] with k = k_io the synapse's integer
// offset (0 for axonal layers) and z_v the axonal interpolation of the source's spikes
// (v = min(k, MM), the base lags that synapse can reach).  For each k this is one plain
// GEMM over the T*B rows with the gr rows shifted by k*B, so the layer's dW is K+1 GEMMs
// P_k = gr_k^T z_{v(k)} followed by a per-synapse pick dW[i,o] = P_{k_io}[i,o].
// The fp32 operands are split into bf16 pairs x = hi + lo (hi = bf16(x),
// lo = bf16(x - hi)) and P_k = hi.hi + hi.lo + lo.hi with fp32 accumulation (each operand
// carries ~16 mantissa bits; the dropped lo.lo term is below 2^-16 relative).
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace delrec {

__global__ void k_split_bf16(const float* __restrict__ x, size_t n, __nv_bfloat16* __restrict__ hi,
                             __nv_bfloat16* __restrict__ lo) {
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
    const float v = x[e];
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[e] = h;
    lo[e] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

// hi + lo bf16 pieces of a (rows, N) fp32 matrix written with row stride Np >= N (the
// GEMM operand layout; columns N..Np-1 are zero)
// (blocks stride over rows, threads over groups of 4 columns: no per-element 64-bit
// index division; 16-byte loads and 8-byte stores when N is a multiple of 4)
__global__ void k_split_bf16_rows(const float* __restrict__ x, size_t rows, int N, int Np,
                                  __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
  const bool vec = (N & 3) == 0 && (((uintptr_t)x) & 15) == 0;
  for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = x + r * N;
    __nv_bfloat16* hr = hi + r * Np;
    __nv_bfloat16* lr = lo + r * Np;
    for (int c = threadIdx.x * 4; c < Np; c += blockDim.x * 4) {
      float v[4];
      if (vec && c + 4 <= N) {
        const float4 f = __ldcs((const float4*)(xr + c));
        v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = c + q < N ? xr[c + q] : 0.f;
      }
      __nv_bfloat16 h[4], l[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        h[q] = __float2bfloat16_rn(v[q]);
        l[q] = __float2bfloat16_rn(v[q] - __bfloat162float(h[q]));
      }
      if (c + 4 <= Np) {   // Np is a multiple of 8: 8-byte aligned groups
        *(uint2*)(hr + c) = *(const uint2*)h;
        *(uint2*)(lr + c) = *(const uint2*)l;
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (c + q < Np) { hr[c + q] = h[q]; lr[c + q] = l[q]; }
      }
    }
  }
}

// One reverse step of an axonal layer run step by step (layers too wide for the
// single-wave scans): for every (b, o),
//   gfut = sum_j w_o[j] gz(t + l_j)[b, o]  (gz of later steps, from the per-step GEMMs),
//   LIF backward with the carried lam, gr = du * keep,
// writing dx(t), gr(t) and the bf16 pieces of gr(t) laid out as the GEMM operand row
// [hi | hi | lo] (3N per sample) for gz(t) = [hi hi lo] . [W_hi; W_lo; W_hi].
__global__ void k_step_lif_bwd(int t, int T, int B, int N, int TAPS, const float* __restrict__ gy,
                               const float* __restrict__ u, const float* __restrict__ keep,
                               const int* __restrict__ l0, const int* __restrict__ nt,
                               const float* __restrict__ tw, const float* __restrict__ gz,
                               float* __restrict__ lam, float* __restrict__ dx, float* __restrict__ gr,
                               __nv_bfloat16* __restrict__ g3, LifK lif) {
  asm volatile("griddepcontrol.wait;" ::: "memory");   // no-op unless launched as a dependent
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const size_t BN = (size_t)B * N;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < BN; e += (size_t)gridDim.x * blockDim.x) {
    const int o = (int)(e % N), b = (int)(e / N);
    const size_t idx = (size_t)t * BN + e;
    const int lo = l0[o], n = nt[o];
    float gfut = 0.f;
    for (int j = 0; j < n; ++j) {
      const int l = lo + j;
      if (l >= 1 && t + l < T) gfut = fmaf(tw[(size_t)o * TAPS + j], gz[idx + (size_t)l * BN], gfut);
    }
    const float gY = __fadd_rn(gy[idx], gfut);
    const float du = lif_backward(gY, u[idx], lam[e], lif);
    lam[e] = lif_carry(du, lif);
    const float g = keep ? __fmul_rn(du, keep[e]) : du;
    dx[idx] = du;
    gr[idx] = g;
    const __nv_bfloat16 h = __float2bfloat16_rn(g);
    const __nv_bfloat16 l = __float2bfloat16_rn(g - __bfloat162float(h));
    __nv_bfloat16* row = g3 + (size_t)b * 3 * N;
    row[o] = h;
    row[N + o] = h;
    row[2 * N + o] = l;
  }
}

// dW[i*N + o] = P[k_io][i*N + o]
__global__ void k_pick_by_offset(int N, const uint8_t* __restrict__ offT, const float* __restrict__ P,
                                 float* __restrict__ dW) {
  const size_t nn = (size_t)N * N;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < nn; e += (size_t)gridDim.x * blockDim.x) {
    const int i = (int)(e / N), o = (int)(e % N);
    const int k = offT[(size_t)o * N + i];
    dW[e] = P[(size_t)k * nn + e];
  }
}

}  // namespace delrec
