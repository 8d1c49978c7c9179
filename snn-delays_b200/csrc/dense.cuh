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
