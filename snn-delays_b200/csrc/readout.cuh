// Readout projection + time sum of the training loss, fused.
//
// The model zoo ends in a Linear readout applied at every step (networks.py:140-181), and
// the SSC / PS-MNIST loss sums its output over time before the cross-entropy
// (utils.py:188-200, calc_loss_SSC).  The sum commutes with the projection:
//   out[b][c] = sum_t (W y_t + bias)[b][c] = sum_n W[c][n] ysum[b][n] + T bias[c],
//   ysum[b][n] = sum_t y[t][b][n],
// so the (T,B,C) readout, its bf16 operand packing and its GEMMs are never formed.  The
// backward of out with upstream g (B,C):
//   dy[t][b][n] = gs[b][n] = sum_c g[b][c] W[c][n]   (the same for every t)
//   dW[c][n]    = sum_b g[b][c] ysum[b][n]
//   dbias[c]    = T sum_b g[b][c]
// All sums are fp32 in a fixed order (time, then the reduction index ascending).
#pragma once

#include "common.cuh"

namespace delrec {

// ysum[b][n] = sum_t y[t][b][n]  (one thread per (b, n), coalesced over n)
__global__ void k_time_sum(int T, size_t BN, const float* __restrict__ y, float* __restrict__ ysum) {
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < BN; e += (size_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    int t = 0;
    for (; t + 4 <= T; t += 4) {   // four loads in flight, added in time order
      const float a0 = __ldcs(y + (size_t)t * BN + e), a1 = __ldcs(y + (size_t)(t + 1) * BN + e);
      const float a2 = __ldcs(y + (size_t)(t + 2) * BN + e), a3 = __ldcs(y + (size_t)(t + 3) * BN + e);
      s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, a0), a1), a2), a3);
    }
    for (; t < T; ++t) s = __fadd_rn(s, __ldcs(y + (size_t)t * BN + e));
    ysum[e] = s;
  }
}

// out[b][c] = sum_n ysum[b][n] W[c][n] + T bias[c]: a warp per output, lanes over n, the
// lane partials combined by a fixed butterfly
__global__ void k_readout_sum(int T, int B, int N, int C, const float* __restrict__ ysum,
                              const float* __restrict__ W, const float* __restrict__ bias, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const size_t nw = (size_t)gridDim.x * (blockDim.x >> 5);
  for (size_t w = blockIdx.x * (size_t)(blockDim.x >> 5) + (threadIdx.x >> 5); w < (size_t)B * C; w += nw) {
    const int b = (int)(w / C), c = (int)(w % C);
    const float* ys = ysum + (size_t)b * N;
    const float* wr = W + (size_t)c * N;
    float s = 0.f;
    for (int n = lane; n < N; n += 32) s = fmaf(ys[n], wr[n], s);
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    if (lane == 0) out[w] = bias ? fmaf((float)T, bias[c], s) : s;
  }
}

// gs[b][n] = sum_c g[b][c] W[c][n], written to dy[t][b][n] for every t
__global__ void k_readout_sum_dy(int T, int B, int N, int C, const float* __restrict__ g,
                                 const float* __restrict__ W, float* __restrict__ dy) {
  const size_t BN = (size_t)B * N;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < BN; e += (size_t)gridDim.x * blockDim.x) {
    const int b = (int)(e / N), n = (int)(e % N);
    float s = 0.f;
    for (int c = 0; c < C; ++c) s = fmaf(g[(size_t)b * C + c], W[(size_t)c * N + n], s);
    for (int t = 0; t < T; ++t) __stcs(dy + (size_t)t * BN + e, s);
  }
}

// dW[c][n] = sum_b g[b][c] ysum[b][n];  dbias[c] = T sum_b g[b][c]
__global__ void k_readout_sum_dw(int T, int B, int N, int C, const float* __restrict__ g,
                                 const float* __restrict__ ysum, float* __restrict__ dW, float* __restrict__ dbias) {
  const size_t CN = (size_t)C * N;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < CN + C; e += (size_t)gridDim.x * blockDim.x) {
    if (e < CN) {
      if (!dW) continue;
      const int c = (int)(e / N), n = (int)(e % N);
      float s = 0.f;
      int b = 0;
      for (; b + 8 <= B; b += 8) {   // eight loads of each operand in flight, summed in order
        float gv[8], yv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          gv[j] = g[(size_t)(b + j) * C + c];
          yv[j] = ysum[(size_t)(b + j) * N + n];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) s = fmaf(gv[j], yv[j], s);
      }
      for (; b < B; ++b) s = fmaf(g[(size_t)b * C + c], ysum[(size_t)b * N + n], s);
      dW[e] = s;
    } else if (dbias) {
      const int c = (int)(e - CN);
      float s = 0.f;
      for (int b = 0; b < B; ++b) s = __fadd_rn(s, g[(size_t)b * C + c]);
      dbias[c] = __fmul_rn((float)T, s);
    }
  }
}

}  // namespace delrec
