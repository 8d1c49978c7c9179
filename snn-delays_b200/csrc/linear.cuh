// Feedforward projection out = x W^T + bias (torch.nn.Linear layout, W (N,K)) on bf16
// tensor cores with fp32 accuracy.
//
// Every fp32 operand v is split exactly into three bf16 pieces v = p0 + p1 + p2
// (p0 = bf16(v), p1 = bf16(v - p0), p2 = bf16(v - p0 - p1); each difference is exact in
// fp32 and 3 x 8 significand bits cover fp32's 24).  A product a.b is then the sum of
// the piece products a_i.b_j with i + j <= 2 (six products; the dropped ones are below
// 2^-24 relative), accumulated in fp32 by the tensor cores.  Operands in {0, 1} (spike
// trains) are exact in one bf16 piece, so a product with them needs three products only.
//
// Each operand's pieces are stored once, side by side in its rows ([x0 x1 x2], or [x]
// for spikes; [W0 W1 W2]), and ONE launch of the library's tcgen05 GEMM sums the piece
// products, each product pairing a piece of one operand with a piece of the other
// (gemm_tc.cuh: GemmArgs pa / pb):
//   forward   out (M,N) = sum x_i . W_j^T over i + j <= 2 (real x: 6 products) or over
//             j (spikes: 3 products); the bias rides along as column K: 1 in x0 (the
//             pieces of 1 are 1, 0, 0), the bias pieces in W0..W2;
//   input gradient  dx (M,K) = sum g_i . W_j over i + j <= 2, with G = [g0 g1 g2] of gout
//     and the pieces of W stored transposed (their rows along the reduction);
//   weight gradient D (3*Np, Kp) = sum_a x_a^T G[:, 0 : (3-a)*Np]  (one GEMM for spikes,
//     three for real x), then dW = D[0:N] + D[Np:Np+N] + D[2Np:2Np+N] and dbias = its
//     column K.
// Kp = roundup(K + 1, 8) and Np = roundup(N, 8) keep every bf16 row 16-byte aligned.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace delrec {

struct Pieces3 {
  __nv_bfloat16 p[3];
};
__device__ __forceinline__ Pieces3 split3(float v) {
  Pieces3 r;
  r.p[0] = __float2bfloat16_rn(v);
  const float r1 = __fsub_rn(v, __bfloat162float(r.p[0]));
  r.p[1] = __float2bfloat16_rn(r1);
  const float r2 = __fsub_rn(r1, __bfloat162float(r.p[1]));
  r.p[2] = __float2bfloat16_rn(r2);
  return r;
}

// Block pattern (piece index of block q, two bits per block): pieces 0, 1, 2 in order.
constexpr unsigned kPatDistinct3 = (0u << 0) | (1u << 2) | (2u << 4);

// out[r][q*Wd + c] = piece pat(q) of
//   src[r*lds + c]                      c <  K
//   extra ? extra[r] : (ones ? 1 : 0)   c == K  (the pieces of 1 are 1, 0, 0)
//   0                                   K < c < Wd
// for rows r < R.  binary != 0: values of src must be 0 or 1 (else ST_SHAPE is set).
// Wd is a multiple of 8: a thread packs 8 consecutive columns (16-byte stores).
__device__ __forceinline__ uint32_t pack_bf16x2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}
__global__ void k_pack_rows(int R, int K, int Wd, const float* __restrict__ src, int lds,
                            const float* __restrict__ extra, int ones, int nb, unsigned pat,
                            int binary, __nv_bfloat16* __restrict__ out) {
  const int groups = Wd >> 3;
  const size_t total = (size_t)R * groups;
  const size_t row_out = (size_t)nb * Wd;
  const bool vec = (lds & 3) == 0 && ((uintptr_t)src & 15) == 0;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / groups), c0 = (int)(e % groups) * 8;
    float v[8];
    const float* sp = src + (size_t)r * lds + c0;
    if (vec && c0 + 8 <= K) {
      const float4 x0 = __ldcs((const float4*)sp), x1 = __ldcs((const float4*)sp + 1);
      v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
      v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int c = c0 + q;
        v[q] = c < K ? sp[q] : (c == K ? (extra ? extra[r] : (ones ? 1.f : 0.f)) : 0.f);
      }
    }
    Pieces3 p[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (binary && c0 + q < K && !(v[q] == 0.f || v[q] == 1.f)) flag_status(ST_SHAPE);
      p[q] = split3(v[q]);
    }
    uint4* o = (uint4*)(out + (size_t)r * row_out + c0);
#pragma unroll 1
    for (int b = 0; b < nb; ++b) {
      const int pi = (pat >> (2 * b)) & 3;
      uint4 w;
      w.x = pack_bf16x2(p[0].p[pi], p[1].p[pi]);
      w.y = pack_bf16x2(p[2].p[pi], p[3].p[pi]);
      w.z = pack_bf16x2(p[4].p[pi], p[5].p[pi]);
      w.w = pack_bf16x2(p[6].p[pi], p[7].p[pi]);
      o[(size_t)b * (Wd >> 3)] = w;
    }
  }
}

// W''[q*Np + n][c] = piece pat(q) of W[n*K + c] (c < K, n < N), else 0.   (nb*Np rows, Kp cols)
__global__ void k_pack_wt(int N, int K, int Np, int Kp, const float* __restrict__ W, unsigned pat, int nb,
                          __nv_bfloat16* __restrict__ out) {
  const int groups = Kp >> 3;
  const size_t total = (size_t)Np * groups;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(e / groups), c0 = (int)(e % groups) * 8;
    Pieces3 p[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int c = c0 + q;
      p[q] = split3((n < N && c < K) ? W[(size_t)n * K + c] : 0.f);
    }
#pragma unroll 1
    for (int b = 0; b < nb; ++b) {
      const int pi = (pat >> (2 * b)) & 3;
      uint4 w;
      w.x = pack_bf16x2(p[0].p[pi], p[1].p[pi]);
      w.y = pack_bf16x2(p[2].p[pi], p[3].p[pi]);
      w.z = pack_bf16x2(p[4].p[pi], p[5].p[pi]);
      w.w = pack_bf16x2(p[6].p[pi], p[7].p[pi]);
      *(uint4*)(out + ((size_t)b * Np + n) * Kp + c0) = w;
    }
  }
}

// Wide axonal layers run their forward step by step with rec(t) on the tensor cores as
//   rec(t)[b, i] = sum_q sum_j Y_q(t)[b, j] * (W[i, j] h_j(q)),
// where q walks source j's positive taps (weights h_j(q) > 0 of its triangle, in lag
// order from lag f_j; at most TF of them) and Y_q(t)[b, j] = y(t - f_j - q)[b, j] is a
// spike (0 or 1, exact in bf16).  W h_j(q) is split into three bf16 pieces whose sum is
// its fp32 value, so every product is exact and only the additions round.

// (first positive tap's lag, number of positive taps) per source, from the tap tables
__global__ void k_pos_taps(int N, int TAPS, const int* __restrict__ l0, const int* __restrict__ nt,
                           const float* __restrict__ tw, int TF, int2* __restrict__ fp) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= N) return;
  int first = -1, np = 0;
  for (int q = 0; q < nt[j]; ++q)
    if (tw[(size_t)j * TAPS + q] > 0.f) {
      if (first < 0) first = q;
      ++np;
    }
  if (np > TF) { flag_status(ST_LAG_RANGE); np = TF; }
  fp[j] = make_int2(first < 0 ? 1 : l0[j] + first, np);
}

// B operand of the step GEMM: row i, column q*N + j = the pieces of fl(W[i, j] h_j(q))
// (zero for q >= npos_j and in the padding up to Kp)
__global__ void k_wtap_pieces(int N, int TAPS, int TF, int Kp, const float* __restrict__ W,
                              const int* __restrict__ l0, const float* __restrict__ tw,
                              const int2* __restrict__ fp, __nv_bfloat16* __restrict__ p0,
                              __nv_bfloat16* __restrict__ p1, __nv_bfloat16* __restrict__ p2) {
  const size_t total = (size_t)N * Kp;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int i = (int)(e / Kp), c = (int)(e % Kp);
    const int q = c / N, j = c - q * N;
    float v = 0.f;
    if (q < TF && q < fp[j].y) {
      const int slot = fp[j].x - l0[j] + q;   // index of the tap in j's table
      v = __fmul_rn(W[(size_t)i * N + j], tw[(size_t)j * TAPS + slot]);
    }
    const Pieces3 r = split3(v);
    p0[e] = r.p[0];
    p1[e] = r.p[1];
    p2[e] = r.p[2];
  }
}

// One forward step: for every (b, n), rec(t) = the fixed-order sum of the step GEMM's
// ksplit partials (0 at t = 0), the LIF update at t, and the A operand row of step t+1:
// A[b, q*N + n] = Y_q(t+1)[b, n] (n as a source).
__global__ void k_step_lif_fwd(int t, int T, int B, int N, int TF, const float* __restrict__ x,
                               const float* __restrict__ part, int ksplit, const float* __restrict__ bias,
                               const float* __restrict__ keep, const int2* __restrict__ fp,
                               float* __restrict__ v, float* __restrict__ y, float* __restrict__ u,
                               __nv_bfloat16* __restrict__ A, int Kp, LifK lif) {
  asm volatile("griddepcontrol.wait;" ::: "memory");   // no-op unless launched as a dependent
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const size_t BN = (size_t)B * N;
  const __nv_bfloat16 one = __float2bfloat16_rn(1.f), zero = __float2bfloat16_rn(0.f);
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < BN; e += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(e % N);
    const size_t b = e / N;
    const size_t idx = (size_t)t * BN + e;
    float rec = 0.f;
    if (t > 0) {
      // 4 partials' loads in flight at a time, added in split order
      int k = 0;
      for (; k + 4 <= ksplit; k += 4) {
        const float p0 = __ldcg(part + (size_t)k * BN + e), p1 = __ldcg(part + (size_t)(k + 1) * BN + e);
        const float p2 = __ldcg(part + (size_t)(k + 2) * BN + e), p3 = __ldcg(part + (size_t)(k + 3) * BN + e);
        rec = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(rec, p0), p1), p2), p3);
      }
      for (; k < ksplit; ++k) rec = __fadd_rn(rec, __ldcg(part + (size_t)k * BN + e));
    }
    const float bs = bias ? bias[n] : 0.f;
    const float kp = keep ? keep[e] : 1.f;
    const float r = __fmul_rn(__fadd_rn(rec, bs), kp);
    const float av = __fadd_rn(x[idx], r);
    const float uu = lif_charge(v[e], av, lif);
    const bool sp = lif_fire(uu, lif);
    v[e] = lif_reset(uu, sp, lif);
    y[idx] = sp ? 1.f : 0.f;
    u[idx] = uu;
    if (t + 1 < T) {
      const int2 f = fp[n];
      for (int q = 0; q < TF; ++q) {
        const int ts = t + 1 - (f.x + q);
        bool s = false;
        if (q < f.y && ts >= 0) s = ts == t ? sp : (y[(size_t)ts * BN + e] != 0.f);
        A[b * Kp + (size_t)q * N + n] = s ? one : zero;
      }
    }
  }
}

__global__ void k_fill_f32(float* __restrict__ p, size_t n, float value) {
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
    p[e] = value;
}

// *count += number of entries of x[0..n) that are neither 0 nor 1 (x 16-byte aligned)
__global__ void k_count_nonbinary(const float* __restrict__ x, size_t n, unsigned int* __restrict__ count) {
  unsigned int c = 0;
  const size_t n4 = n / 4;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n4; e += (size_t)gridDim.x * blockDim.x) {
    const float4 v = __ldcs((const float4*)x + e);
    c += !(v.x == 0.f || v.x == 1.f);
    c += !(v.y == 0.f || v.y == 1.f);
    c += !(v.z == 0.f || v.z == 1.f);
    c += !(v.w == 0.f || v.w == 1.f);
  }
  for (size_t e = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
    c += !(x[e] == 0.f || x[e] == 1.f);
  for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(count, c);
}

// dW[n*K + c] = D[n][c] + D[Np+n][c] + D[2Np+n][c];  dbias[n] = the same at c = K.
// D is (3*Np, Kp) row-major (the column-major Kp x 3Np GEMM output).
__global__ void k_linear_dw_reduce(int N, int K, int Np, int Kp, const float* __restrict__ D,
                                   float* __restrict__ dW, float* __restrict__ dbias) {
  const size_t total = (size_t)N * (K + 1);
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(e / (K + 1)), c = (int)(e % (K + 1));
    const float v = D[(size_t)n * Kp + c] + D[((size_t)Np + n) * Kp + c] + D[((size_t)2 * Np + n) * Kp + c];
    if (c < K) {
      if (dW) dW[(size_t)n * K + c] = v;
    } else if (dbias) {
      dbias[n] = v;
    }
  }
}

}  // namespace delrec
