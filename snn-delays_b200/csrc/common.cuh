// Shared device-side pieces of the delay-LIF kernels: LIF charge/fire/reset and its
// BPTT step, the surrogate derivatives, and the triangular delay kernel with the
// subgradient conventions of torch autograd.  All arithmetic is written with explicit
// round-to-nearest intrinsics so the compiler does not contract it into FMAs: the
// forward membrane then reproduces the reference's fp32 evaluation order
// (SpikingJelly LIFNode, delrec/triton_kernels/lif.py:24-56).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/delrec_b200.h"

namespace delrec {

// ---------------------------------------------------------------------------------
// device status word (no traps: kernels record and skip)
// ---------------------------------------------------------------------------------
// the library is one translation unit (api.cu), which owns this definition
__device__ int g_status = 0;
enum : int { ST_LAG_RANGE = 1 << 0, ST_INDEX_RANGE = 1 << 1, ST_SHAPE = 1 << 2, ST_TIMEOUT = 1 << 3 };
__device__ __forceinline__ void flag_status(int bit) { atomicOr(&g_status, bit); }

// ---------------------------------------------------------------------------------
// LIF parameters prepared on the host
// ---------------------------------------------------------------------------------
struct LifK {
  float decay;      // (float)(1 - 1/tau)
  float tau;        // (float)tau
  float vth;
  float vr;         // hard reset value (0 for soft)
  float v0;         // initial membrane
  int hard_nz;      // 1: hard reset with v_reset != 0 -> charge v - (v - vr)/tau + a
  int soft;
  int detach;
  int surr;         // DELREC_SURR_*
  float tri_c;      // (1/gamma)^2
  float gamma;
  float atan_c;     // pi/2 * alpha
  float atan_h;     // alpha / 2
};

inline LifK make_lif(const delrec_lif& l) {
  LifK k;
  const double tau = l.tau;
  k.decay = (float)(1.0 - 1.0 / tau);
  k.tau = (float)tau;
  k.vth = l.v_threshold;
  k.soft = l.soft_reset ? 1 : 0;
  k.vr = k.soft ? 0.f : l.v_reset;
  k.v0 = k.soft ? 0.f : l.v_reset;
  k.hard_nz = (!k.soft && l.v_reset != 0.f) ? 1 : 0;
  k.detach = l.detach_reset ? 1 : 0;
  k.surr = l.surrogate;
  const double g = l.gamma;
  k.tri_c = (float)((1.0 / g) * (1.0 / g));
  k.gamma = (float)g;
  const double a = l.alpha;
  k.atan_c = (float)(3.14159265358979323846 / 2.0 * a);
  k.atan_h = (float)(a / 2.0);
  return k;
}

// charge: u = v*(1-1/tau) + a, or v - (v - vr)/tau + a for a nonzero hard reset
__device__ __forceinline__ float lif_charge(float v, float a, const LifK& p) {
  if (p.hard_nz) return __fadd_rn(__fsub_rn(v, __fdiv_rn(__fsub_rn(v, p.vr), p.tau)), a);
  return __fadd_rn(__fmul_rn(v, p.decay), a);
}
// fire: spike when u - v_th >= 0 (ties fire)
__device__ __forceinline__ bool lif_fire(float u, const LifK& p) {
  return __fsub_rn(u, p.vth) >= 0.f;
}
// reset
__device__ __forceinline__ float lif_reset(float u, bool s, const LifK& p) {
  if (p.soft) return s ? __fsub_rn(u, p.vth) : u;
  return s ? p.vr : u;
}

// surrogate derivative at x = u - v_th
__device__ __forceinline__ float surrogate_grad(float x, const LifK& p) {
  if (p.surr == DELREC_SURR_ATAN) {
    const float t = __fmul_rn(p.atan_c, x);
    const float den = __fadd_rn(1.f, __fmul_rn(t, t));
    return __fmul_rn(__fdiv_rn(1.f, den), p.atan_h);
  }
  const float c = fmaxf(__fsub_rn(p.gamma, fabsf(x)), 0.f);
  return __fmul_rn(p.tri_c, c);
}

// One reverse LIF step.  gY = dL/dspike (output + recurrence), lam = dL/dv(t) carried
// from t+1.  Returns du = dL/du(t); the caller sets lam(t-1) = decay * du for the
// reset0/soft charge, or (1 - 1/tau) * du for the nonzero hard reset (same value).
__device__ __forceinline__ float lif_backward(float gY, float u, float lam, const LifK& p) {
  const float x = __fsub_rn(u, p.vth);
  const bool s = x >= 0.f;
  const float sg = surrogate_grad(x, p);
  if (p.soft) {
    const float gS = p.detach ? gY : __fsub_rn(gY, __fmul_rn(lam, p.vth));
    return __fadd_rn(lam, __fmul_rn(gS, sg));
  }
  const float gS = p.detach ? gY : __fadd_rn(gY, __fmul_rn(lam, __fsub_rn(p.vr, u)));
  return __fadd_rn(s ? 0.f : lam, __fmul_rn(gS, sg));
}
// lif_backward split in two: the part that depends on u only (surrogate derivative, spike,
// reset term), computed ahead of time, and the part that needs the incoming gradient.
// lif_backward_pre(gY, lam, lif_bwd_prep(u, p), p) == lif_backward(gY, u, lam, p) bit for bit.
struct LifPre {
  float sg;     // surrogate derivative at u - vth
  float vr_u;   // vr - u (hard reset)
  bool s;       // spike
};
__device__ __forceinline__ LifPre lif_bwd_prep(float u, const LifK& p) {
  LifPre q;
  const float x = __fsub_rn(u, p.vth);
  q.s = x >= 0.f;
  q.sg = surrogate_grad(x, p);
  q.vr_u = __fsub_rn(p.vr, u);
  return q;
}
__device__ __forceinline__ float lif_backward_pre(float gY, float lam, const LifPre& q, const LifK& p) {
  if (p.soft) {
    const float gS = p.detach ? gY : __fsub_rn(gY, __fmul_rn(lam, p.vth));
    return __fadd_rn(lam, __fmul_rn(gS, q.sg));
  }
  const float gS = p.detach ? gY : __fadd_rn(gY, __fmul_rn(lam, q.vr_u));
  return __fadd_rn(q.s ? 0.f : lam, __fmul_rn(gS, q.sg));
}
__device__ __forceinline__ float lif_carry(float du, const LifK& p) {
  return __fmul_rn(p.decay, du);
}

// ---------------------------------------------------------------------------------
// triangular delay kernel  h(l) = max(0, s - |l - (1 + d)|) / (s*s)
// ---------------------------------------------------------------------------------
struct Tri {
  float onepd;  // fl(1 + d)
  float s;      // half-width
  float s2;     // fl(s*s)
};
__device__ __forceinline__ Tri make_tri(float d, float s) {
  Tri t;
  t.onepd = __fadd_rn(1.f, d);
  t.s = s;
  t.s2 = __fmul_rn(s, s);
  return t;
}
// first lag with a possibly nonzero weight (>= 1) and the last one (<= Lm1)
__device__ __forceinline__ int tri_lo(const Tri& t) {
  int lo = (int)floorf(__fsub_rn(t.onepd, t.s));
  return lo < 1 ? 1 : lo;
}
__device__ __forceinline__ int tri_hi(const Tri& t, int Lm1) {
  int hi = (int)ceilf(__fadd_rn(t.onepd, t.s));
  return hi > Lm1 ? Lm1 : hi;
}
__device__ __forceinline__ float tri_clamped(const Tri& t, int l) {
  return __fsub_rn(t.s, fabsf(__fsub_rn((float)l, t.onepd)));
}
__device__ __forceinline__ float tri_h(const Tri& t, int l) {
  const float c = fmaxf(tri_clamped(t, l), 0.f);
  return __fdiv_rn(c, t.s2);
}
// d h / d d  (autograd through clamp(min=0) passes where c >= 0, abs'(0) = 0)
__device__ __forceinline__ float tri_dh_dd(const Tri& t, int l) {
  const float a = __fsub_rn((float)l, t.onepd);
  const float c = __fsub_rn(t.s, fabsf(a));
  if (!(c >= 0.f)) return 0.f;
  const float sg = a > 0.f ? 1.f : (a < 0.f ? -1.f : 0.f);
  return __fdiv_rn(sg, t.s2);
}
// d h / d s = [c>=0]/s^2 - 2 s c / s^4   (c clamped)
__device__ __forceinline__ float tri_dh_ds(const Tri& t, int l) {
  const float cr = tri_clamped(t, l);
  if (!(cr >= 0.f)) return 0.f;
  const float inv = __fdiv_rn(1.f, t.s2);
  const float h = __fdiv_rn(cr, t.s2);
  return __fsub_rn(inv, __fmul_rn(__fmul_rn(2.f, t.s), __fdiv_rn(h, t.s2)));
}

// ---------------------------------------------------------------------------------
// small helpers
// ---------------------------------------------------------------------------------
__host__ __device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ __forceinline__ size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// A bump allocator over the caller's workspace (256-byte aligned slices).
struct Carve {
  char* base;
  size_t cap;
  size_t off;
  bool ok;
  __host__ Carve(void* p, size_t c) : base((char*)p), cap(c), off(0), ok(true) {}
  template <class T>
  __host__ T* take(size_t count) {
    size_t bytes = align256(count * sizeof(T));
    if (off + bytes > cap) { ok = false; return nullptr; }
    T* r = base ? (T*)(base + off) : nullptr;
    off += bytes;
    return r;
  }
};

}  // namespace delrec
