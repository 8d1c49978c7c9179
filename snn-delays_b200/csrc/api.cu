// extern "C" entry points of libdelrec_b200.so: argument checks, workspace carving,
// launch planning (block sizes, cluster shapes, shared-memory budgets) and the kernel
// sequences of each layer forward / backward.  No allocation happens here: all
// scratch comes from the caller's workspace.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <cstdio>
#include <cstring>

#include "backward.cuh"
#include "backward_hybrid.cuh"
#include "backward_hybrid64.cuh"
#include "backward_axonal_mma.cuh"
#include "backward_chunk.cuh"
#include "backward_chunk_local.cuh"
#include "dense.cuh"
#include "forward.cuh"
#include "gemm_tc.cuh"
#include "grads.cuh"
#include "linear.cuh"
#include "misc.cuh"
#include "prep.cuh"
#include "readout.cuh"

namespace delrec {

static constexpr size_t kSmemLimit = 227 * 1024;  // opt-in dynamic shared memory per block
static constexpr int kSMs = 148;
static constexpr int kTapsMax = 16;               // widest axonal tap window supported

static inline int pow2_at_least(int x) {
  int r = 1;
  while (r < x) r <<= 1;
  return r;
}

#define DR_CUDA(call)                                                      \
  do {                                                                     \
    cudaError_t _e = (call);                                               \
    if (_e != cudaSuccess) {                                               \
      fprintf(stderr, "delrec_b200: %s failed: %s\n", #call, cudaGetErrorString(_e)); \
      return DELREC_ERR_CUDA;                                              \
    }                                                                      \
  } while (0)
static unsigned long long g_launches = 0;  // kernels issued by this library (host counter)

// Optional timing of the reverse-scan kernels: CUDA events recorded on the launching
// stream around each scan launch while enabled (delrec_scan_timing).
static bool g_scan_timing = false;
// part 0: whole reverse-scan launches (or the whole chunked scan of a layer); 1: the step
// launches of the chunked scan; 2: its chunk GEMM launches
static constexpr int kTimeParts = 3, kTimeSlots = 1024;
static cudaEvent_t g_ev[kTimeParts][kTimeSlots][2];
static int g_ev_n[kTimeParts] = {0, 0, 0};
static void scan_mark(int which, cudaStream_t st, int part = 0) {
  if (!g_scan_timing || part < 0 || part >= kTimeParts || g_ev_n[part] >= kTimeSlots) return;
  cudaEvent_t& e = g_ev[part][g_ev_n[part]][which];
  if (!e) cudaEventCreate(&e);
  cudaEventRecord(e, st);
  if (which == 1) ++g_ev_n[part];
}

#define DR_LAUNCHED()                                                      \
  do {                                                                     \
    ++g_launches;                                                          \
    cudaError_t _e = cudaGetLastError();                                   \
    if (_e != cudaSuccess) {                                               \
      fprintf(stderr, "delrec_b200: launch failed at %s:%d: %s\n", __FILE__, __LINE__, \
              cudaGetErrorString(_e));                                     \
      return DELREC_ERR_CUDA;                                              \
    }                                                                      \
  } while (0)

static inline int grid_for(size_t n, int threads) {
  size_t g = (n + threads - 1) / threads;
  if (g > (size_t)kSMs * 16) g = (size_t)kSMs * 16;
  return (int)std::max<size_t>(g, 1);
}

// --------------------------------------------------------------------------------
// layer descriptor validation
// --------------------------------------------------------------------------------
static int check_layer(const delrec_layer* ly, int kind) {
  if (!ly || ly->kind != kind) return DELREC_ERR_ARG;
  if (ly->T < 1 || ly->B < 1 || ly->N < 1 || ly->L < 1) return DELREC_ERR_ARG;
  if (kind == DELREC_HYBRID && (ly->K < 0 || ly->K > 255)) return DELREC_ERR_ARG;
  if (ly->N > 8192) return DELREC_ERR_UNSUPPORTED;
  if (!(ly->s_max >= 1.f) || ly->s_max > 6.f) return DELREC_ERR_UNSUPPORTED;
  return DELREC_OK;
}

// number of lags in an axonal tap window: [floor(1+d-s)-1, ceil(1+d+s)+1]
static inline int taps_for(const delrec_layer* ly) {
  const int w = 2 * (int)ceilf(ly->s_max) + 5;
  // hybrid base windows may start below lag 1, so only the axonal window is capped by L-1
  const int cap = ly->kind == DELREC_HYBRID ? w : std::min(ly->L - 1, w);
  return std::max(1, std::min(cap, kTapsMax));
}

// Hybrid backward: the base's tap window may reach lags l <= 0 (a synapse with integer
// offset k receives base lag l when l + k >= 1).  MM = 1 - (smallest such lag) over all
// sources, evaluated with the device's float32 arithmetic on (min base, max width),
// which bounds every source's window from below.  0 when every tap lag is >= 1.
static int hybrid_mm(const delrec_layer* ly) {
  const float onepd = 1.0f + ly->d_min;
  const float s = ly->s_max;
  int l = (int)floorf(onepd - s) - 1;
  while (!(s - fabsf((float)l - onepd) >= 0.f) && l < 1) ++l;
  int mm = 1 - l;
  if (mm < 0) mm = 0;
  if (mm > ly->K) mm = ly->K;
  return mm;
}
// The factored hybrid backward keeps gz_m(tau) = sum_{k >= m} W_k gr(tau + k) for tau >= 0
// only.  A base tap at lag l = 1 - m <= -1 needs gz_m(t + l) at t + l < 0 for the first
// steps (t < m - 1), so layers whose base reaches two or more lags below lag 1 (MM >= 2)
// take the per-synapse path on the materialised delay instead.
static constexpr int kMMMax = 1;

// --------------------------------------------------------------------------------
// forward planning
// --------------------------------------------------------------------------------
struct FwdPlan {
  int nth, ipt, R, NW, TAPS;
  size_t smem;
  int ring_smem;
};

static FwdPlan plan_forward(const delrec_layer* ly, int kind) {
  FwdPlan p;
  const int N = ly->N;
  p.nth = std::min(512, ((N + 31) / 32) * 32);
  p.ipt = cdiv(N, p.nth);
  if (p.ipt > 2 && p.ipt <= 4) p.ipt = 4;
  else if (p.ipt > 4) p.ipt = 8;
  p.NW = cdiv(N, 32);
  p.R = pow2_at_least(std::max(ly->L, 2));
  p.TAPS = taps_for(ly);
  if (kind == DELREC_AXONAL) {
    p.ring_smem = 0;
    p.smem = (size_t)p.R * p.NW * 4 + (size_t)N * (2 + p.TAPS) * 4 + (size_t)N * 8;
  } else {
    const size_t ring = (size_t)ly->L * N * 4;
    // event list, s, base; hybrid: the base's tap table
    const size_t rest = (size_t)N * 4 * 3 + (kind == DELREC_HYBRID ? (size_t)N * 4 * (2 + p.TAPS) : 0);
    p.ring_smem = (ring + rest <= 160 * 1024) ? 1 : 0;
    p.smem = (p.ring_smem ? ring : 0) + rest;
  }
  return p;
}

template <class K>
static int set_smem(K kernel, size_t bytes) {
  if (bytes > kSmemLimit) return DELREC_ERR_UNSUPPORTED;
  DR_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return DELREC_OK;
}

template <int IPT>
static int launch_fwd_axonal(const FwdArgs& a, const FwdPlan& p, cudaStream_t st) {
  int rc = set_smem(k_fwd_axonal<IPT>, p.smem);
  if (rc) return rc;
  k_fwd_axonal<IPT><<<a.B, p.nth, p.smem, st>>>(a);
  DR_LAUNCHED();
  return DELREC_OK;
}
// the 4-neurons-per-thread axonal forward: N % 4 == 0, N <= 1024, 16-byte aligned rows
static bool fwd_axonal4_ok(const delrec_layer* ly, const FwdArgs& a) {
  const auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  return ly->N % 4 == 0 && ly->N <= 1024 && al(a.x) && al(a.y) && al(a.u) && al(a.WT);
}
static int launch_fwd_axonal4(const FwdArgs& a, const FwdPlan& p, cudaStream_t st) {
  int rc = set_smem(k_fwd_axonal4<32>, p.smem);
  if (rc) return rc;
  const int nth = ((a.N / 4 + 31) / 32) * 32;
  k_fwd_axonal4<32><<<a.B, nth, p.smem, st>>>(a);
  DR_LAUNCHED();
  return DELREC_OK;
}
template <int IPT, bool HYB>
static int launch_fwd_syn(const FwdArgs& a, const FwdPlan& p, cudaStream_t st) {
  int rc = set_smem(k_fwd_synaptic<IPT, HYB>, p.smem);
  if (rc) return rc;
  k_fwd_synaptic<IPT, HYB><<<a.B, p.nth, p.smem, st>>>(a);
  DR_LAUNCHED();
  return DELREC_OK;
}

// Programmatic dependent launch (the chunk loop's and the step loops' kernels): the kernel
// may start while the previous kernel on the stream finishes; its griddepcontrol.wait
// orders every read of that kernel's results after its completion.
static cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                                     cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Wide axonal layers (N > 512) run their forward step by step: per step one LIF kernel
// (which also lays out the next step's spike operand) and one tensor-core GEMM
// rec(t+1) = [Y_0 .. Y_TF-1](t+1) . [W h(0) .. W h(TF-1)]^T over the positive taps, the
// tap-weighted W in three exact bf16 pieces (linear.cuh).  The GEMM leaves its reduction
// split's fp32 partials for the LIF kernel, which adds them in a fixed order: no partial
// sums more than ~1536 piece products, so the tensor core's fp32 accumulation stays
// within the 1e-5 membrane contract at any width and batch.
static bool axstep_fwd(const delrec_layer* ly) { return ly->kind == DELREC_AXONAL && ly->N > 512; }
static constexpr int kFwdStepSplit = 16;
struct FwdStepPlan {
  int TF, Kp, BN, ksplit;
};
static FwdStepPlan plan_fwd_step(const delrec_layer* ly) {
  FwdStepPlan p;
  // positive taps of a triangle of half-width s lie in an open interval of length 2s
  p.TF = std::max(1, (int)std::ceil(2.0 * (double)ly->s_max - 1e-6));
  p.Kp = (p.TF * ly->N + 7) / 8 * 8;
  p.BN = gemm_pick_bn(ly->N);
  p.ksplit = gemm_pick_ksplit(ly->B, ly->N, p.Kp, 3, 1, 1, p.BN, kFwdStepSplit, 4);
  // accuracy floor (large batches fill the GPU without splitting): at most ~1536 piece
  // products per accumulator
  const int cap = std::max(1, std::min(kFwdStepSplit, 3 * ((p.Kp + 63) / 64) / 4));
  p.ksplit = std::max(p.ksplit, std::min((3 * p.Kp + 1535) / 1536, cap));
  return p;
}
static size_t fwd_step_ws(const delrec_layer* ly) {
  const FwdStepPlan p = plan_fwd_step(ly);
  const size_t N = ly->N, BN = (size_t)ly->B * N;
  Carve c(nullptr, (size_t)-1);
  c.take<int2>(N);                                    // positive taps
  c.take<float>(BN);                                  // v
  c.take<__nv_bfloat16>((size_t)ly->B * p.Kp);       // spike operand
  c.take<__nv_bfloat16>(3 * N * p.Kp);               // tap-weighted W pieces
  c.take<unsigned char>(gemm_partial_bytes(ly->B, ly->N, p.ksplit, 1, true));
  return c.off;
}
static int run_axstep_fwd(const delrec_layer* ly, const FwdArgs& a, const float* W, Carve& c, cudaStream_t st) {
  const int N = ly->N, B = ly->B, T = ly->T;
  const FwdStepPlan p = plan_fwd_step(ly);
  const size_t BN = (size_t)B * N, nk = (size_t)N * p.Kp;
  int2* fp = c.take<int2>(N);
  float* v = c.take<float>(BN);
  __nv_bfloat16* A16 = c.take<__nv_bfloat16>((size_t)B * p.Kp);
  __nv_bfloat16* Wp = c.take<__nv_bfloat16>(3 * nk);
  float* part = (float*)c.take<unsigned char>(gemm_partial_bytes(B, N, p.ksplit, 1, true));
  if (!c.ok) return DELREC_ERR_WORKSPACE;
  k_pos_taps<<<cdiv(N, 256), 256, 0, st>>>(N, a.TAPS, a.tap_l0, a.tap_nt, a.tap_w, p.TF, fp);
  DR_LAUNCHED();
  k_wtap_pieces<<<grid_for(nk, 256), 256, 0, st>>>(N, a.TAPS, p.TF, p.Kp, W, a.tap_l0, a.tap_w, fp, Wp, Wp + nk,
                                                   Wp + 2 * nk);
  DR_LAUNCHED();
  DR_CUDA(cudaMemsetAsync(A16, 0, (size_t)B * p.Kp * sizeof(__nv_bfloat16), st));
  k_fill_f32<<<grid_for(BN, 256), 256, 0, st>>>(v, BN, a.lif.v0);
  DR_LAUNCHED();
  GemmSide As{}, Ws{};   // K-major bf16 operands: rows x Kp, row stride Kp
  As.p[0] = A16; As.n = 1; As.rows = B; As.cols = p.Kp; As.ld = p.Kp;
  Ws.p[0] = Wp; Ws.p[1] = Wp + nk; Ws.p[2] = Wp + 2 * nk; Ws.n = 3;
  Ws.rows = N; Ws.cols = p.Kp; Ws.ld = p.Kp;
  GemmArgs g{};
  g.M = B; g.N = N; g.K = p.Kp; g.nprod = 3; g.nseg = 1;
  g.pa[0] = g.pa[1] = g.pa[2] = 0;
  g.pb[0] = 0; g.pb[1] = 1; g.pb[2] = 2;
  g.ksplit = p.ksplit;
  g.D = part; g.ldd = N; g.mode = GEMM_PARTIALS;
  GemmLaunch gl;
  int rc = gemm_prepare(As, Ws, g, 1, p.BN, part, &gl);   // tensor maps encoded once
  if (rc) return rc;
  // every launch after the first is a programmatic dependent of the one before it
  for (int t = 0; t < T; ++t) {
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(dim3(grid_for(BN, 256)), dim3(256), 0, st, t > 0, attr);
    DR_CUDA(cudaLaunchKernelEx(&cfg, k_step_lif_fwd, t, T, B, N, p.TF, a.x, (const float*)part, p.ksplit, a.bias,
                               a.keep, (const int2*)fp, v, a.y, a.u, A16, p.Kp, a.lif));
    DR_LAUNCHED();
    if (t + 1 < T) {
      rc = gemm_exec(gl, nullptr, st, &g_launches, true);
      if (rc) return rc;
    }
  }
  return DELREC_OK;
}

static size_t forward_ws(const delrec_layer* ly, int kind, bool allow_step = true) {
  const FwdPlan p = plan_forward(ly, kind);
  const size_t N = ly->N;
  Carve c(nullptr, (size_t)-1);
  c.take<float>(N * N);                             // WT
  if (kind == DELREC_AXONAL) {
    c.take<int>(N); c.take<int>(N); c.take<float>(N * p.TAPS);
    if (allow_step && axstep_fwd(ly)) c.take<unsigned char>(fwd_step_ws(ly));   // step-by-step forward
  } else if (kind == DELREC_SYNAPTIC) {
    c.take<float>(N * N);                           // dT
    c.take<int4>(N * N);                            // scatter records
  } else {
    c.take<uint8_t>(N * N);                         // offT
    c.take<int>(N); c.take<int>(N); c.take<float>(N * p.TAPS);   // base taps
    c.take<int4>(N * N);                            // scatter records
  }
  if (kind != DELREC_AXONAL && !p.ring_smem) c.take<float>((size_t)ly->B * ly->L * N);
  return c.off;
}

static int run_forward(const delrec_layer* ly, int kind, const delrec_lif* lif, const float* x,
                       const float* W, const float* bias, const float* d, const float* offsets,
                       const float* s, const float* keep, float* y, float* u, void* ws,
                       size_t wsb, cudaStream_t st, bool allow_step = true) {
  int rc = check_layer(ly, kind);
  if (rc) return rc;
  if (!lif || !x || !W || !d || !s || !y || !u) return DELREC_ERR_ARG;
  if (kind == DELREC_HYBRID && !offsets) return DELREC_ERR_ARG;
  if (ly->has_bias && !bias) return DELREC_ERR_ARG;
  if (ly->has_keep && !keep) return DELREC_ERR_ARG;
  if (((uintptr_t)ws & 255) != 0) return DELREC_ERR_WORKSPACE;
  if (wsb < forward_ws(ly, kind, allow_step)) return DELREC_ERR_WORKSPACE;
  const FwdPlan p = plan_forward(ly, kind);
  const int N = ly->N;
  Carve c(ws, wsb);
  FwdArgs a{};
  a.T = ly->T; a.B = ly->B; a.N = N; a.L = ly->L; a.R = p.R; a.NW = p.NW; a.TAPS = p.TAPS;
  a.x = x; a.bias = ly->has_bias ? bias : nullptr; a.keep = ly->has_keep ? keep : nullptr; a.s = s;
  a.y = y; a.u = u; a.lif = make_lif(*lif); a.ring_smem = p.ring_smem;
  float* WT = c.take<float>((size_t)N * N);
  dim3 tb(32, 8), tg(cdiv(N, 32), cdiv(N, 32));
  k_transpose<<<tg, tb, 0, st>>>(W, WT, N, N);
  DR_LAUNCHED();
  a.WT = WT;
  if (kind == DELREC_AXONAL) {
    int* l0 = c.take<int>(N);
    int* nt = c.take<int>(N);
    float* w = c.take<float>((size_t)N * p.TAPS);
    k_taps<<<cdiv(N, 256), 256, 0, st>>>(d, s, N, ly->L - 1, p.TAPS, 1, l0, nt, w);
    DR_LAUNCHED();
    a.tap_l0 = l0; a.tap_nt = nt; a.tap_w = w;
    if (allow_step && axstep_fwd(ly)) return run_axstep_fwd(ly, a, W, c, st);
    if (fwd_axonal4_ok(ly, a)) return launch_fwd_axonal4(a, p, st);
    switch (p.ipt) {
      case 1: return launch_fwd_axonal<1>(a, p, st);
      case 2: return launch_fwd_axonal<2>(a, p, st);
      case 4: return launch_fwd_axonal<4>(a, p, st);
      default: return launch_fwd_axonal<8>(a, p, st);
    }
  }
  if (kind == DELREC_SYNAPTIC) {
    float* dT = c.take<float>((size_t)N * N);
    k_transpose<<<tg, tb, 0, st>>>(d, dT, N, N);
    DR_LAUNCHED();
    a.dT = dT;
    int4* rec = c.take<int4>((size_t)N * N);
    k_syn_records_syn<<<grid_for((size_t)N * N, 256), 256, 0, st>>>(N, ly->L, dT, s, WT, rec);
    DR_LAUNCHED();
    a.rec = rec;
  } else {
    uint8_t* offT = c.take<uint8_t>((size_t)N * N);
    k_offsets_u8T<<<tg, tb, 0, st>>>(offsets, offT, N, ly->K);
    DR_LAUNCHED();
    a.offT = offT;
    a.base = d;
    // base taps from lag 1-K: a base lag l' <= 0 reaches the synapses with offset >= 1-l'
    int* l0 = c.take<int>(N);
    int* nt = c.take<int>(N);
    float* w = c.take<float>((size_t)N * p.TAPS);
    k_taps<<<cdiv(N, 256), 256, 0, st>>>(d, s, N, ly->L - 1, p.TAPS, 1 - ly->K, l0, nt, w);
    DR_LAUNCHED();
    a.tap_l0 = l0; a.tap_nt = nt; a.tap_w = w;
    int4* rec = c.take<int4>((size_t)N * N);
    k_syn_records<<<grid_for((size_t)N * N, 256), 256, 0, st>>>(N, ly->L, offT, WT, l0, nt, w, p.TAPS, rec);
    DR_LAUNCHED();
    a.rec = rec;
  }
  if (!p.ring_smem) a.ring_g = c.take<float>((size_t)ly->B * ly->L * N);
  const bool hyb = kind == DELREC_HYBRID;
  switch (p.ipt) {
    case 1: return hyb ? launch_fwd_syn<1, true>(a, p, st) : launch_fwd_syn<1, false>(a, p, st);
    case 2: return hyb ? launch_fwd_syn<2, true>(a, p, st) : launch_fwd_syn<2, false>(a, p, st);
    case 4: return hyb ? launch_fwd_syn<4, true>(a, p, st) : launch_fwd_syn<4, false>(a, p, st);
    default: return hyb ? launch_fwd_syn<8, true>(a, p, st) : launch_fwd_syn<8, false>(a, p, st);
  }
}

// --------------------------------------------------------------------------------
// backward planning
// --------------------------------------------------------------------------------
struct BwdPlan {
  int mode, CS, NT, BT, KS, PPT, KH, NKEY, CAP, PADM, TAPS, w_smem, MM;
  size_t smem;
  bool ok;
};

static BwdPlan plan_backward(const delrec_layer* ly, int kind) {
  const int N = ly->N, B = ly->B;
  const int mode = kind == DELREC_AXONAL ? 0 : (kind == DELREC_HYBRID ? 1 : 2);
  BwdPlan best{};
  best.ok = false;
  double best_cost = 1e300;
  const int TAPS = taps_for(ly);
  const int KH = ly->K + 1;
  const int MM = mode == 1 ? hybrid_mm(ly) : 0;
  const int bts[3] = {32, 16, 8};
  const int css[5] = {1, 2, 4, 8, 16};
  for (int bi = 0; bi < 3; ++bi) {
    const int BT = bts[bi];
    for (int ci = 0; ci < 5; ++ci) {
      const int CS = css[ci];
      int NT = ((cdiv(N, CS) + 3) / 4) * 4;
      if (CS > 1 && (CS - 1) * NT >= N) continue;     // an empty rank
      if (NT * BT > 1024) continue;                    // PPT <= 4 with 256 threads
      const int tiles = (BT / 4) * (NT / 4);
      if (mode == 0 && tiles > 256) continue;
      const int KS = mode == 0 ? std::max(1, std::min(256 / tiles, N)) : 1;
      int w_smem = 1;
      BwdSmem sm = bwd_smem_plan(mode, N, NT, BT, KS, KH, ly->L, TAPS, w_smem, MM);
      if (sm.total > kSmemLimit && mode == 0) {
        w_smem = 0;
        sm = bwd_smem_plan(mode, N, NT, BT, KS, KH, ly->L, TAPS, w_smem, MM);
      }
      if (sm.total > kSmemLimit) continue;
      const int ctas = CS * cdiv(B, BT);
      const int per_wave = (kSMs / CS) * CS;
      const int waves = cdiv(ctas, per_wave);
      // per-step work of one block (synapse-sample products) plus a cluster overhead
      const double work = (double)NT * BT * (N + 64) * (mode == 0 ? 1.0 : 2.0) * (w_smem ? 1.0 : 2.0);
      const double cost = waves * (work + 4000.0 * CS + 20000.0);
      if (cost < best_cost) {
        best_cost = cost;
        best.ok = true;
        best.mode = mode; best.CS = CS; best.NT = NT; best.BT = BT; best.KS = KS;
        best.PPT = cdiv(NT * BT, 256); best.KH = KH; best.TAPS = TAPS; best.w_smem = w_smem;
        best.MM = MM;
        best.smem = sm.total;
      }
    }
  }
  best.NKEY = mode == 1 ? KH : ly->L;
  best.PADM = best.ok ? 4 * (32 / best.BT) : 4;
  // room for the padding of either backward kernel (the specialised hybrid one pads to 8)
  best.CAP = (mode == 1 ? N : N * std::min(ly->L, 2 * kTapsMax)) + best.NKEY * std::max(best.PADM, 8);
  best.CAP = (best.CAP + 7) / 8 * 8;   // rows start 16-byte aligned for 8-byte entries (4-entry vectors)
  return best;
}

// Specialised hybrid reverse scan (backward_hybrid.cuh): 32 sources per block, batch
// tiles of 32, resident bucket lists.  Usable when N <= 512, K <= 8, MM <= 1 and the
// lists fit in shared memory.
struct HybPlan {
  bool ok, coop;
  int CS, NT, CAPS, KMAX, tiles;
  size_t smem;
};
static HybPlan plan_hybrid_fast(const delrec_layer* ly, const BwdPlan& bp) {
  HybPlan h{};
  h.ok = false;
  if (ly->kind != DELREC_HYBRID || bp.MM > ly->K || ly->K > 8) return h;
  if (ly->N > 512) return h;   // 16-bit byte offsets of the gr rows (512 rows of 128 B)
  h.NT = 32;
  h.CS = cdiv(ly->N, h.NT);
  h.tiles = cdiv(ly->B, 32);
  // one wave: a cooperative launch when every block fits on its own SM, else clusters
  h.coop = h.CS * h.tiles <= kSMs;
  if (!h.coop && h.CS > 16) return h;
  h.CAPS = ((ly->N + 7 * (ly->K + 1)) + 7) / 8 * 8;   // buckets padded to 8 entries
  h.KMAX = ly->K <= 4 ? 5 : 9;
  h.smem = hyb_smem_plan(ly->N, h.NT, h.CAPS, ly->K, bp.TAPS, h.KMAX).total;
  h.ok = h.smem <= kSmemLimit;
  return h;
}

template <int KMAX>
static int launch_hyb_t(const HybArgs& a, const HybPlan& h, cudaStream_t st) {
  if (h.coop) {
    auto kern = k_bwd_hybrid<KMAX, true>;
    int rc = set_smem(kern, h.smem);
    if (rc) return rc;
    int per_sm = 0;
    DR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 512, h.smem));
    if (per_sm >= 1 && h.CS * h.tiles <= per_sm * kSMs) {
      DR_CUDA(cudaMemsetAsync(a.arrive, 0, sizeof(unsigned int) * h.tiles, st));
      HybArgs ac = a;
      void* args[] = {(void*)&ac};
      scan_mark(0, st);
      DR_CUDA(cudaLaunchCooperativeKernel((const void*)kern, dim3(h.CS * h.tiles), dim3(512), args, h.smem, st));
      scan_mark(1, st);
      ++g_launches;
      return DELREC_OK;
    }
    if (h.CS > 16) return DELREC_ERR_UNSUPPORTED;
  }
  auto kern = k_bwd_hybrid<KMAX, false>;
  int rc = set_smem(kern, h.smem);
  if (rc) return rc;
  if (h.CS > 8) DR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(h.CS * cdiv(a.B, 32));
  cfg.blockDim = dim3(512);
  cfg.dynamicSmemBytes = h.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = h.CS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  scan_mark(0, st);
  DR_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
  scan_mark(1, st);
  ++g_launches;
  return DELREC_OK;
}

// Hybrid reverse scan with 64-sample tiles and deferred synapse sums
// (backward_hybrid64.cuh): cooperative single wave, every base tap at lag >= 1 (MM = 0),
// K <= 8, N <= 512 (gr of a tile staged in shared memory), at most 8 taps per source.
struct Hyb64Plan {
  bool ok;
  int CS, NT, tiles, CAPS, KMAX, K, NKEY, CAP;
  size_t smem;
};
static constexpr int kH64Taps = 8;
// Axonal layers run the same scan as a hybrid layer whose offsets are all 0 (one bucket
// per source holding all its synapses).
static Hyb64Plan plan_hybrid64(const delrec_layer* ly, const BwdPlan& bp) {
  Hyb64Plan h{};
  h.ok = false;
  if (ly->kind == DELREC_SYNAPTIC) return h;
  h.K = ly->kind == DELREC_HYBRID ? ly->K : 0;
  if (bp.MM != 0 || h.K > 8 || ly->N > 512 || bp.TAPS > kH64Taps) return h;
  if (ly->B <= 32) return h;   // a 32-sample tile wastes no lanes there
  h.tiles = cdiv(ly->B, kH64BT);
  // sources per block: fill the SMs (every block stages all N rows of gr, so not fewer
  // than 12 sources per block)
  h.NT = std::max(12, cdiv(ly->N * h.tiles, kSMs));
  if (h.NT > kH64NTMax) return h;
  h.CS = cdiv(ly->N, h.NT);
  if (h.CS * h.tiles > kSMs) return h;
  // small axonal layers keep the generic cluster scan (a few 64-sample blocks run slower)
  if (ly->kind == DELREC_AXONAL && h.CS * h.tiles < 32) return h;
  h.CAPS = ((ly->N + 7 * (h.K + 1)) + 7) / 8 * 8;
  h.NKEY = h.K + 1;
  h.CAP = ly->kind == DELREC_HYBRID ? bp.CAP : h.CAPS;
  h.KMAX = h.K <= 4 ? 6 : 10;
  h.smem = hyb64_smem_plan(ly->N, h.NT, h.CAPS, h.K, bp.TAPS, h.KMAX).total;
  h.ok = h.smem <= kSmemLimit;
  return h;
}

// Synaptic layers in the 64-sample-tile scan: bucket k holds the synapse taps at lag k+1
// (weight W*h), one unit base tap at lag 1; lags up to 31 (ring of 32 slots).
static constexpr int kSynKmax = 32;
static Hyb64Plan plan_syn64(const delrec_layer* ly) {
  Hyb64Plan h{};
  h.ok = false;
  if (ly->kind != DELREC_SYNAPTIC || ly->N > 512 || ly->B <= 32) return h;
  h.K = ly->L - 2;
  if (h.K < 0 || h.K + 2 > kSynKmax) return h;
  const int maxtaps = (int)ceilf(2.f * ly->s_max) + 1;   // integer lags inside one triangle
  h.CAPS = (ly->N * maxtaps + 7 * (h.K + 1) + 7) / 8 * 8;
  h.NKEY = ly->L;
  h.KMAX = kSynKmax;
  h.tiles = cdiv(ly->B, kH64BT);
  int fit = 0;
  for (int nt = kH64NTMax; nt >= 1 && !fit; --nt)
    if (hyb64_smem_plan(ly->N, nt, h.CAPS, h.K, 1, h.KMAX).total <= kSmemLimit) fit = nt;
  h.NT = std::max(4, cdiv(ly->N * h.tiles, kSMs));
  if (fit == 0 || h.NT > fit) return h;
  h.CS = cdiv(ly->N, h.NT);
  if (h.CS * h.tiles > kSMs) return h;
  h.smem = hyb64_smem_plan(ly->N, h.NT, h.CAPS, h.K, 1, h.KMAX).total;
  h.ok = true;
  return h;
}

// Axonal layers with the per-step contraction on tensor cores (backward_axonal_mma.cuh):
// the same one-wave tiling as the 64-sample scan, 16 sources per block.
struct AxMmaPlan {
  bool ok;
  int CS, tiles;
  size_t smem;
};
static AxMmaPlan plan_axmma(const delrec_layer* ly, const BwdPlan& bp) {
  AxMmaPlan h{};
  h.ok = false;
  if (ly->kind != DELREC_AXONAL || bp.MM != 0 || ly->N % 4 != 0 || ly->N > 1024 || bp.TAPS > kH64Taps) return h;
  if (ly->B <= 32) return h;
  h.CS = cdiv(ly->N, kAxNT);
  h.tiles = cdiv(ly->B, kAxBT);
  if (h.CS * h.tiles > kSMs || h.CS * h.tiles < 32) return h;
  h.smem = axmma_smem_plan(ly->N, bp.TAPS).total;
  h.ok = h.smem <= kSmemLimit;
  return h;
}
static int launch_axmma(const AxMmaArgs& a, const AxMmaPlan& h, cudaStream_t st) {
  auto kern = k_bwd_axonal_mma<kH64Taps>;
  int rc = set_smem(kern, h.smem);
  if (rc) return rc;
  int per_sm = 0;
  DR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kAxThreads, h.smem));
  if (per_sm < 1 || h.CS * h.tiles > per_sm * kSMs) return DELREC_ERR_UNSUPPORTED;
  DR_CUDA(cudaMemsetAsync(a.arrive, 0, sizeof(unsigned int) * h.tiles, st));
  AxMmaArgs ac = a;
  void* args[] = {(void*)&ac};
  scan_mark(0, st);
  DR_CUDA(cudaLaunchCooperativeKernel((const void*)kern, dim3(h.CS * h.tiles), dim3(kAxThreads), args, h.smem, st));
  scan_mark(1, st);
  ++g_launches;
  return DELREC_OK;
}

template <int KMAX>
static int launch_hyb64_t(const Hyb64Args& a, const Hyb64Plan& h, cudaStream_t st) {
  auto kern = k_bwd_hybrid64<KMAX, kH64Taps>;
  int rc = set_smem(kern, h.smem);
  if (rc) return rc;
  int per_sm = 0;
  DR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kH64Threads, h.smem));
  if (per_sm < 1 || h.CS * h.tiles > per_sm * kSMs) return DELREC_ERR_UNSUPPORTED;
  DR_CUDA(cudaMemsetAsync(a.arrive, 0, sizeof(unsigned int) * h.tiles, st));
  Hyb64Args ac = a;
  void* args[] = {(void*)&ac};
  scan_mark(0, st);
  DR_CUDA(cudaLaunchCooperativeKernel((const void*)kern, dim3(h.CS * h.tiles), dim3(kH64Threads), args, h.smem,
                                      st));
  scan_mark(1, st);
  ++g_launches;
  return DELREC_OK;
}

template <int MODE, int BT, int PPT>
static int launch_bwd_t(const BwdArgs& a, const BwdPlan& p, cudaStream_t st) {
  auto kern = k_bwd<MODE, BT, PPT>;
  int rc = set_smem(kern, p.smem);
  if (rc) return rc;
  if (p.CS > 8) DR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.CS * cdiv(a.B, BT));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.CS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  scan_mark(0, st);
  DR_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
  scan_mark(1, st);
  ++g_launches;
  return DELREC_OK;
}

template <int MODE, int BT>
static int launch_bwd_ppt(const BwdArgs& a, const BwdPlan& p, cudaStream_t st) {
  switch (p.PPT) {
    case 1: return launch_bwd_t<MODE, BT, 1>(a, p, st);
    case 2: return launch_bwd_t<MODE, BT, 2>(a, p, st);
    default: return launch_bwd_t<MODE, BT, 4>(a, p, st);
  }
}
template <int MODE>
static int launch_bwd_mode(const BwdArgs& a, const BwdPlan& p, cudaStream_t st) {
  switch (p.BT) {
    case 32: return launch_bwd_ppt<MODE, 32>(a, p, st);
    case 16: return launch_bwd_ppt<MODE, 16>(a, p, st);
    default: return launch_bwd_ppt<MODE, 8>(a, p, st);
  }
}

// Synaptic weight-gradient lag window: the lags from max(1, floor(1 + d - s) - 1) that the
// triangle (and its derivatives) of a synapse can touch, as a template width 4, 8 or 16.
static int syn_window(const delrec_layer* ly) {
  const int tw = std::min(std::max(std::min(ly->L - 1, 2 * (int)ceilf(ly->s_max) + 4), 1), 16);
  return tw <= 4 ? 4 : (tw <= 8 ? 8 : 16);
}

struct SrcPlan { int splits, tsplit; };
static SrcPlan plan_src(const delrec_layer* ly) {
  SrcPlan p;
  // one partial row per chunk of 8 samples and time chunk (time chunks: the fused pass
  // of the axonal / hybrid layers, so that enough threads stream)
  p.tsplit = ly->kind == DELREC_SYNAPTIC ? 1 : std::max(1, std::min(4, ly->T / 64));
  p.splits = cdiv(ly->B, 8) * p.tsplit;
  return p;
}

// ---- tensor-core dW (dense.cuh) -------------------------------------------------
static inline int pad8(int n) { return (n + 7) / 8 * 8; }
// k_split_bf16_rows launch: a block per row (grid-stride), a thread per 4 columns
static inline int split_rows_block(int N) { return std::min(256, std::max(32, (cdiv(pad8(N), 4) + 31) / 32 * 32)); }
static inline int split_rows_grid(size_t rows) { return (int)std::max<size_t>(1, std::min<size_t>(rows, (size_t)kSMs * 16)); }
// Split of the dW-type reductions (over the T*B rows) and its tile width.
static int dw_bn(const delrec_layer* ly) { return gemm_pick_bn(ly->N); }
static int dw_ksplit(const delrec_layer* ly, int nprod, int nslices) {
  return gemm_pick_ksplit(ly->N, ly->N, ly->T * ly->B, nprod, 1, nslices, dw_bn(ly));
}

// bytes of the tensor-core dW path: bf16 pieces of gr and of each z variant, the
// split-reduction partials, and (synaptic) the L lag products
static size_t dense_dw_ws(const delrec_layer* ly, int nz, int nk) {
  const size_t TBN = (size_t)ly->T * ly->B * pad8(ly->N), nn = (size_t)ly->N * ly->N;
  Carve c(nullptr, (size_t)-1);
  c.take<__nv_bfloat16>(TBN * 2);
  c.take<__nv_bfloat16>(TBN * 2 * nz);
  if (ly->kind == DELREC_SYNAPTIC) c.take<float>(nn * nk);
  const int np = ly->kind == DELREC_SYNAPTIC ? 2 : 3;
  c.take<unsigned char>(gemm_partial_bytes(ly->N, ly->N, dw_ksplit(ly, np, nk), nk));
  return c.off;
}

// Buffers of the tensor-core dW path (inside the caller's workspace).  The bf16 pieces
// are (T*B, Np) with Np = N rounded up to 8 (16-byte rows for the tensor maps).
struct DenseBufs {
  __nv_bfloat16* g16;   // gr pieces: hi [T*B*Np], lo [T*B*Np]
  __nv_bfloat16* z16;   // z variant v: hi at v*2*T*B*Np, lo T*B*Np after it
  float* P;             // synaptic: (L, N, N) lag products
  float* part;          // split-reduction partials
};
static bool dense_carve(const delrec_layer* ly, int nz, int nk, Carve& c, DenseBufs* d) {
  const size_t TBN = (size_t)ly->T * ly->B * pad8(ly->N), nn = (size_t)ly->N * ly->N;
  d->g16 = c.take<__nv_bfloat16>(TBN * 2);
  d->z16 = c.take<__nv_bfloat16>(TBN * 2 * nz);
  d->P = ly->kind == DELREC_SYNAPTIC ? c.take<float>(nn * nk) : nullptr;
  const int np = ly->kind == DELREC_SYNAPTIC ? 2 : 3;
  d->part = (float*)c.take<unsigned char>(gemm_partial_bytes(ly->N, ly->N, dw_ksplit(ly, np, nk), nk));
  return c.ok;
}

// A (T*B, N) activation's bf16 pieces as an MN-major GEMM operand (reduced over T*B).
static GemmSide rows_operand(const __nv_bfloat16* p0, const __nv_bfloat16* p1, int n, const delrec_layer* ly) {
  GemmSide s{};
  s.p[0] = p0;
  s.p[1] = p1;
  s.n = n;
  s.rows = (long long)ly->T * ly->B;
  s.cols = ly->N;
  s.ld = pad8(ly->N);
  s.mn_major = 1;
  return s;
}

// dW (N,N) from gr (T,B,N) and the z variants (already in d.z16), v = min(k, nz-1) for
// offset k:  dW[i,o] = sum_r gr[r + k_io*B, i] z_v[r, o] over the T*B rows r, on the
// tensor cores as three bf16 piece products (hi.hi + hi.lo + lo.hi) with the offset k as
// the batch index (a row shift of the gr operand; rows past T*B read as zero) and each
// batch writing only the synapses whose offset is k.
static int dense_dw(const delrec_layer* ly, const float* gr, int nz, int nk, const uint8_t* offT, float* dW,
                    const DenseBufs& d, cudaStream_t st) {
  const int N = ly->N, T = ly->T, B = ly->B;
  const size_t TBN = (size_t)T * B * pad8(N);
  k_split_bf16_rows<<<split_rows_grid((size_t)T * B), split_rows_block(N), 0, st>>>(gr, (size_t)T * B, N, pad8(N), d.g16, d.g16 + TBN);
  DR_LAUNCHED();
  const GemmSide A = rows_operand(d.g16, d.g16 + TBN, 2, ly);
  const int BN = dw_bn(ly);
  // offsets k < nz-1 use z variant k alone; k >= nz-1 share variant nz-1 (one batch)
  for (int k0 = 0; k0 < nk;) {
    const int v = k0 < nz - 1 ? k0 : nz - 1;
    const int count = k0 < nz - 1 ? 1 : nk - k0;
    const __nv_bfloat16* Zh = d.z16 + (size_t)v * 2 * TBN;
    const GemmSide Bz = rows_operand(Zh, Zh + TBN, 2, ly);
    GemmArgs g{};
    g.M = N; g.N = N; g.K = T * B; g.nprod = 3; g.nseg = 1;
    g.pa[0] = 0; g.pb[0] = 0; g.pa[1] = 0; g.pb[1] = 1; g.pa[2] = 1; g.pb[2] = 0;
    g.a_k_z = B;            // offset k: gr rows shifted by k steps
    g.z0 = k0;
    g.ksplit = dw_ksplit(ly, 3, nk);
    g.D = dW; g.ldd = N; g.d_z = 0;
    g.mode = nk > 1 ? GEMM_MASKED : GEMM_STORE;
    g.mask = offT; g.ldmask = 1; g.mask_cs = N;    // offT[o*N + i]: the offset of synapse (i, o)
    const int rc = gemm_run(A, Bz, g, count, BN, d.part, st, &g_launches);
    if (rc) return rc;
    k0 += count;
  }
  return DELREC_OK;
}

// Synaptic layers: the per-lag correlation stack C_l = sum_r gr[r + l*B] (x) y[r] for all
// lags l = 0..L-1 (the reference's Cstack), as one batched GEMM over the T*B rows: gr in
// hi + lo pieces, the spikes exact in one piece, the lag as the batch index (a row shift
// of the gr operand).  d.P receives C (L, N, N).
static int syn_cstack(const delrec_layer* ly, const float* gr, const float* y, const DenseBufs& d, cudaStream_t st) {
  const int N = ly->N, T = ly->T, B = ly->B, nk = ly->L;
  const size_t TBN = (size_t)T * B * pad8(N), nn = (size_t)N * N;
  k_split_bf16_rows<<<split_rows_grid((size_t)T * B), split_rows_block(N), 0, st>>>(gr, (size_t)T * B, N, pad8(N), d.g16, d.g16 + TBN);
  DR_LAUNCHED();
  k_split_bf16_rows<<<split_rows_grid((size_t)T * B), split_rows_block(N), 0, st>>>(y, (size_t)T * B, N, pad8(N), d.z16, d.z16 + TBN);
  DR_LAUNCHED();
  const GemmSide A = rows_operand(d.g16, d.g16 + TBN, 2, ly);
  const GemmSide Y = rows_operand(d.z16, nullptr, 1, ly);
  GemmArgs g{};
  g.M = N; g.N = N; g.K = T * B; g.nprod = 2; g.nseg = 1;
  g.pa[0] = 0; g.pb[0] = 0; g.pa[1] = 1; g.pb[1] = 0;
  g.a_k_z = B;
  g.ksplit = dw_ksplit(ly, 2, nk);
  g.D = d.P; g.ldd = N; g.d_z = (long long)nn;
  g.mode = GEMM_STORE;
  return gemm_run(A, Y, g, nk, dw_bn(ly), d.part, st, &g_launches);
}

// ---- feedforward projection on tensor cores (linear.cuh) ------------------------
struct LinPlan {
  int Kp, Np, nbx;       // padded widths, x pieces (1 for spikes, else 3)
};
static LinPlan plan_linear(int K, int N, int x_binary) {
  LinPlan p;
  p.Kp = (K + 1 + 7) / 8 * 8;
  p.Np = (N + 7) / 8 * 8;
  p.nbx = x_binary ? 1 : 3;
  return p;
}
// The piece products with i + j <= 2 of two 3-piece operands (or the 3 products of a
// 1-piece spike operand with the 3 pieces of the other), each operand's pieces stored once
static void lin_products(GemmArgs* g, int a_pieces) {
  static const int pa6[6] = {0, 1, 2, 0, 1, 0}, pb6[6] = {0, 0, 0, 1, 1, 2};
  g->nprod = a_pieces == 1 ? 3 : 6;
  for (int q = 0; q < g->nprod; ++q) {
    g->pa[q] = a_pieces == 1 ? 0 : pa6[q];
    g->pb[q] = a_pieces == 1 ? q : pb6[q];
  }
}
static int lin_ksplit(int M, int N, int K, int nprod) {
  return gemm_pick_ksplit(M, N, K, nprod, 1, 1, gemm_pick_bn(N), 8);
}
// K-major bf16 operand: rows x cols, row stride ld
static GemmSide kmajor_operand(const void* p, long long rows, long long cols, long long ld) {
  GemmSide s{};
  s.p[0] = p;
  s.n = 1;
  s.rows = rows;
  s.cols = cols;
  s.ld = ld;
  s.mn_major = 0;
  return s;
}
// MN-major bf16 operand: krows (reduction) x cols, row stride ld
static GemmSide mnmajor_operand(const void* p, long long krows, long long cols, long long ld) {
  GemmSide s = kmajor_operand(p, krows, cols, ld);
  s.mn_major = 1;
  return s;
}
// one-product GEMM D (M x Nn) (mode) = A . B^T over K, split as gemm_pick_ksplit decides
static int gemm1(const GemmSide& A, const GemmSide& B, int M, int Nn, int K, float* D, long long ldd, int mode,
                 float* part, int max_ks, cudaStream_t st) {
  GemmArgs g{};
  g.M = M; g.N = Nn; g.K = K; g.nprod = 1; g.nseg = 1;
  const int BN = gemm_pick_bn(Nn);
  g.ksplit = gemm_pick_ksplit(M, Nn, K, 1, 1, 1, BN, max_ks);
  g.D = D; g.ldd = ldd; g.mode = mode;
  return gemm_run(A, B, g, 1, BN, part, st, &g_launches);
}
static size_t gemm1_part_bytes(int M, int Nn, int K, int max_ks) {
  return gemm_partial_bytes(M, Nn, gemm_pick_ksplit(M, Nn, K, 1, 1, 1, gemm_pick_bn(Nn), max_ks), 1);
}
static constexpr int kLinMaxSplit = 8;

static size_t linear_fwd_ws(int M, int K, int N, int xb) {
  const LinPlan p = plan_linear(K, N, xb);
  Carve c(nullptr, (size_t)-1);
  c.take<__nv_bfloat16>((size_t)M * p.nbx * p.Kp);
  c.take<__nv_bfloat16>((size_t)N * 3 * p.Kp);
  c.take<unsigned char>(gemm_partial_bytes(M, N, lin_ksplit(M, N, p.Kp, p.nbx == 1 ? 3 : 6), 1));
  return c.off;
}
static size_t linear_bwd_ws(int M, int K, int N, int xb) {
  const LinPlan p = plan_linear(K, N, xb);
  Carve c(nullptr, (size_t)-1);
  c.take<__nv_bfloat16>((size_t)M * p.nbx * p.Kp);
  c.take<__nv_bfloat16>((size_t)M * 3 * p.Np);
  c.take<__nv_bfloat16>((size_t)3 * p.Np * p.Kp);
  c.take<float>((size_t)3 * p.Np * p.Kp);
  c.take<unsigned char>(std::max(gemm_partial_bytes(M, K, lin_ksplit(M, K, p.Np, 6), 1),
                                 gemm1_part_bytes(3 * p.Np, p.Kp, M, kLinMaxSplit)));
  return c.off;
}
static int run_linear_forward(int M, int K, int N, const float* x, const float* W, const float* bias, int xb,
                              float* out, void* ws, size_t wsb, cudaStream_t st) {
  if (M <= 0 || K <= 0 || N <= 0 || !x || !W || !out) return DELREC_ERR_ARG;
  if (((uintptr_t)ws & 255) != 0 || wsb < linear_fwd_ws(M, K, N, xb)) return DELREC_ERR_WORKSPACE;
  const LinPlan p = plan_linear(K, N, xb);
  Carve c(ws, wsb);
  __nv_bfloat16* X = c.take<__nv_bfloat16>((size_t)M * p.nbx * p.Kp);
  __nv_bfloat16* Wp = c.take<__nv_bfloat16>((size_t)N * 3 * p.Kp);
  const int nprod = p.nbx == 1 ? 3 : 6, ks = lin_ksplit(M, N, p.Kp, nprod);
  float* part = (float*)c.take<unsigned char>(gemm_partial_bytes(M, N, ks, 1));
  if (!c.ok) return DELREC_ERR_WORKSPACE;
  // rows [x0 (x1 x2)] and [W0 W1 W2], the ones / bias column at K
  k_pack_rows<<<grid_for((size_t)M * p.Kp / 8, 256), 256, 0, st>>>(M, K, p.Kp, x, K, nullptr, 1, p.nbx,
                                                                   kPatDistinct3, xb, X);
  DR_LAUNCHED();
  k_pack_rows<<<grid_for((size_t)N * p.Kp / 8, 256), 256, 0, st>>>(N, K, p.Kp, W, K, bias, 0, 3, kPatDistinct3, 0,
                                                                   Wp);
  DR_LAUNCHED();
  // out[m][n] = sum over the piece products of X_i[m][.] W_j[n][.]
  GemmSide A{}, Bw{};
  for (int i = 0; i < 3; ++i) {
    A.p[i] = X + (size_t)std::min(i, p.nbx - 1) * p.Kp;
    Bw.p[i] = Wp + (size_t)i * p.Kp;
  }
  A.n = p.nbx; A.rows = M; A.cols = p.Kp; A.ld = (long long)p.nbx * p.Kp;
  Bw.n = 3; Bw.rows = N; Bw.cols = p.Kp; Bw.ld = 3LL * p.Kp;
  GemmArgs g{};
  g.M = M; g.N = N; g.K = p.Kp; g.nseg = 1;
  lin_products(&g, p.nbx);
  g.ksplit = ks;
  g.D = out; g.ldd = N; g.mode = GEMM_STORE;
  return gemm_run(A, Bw, g, 1, gemm_pick_bn(N), part, st, &g_launches);
}

static int run_linear_backward(int M, int K, int N, const float* x, const float* W, const float* gout, int xb,
                               float* dx, float* dW, float* dbias, void* ws, size_t wsb, cudaStream_t st) {
  if (M <= 0 || K <= 0 || N <= 0 || !gout || (dx && !W) || ((dW || dbias) && !x)) return DELREC_ERR_ARG;
  if (((uintptr_t)ws & 255) != 0 || wsb < linear_bwd_ws(M, K, N, xb)) return DELREC_ERR_WORKSPACE;
  const LinPlan p = plan_linear(K, N, xb);
  Carve c(ws, wsb);
  __nv_bfloat16* X = c.take<__nv_bfloat16>((size_t)M * p.nbx * p.Kp);
  __nv_bfloat16* G = c.take<__nv_bfloat16>((size_t)M * 3 * p.Np);
  __nv_bfloat16* Wt = c.take<__nv_bfloat16>((size_t)3 * p.Np * p.Kp);
  float* D = c.take<float>((size_t)3 * p.Np * p.Kp);
  const int ksx = lin_ksplit(M, K, p.Np, 6);
  float* part = (float*)c.take<unsigned char>(std::max(gemm_partial_bytes(M, K, ksx, 1),
                                                       gemm1_part_bytes(3 * p.Np, p.Kp, M, kLinMaxSplit)));
  if (!c.ok) return DELREC_ERR_WORKSPACE;
  // G = [g0 g1 g2] per row (gb blocks): the three pieces of gout, each stored once
  const int gb = 3;
  k_pack_rows<<<grid_for((size_t)M * p.Np / 8, 256), 256, 0, st>>>(M, N, p.Np, gout, N, nullptr, 0, gb,
                                                                   kPatDistinct3, 0, G);
  DR_LAUNCHED();
  if (dx) {
    k_pack_wt<<<grid_for((size_t)p.Np * p.Kp / 8, 256), 256, 0, st>>>(N, K, p.Np, p.Kp, W, kPatDistinct3, 3, Wt);
    DR_LAUNCHED();
    // dx[m][k] = sum over the piece products of G_i[m][.] W_j[.][k]  (W pieces: rows along
    // the reduction, MN-major)
    GemmSide A{}, Bw{};
    for (int i = 0; i < 3; ++i) {
      A.p[i] = G + (size_t)i * p.Np;
      Bw.p[i] = Wt + (size_t)i * p.Np * p.Kp;
    }
    A.n = 3; A.rows = M; A.cols = p.Np; A.ld = 3LL * p.Np;
    Bw.n = 3; Bw.rows = p.Np; Bw.cols = K; Bw.ld = p.Kp; Bw.mn_major = 1;
    GemmArgs g{};
    g.M = M; g.N = K; g.K = p.Np; g.nseg = 1;
    lin_products(&g, 3);
    g.ksplit = ksx;
    g.D = dx; g.ldd = K; g.mode = GEMM_STORE;
    const int rc = gemm_run(A, Bw, g, 1, gemm_pick_bn(K), part, st, &g_launches);
    if (rc) return rc;
  }
  if (dW || dbias) {
    k_pack_rows<<<grid_for((size_t)M * p.Kp / 8, 256), 256, 0, st>>>(M, K, p.Kp, x, K, nullptr, 1, p.nbx,
                                                                     kPatDistinct3, xb, X);
    DR_LAUNCHED();
    // D[c][k'] (+)= sum_m G'[m][c] X_a[m][k'] over the M rows, c < (3-a) Np
    for (int a = 0; a < p.nbx; ++a) {
      const int rc = gemm1(mnmajor_operand(G, M, (long long)(3 - a) * p.Np, (long long)gb * p.Np),
                           mnmajor_operand(X + (size_t)a * p.Kp, M, p.Kp, (long long)p.nbx * p.Kp), (3 - a) * p.Np,
                           p.Kp, M, D, p.Kp, a == 0 ? GEMM_STORE : GEMM_ACCUM, part, kLinMaxSplit, st);
      if (rc) return rc;
    }
    k_linear_dw_reduce<<<grid_for((size_t)N * (K + 1), 256), 256, 0, st>>>(N, K, p.Np, p.Kp, D, dW, dbias);
    DR_LAUNCHED();
  }
  return DELREC_OK;
}

// Axonal layers too wide for the single-wave scans run step by step: per reverse step one
// LIF-backward kernel and one bf16 GEMM gz(t) = [hi hi lo](gr(t)) . [W_hi; W_lo; W_hi].
static bool plan_axstep(const delrec_layer* ly, const BwdPlan& bp, bool single_wave_ok) {
  // (the per-step GEMM's operands need 16-byte rows: N a multiple of 8)
  return ly->kind == DELREC_AXONAL && !single_wave_ok && ly->N > 512 && bp.MM == 0 && ly->N % 8 == 0;
}
static constexpr int kStepMaxSplit = 16;   // the per-step GEMM fills the GPU by splitting
static int axstep_ksplit(const delrec_layer* ly) {
  return gemm_pick_ksplit(ly->B, ly->N, 3 * ly->N, 1, 1, 1, gemm_pick_bn(ly->N), kStepMaxSplit, 4);
}
static size_t axstep_ws(const delrec_layer* ly) {
  const size_t N = ly->N, BN = (size_t)ly->B * N;
  Carve c(nullptr, (size_t)-1);
  c.take<float>(BN);                          // lam
  c.take<__nv_bfloat16>(3 * N * N);           // [W_hi; W_lo; W_hi]
  c.take<__nv_bfloat16>(3 * BN);              // [hi | hi | lo] of gr(t)
  c.take<unsigned char>(gemm_partial_bytes(ly->B, ly->N, axstep_ksplit(ly), 1));
  return c.off;
}
static int run_axstep(const delrec_layer* ly, const delrec_lif* lif, const float* gy, const float* u,
                      const float* keep, const float* W, const int* tl0, const int* tnt, const float* tw,
                      int TAPS, float* gz, float* gr, float* dx, Carve& c, cudaStream_t st) {
  const int N = ly->N, B = ly->B, T = ly->T;
  const size_t BN = (size_t)B * N, nn = (size_t)N * N;
  float* lam = c.take<float>(BN);
  __nv_bfloat16* Wp = c.take<__nv_bfloat16>(3 * nn);
  __nv_bfloat16* g3 = c.take<__nv_bfloat16>(3 * BN);
  float* part = (float*)c.take<unsigned char>(gemm_partial_bytes(B, N, axstep_ksplit(ly), 1));
  if (!c.ok) return DELREC_ERR_WORKSPACE;
  DR_CUDA(cudaMemsetAsync(lam, 0, BN * sizeof(float), st));
  k_split_bf16<<<grid_for(nn, 256), 256, 0, st>>>(W, nn, Wp, Wp + nn);
  DR_LAUNCHED();
  DR_CUDA(cudaMemcpyAsync(Wp + 2 * nn, Wp, nn * sizeof(__nv_bfloat16), cudaMemcpyDeviceToDevice, st));
  const LifK lk = make_lif(*lif);
  // gz(t)[b][o] = sum_c g3[b][c] Wp[c][o], c over the 3N piece rows (W rows: MN-major operand)
  const GemmSide A = kmajor_operand(g3, B, 3 * N, 3 * N);
  const GemmSide Wm = mnmajor_operand(Wp, 3 * N, N, N);
  GemmArgs g{};   // one product over K = 3N; the per-step output row block of gz
  g.M = B; g.N = N; g.K = 3 * N; g.nprod = 1; g.nseg = 1;
  const int BNt = gemm_pick_bn(N);
  g.ksplit = axstep_ksplit(ly);
  g.D = gz; g.ldd = N; g.mode = GEMM_STORE;
  GemmLaunch gl;
  int rc = gemm_prepare(A, Wm, g, 1, BNt, part, &gl);   // tensor maps encoded once
  if (rc) return rc;
  scan_mark(0, st);
  // every launch after the first is a programmatic dependent of the one before it
  for (int t = T - 1; t >= 0; --t) {
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(dim3(grid_for(BN, 256)), dim3(256), 0, st, t < T - 1, attr);
    DR_CUDA(cudaLaunchKernelEx(&cfg, k_step_lif_bwd, t, T, B, N, TAPS, gy, u, keep, tl0, tnt, tw, (const float*)gz,
                               lam, dx, gr, g3, lk));
    DR_LAUNCHED();
    rc = gemm_exec(gl, gz + (size_t)t * BN, st, &g_launches, true);
    if (rc) return rc;
  }
  scan_mark(1, st);
  return DELREC_OK;
}

// ---- chunked reverse scan (backward_chunk.cuh) ----------------------------------------
// 0: hybrid layers run the chunked scan where the shape allows it, its steps in the
// sample-local form; 1: every layer runs the step-by-step scans; 2: the chunked scan with
// the steps exchanging gr between blocks (delrec_set_reverse_scan).
static std::atomic<int> g_reverse_scan{0};

struct ChunkPlan {
  bool ok, exch;     // ok: the sample-local chunked scan applies; exch: so does its exchange form
  int KP1, ntiles, nchunks, Np, S;
  size_t smem;       // exchange form's step kernel
};
// Shape test only (the workspace query does not depend on the selected variant): a hybrid
// layer whose base taps are all at lag >= 1, offsets within two chunks (K + 1 <= 9), at
// most 8 taps per source, N <= 1024.  The exchange form also needs the 64-sample tiling.
// S: samples per step block, 1 while the batch fills at most one wave of blocks.
static ChunkPlan plan_chunk(const delrec_layer* ly, const BwdPlan& bp, const Hyb64Plan& h64) {
  ChunkPlan c{};
  c.ok = c.exch = false;
  if (ly->kind != DELREC_HYBRID || !bp.ok || bp.MM != 0 || ly->N > 1024) return c;
  c.KP1 = ly->K + 1;
  if (c.KP1 > kChunk + 1 || bp.TAPS > kH64Taps) return c;
  c.ntiles = cdiv(ly->N, gz_ntg(c.KP1));
  c.nchunks = cdiv(ly->T, kChunk);
  c.Np = pad8(ly->N);
  c.S = ly->B <= kSMs ? 1 : kLocSMax;
  if (loc_smem_plan(ly->N, bp.TAPS, c.S).fixed + 512 > kSmemLimit) return c;
  c.ok = true;
  if (h64.ok) {
    c.smem = hyb64_smem_plan(ly->N, h64.NT, h64.CAPS, h64.K, bp.TAPS, kChunk).total;
    c.exch = c.smem <= kSmemLimit;
  }
  return c;
}
static size_t chunk_ws(const delrec_layer* ly, const ChunkPlan& cp) {
  Carve c(nullptr, (size_t)-1);
  const size_t rows = (size_t)ly->B * ly->T;
  c.take<__nv_bfloat16>(rows * cp.Np);                       // gr pieces (B, T, Np)
  c.take<__nv_bfloat16>(rows * cp.Np);
  c.take<__nv_bfloat16>((size_t)cp.ntiles * kGzCols * cp.Np);   // masked W pieces
  c.take<__nv_bfloat16>((size_t)cp.ntiles * kGzCols * cp.Np);
  c.take<float>((size_t)ly->B * ly->N);                       // LIF carry between chunks
  c.take<uint16_t>((size_t)ly->N * plan_backward(ly, DELREC_HYBRID).CAP);   // short entries
  c.take<float>((size_t)ly->N * plan_backward(ly, DELREC_HYBRID).CAP);
  const int ecap = loc_entry_cap(kSmemLimit, loc_smem_plan(ly->N, plan_backward(ly, DELREC_HYBRID).TAPS, cp.S));
  c.take<uint16_t>((size_t)std::max(ecap, 8));                // compact cache
  c.take<float>((size_t)std::max(ecap, 8));
  c.take<int4>((size_t)ly->N * kChunk);                       // (source, bucket) pairs
  c.take<int>(16);                                            // pair counts, meta
  return c.off;
}

// (B, T, N) bf16 pieces read as boxes of 32 targets x 8 steps x 16 samples (64-byte swizzle)
static bool tmap_bf16_btn(CUtensorMap* m, const void* base, int N, int T, int B, int Np) {
  TmapEncodeFn fn = tmap_encoder();
  if (!fn || !base || ((uintptr_t)base & 15) || (Np % 8)) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[2] = {(cuuint64_t)Np * 2, (cuuint64_t)T * Np * 2};
  const cuuint32_t box[3] = {(cuuint32_t)kGzK, (cuuint32_t)kChunk, (cuuint32_t)kGzSamples};
  const cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A bf16 matrix of `rows` x `cols` (row stride ld elements) read as 32-column x box_rows
// boxes with the 64-byte swizzle (the chunk GEMM's B operand)
static bool tmap_bf16_k32(CUtensorMap* m, const void* base, long long cols, long long rows, long long ld,
                          int box_rows) {
  TmapEncodeFn fn = tmap_encoder();
  if (!fn || !base || cols < 1 || rows < 1 || box_rows < 8 || box_rows > 256 || ((uintptr_t)base & 15) ||
      ((ld * 2) & 15) || ld < cols)
    return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)kGzK, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KP1>
static int launch_gz_t(const CUtensorMap* m, const GzArgs& g, int ntiles, cudaStream_t st, bool pdl) {
  auto kern = k_chunk_gz<KP1>;
  int rc = set_smem(kern, kGzSmem);
  if (rc) return rc;
  GzArgs ga = g;
  ga.ntiles = ntiles;
  const int total = gz_items(cdiv(g.B, kGzSamples), ntiles, g.ncl);
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = pdl_config(dim3(std::min(total, kSMs)), dim3(kGzThreads), kGzSmem, st, pdl, attr);
  DR_CUDA(cudaLaunchKernelEx(&cfg, kern, m[0], m[1], m[2], m[3], m[4], m[5], ga));
  DR_LAUNCHED();
  return DELREC_OK;
}
static int launch_gz(int KP1, const CUtensorMap* m, const GzArgs& g, int ntiles, cudaStream_t st, bool pdl) {
  switch (KP1) {
    case 1: return launch_gz_t<1>(m, g, ntiles, st, pdl);
    case 2: return launch_gz_t<2>(m, g, ntiles, st, pdl);
    case 3: return launch_gz_t<3>(m, g, ntiles, st, pdl);
    case 4: return launch_gz_t<4>(m, g, ntiles, st, pdl);
    case 5: return launch_gz_t<5>(m, g, ntiles, st, pdl);
    case 6: return launch_gz_t<6>(m, g, ntiles, st, pdl);
    case 7: return launch_gz_t<7>(m, g, ntiles, st, pdl);
    case 8: return launch_gz_t<8>(m, g, ntiles, st, pdl);
    case 9: return launch_gz_t<9>(m, g, ntiles, st, pdl);
    default: return DELREC_ERR_UNSUPPORTED;
  }
}

// The chunked reverse scan of one layer: for each chunk of 8 steps, from the last, the
// SIMT steps (k_bwd_chunk) and the tensor-core delayed-gradient GEMM (k_chunk_gz).
// `base` carries the 64-sample scan's arguments (taps, buckets, exchange buffers).
static int run_chunked(const delrec_layer* ly, const Hyb64Plan& h64, const ChunkPlan& cp, const Hyb64Args& base,
                       const float* W, const uint8_t* offT, float* gz, Carve& c, cudaStream_t st) {
  const int N = ly->N, T = ly->T, B = ly->B, Np = cp.Np;
  const size_t rows = (size_t)B * T, wrows = (size_t)cp.ntiles * kGzCols;
  __nv_bfloat16* ga_hi = c.take<__nv_bfloat16>(rows * Np);
  __nv_bfloat16* ga_lo = c.take<__nv_bfloat16>(rows * Np);
  __nv_bfloat16* wm_hi = c.take<__nv_bfloat16>(wrows * Np);
  __nv_bfloat16* wm_lo = c.take<__nv_bfloat16>(wrows * Np);
  float* lam = c.take<float>((size_t)B * N);
  uint16_t* sh_idx = c.take<uint16_t>((size_t)N * base.CAP);
  float* sh_w = c.take<float>((size_t)N * base.CAP);
  const LocSmem lplan = loc_smem_plan(N, base.TAPS, cp.S);
  const size_t lsmem = kSmemLimit;   // the fixed part, the rest caches the short entries
  const int lecap = loc_entry_cap(lsmem, lplan);
  uint16_t* c_idx = c.take<uint16_t>((size_t)std::max(lecap, 8));
  float* c_w = c.take<float>((size_t)std::max(lecap, 8));
  int4* pairs = c.take<int4>((size_t)N * kChunk);
  int* pcnt = c.take<int>(16);
  if (!c.ok) return DELREC_ERR_WORKSPACE;
  k_mask_w<<<grid_for(wrows * Np, 256), 256, 0, st>>>(N, Np, cp.KP1, (int)wrows, W, offT, wm_hi, wm_lo);
  DR_LAUNCHED();
  DR_CUDA(cudaMemsetAsync(gz, 0, (size_t)T * B * N * sizeof(float), st));
  // the last column tile's sources, and its MMA width (used columns rounded up to 16)
  const int ncl = std::min(kGzCols, ((N - (cp.ntiles - 1) * gz_ntg(cp.KP1)) * cp.KP1 + 15) & ~15);
  CUtensorMap maps[6];
  if (!tmap_bf16_btn(&maps[0], ga_hi, N, T, B, Np) || !tmap_bf16_btn(&maps[1], ga_lo, N, T, B, Np) ||
      !tmap_bf16_k32(&maps[2], wm_hi, N, (long long)wrows, Np, kGzCols) ||
      !tmap_bf16_k32(&maps[3], wm_lo, N, (long long)wrows, Np, kGzCols) ||
      !tmap_bf16_k32(&maps[4], wm_hi, N, (long long)wrows, Np, ncl) ||
      !tmap_bf16_k32(&maps[5], wm_lo, N, (long long)wrows, Np, ncl))
    return DELREC_ERR_ARG;
  // steps: the sample-local kernel (no exchange) unless the exchange form is selected
  const bool local = g_reverse_scan.load() != 2 || !cp.exch;
  // one (sample, source) pair per thread where it fits in a block of 1024, else 512 threads
  const int S = cp.S;
  const int lnth = S * N <= 1024 ? 1024 : kLocThreads;
  const int lppt = cdiv(S * N, lnth);
  auto kern = k_bwd_chunk<kH64Taps>;
  // taps per source: the integer lags inside one triangle, at most 2*ceil(s_max) + 1
  const bool tap4 = 2 * (int)ceilf(ly->s_max) + 1 <= 4;
  auto lkern = S == 1 ? (lnth == 1024 ? (tap4 ? k_bwd_chunk_local<4, 1, 1024, 1> : k_bwd_chunk_local<kH64Taps, 1, 1024, 1>)
                                       : k_bwd_chunk_local<kH64Taps, 2, kLocThreads, 1>)
                      : (lnth == 1024 ? (tap4 ? k_bwd_chunk_local<4, 1, 1024, 2> : k_bwd_chunk_local<kH64Taps, 1, 1024, 2>)
                                      : (lppt <= 2 ? k_bwd_chunk_local<kH64Taps, 2, kLocThreads, 2>
                                                   : k_bwd_chunk_local<kH64Taps, 4, kLocThreads, 2>));
  int rc = DELREC_OK;
  if (local) {
    if (lppt > 4 || lplan.fixed + 512 > lsmem) return DELREC_ERR_UNSUPPORTED;
    rc = set_smem(lkern, lsmem);
    if (rc) return rc;
    k_short_entries<<<N, 64, 0, st>>>(N, ly->K, base.CAP, base.boff_stride, base.ent, base.boff, base.tap_l0, sh_idx,
                                      sh_w);
    DR_LAUNCHED();
    k_short_pairs<<<1, kLocThreads, 0, st>>>(N, ly->K, base.CAP, base.boff_stride, base.boff, base.tap_l0, sh_idx, sh_w,
                                             lecap, c_idx, c_w, pairs, pcnt, pcnt + 8);
    DR_LAUNCHED();
  } else {
    rc = set_smem(kern, cp.smem);
    if (rc) return rc;
    int per_sm = 0;
    DR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kH64Threads, cp.smem));
    if (per_sm < 1 || h64.CS * h64.tiles > per_sm * kSMs) return DELREC_ERR_UNSUPPORTED;
  }
  ChunkArgs a{};
  a.T = T; a.B = B; a.N = N; a.K = ly->K; a.CS = h64.CS; a.NT = h64.NT; a.TAPS = base.TAPS;
  a.CAPS = h64.CAPS; a.CAP = base.CAP; a.boff_stride = base.boff_stride;
  a.gy = base.gy; a.u = base.u; a.keep = base.keep;
  a.tap_l0 = base.tap_l0; a.tap_nt = base.tap_nt; a.tap_w = base.tap_w; a.ent = base.ent; a.boff = base.boff;
  a.dx = base.dx; a.gr = base.gr; a.gz = gz; a.ga_hi = ga_hi; a.ga_lo = ga_lo; a.Np = Np; a.lam = lam;
  a.lif = base.lif; a.grx = base.grx; a.arrive = base.arrive; a.spin_limit = base.spin_limit;
  GzArgs g{};
  g.T = T; g.B = B; g.N = N; g.ncl = ncl; g.gz = gz; g.spin_ns = 2000000000ll;
  if (!local) DR_CUDA(cudaMemsetAsync(a.arrive, 0, sizeof(unsigned int) * h64.tiles, st));
  scan_mark(0, st);
  for (int ch = cp.nchunks - 1; ch >= 0; --ch) {
    a.t0 = ch * kChunk;
    a.t_hi = std::min(T - 1, a.t0 + kChunk - 1);
    a.arr_base = (unsigned int)((T - 1 - a.t_hi) * h64.CS);
    scan_mark(0, st, 1);
    if (local) {
      LocArgs la{a, sh_idx, sh_w, c_idx, c_w, pairs, pcnt, pcnt + 8, lecap};
      // the first chunk follows the kernels that build its tables: an ordinary launch
      cudaLaunchAttribute attr[1];
      const cudaLaunchConfig_t cfg =
          pdl_config(dim3(cdiv(B, S)), dim3(lnth), lsmem, st, ch < cp.nchunks - 1 && !g_scan_timing, attr);
      DR_CUDA(cudaLaunchKernelEx(&cfg, lkern, la));
    } else {
      ChunkArgs ac = a;
      void* args[] = {(void*)&ac};
      DR_CUDA(cudaLaunchCooperativeKernel((const void*)kern, dim3(h64.CS * h64.tiles), dim3(kH64Threads), args,
                                          cp.smem, st));
    }
    scan_mark(1, st, 1);
    ++g_launches;
    g.t0 = a.t0;
    scan_mark(0, st, 2);
    rc = launch_gz(cp.KP1, maps, g, cp.ntiles, st, local && !g_scan_timing);
    scan_mark(1, st, 2);
    if (rc) return rc;
  }
  scan_mark(1, st);
  return DELREC_OK;
}

// Hard-tap forms of the axonal backward (AxonalRecdelTriton with ste_mode / approx,
// recdel_base.py:350-445).  dw_d: the weight gradient correlates gr with the z of the
// triangle (dw_d, half-width 1) -- the hard forward's taps -- instead of the soft one;
// st_dd: dd straight-through from the single tap at l = 1 + d.
struct HardBwd {
  const float* dw_d;
  int st_dd;
};

static size_t backward_ws(const delrec_layer* ly, int kind, bool hard = false) {
  const BwdPlan bp = plan_backward(ly, kind);
  const SrcPlan sp = plan_src(ly);
  const size_t N = ly->N, TBN = (size_t)ly->T * ly->B * N;
  Carve c(nullptr, (size_t)-1);
  c.take<float>(TBN);                                  // gr
  if (kind != DELREC_SYNAPTIC) {
    c.take<float>(TBN * (bp.MM + 1));                  // gz_m
    c.take<int>(N); c.take<int>(N); c.take<float>(N * bp.TAPS);
  }
  if (kind == DELREC_HYBRID) c.take<uint8_t>(N * N);   // offT
  if (kind == DELREC_SYNAPTIC) c.take<float>(N * N);   // dT
  if (kind != DELREC_AXONAL) {
    c.take<int2>(N * (size_t)bp.CAP);
    c.take<int>(N * (size_t)(bp.NKEY + 1));
  }
  if (kind == DELREC_HYBRID) {
    c.take<float>((size_t)2 * cdiv(ly->B, 64) * N * 64);   // gr exchange (cooperative modes)
    c.take<unsigned int>((size_t)cdiv(ly->B, 32));         // arrival counters
  }
  if (kind == DELREC_SYNAPTIC) {
    const Hyb64Plan s64 = plan_syn64(ly);
    if (s64.ok) {
      c.take<int>(N); c.take<int>(N); c.take<float>(N);   // unit taps
      c.take<float>((size_t)2 * s64.tiles * N * 64);
      c.take<unsigned int>((size_t)s64.tiles);
    }
  }
  if (plan_axstep(ly, bp, plan_axmma(ly, bp).ok || plan_hybrid64(ly, bp).ok)) c.take<unsigned char>(axstep_ws(ly));
  if (kind == DELREC_HYBRID) {
    const ChunkPlan cp = plan_chunk(ly, bp, plan_hybrid64(ly, bp));
    if (cp.ok) c.take<unsigned char>(chunk_ws(ly, cp));
  }
  if (kind == DELREC_AXONAL && plan_axmma(ly, bp).ok) {
    const AxMmaPlan am = plan_axmma(ly, bp);
    c.take<float>((size_t)2 * am.tiles * N * 64);
    c.take<unsigned int>((size_t)am.tiles);
  } else if (kind == DELREC_AXONAL) {
    const Hyb64Plan h64 = plan_hybrid64(ly, bp);
    if (h64.ok) {
      c.take<uint8_t>(N * N);                              // zero offsets
      c.take<int2>(N * (size_t)h64.CAP);
      c.take<int>(N * (size_t)(h64.NKEY + 1));
      c.take<float>((size_t)2 * h64.tiles * N * 64);
      c.take<unsigned int>((size_t)h64.tiles);
    }
  }
  if (kind == DELREC_SYNAPTIC) c.take<unsigned char>(dense_dw_ws(ly, 1, ly->L));   // lag correlation stack
  if (kind != DELREC_SYNAPTIC) {
    const size_t dws = dense_dw_ws(ly, bp.MM + 1, kind == DELREC_HYBRID ? ly->K + 1 : 1);
    c.take<unsigned char>(dws);
  }
  if (kind == DELREC_SYNAPTIC) c.take<float>(N * N);   // ds per pair, summed
  c.take<float>((size_t)sp.splits * N * (bp.TAPS + 1)); // source partials
  if (hard) {                                          // the hard taps and their pass
    c.take<int>(N); c.take<int>(N); c.take<float>(N * bp.TAPS); c.take<float>(N);
    c.take<float>((size_t)sp.splits * N * (bp.TAPS + 1));
  }
  return c.off;
}

static int run_backward(const delrec_layer* ly, int kind, const delrec_lif* lif, const float* gy,
                        const float* u, const float* y, const float* W, const float* d,
                        const float* offsets, const float* s, const float* keep,
                        const delrec_grads* g, void* ws, size_t wsb, cudaStream_t st,
                        const HardBwd* hb = nullptr) {
  int rc = check_layer(ly, kind);
  if (rc) return rc;
  if (!lif || !gy || !u || !y || !W || !d || !s || !g || !g->dx) return DELREC_ERR_ARG;
  if (kind == DELREC_HYBRID && !offsets) return DELREC_ERR_ARG;
  if (ly->has_keep && !keep) return DELREC_ERR_ARG;
  if (((uintptr_t)ws & 255) != 0) return DELREC_ERR_WORKSPACE;
  if (hb && (kind != DELREC_AXONAL || (hb->st_dd && g->ds))) return DELREC_ERR_ARG;
  if (wsb < backward_ws(ly, kind, hb != nullptr)) return DELREC_ERR_WORKSPACE;
  const BwdPlan bp = plan_backward(ly, kind);
  if (!bp.ok || bp.MM > kMMMax) return DELREC_ERR_UNSUPPORTED;
  // k_source_pass keeps each neuron's spike history in 128 bits
  if (kind != DELREC_SYNAPTIC && ly->L - 1 + bp.MM > 127) return DELREC_ERR_UNSUPPORTED;
  const int N = ly->N, T = ly->T, B = ly->B;
  const size_t TBN = (size_t)T * B * N;
  Carve c(ws, wsb);
  float* gr = c.take<float>(TBN);
  // without dropout gr = du * 1 = dx: the scans' gr is dx itself (one array written once)
  if (!ly->has_keep) gr = g->dx;
  float *gz = nullptr, *tw = nullptr;
  int *tl0 = nullptr, *tnt = nullptr;
  if (kind != DELREC_SYNAPTIC) {
    gz = c.take<float>(TBN * (bp.MM + 1));
    tl0 = c.take<int>(N);
    tnt = c.take<int>(N);
    tw = c.take<float>((size_t)N * bp.TAPS);
    const int lmin = kind == DELREC_HYBRID ? 1 - ly->K : 1;
    k_taps<<<cdiv(N, 256), 256, 0, st>>>(d, s, N, ly->L - 1, bp.TAPS, lmin, tl0, tnt, tw);
    DR_LAUNCHED();
  }
  dim3 tb(32, 8), tg(cdiv(N, 32), cdiv(N, 32));
  uint8_t* offT = nullptr;
  float* dT = nullptr;
  if (kind == DELREC_HYBRID) {
    offT = c.take<uint8_t>((size_t)N * N);
    k_offsets_u8T<<<tg, tb, 0, st>>>(offsets, offT, N, ly->K);
    DR_LAUNCHED();
  }
  if (kind == DELREC_SYNAPTIC) {
    dT = c.take<float>((size_t)N * N);
    k_transpose<<<tg, tb, 0, st>>>(d, dT, N, N);
    DR_LAUNCHED();
  }
  int2* ent = nullptr;
  int* boff = nullptr;
  const HybPlan hp = plan_hybrid_fast(ly, bp);
  const AxMmaPlan am = plan_axmma(ly, bp);
  Hyb64Plan h64 = plan_hybrid64(ly, bp);
  if (am.ok) h64.ok = false;   // the tensor-core scan takes the axonal layer
  const bool axstep = plan_axstep(ly, bp, am.ok || h64.ok);
  const Hyb64Plan s64 = plan_syn64(ly);
  if (kind == DELREC_AXONAL && h64.ok) {
    // offsets all 0: one bucket per source with all its synapses
    offT = c.take<uint8_t>((size_t)N * N);
    DR_CUDA(cudaMemsetAsync(offT, 0, (size_t)N * N, st));
    ent = c.take<int2>((size_t)N * h64.CAP);
    boff = c.take<int>((size_t)N * (h64.NKEY + 1));
    const int nth = std::min(256, ((N + 31) / 32) * 32);
    k_buckets<1><<<N, nth, (size_t)nth * 8, st>>>(N, h64.NKEY, h64.CAP, 8, W, offT, nullptr, s, ent, boff);
    DR_LAUNCHED();
  }
  if (kind != DELREC_AXONAL) {
    ent = c.take<int2>((size_t)N * bp.CAP);
    boff = c.take<int>((size_t)N * (bp.NKEY + 1));
    const int nth = std::min(256, ((N + 31) / 32) * 32);
    const size_t sm = (size_t)nth * 8;
    const int padm = (hp.ok || h64.ok || s64.ok) ? 8 : bp.PADM;
    if (kind == DELREC_HYBRID)
      k_buckets<1><<<N, nth, sm, st>>>(N, bp.NKEY, bp.CAP, padm, W, offT, nullptr, s, ent, boff);
    else
      k_buckets<2><<<N, nth, sm, st>>>(N, bp.NKEY, bp.CAP, padm, W, nullptr, dT, s, ent, boff);
    DR_LAUNCHED();
  }
  // ---- reverse scan
  BwdArgs a{};
  a.T = T; a.B = B; a.N = N; a.L = ly->L; a.KH = bp.KH; a.CS = bp.CS; a.NT = bp.NT;
  a.TAPS = bp.TAPS; a.NKEY = bp.NKEY; a.CAP = bp.CAP; a.KS = bp.KS; a.MM = bp.MM;
  a.gy = gy; a.u = u; a.keep = ly->has_keep ? keep : nullptr; a.W = W;
  a.tap_l0 = tl0; a.tap_nt = tnt; a.tap_w = tw; a.ent = ent; a.boff = boff;
  a.dx = g->dx; a.gr = gr; a.gz = gz; a.w_smem = bp.w_smem; a.lif = make_lif(*lif);
  float* grx = nullptr;
  unsigned int* arrive = nullptr;
  if (kind == DELREC_HYBRID) {
    grx = c.take<float>((size_t)2 * cdiv(B, 64) * N * 64);
    arrive = c.take<unsigned int>((size_t)cdiv(B, 32));
  } else if (kind == DELREC_AXONAL && h64.ok) {
    grx = c.take<float>((size_t)2 * h64.tiles * N * 64);
    arrive = c.take<unsigned int>((size_t)h64.tiles);
  } else if (kind == DELREC_SYNAPTIC && s64.ok) {
    grx = c.take<float>((size_t)2 * s64.tiles * N * 64);
    arrive = c.take<unsigned int>((size_t)s64.tiles);
  } else if (am.ok) {
    grx = c.take<float>((size_t)2 * am.tiles * N * 64);
    arrive = c.take<unsigned int>((size_t)am.tiles);
  }
  if (axstep) {
    const size_t sws = axstep_ws(ly);
    unsigned char* region = c.take<unsigned char>(sws);
    Carve sc(region, sws);
    rc = run_axstep(ly, lif, gy, u, ly->has_keep ? keep : nullptr, W, tl0, tnt, tw, bp.TAPS, gz, gr, g->dx, sc, st);
  } else if (am.ok) {
    AxMmaArgs h{};
    h.T = T; h.B = B; h.N = N; h.CS = am.CS; h.TAPS = bp.TAPS;
    h.gy = gy; h.u = u; h.keep = ly->has_keep ? keep : nullptr; h.W = W;
    h.tap_l0 = tl0; h.tap_nt = tnt; h.tap_w = tw;
    h.dx = g->dx; h.gr = gr; h.gz = gz; h.lif = a.lif;
    h.grx = grx; h.arrive = arrive; h.spin_limit = 1ll << 22;
    rc = launch_axmma(h, am, st);
  } else if (kind == DELREC_SYNAPTIC && s64.ok) {
    int* ul0 = c.take<int>(N);
    int* unt = c.take<int>(N);
    float* uw = c.take<float>(N);
    k_unit_taps<<<cdiv(N, 256), 256, 0, st>>>(N, ul0, unt, uw);
    DR_LAUNCHED();
    Hyb64Args h{};
    h.T = T; h.B = B; h.N = N; h.K = s64.K; h.CS = s64.CS; h.NT = s64.NT; h.TAPS = 1; h.CAPS = s64.CAPS;
    h.CAP = bp.CAP;
    h.gy = gy; h.u = u; h.keep = ly->has_keep ? keep : nullptr;
    h.tap_l0 = ul0; h.tap_nt = unt; h.tap_w = uw;
    h.ent = ent; h.boff = boff + 1; h.boff_stride = bp.NKEY + 1;   // key 0 (lag 0) is empty
    h.dx = g->dx; h.gr = gr; h.gz = nullptr; h.lif = a.lif;
    h.grx = grx; h.arrive = arrive; h.spin_limit = 1ll << 22;
    rc = launch_hyb64_t<kSynKmax>(h, s64, st);
  } else if (h64.ok || (kind == DELREC_HYBRID && plan_chunk(ly, bp, h64).ok && g_reverse_scan.load() != 1)) {
    const ChunkPlan cp = plan_chunk(ly, bp, h64);
    Hyb64Args h{};
    h.T = T; h.B = B; h.N = N; h.K = ly->K; h.CS = h64.CS; h.NT = h64.NT; h.TAPS = bp.TAPS; h.CAPS = h64.CAPS;
    h.CAP = bp.CAP; h.boff_stride = ly->K + 2;
    h.gy = gy; h.u = u; h.keep = ly->has_keep ? keep : nullptr;
    h.tap_l0 = tl0; h.tap_nt = tnt; h.tap_w = tw; h.ent = ent; h.boff = boff;
    h.dx = g->dx; h.gr = gr; h.gz = gz; h.lif = a.lif;
    h.grx = grx; h.arrive = arrive; h.spin_limit = 1ll << 22;
    if (cp.ok && g_reverse_scan.load() == 0) {
      const size_t cws = chunk_ws(ly, cp);
      unsigned char* region = c.take<unsigned char>(cws);
      Carve cc(region, cws);
      rc = c.ok ? run_chunked(ly, h64, cp, h, W, offT, gz, cc, st) : DELREC_ERR_WORKSPACE;
    } else {
      rc = h64.KMAX == 6 ? launch_hyb64_t<6>(h, h64, st) : launch_hyb64_t<10>(h, h64, st);
    }
  } else if (hp.ok) {
    HybArgs h{};
    h.grx = grx; h.arrive = arrive; h.spin_limit = 1ll << 22;
    h.T = T; h.B = B; h.N = N; h.K = ly->K; h.CS = hp.CS; h.NT = hp.NT; h.TAPS = bp.TAPS; h.MM = bp.MM;
    h.CAPS = hp.CAPS; h.gy = gy; h.u = u; h.keep = ly->has_keep ? keep : nullptr;
    h.tap_l0 = tl0; h.tap_nt = tnt; h.tap_w = tw; h.ent = ent; h.boff = boff; h.CAP = bp.CAP;
    h.dx = g->dx; h.gr = gr; h.gz = gz; h.lif = a.lif;
    if (hp.KMAX == 5) rc = launch_hyb_t<5>(h, hp, st);
    else rc = launch_hyb_t<9>(h, hp, st);
  } else if (bp.mode == 0) rc = launch_bwd_mode<0>(a, bp, st);
  else if (bp.mode == 1) rc = launch_bwd_mode<1>(a, bp, st);
  else rc = launch_bwd_mode<2>(a, bp, st);
  if (rc) return rc;
  // ---- parameter gradients
  float* dsm = kind == DELREC_SYNAPTIC ? c.take<float>((size_t)N * N) : nullptr;
  const SrcPlan sp = plan_src(ly);
  float* spart = c.take<float>((size_t)sp.splits * N * (bp.TAPS + 1));
  // per-neuron sums: db (all kinds), dd/ds of the axonal / hybrid base
  const bool need_src = g->dbias || (kind != DELREC_SYNAPTIC && (g->dd || g->ds));
  SrcArgs sa{};
  sa.T = T; sa.B = B; sa.N = N; sa.TAPS = bp.TAPS;
  sa.gr = gr; sa.gz = kind != DELREC_SYNAPTIC ? gz : nullptr; sa.y = y; sa.tap_l0 = tl0; sa.tap_nt = tnt;
  sa.tap_w = tw; sa.part = spart; sa.MM = bp.MM; sa.Np = pad8(N);
  const dim3 sgrid(cdiv(N, 32), cdiv(B, 8), sp.tsplit);
  if (kind != DELREC_SYNAPTIC) {
    // one pass over (gr, y, gz at spikes) -> db/dmask partials and the bf16 z pieces of
    // the tensor-core dW (K+1 shifted GEMMs and a per-synapse pick)
    const int nz = bp.MM + 1, nk = kind == DELREC_HYBRID ? ly->K + 1 : 1;
    DenseBufs dbf{};
    if (g->dW) {
      const size_t dws = dense_dw_ws(ly, nz, nk);
      unsigned char* region = c.take<unsigned char>(dws);
      Carve dc(region, dws);
      if (!dense_carve(ly, nz, nk, dc, &dbf)) return DELREC_ERR_WORKSPACE;
      // the source pass writes columns < N of the z pieces; the row padding stays zero
      if (pad8(N) != N)
        DR_CUDA(cudaMemsetAsync(dbf.z16, 0, (size_t)T * B * pad8(N) * 2 * nz * sizeof(__nv_bfloat16), st));
    }
    const int warm = ly->L - 1 + bp.MM;
    auto src_pass = [&](const SrcArgs& a_, int wz) {
      if (bp.MM == 0) {
        if (bp.TAPS <= 4) k_source_pass<4, 0><<<sgrid, 256, 0, st>>>(a_, wz, warm, dbf.z16);
        else if (bp.TAPS <= 8) k_source_pass<8, 0><<<sgrid, 256, 0, st>>>(a_, wz, warm, dbf.z16);
        else k_source_pass<16, 0><<<sgrid, 256, 0, st>>>(a_, wz, warm, dbf.z16);
      } else {
        if (bp.TAPS <= 4) k_source_pass<4, 3><<<sgrid, 256, 0, st>>>(a_, wz, warm, dbf.z16);
        else if (bp.TAPS <= 8) k_source_pass<8, 3><<<sgrid, 256, 0, st>>>(a_, wz, warm, dbf.z16);
        else k_source_pass<16, 3><<<sgrid, 256, 0, st>>>(a_, wz, warm, dbf.z16);
      }
    };
    // hard-tap weight gradient: the soft pass gives the sums, a second pass over the
    // hard taps writes the z pieces (its partial sums are not used)
    const bool hard_dw = hb && hb->dw_d && g->dW;
    if (need_src || (g->dW && !hard_dw)) {
      src_pass(sa, g->dW && !hard_dw ? 1 : 0);
      DR_LAUNCHED();
    }
    if (hard_dw) {
      int* hl0 = c.take<int>(N);
      int* hnt = c.take<int>(N);
      float* hw = c.take<float>((size_t)N * bp.TAPS);
      float* ones = c.take<float>(N);
      float* hpart = c.take<float>((size_t)sp.splits * N * (bp.TAPS + 1));
      if (!c.ok) return DELREC_ERR_WORKSPACE;
      k_fill_f32<<<cdiv(N, 256), 256, 0, st>>>(ones, N, 1.f);
      DR_LAUNCHED();
      k_taps<<<cdiv(N, 256), 256, 0, st>>>(hb->dw_d, ones, N, ly->L - 1, bp.TAPS, 1, hl0, hnt, hw);
      DR_LAUNCHED();
      SrcArgs sh = sa;
      sh.tap_l0 = hl0; sh.tap_nt = hnt; sh.tap_w = hw; sh.part = hpart;
      src_pass(sh, 1);
      DR_LAUNCHED();
    }
    if (g->dW) {
      rc = dense_dw(ly, gr, nz, nk, offT, g->dW, dbf, st);
      if (rc) return rc;
    }
  } else {
    if (g->dW || g->dd || g->ds) {
      // synaptic: the per-lag correlation stack on the tensor cores, then per synapse the
      // triangle-weighted sums over its lag window: dW, dd, ds
      const int nk = ly->L;
      const size_t dws = dense_dw_ws(ly, 1, nk);
      unsigned char* region = c.take<unsigned char>(dws);
      Carve dc(region, dws);
      DenseBufs dbf{};
      if (!c.ok || !dense_carve(ly, 1, nk, dc, &dbf)) return DELREC_ERR_WORKSPACE;
      rc = syn_cstack(ly, gr, y, dbf, st);
      if (rc) return rc;
      const size_t nn = (size_t)N * N;
      float* dsmo = g->ds ? dsm : nullptr;
      const int tw = syn_window(ly);
      if (tw == 4)
        k_syn_cstack_combine<4><<<grid_for(nn, 256), 256, 0, st>>>(N, ly->L - 1, dT, s, W, dbf.P, g->dW, g->dd, dsmo);
      else if (tw == 8)
        k_syn_cstack_combine<8><<<grid_for(nn, 256), 256, 0, st>>>(N, ly->L - 1, dT, s, W, dbf.P, g->dW, g->dd, dsmo);
      else
        k_syn_cstack_combine<16><<<grid_for(nn, 256), 256, 0, st>>>(N, ly->L - 1, dT, s, W, dbf.P, g->dW, g->dd, dsmo);
      DR_LAUNCHED();
      if (g->ds) {
        k_colsum<<<cdiv(N, 128), 128, 0, st>>>(dsm, N, N, g->ds);
        DR_LAUNCHED();
      }
    }
    if (need_src) {
      if (bp.TAPS <= 4) k_source_reduce<4><<<sgrid, 256, 0, st>>>(sa);
      else if (bp.TAPS <= 8) k_source_reduce<8><<<sgrid, 256, 0, st>>>(sa);
      else k_source_reduce<16><<<sgrid, 256, 0, st>>>(sa);
      DR_LAUNCHED();
    }
  }
  if (need_src) {
    const bool src_dd = kind != DELREC_SYNAPTIC;
    k_source_finalize<<<cdiv(N, 128), 128, 0, st>>>(N, bp.TAPS, sp.splits, spart, d, s, tl0, tnt,
                                                     g->dbias, src_dd ? g->dd : nullptr,
                                                     src_dd ? g->ds : nullptr, hb ? hb->st_dd : 0);
    DR_LAUNCHED();
  }
  return DELREC_OK;
}

}  // namespace delrec

using namespace delrec;

extern "C" {

const char* delrec_version(void) { return "delrec_b200 0.1 (sm_100a)"; }

unsigned long long delrec_launch_count(void) { return g_launches; }

int delrec_scan_timing(int enable) {
  g_scan_timing = enable != 0;
  for (int p = 0; p < kTimeParts; ++p) g_ev_n[p] = 0;
  return DELREC_OK;
}
int delrec_scan_time_part(int part, double* total_ms, int* launches) {
  if (!total_ms || !launches || part < 0 || part >= kTimeParts) return DELREC_ERR_ARG;
  double sum = 0.0;
  for (int i = 0; i < g_ev_n[part]; ++i) {
    DR_CUDA(cudaEventSynchronize(g_ev[part][i][1]));
    float ms = 0.f;
    DR_CUDA(cudaEventElapsedTime(&ms, g_ev[part][i][0], g_ev[part][i][1]));
    sum += ms;
  }
  *total_ms = sum;
  *launches = g_ev_n[part];
  g_ev_n[part] = 0;
  return DELREC_OK;
}
int delrec_scan_time(double* total_ms, int* launches) { return delrec_scan_time_part(0, total_ms, launches); }

// The reverse scans' exchange alone (k_exchange_floor) on the tiling the 64-sample scans
// use for this layer: a measurement of the per-step latency floor.
static int floor_plan(const delrec_layer* ly, Hyb64Plan* h) {
  if (!ly || ly->T < 1 || ly->B < 1 || ly->N < 1) return DELREC_ERR_ARG;
  delrec_layer l = *ly;
  l.kind = DELREC_HYBRID;
  if (l.K < 0) l.K = 0;
  const BwdPlan bp = plan_backward(&l, DELREC_HYBRID);
  *h = plan_hybrid64(&l, bp);
  return h->ok ? DELREC_OK : DELREC_ERR_UNSUPPORTED;
}
size_t delrec_exchange_floor_workspace(const delrec_layer* ly) {
  Hyb64Plan h{};
  if (floor_plan(ly, &h)) return 0;
  Carve c(nullptr, (size_t)-1);
  c.take<float>((size_t)2 * h.tiles * ly->N * kH64BT);
  c.take<unsigned int>((size_t)h.tiles);
  return c.off;
}
int delrec_exchange_floor(const delrec_layer* ly, void* ws, size_t wsb, void* stream) {
  Hyb64Plan h{};
  int rc = floor_plan(ly, &h);
  if (rc) return rc;
  if (((uintptr_t)ws & 255) != 0 || wsb < delrec_exchange_floor_workspace(ly)) return DELREC_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  Carve c(ws, wsb);
  float* grx = c.take<float>((size_t)2 * h.tiles * ly->N * kH64BT);
  unsigned int* arrive = c.take<unsigned int>((size_t)h.tiles);
  if (!c.ok) return DELREC_ERR_WORKSPACE;
  rc = set_smem(k_exchange_floor, h.smem);
  if (rc) return rc;
  int per_sm = 0;
  DR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_exchange_floor, kH64Threads, h.smem));
  if (per_sm < 1 || h.CS * h.tiles > per_sm * kSMs) return DELREC_ERR_UNSUPPORTED;
  DR_CUDA(cudaMemsetAsync(arrive, 0, sizeof(unsigned int) * h.tiles, st));
  int T = ly->T, N = ly->N, CS = h.CS, NT = h.NT;
  long long spin = 1ll << 22;
  void* args[] = {(void*)&T, (void*)&N, (void*)&CS, (void*)&NT, (void*)&grx, (void*)&arrive, (void*)&spin};
  DR_CUDA(cudaLaunchCooperativeKernel((const void*)k_exchange_floor, dim3(h.CS * h.tiles), dim3(kH64Threads), args,
                                      h.smem, st));
  ++g_launches;
  return DELREC_OK;
}

int delrec_set_reverse_scan(int variant) {
  if (variant < 0 || variant > 2) return DELREC_ERR_ARG;
  g_reverse_scan.store(variant);
  return DELREC_OK;
}

int delrec_get_status(int* out) {
  if (!out) return DELREC_ERR_ARG;
  DR_CUDA(cudaDeviceSynchronize());
  DR_CUDA(cudaMemcpyFromSymbol(out, g_status, sizeof(int)));
  return DELREC_OK;
}
int delrec_clear_status(void) {
  const int z = 0;
  DR_CUDA(cudaMemcpyToSymbol(g_status, &z, sizeof(int)));
  return DELREC_OK;
}

int delrec_build_mask(int R, int L, const float* d, const float* s, int s_period, float* out, void* stream) {
  if (R < 1 || L < 1 || s_period < 1 || !d || !s || !out) return DELREC_ERR_ARG;
  k_build_mask<<<grid_for((size_t)R * L, 256), 256, 0, (cudaStream_t)stream>>>(R, L, d, s, s_period, out);
  DR_LAUNCHED();
  return DELREC_OK;
}

size_t delrec_axonal_forward_workspace(const delrec_layer* ly) { return ly ? forward_ws(ly, DELREC_AXONAL) : 0; }
size_t delrec_synaptic_forward_workspace(const delrec_layer* ly) { return ly ? forward_ws(ly, DELREC_SYNAPTIC) : 0; }
size_t delrec_hybrid_forward_workspace(const delrec_layer* ly) { return ly ? forward_ws(ly, DELREC_HYBRID) : 0; }
size_t delrec_axonal_backward_workspace(const delrec_layer* ly) { return ly ? backward_ws(ly, DELREC_AXONAL) : 0; }
size_t delrec_synaptic_backward_workspace(const delrec_layer* ly) { return ly ? backward_ws(ly, DELREC_SYNAPTIC) : 0; }
size_t delrec_hybrid_backward_workspace(const delrec_layer* ly) { return ly ? backward_ws(ly, DELREC_HYBRID) : 0; }

int delrec_axonal_forward(const delrec_layer* ly, const delrec_lif* lif, const float* x, const float* W,
                          const float* bias, const float* d, const float* s, const float* keep, float* y,
                          float* u, void* ws, size_t wsb, void* stream) {
  return run_forward(ly, DELREC_AXONAL, lif, x, W, bias, d, nullptr, s, keep, y, u, ws, wsb, (cudaStream_t)stream);
}
int delrec_synaptic_forward(const delrec_layer* ly, const delrec_lif* lif, const float* x, const float* W,
                            const float* bias, const float* d, const float* s, const float* keep, float* y,
                            float* u, void* ws, size_t wsb, void* stream) {
  return run_forward(ly, DELREC_SYNAPTIC, lif, x, W, bias, d, nullptr, s, keep, y, u, ws, wsb, (cudaStream_t)stream);
}
int delrec_hybrid_forward(const delrec_layer* ly, const delrec_lif* lif, const float* x, const float* W,
                          const float* bias, const float* base, const float* offsets, const float* s,
                          const float* keep, float* y, float* u, void* ws, size_t wsb, void* stream) {
  return run_forward(ly, DELREC_HYBRID, lif, x, W, bias, base, offsets, s, keep, y, u, ws, wsb, (cudaStream_t)stream);
}

int delrec_axonal_backward(const delrec_layer* ly, const delrec_lif* lif, const float* gy, const float* u,
                           const float* y, const float* W, const float* d, const float* s, const float* keep,
                           const delrec_grads* g, void* ws, size_t wsb, void* stream) {
  return run_backward(ly, DELREC_AXONAL, lif, gy, u, y, W, d, nullptr, s, keep, g, ws, wsb, (cudaStream_t)stream);
}
size_t delrec_axonal_backward_hard_workspace(const delrec_layer* ly) {
  return ly ? backward_ws(ly, DELREC_AXONAL, true) : 0;
}
int delrec_axonal_backward_hard(const delrec_layer* ly, const delrec_lif* lif, int mode, const float* gy,
                                const float* u, const float* y, const float* W, const float* d,
                                const float* s, const float* d_hard, const float* keep,
                                const delrec_grads* g, void* ws, size_t wsb, void* stream) {
  HardBwd hb{};
  if (mode == DELREC_HARD_STE) {
    if (!d_hard) return DELREC_ERR_ARG;
    hb.dw_d = d_hard;
  } else if (mode == DELREC_HARD_APPROX) {
    hb.st_dd = 1;
  } else {
    return DELREC_ERR_ARG;
  }
  return run_backward(ly, DELREC_AXONAL, lif, gy, u, y, W, d, nullptr, s, keep, g, ws, wsb,
                      (cudaStream_t)stream, &hb);
}
int delrec_synaptic_backward(const delrec_layer* ly, const delrec_lif* lif, const float* gy, const float* u,
                             const float* y, const float* W, const float* d, const float* s, const float* keep,
                             const delrec_grads* g, void* ws, size_t wsb, void* stream) {
  return run_backward(ly, DELREC_SYNAPTIC, lif, gy, u, y, W, d, nullptr, s, keep, g, ws, wsb, (cudaStream_t)stream);
}
int delrec_hybrid_backward(const delrec_layer* ly, const delrec_lif* lif, const float* gy, const float* u,
                           const float* y, const float* W, const float* base, const float* offsets,
                           const float* s, const float* keep, const delrec_grads* g, void* ws, size_t wsb,
                           void* stream) {
  return run_backward(ly, DELREC_HYBRID, lif, gy, u, y, W, base, offsets, s, keep, g, ws, wsb, (cudaStream_t)stream);
}

int delrec_readout_sum_forward(int T, int B, int N, int C, const float* y, const float* W, const float* bias,
                               float* ysum, float* out, void* stream) {
  if (T < 1 || B < 1 || N < 1 || C < 1 || !y || !W || !ysum || !out) return DELREC_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t BN = (size_t)B * N;
  k_time_sum<<<grid_for(BN, 256), 256, 0, st>>>(T, BN, y, ysum);
  DR_LAUNCHED();
  const size_t warps = (size_t)B * C;
  k_readout_sum<<<(int)std::min<size_t>((warps + 7) / 8, (size_t)kSMs * 16), 256, 0, st>>>(T, B, N, C, ysum, W,
                                                                                              bias, out);
  DR_LAUNCHED();
  return DELREC_OK;
}

int delrec_readout_sum_backward(int T, int B, int N, int C, const float* ysum, const float* W, const float* g,
                                float* dy, float* dW, float* dbias, void* stream) {
  if (T < 1 || B < 1 || N < 1 || C < 1 || !g || (dy && !W) || (dW && !ysum)) return DELREC_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t BN = (size_t)B * N, CN = (size_t)C * N;
  if (dy) {
    k_readout_sum_dy<<<grid_for(BN, 256), 256, 0, st>>>(T, B, N, C, g, W, dy);
    DR_LAUNCHED();
  }
  if (dW || dbias) {
    k_readout_sum_dw<<<grid_for(CN + C, 256), 256, 0, st>>>(T, B, N, C, g, ysum, dW, dbias);
    DR_LAUNCHED();
  }
  return DELREC_OK;
}

int delrec_count_nonbinary(const float* x, size_t n, unsigned int* count, void* stream) {
  if (!count || (n && !x) || ((uintptr_t)x & 15) != 0) return DELREC_ERR_ARG;
  const cudaStream_t st = (cudaStream_t)stream;
  DR_CUDA(cudaMemsetAsync(count, 0, sizeof(unsigned int), st));
  if (n == 0) return DELREC_OK;
  k_count_nonbinary<<<grid_for(n / 4 + 1, 256), 256, 0, st>>>(x, n, count);
  DR_LAUNCHED();
  return DELREC_OK;
}
size_t delrec_linear_forward_workspace(int M, int K, int N, int x_binary) {
  return (M > 0 && K > 0 && N > 0) ? linear_fwd_ws(M, K, N, x_binary ? 1 : 0) : 0;
}
size_t delrec_linear_backward_workspace(int M, int K, int N, int x_binary) {
  return (M > 0 && K > 0 && N > 0) ? linear_bwd_ws(M, K, N, x_binary ? 1 : 0) : 0;
}
int delrec_linear_forward(int M, int K, int N, const float* x, const float* W, const float* bias, int x_binary,
                          float* out, void* ws, size_t wsb, void* stream) {
  return run_linear_forward(M, K, N, x, W, bias, x_binary ? 1 : 0, out, ws, wsb, (cudaStream_t)stream);
}
int delrec_linear_backward(int M, int K, int N, const float* x, const float* W, const float* gout, int x_binary,
                           float* dx, float* dW, float* dbias, void* ws, size_t wsb, void* stream) {
  return run_linear_backward(M, K, N, x, W, gout, x_binary ? 1 : 0, dx, dW, dbias, ws, wsb,
                             (cudaStream_t)stream);
}

int delrec_hybrid_delay_grad(int N, int LM, const float* C, const float* W, const float* d, float sigma,
                             float* dd, void* stream) {
  if (N < 1 || LM < 1 || !C || !W || !d || !dd) return DELREC_ERR_ARG;
  k_hybrid_delay_grad<<<grid_for((size_t)N * N, 256), 256, 0, (cudaStream_t)stream>>>(N, LM, C, W, d, 1.f + sigma, dd);
  DR_LAUNCHED();
  return DELREC_OK;
}

int delrec_lif_forward(int T, int M, const delrec_lif* lif, const float* x, float* y, float* u, void* stream) {
  if (T < 1 || M < 1 || !lif || !x || !y) return DELREC_ERR_ARG;
  k_lif_fwd<<<cdiv(M, 256), 256, 0, (cudaStream_t)stream>>>(T, M, make_lif(*lif), x, y, u);
  DR_LAUNCHED();
  return DELREC_OK;
}
int delrec_lif_backward(int T, int M, const delrec_lif* lif, const float* gy, const float* u, float* dx,
                        void* stream) {
  if (T < 1 || M < 1 || !lif || !gy || !u || !dx) return DELREC_ERR_ARG;
  k_lif_bwd<<<cdiv(M, 256), 256, 0, (cudaStream_t)stream>>>(T, M, make_lif(*lif), gy, u, dx);
  DR_LAUNCHED();
  return DELREC_OK;
}

static int dcls_check(int T, int B, int Cin, int Cout, int groups, int K, int lpad) {
  if (T < 1 || B < 1 || Cin < 1 || Cout < 1 || groups < 1 || K < 1 || lpad < 0) return DELREC_ERR_ARG;
  if (Cin % groups || Cout % groups) return DELREC_ERR_ARG;
  if (K > 64) return DELREC_ERR_UNSUPPORTED;
  return DELREC_OK;
}

int delrec_dcls_forward(int T, int B, int Cin, int Cout, int groups, int K, int lpad, const float* x,
                        const float* weight, const float* P, const float* SIG, const float* bias, float* ker,
                        float* out, void* stream) {
  int rc = dcls_check(T, B, Cin, Cout, groups, K, lpad);
  if (rc) return rc;
  if (!x || !weight || !P || !SIG || !ker || !out) return DELREC_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int rows = Cout * (Cin / groups);
  k_dcls_build<<<cdiv(rows, 128), 128, 0, st>>>(rows, K, weight, P, SIG, ker);
  DR_LAUNCHED();
  k_dcls_conv<<<grid_for((size_t)T * B * Cout, 256), 256, 0, st>>>(T, B, Cin, Cout, groups, K, lpad, x, ker, bias, out);
  DR_LAUNCHED();
  return DELREC_OK;
}

size_t delrec_dcls_backward_workspace(int T, int B, int Cin, int Cout, int groups, int K) {
  (void)T; (void)B;
  if (groups < 1) return 0;
  Carve c(nullptr, (size_t)-1);
  c.take<float>((size_t)Cout * (Cin / groups) * K);  // ker
  c.take<float>((size_t)Cout * (Cin / groups) * K);  // dker
  return c.off;
}

int delrec_dcls_backward(int T, int B, int Cin, int Cout, int groups, int K, int lpad, const float* x,
                         const float* weight, const float* P, const float* SIG, const float* gout, float* dx,
                         float* dweight, float* dP, float* dSIG, float* dbias, void* ws, size_t wsb,
                         void* stream) {
  int rc = dcls_check(T, B, Cin, Cout, groups, K, lpad);
  if (rc) return rc;
  if (!x || !weight || !P || !SIG || !gout) return DELREC_ERR_ARG;
  if (((uintptr_t)ws & 255) != 0 || wsb < delrec_dcls_backward_workspace(T, B, Cin, Cout, groups, K))
    return DELREC_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const int rows = Cout * (Cin / groups);
  Carve c(ws, wsb);
  float* ker = c.take<float>((size_t)rows * K);
  float* dker = c.take<float>((size_t)rows * K);
  k_dcls_build<<<cdiv(rows, 128), 128, 0, st>>>(rows, K, weight, P, SIG, ker);
  DR_LAUNCHED();
  if (dx) {
    k_dcls_dx<<<grid_for((size_t)T * B * Cin, 256), 256, 0, st>>>(T, B, Cin, Cout, groups, K, lpad, gout, ker, dx);
    DR_LAUNCHED();
  }
  if (dweight || dP || dSIG) {
    k_dcls_dker<<<rows * K, 256, 0, st>>>(T, B, Cin, Cout, groups, K, lpad, x, gout, dker);
    DR_LAUNCHED();
    k_dcls_params<<<cdiv(rows, 128), 128, 0, st>>>(rows, K, weight, P, SIG, dker, dweight, dP, dSIG);
    DR_LAUNCHED();
  }
  if (dbias) {
    k_dcls_dbias<<<cdiv(Cout, 32), 1024, 0, st>>>(T * B, Cout, gout, dbias);
    DR_LAUNCHED();
  }
  return DELREC_OK;
}

// ---- the library's tensor-core GEMM, exposed for testing and for callers' own use ----
size_t delrec_tc_gemm_workspace(int M, int N, int ksplit) {
  return (M > 0 && N > 0 && ksplit > 0) ? gemm_partial_bytes(M, N, ksplit, 1) : 0;
}

int delrec_tc_gemm(int M, int N, int K, int layout, int a_pieces, const void* const* A, long long lda,
                   int b_pieces, const void* const* B, long long ldb, int nprod, const int* prod_a,
                   const int* prod_b, int ksplit, int block_n, float* D, long long ldd, int accumulate, void* ws,
                   size_t wsb, void* stream) {
  if (M < 1 || N < 1 || K < 1 || !A || !B || !D || !prod_a || !prod_b) return DELREC_ERR_ARG;
  if (a_pieces < 1 || a_pieces > 3 || b_pieces < 1 || b_pieces > 3 || nprod < 1 || nprod > kGemmMaxProd)
    return DELREC_ERR_ARG;
  if (ksplit < 1 || ldd < N) return DELREC_ERR_ARG;
  if (ksplit > 1 && (((uintptr_t)ws & 255) != 0 || wsb < gemm_partial_bytes(M, N, ksplit, 1)))
    return DELREC_ERR_WORKSPACE;
  GemmSide as{}, bs{};
  as.n = a_pieces; as.ld = lda; as.mn_major = (layout & 1) ? 1 : 0;
  as.rows = as.mn_major ? K : M; as.cols = as.mn_major ? M : K;
  bs.n = b_pieces; bs.ld = ldb; bs.mn_major = (layout & 2) ? 1 : 0;
  bs.rows = bs.mn_major ? K : N; bs.cols = bs.mn_major ? N : K;
  for (int i = 0; i < a_pieces; ++i) as.p[i] = A[i];
  for (int i = 0; i < b_pieces; ++i) bs.p[i] = B[i];
  GemmArgs g{};
  g.M = M; g.N = N; g.K = K; g.nprod = nprod; g.nseg = 1; g.ksplit = ksplit;
  for (int p = 0; p < nprod; ++p) { g.pa[p] = prod_a[p]; g.pb[p] = prod_b[p]; }
  g.D = D; g.ldd = ldd; g.mode = accumulate ? GEMM_ACCUM : GEMM_STORE;
  return gemm_run(as, bs, g, 1, block_n, (float*)ws, (cudaStream_t)stream, &g_launches);
}

// ---- allocation-free variant of the axonal forward --------------------------------
// Some callers cannot call cudaMalloc while they run this layer: a host that hands all
// device memory to its own allocator up front and keeps none spare, a training loop that
// must not add the device-wide synchronisation cudaMalloc/cudaFree imply, or a plugin
// runtime that forbids allocation after start-up.  For them the scratch of the axonal
// forward (transposed weights and the per-source tap table) lives in this fixed device
// array, which every GPU that loads the library holds until the process exits.
static constexpr size_t kNoAllocScratchBytes = 8u << 20;   // 8 MiB
static constexpr int kNoAllocMaxN = 1024;                  // widest layer it accepts
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static std::atomic<void*> g_noalloc_ptr[64];
static std::mutex g_noalloc_mu;

int delrec_axonal_forward_noalloc(const delrec_layer* ly, const delrec_lif* lif, const float* x,
                                  const float* W, const float* bias, const float* d, const float* s,
                                  const float* keep, float* y, float* u, void* stream) {
  if (!ly) return DELREC_ERR_ARG;
  if (ly->N > kNoAllocMaxN || forward_ws(ly, DELREC_AXONAL, false) > kNoAllocScratchBytes) {
    fprintf(stderr, "delrec_b200: delrec_axonal_forward_noalloc supports N <= %d neurons (its fixed "
                    "%zu-byte scratch array); N=%d needs the workspace entry point delrec_axonal_forward\n",
            kNoAllocMaxN, kNoAllocScratchBytes, (int)ly->N);
    return DELREC_ERR_WORKSPACE;
  }
  // the per-sample scan keeps the spike history of its sample in shared memory
  if (ly->N >= 1 && ly->L >= 1 && plan_forward(ly, DELREC_AXONAL).smem > kSmemLimit) {
    fprintf(stderr, "delrec_b200: delrec_axonal_forward_noalloc: ring length L=%d is too long for the "
                    "per-sample scan at N=%d\n", (int)ly->L, (int)ly->N);
    return DELREC_ERR_UNSUPPORTED;
  }
  int dev = 0;
  DR_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return DELREC_ERR_UNSUPPORTED;
  void* scratch = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (!scratch) {
    // once per device, with that device current: the symbol's device address (host
    // threads making their first call together take turns here)
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    scratch = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
    if (!scratch) {
      DR_CUDA(cudaGetSymbolAddress(&scratch, g_noalloc_scratch));
      g_noalloc_ptr[dev].store(scratch, std::memory_order_release);
    }
  }
  // the per-sample scan only: the step-by-step forward of wide layers needs more scratch
  return run_forward(ly, DELREC_AXONAL, lif, x, W, bias, d, nullptr, s, keep, y, u, scratch,
                     kNoAllocScratchBytes, (cudaStream_t)stream, false);
}

}  // extern "C"
