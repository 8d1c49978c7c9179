/*
 * delrec_b200: C-ABI of the B200-native delay-LIF hot path (DelRec).
 *
 * All pointers are device pointers, tensors are fp32, contiguous, time-major (T,B,N).
 * Weights follow the reference's convention W[i,o] (row = target neuron i, column =
 * source neuron o): rec[b,i] = sum_o W[i,o] * (delayed spike of o).
 * Every entry point launches on `stream` (a cudaStream_t; NULL = legacy default stream)
 * and returns DELREC_OK or an error code.  Scratch memory is passed in by the caller:
 * query its size with the matching *_workspace function.  Weight gradients, the
 * synaptic lag stack, the projections, the chunked reverse scan and the step-by-step
 * forward and reverse scans of axonal layers wider than 512 neurons run on the library's
 * own tcgen05 GEMM; the library calls no vendor math library.
 *
 * Reference interfaces replaced (paths are inside ZiyadBekrar/SNN-delays):
 *   delrec_build_mask             triton_kernels/delays.py:13-29, 48-63 (build_mask,
 *                                 build_syn_mask)
 *   delrec_axonal_forward         triton_kernels/recdel_base.py:136-182 (recdel_triton_forward,
 *                                 launching recdel_fwd_kernel :34-129)
 *   delrec_axonal_backward        recdel_base.py:288-342 (recdel_triton_backward: recdel_bwd_kernel
 *                                 :189-285 + host dW/db/dmask) and the dmask->dd/dp autograd
 *                                 of AxonalRecdelTriton.backward :402-439
 *   delrec_synaptic_forward       triton_kernels/synaptic_eventdriven.py:386-416 (EventDrivenSyn
 *                                 .forward launching _ed_scatter_compact_kernel :106-164)
 *   delrec_synaptic_backward      synaptic_eventdriven.py:419-471 (EventDrivenSyn.backward:
 *                                 _ed_bwd_kernel :323-364 + Cstack GEMMs + autograd dd/dp)
 *   delrec_hybrid_forward         triton_kernels/synaptic_hybrid.py:139-172 (HybridSynDelay.forward)
 *   delrec_hybrid_backward        synaptic_hybrid.py:175-211 (HybridSynDelay.backward incl.
 *                                 _hybrid_dd_kernel :83-113), with the (N,N) delay gradient
 *                                 already reduced onto the learned (N,) base the way the
 *                                 parametrization networks.py:823-829 does
 *   delrec_hybrid_delay_grad      synaptic_hybrid.py:116-126 (_delay_grad, closed-form dd)
 *   delrec_lif_forward/backward   the multi-step SpikingJelly LIFNode used between layers by
 *                                 the model zoo (networks.py:84-96), no recurrence
 *   delrec_dcls_forward/backward  networks.py:43-50 (dcls_module.forward: DCLS 0.1.1 Gaussian
 *                                 kernel construction + causal conv1d over time)
 *   delrec_linear_forward/backward  the torch.nn.Linear projections between the delay layers
 *                                 and the readout (networks.py:84-96, 140-181)
 */
#ifndef DELREC_B200_H
#define DELREC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------- */
#define DELREC_OK 0
#define DELREC_ERR_ARG 1          /* invalid size / null pointer / bad enum            */
#define DELREC_ERR_CUDA 2         /* a CUDA launch or attribute call failed             */
#define DELREC_ERR_WORKSPACE 3    /* workspace too small or misaligned (256 B)          */
#define DELREC_ERR_UNSUPPORTED 4  /* shape outside the kernels' supported range          */

/* ---- delay kinds ------------------------------------------------------------------ */
#define DELREC_AXONAL 0           /* d (N,): one delay per source neuron                */
#define DELREC_SYNAPTIC 1         /* d (N,N): one delay per connection d[i,o]           */
#define DELREC_HYBRID 2           /* learned base (N,) + frozen integer offsets (N,N)   */

/* surrogate ids: identical to triton_kernels/surrogate.py:_SURR_ID */
#define DELREC_SURR_TRIANGLE 0
#define DELREC_SURR_ATAN 1

/* LIF neuron, SpikingJelly LIFNode semantics with decay_input=False
 * (charge v*(1-1/tau)+a when v_reset is None or 0, else v-(v-v_reset)/tau+a; fire
 * u-v_th >= 0; hard reset to v_reset or soft reset by v_th; initial v = v_reset, or 0
 * for a soft reset). */
typedef struct delrec_lif {
  float tau;
  float v_threshold;
  float v_reset;        /* ignored when soft_reset != 0 */
  int32_t soft_reset;   /* 1: v_reset is None */
  int32_t detach_reset; /* 1: no gradient through the reset */
  int32_t surrogate;    /* DELREC_SURR_* */
  float gamma;          /* Triangle width */
  float alpha;          /* ATan slope */
} delrec_lif;

/* Shape and delay description of one recurrent delay layer. */
typedef struct delrec_layer {
  int32_t kind;         /* DELREC_AXONAL / DELREC_SYNAPTIC / DELREC_HYBRID */
  int32_t T, B, N;
  int32_t L;            /* ring length ceil(1 + max d + max s) + 1 (lags 1..L-1) */
  int32_t K;            /* hybrid: largest integer offset (offsets in [0, K]) */
  int32_t has_bias;     /* bias pointer is read */
  int32_t has_keep;     /* keep (B,N) dropout mask is read */
  float s_max;          /* largest triangle half-width (1 + sigma, or max over s) */
  float d_min;          /* smallest delay (hybrid: smallest learned base; may be negative) */
} delrec_layer;

/* Gradient outputs of a layer backward.  Any pointer may be NULL to skip it. */
typedef struct delrec_grads {
  float* dx;            /* (T,B,N) */
  float* dW;            /* (N,N)   */
  float* dbias;         /* (N,)    */
  float* dd;            /* axonal (N,), synaptic (N,N), hybrid base (N,) */
  float* ds;            /* (N,) gradient w.r.t. the per-source half-width s (use_sig_p) */
} delrec_grads;

/* Triangle delay kernel h[r,l] = max(0, s_r' - |l - (1 + d[r])|) / s_r'^2 for l in [0,L),
 * rows r in [0,R); s_r' = s[r % s_period] (s_period = N for synaptic (N,N) delays whose
 * width is indexed by the source, = R for axonal).  out (R, L). */
int delrec_build_mask(int R, int L, const float* d, const float* s, int s_period,
                      float* out, void* stream);

/* ---- axonal layer ------------------------------------------------------------------ */
/* x (T,B,N), W (N,N), bias (N), d (N), s (N) half-widths, keep (B,N).
 * Outputs y (spikes) and u (pre-reset membrane), both (T,B,N). */
size_t delrec_axonal_forward_workspace(const delrec_layer* layer);
int delrec_axonal_forward(const delrec_layer* layer, const delrec_lif* lif,
                          const float* x, const float* W, const float* bias,
                          const float* d, const float* s, const float* keep,
                          float* y, float* u, void* workspace, size_t workspace_bytes,
                          void* stream);
/* gy (T,B,N) upstream gradient of the spikes; u, y from the forward. */
size_t delrec_axonal_backward_workspace(const delrec_layer* layer);
int delrec_axonal_backward(const delrec_layer* layer, const delrec_lif* lif,
                           const float* gy, const float* u, const float* y,
                           const float* W, const float* d, const float* s,
                           const float* keep, const delrec_grads* grads,
                           void* workspace, size_t workspace_bytes, void* stream);

/* Hard-tap forms of the axonal layer: AxonalRecdelTriton with ste_mode 1 / 2 or approx
 * (triton_kernels/recdel_base.py:350-445, recdel_bwd_kernel APPROX branch :215-278).
 * Their forwards are delrec_axonal_forward at half-width s = 1 with the hard taps written
 * as a delay: the single tap at lag l (lag = clamp(round(d) + 1, 1, .)) is d = l - 1 and
 * the two-tap interpolation (1 - f) at l, f at l + 1 (l = floor(1 + d)) is d = l - 1 + f,
 * i.e. max(d, 0).  Backwards:
 *   DELREC_HARD_STE     the soft triangle's backward over (d, s) -- gfut, dx, dd, ds,
 *                       dbias -- except dW, which correlates gr with the hard forward's z
 *                       (taps of d_hard at half-width 1);
 *   DELREC_HARD_APPROX  the backward of the single-tap forward: d = the hard delays
 *                       (l - 1), s all 1 and the layer's L sized for them; dd is the
 *                       straight-through sum_{t,b} gz[t,b,n] (y[t-l-1,b,n] - y[t-l,b,n]);
 *                       grads->ds must be NULL, d_hard is not read. */
#define DELREC_HARD_STE 1
#define DELREC_HARD_APPROX 2
size_t delrec_axonal_backward_hard_workspace(const delrec_layer* layer);
int delrec_axonal_backward_hard(const delrec_layer* layer, const delrec_lif* lif, int mode,
                                const float* gy, const float* u, const float* y,
                                const float* W, const float* d, const float* s,
                                const float* d_hard, const float* keep,
                                const delrec_grads* grads, void* workspace,
                                size_t workspace_bytes, void* stream);

/* ---- the library's own tensor-core GEMM (tcgen05, bf16 pieces, fp32 accumulate) ------
 * No reference counterpart as an interface: it is the contraction engine behind the
 * weight gradients, the lag-correlation stack and the projections (which the reference
 * runs as torch matmuls / cuBLAS), exposed so it can be tested on its own.
 * D (M,N) = [D +] sum_p A[prod_a[p]] . B[prod_b[p]]^T over K.  layout bit 0: A pieces
 * are stored (K,M) instead of (M,K) (MN-major); bit 1: B pieces (K,N) instead of (N,K).
 * Pieces are bf16, 16-byte aligned, row strides lda / ldb multiples of 8 elements; D fp32
 * row stride ldd.  ksplit > 1 splits the reduction (partials in the workspace, summed in
 * a fixed order); block_n = 64, 128 or 256 output columns per tile. */
size_t delrec_tc_gemm_workspace(int M, int N, int ksplit);
int delrec_tc_gemm(int M, int N, int K, int layout, int a_pieces, const void* const* A, long long lda,
                   int b_pieces, const void* const* B, long long ldb, int nprod, const int* prod_a,
                   const int* prod_b, int ksplit, int block_n, float* D, long long ldd, int accumulate,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Same as delrec_axonal_forward but allocation-free: no reference counterpart.  It is for
 * callers that cannot call cudaMalloc while the layer runs (all device memory handed to
 * their own allocator, no device-wide synchronisation allowed in the loop, or a plugin
 * host that forbids allocation after start-up).  Its scratch is a fixed 8 MiB device
 * array inside the library, held by every GPU that loads the library until the process
 * exits.  Limits: N <= 1024 neurons (wider layers get DELREC_ERR_WORKSPACE); every width
 * runs the per-sample scan, whose spike history lives in shared memory, so very long
 * rings (at N = 1024, L above about 1000) get DELREC_ERR_UNSUPPORTED.  The first call on
 * a device looks the array up (cudaGetSymbolAddress), so make that first call before any
 * stream capture.  All calls share the array: calls that overlap on the GPU (other
 * streams, other threads) race on it.  Every byte it reads is written earlier in the
 * same call, so nothing carries over between calls. */
int delrec_axonal_forward_noalloc(const delrec_layer* layer, const delrec_lif* lif,
                                  const float* x, const float* W, const float* bias,
                                  const float* d, const float* s, const float* keep,
                                  float* y, float* u, void* stream);

/* ---- synaptic layer ---------------------------------------------------------------- */
/* d (N,N) per connection, s (N) per source. */
size_t delrec_synaptic_forward_workspace(const delrec_layer* layer);
int delrec_synaptic_forward(const delrec_layer* layer, const delrec_lif* lif,
                            const float* x, const float* W, const float* bias,
                            const float* d, const float* s, const float* keep,
                            float* y, float* u, void* workspace, size_t workspace_bytes,
                            void* stream);
size_t delrec_synaptic_backward_workspace(const delrec_layer* layer);
int delrec_synaptic_backward(const delrec_layer* layer, const delrec_lif* lif,
                             const float* gy, const float* u, const float* y,
                             const float* W, const float* d, const float* s,
                             const float* keep, const delrec_grads* grads,
                             void* workspace, size_t workspace_bytes, void* stream);

/* ---- hybrid layer ------------------------------------------------------------------ */
/* base (N,) learned per source, offsets (N,N) frozen integers in [0,K] (fp32, as the
 * reference buffer); effective delay d[i,o] = base[o] + offsets[i,o].  s (N). */
size_t delrec_hybrid_forward_workspace(const delrec_layer* layer);
int delrec_hybrid_forward(const delrec_layer* layer, const delrec_lif* lif,
                          const float* x, const float* W, const float* bias,
                          const float* base, const float* offsets, const float* s,
                          const float* keep, float* y, float* u,
                          void* workspace, size_t workspace_bytes, void* stream);
/* The backward factors each synapse's delay into base + offset and supports base tap
 * windows that reach at most one lag below lag 1 (layer->d_min, s_max); a wider window
 * returns DELREC_ERR_UNSUPPORTED -- run such a layer through delrec_synaptic_* on the
 * materialised delay d[i,o] = base[o] + offsets[i,o] (the Python Function does). */
size_t delrec_hybrid_backward_workspace(const delrec_layer* layer);
int delrec_hybrid_backward(const delrec_layer* layer, const delrec_lif* lif,
                           const float* gy, const float* u, const float* y,
                           const float* W, const float* base, const float* offsets,
                           const float* s, const float* keep, const delrec_grads* grads,
                           void* workspace, size_t workspace_bytes, void* stream);

/* Closed-form per-synapse delay gradient of the hybrid/synaptic triangle kernel:
 * dd[i,o] = W[i,o] * sum_{l=1}^{LM-1} C[i,o,l] * g(l - 1 - d[i,o]),
 * g(a) = sign(a)/s^2 where |a| <= s, else 0  (s = 1 + sigma).  C (N,N,LM). */
int delrec_hybrid_delay_grad(int N, int LM, const float* C, const float* W,
                             const float* d, float sigma, float* dd, void* stream);

/* ---- plain multi-step LIF (no recurrence) ------------------------------------------ */
int delrec_lif_forward(int T, int M, const delrec_lif* lif, const float* x,
                       float* y, float* u, void* stream);
int delrec_lif_backward(int T, int M, const delrec_lif* lif, const float* gy,
                        const float* u, float* dx, void* stream);

/* ---- DCLS feedforward delay (Gaussian-interpolated positions, causal conv) ---------- */
/* x (T,B,Cin); weight (Cout, Cin/groups); P, SIG (Cout, Cin/groups); kernel width K;
 * left zero padding lpad (= K-1 for the causal length-preserving layer).  out (T,B,Cout).
 * The constructed dense kernel is written to ker (Cout, Cin/groups, K). */
int delrec_dcls_forward(int T, int B, int Cin, int Cout, int groups, int K, int lpad,
                        const float* x, const float* weight, const float* P,
                        const float* SIG, const float* bias, float* ker, float* out,
                        void* stream);
/* Gradients w.r.t. x, weight, P, SIG, bias (any may be NULL).  gout (T,B,Cout). */
size_t delrec_dcls_backward_workspace(int T, int B, int Cin, int Cout, int groups, int K);
int delrec_dcls_backward(int T, int B, int Cin, int Cout, int groups, int K, int lpad,
                         const float* x, const float* weight, const float* P,
                         const float* SIG, const float* gout, float* dx, float* dweight,
                         float* dP, float* dSIG, float* dbias,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ---- feedforward projection ------------------------------------------------------- */
/* out (M,N) = x (M,K) . W^T + bias, W (N,K) as torch.nn.Linear, bias (N) or NULL.
 * Runs on bf16 tensor cores with fp32 accuracy: each fp32 operand is split exactly into
 * three bf16 pieces and the piece products with i + j <= 2 are summed with fp32
 * accumulation.  x_binary = 1 promises x in {0, 1} (spike trains: three products instead
 * of six); a violated promise sets the status word.  The GEMMs run on the library's
 * tcgen05 GEMM (partials on a slice of the workspace). */
size_t delrec_linear_forward_workspace(int M, int K, int N, int x_binary);
int delrec_linear_forward(int M, int K, int N, const float* x, const float* W, const float* bias,
                          int x_binary, float* out, void* workspace, size_t workspace_bytes,
                          void* stream);
/* gout (M,N); dx (M,K), dW (N,K), dbias (N): any may be NULL (x may be NULL when dW and
 * dbias are, W when dx is). */
size_t delrec_linear_backward_workspace(int M, int K, int N, int x_binary);
int delrec_linear_backward(int M, int K, int N, const float* x, const float* W, const float* gout,
                           int x_binary, float* dx, float* dW, float* dbias, void* workspace,
                           size_t workspace_bytes, void* stream);

/* ---- readout + time sum of the loss ----------------------------------------------- */
/* The model zoo's readout Linear (networks.py:140-181) followed by the SSC / PS-MNIST
 * loss's sum over time (utils.py:188-200, calc_loss_SSC), fused: out (B,C) =
 * sum_t (y_t W^T + bias) = ysum W^T + T bias with ysum (B,N) = sum_t y_t written too; the
 * (T,B,C) readout is never formed.  y (T,B,N), W (C,N) as torch.nn.Linear, bias (C) or
 * NULL.  Backward with g (B,C) = dloss/dout: dy (T,B,N) = g W for every t, dW (C,N) =
 * g^T ysum, dbias (C) = T sum_b g (any output may be NULL).  fp32, fixed summation order. */
int delrec_readout_sum_forward(int T, int B, int N, int C, const float* y, const float* W,
                               const float* bias, float* ysum, float* out, void* stream);
int delrec_readout_sum_backward(int T, int B, int N, int C, const float* ysum, const float* W,
                                const float* g, float* dy, float* dW, float* dbias, void* stream);

/* Sets *count (device) to the number of entries of x[0..n) that are neither 0 nor 1;
 * asynchronous on the stream, x 16-byte aligned.  The projections' spike-input test
 * (x_binary above); no counterpart in the reference, whose projections are fp32 GEMMs. */
int delrec_count_nonbinary(const float* x, size_t n, unsigned int* count, void* stream);

/* ---- device status word ------------------------------------------------------------ */
/* Kernels record internal inconsistencies (an out-of-range lag or index that was
 * skipped) in a device status word instead of trapping.  Reading it synchronizes. */
int delrec_get_status(int* status_out);
int delrec_clear_status(void);
const char* delrec_version(void);
/* Number of kernels this library has launched in this process (host-side counter). */
unsigned long long delrec_launch_count(void);
/* Measurement hooks: while enabled, every reverse-scan launch (the backward's time loop)
 * is bracketed by CUDA events on its stream; delrec_scan_time synchronizes on them and
 * returns the summed milliseconds and the number of launches since enabling. */
int delrec_scan_timing(int enable);
int delrec_scan_time(double* total_ms, int* launches);
/* The same per part: 0 = every reverse scan (a chunked scan counts as one launch per
 * layer), 1 = the step launches of the chunked scans, 2 = their chunk GEMM launches. */
int delrec_scan_time_part(int part, double* total_ms, int* launches);
/* Reverse-scan variant of the layer backwards (process-wide).  0 (default): hybrid layers
 * whose shape allows it run the chunked scan -- the delayed-gradient contraction of every
 * synapse whose lag reaches past the current 8-step chunk as one tensor-core GEMM per
 * chunk, the short-lag synapses step by step in blocks that own whole samples; 1: the
 * step-by-step scans only; 2: the chunked scan with its steps split over source slices
 * that exchange gr through L2 every step (kept for comparison).  All give
 * the reference's gradients within the library's tolerance; the workspace size queries
 * cover either variant.  Replaces no reference call (the reference has one Triton
 * kernel per layer kind, triton_kernels/synaptic_eventdriven.py:323-364). */
int delrec_set_reverse_scan(int variant);
/* Measurement: the per-step latency floor of the reverse scans.  Runs T steps of their
 * exchange alone -- each block publishes its slice of gr to L2, meets its batch tile at an
 * arrival counter and restages the tile's gr into shared memory -- on the grid and tiling
 * the 64-sample scans use for `layer` (N <= 512, B > 32; otherwise
 * DELREC_ERR_UNSUPPORTED), with no LIF step and no synapse sums.  Time it with events on
 * `stream`.  No counterpart in the reference. */
size_t delrec_exchange_floor_workspace(const delrec_layer* layer);
int delrec_exchange_floor(const delrec_layer* layer, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DELREC_B200_H */
