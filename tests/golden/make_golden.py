"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run here (it needs the read-only reference checkout; the GPU box never runs it):

    python tests/golden/make_golden.py <path of the reference checkout> [--hard-only]
                                       [--only NAME[,NAME...]]

(``--only`` regenerates the named cases of CASES and nothing else.)

For every case it runs, on identical seeded inputs,
  * the reference's canonical pure-PyTorch scans ``multi_step_forward_v2``
    (src/delrec/delay_layers_pytorch.py:121-194, 271-325), imported unmodified, driven by
    a minimal host object and the oracle's SpikingJelly-equivalent LIF neuron, with
    gradients from autograd;
  * the reference's own Triton kernels (src/delrec/triton_kernels/recdel_base.py:34-285,
    synaptic_eventdriven.py:106-164, 323-364, synaptic_hybrid.py:83-126) executed on the
    CPU by Triton's interpreter (TRITON_INTERPRET=1), with the host-side reductions of
    their autograd Functions.
The fixtures land in tests/golden/*.pt (small: T*B*N <= ~4k).
"""

import math
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
if len(sys.argv) < 2:
    sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
REF = sys.argv[1]
sys.path.insert(0, os.path.join(REF, "src"))
sys.path.insert(0, REPO)

import torch  # noqa: E402

from delrec import delay_layers_pytorch as ref_scans  # noqa: E402
from delrec.triton_kernels import recdel_base as ref_ax  # noqa: E402
from delrec.triton_kernels import synaptic_eventdriven as ref_ed  # noqa: E402
from delrec.triton_kernels import synaptic_hybrid as ref_hy  # noqa: E402
from delrec.triton_kernels.delays import build_lag, build_lag_interp  # noqa: E402
from delrec.triton_kernels.delays import build_mask, build_syn_mask  # noqa: E402
from oracle.delrec_oracle import OracleLIF, ATanSpike, TriangleSpike  # noqa: E402


class _RecordingLIF(OracleLIF):
    def single_step_forward(self, a):
        s = super().single_step_forward(a)
        self.u_seq.append(self.u)
        return s

    def reset(self):
        super().reset()
        self.u_seq = []


class _Host:
    """Attributes the reference's v2 mixins read (delay_layers.py:100-143)."""

    def __init__(self, kind, W, d, sigma, lif, p_spread, use_sig_p, bias, keep):
        self.recurrent_weights = W
        self.recurrent_delays = d
        self.sigma = sigma
        self.neuron_module = lif
        self.use_sig_p = use_sig_p
        self.p_spread = p_spread
        self.round_delays = False
        self.use_rec_bias = bias is not None
        self.recurrent_bias = bias
        self.store_v_seq = False
        self.neurons = W.shape[0]
        self._keep = keep
        self._kind = kind

    def dropout(self, r):
        return r if self._keep is None else r * self._keep


class AxHost(_Host, ref_scans.AxonalTorchScans):
    pass


class SynHost(_Host, ref_scans.SynapticTorchScans):
    pass


def _surr(surr):
    return ATanSpike(2.0) if surr == "atan" else TriangleSpike(1.0)


def _lif_consts(tau, v_reset):
    decay = 1.0 - 1.0 / tau
    charge = 0.0 if (v_reset is None or v_reset == 0.0) else float(v_reset) / tau
    return decay, charge, (0.0 if v_reset is None else float(v_reset)), v_reset is None


def make_inputs(seed, T, B, N, kind, sigma, use_sig_p, bias, dropout, dmax, K=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, B, N, generator=g) * 0.9 + 0.35
    W = torch.randn(N, N, generator=g) * (1.2 / math.sqrt(N))
    if kind == "axonal":
        d = torch.rand(N, generator=g) * dmax
    elif kind == "synaptic":
        d = torch.rand(N, N, generator=g) * dmax
    else:
        d = torch.rand(N, generator=g) * dmax          # hybrid base (N,)
    p = torch.randn(N, generator=g) if use_sig_p else torch.zeros(N)
    b = torch.randn(N, generator=g) * 0.2 if bias else None
    keep = None
    if dropout:
        keep = (torch.rand(B, N, generator=g) > 0.3).float() / 0.7
    gy = torch.randn(T, B, N, generator=g)
    off = torch.randint(K + 1, (N, N), generator=g).float() if kind == "hybrid" else None
    return dict(x=x, W=W, d=d, p=p, bias=b, keep=keep, gy=gy, offsets=off)


def run_v2(kind, inp, sigma, use_sig_p, tau, v_reset, surr, detach_reset):
    x = inp["x"].clone().requires_grad_(True)
    W = inp["W"].clone().requires_grad_(True)
    base = inp["d"].clone().requires_grad_(True)
    d = base + 0.0 + 1.0 * inp["offsets"] if kind == "hybrid" else base
    p = inp["p"].clone().requires_grad_(use_sig_p)
    b = inp["bias"].clone().requires_grad_(True) if inp["bias"] is not None else None
    lif = _RecordingLIF(tau=tau, v_threshold=1.0, v_reset=v_reset, surrogate=_surr(surr),
                        detach_reset=detach_reset)
    cls = AxHost if kind == "axonal" else SynHost
    host = cls(kind, W, d, sigma, lif, p, use_sig_p, b, inp["keep"])
    y = host.multi_step_forward_v2(x)
    u = torch.stack(lif.u_seq)
    (y * inp["gy"]).sum().backward()
    out = dict(y=y.detach(), u=u.detach(), dx=x.grad, dW=W.grad, dd=base.grad)
    if use_sig_p:
        out["dp"] = p.grad
    if b is not None:
        out["dbias"] = b.grad
    return out


def run_triton_axonal(inp, sigma, use_sig_p, tau, v_reset, surr, detach_reset):
    """Reference Triton axonal scan (recdel_base.py) on the CPU interpreter, with the
    host-side reductions of recdel_triton_backward / AxonalRecdelTriton.backward."""
    x, W, d, p = inp["x"], inp["W"], inp["d"], inp["p"]
    T, B, N = x.shape
    decay, charge, vr, soft = _lif_consts(tau, v_reset)
    mask, L = build_mask(d, sigma, p, use_sig_p)
    keep = inp["keep"] if inp["keep"] is not None else torch.ones(B, N)
    drop = keep.unsqueeze(0).expand(T, B, N).contiguous()
    bias = inp["bias"] if inp["bias"] is not None else torch.zeros(N)
    Wt = W.t().contiguous()
    y, u, rec, z = (torch.empty_like(x) for _ in range(4))
    lag = torch.ones(N, dtype=torch.int32)
    frac = torch.zeros(N)
    BN = 1 << (N - 1).bit_length()
    bk = min(64, BN)
    ref_ax.recdel_fwd_kernel[(triton_cdiv(B, 16),)](
        x, drop, Wt, bias, mask, lag, frac, y, u, rec, z, T, B, N,
        x.stride(0), x.stride(1), x.stride(2), Wt.stride(0), Wt.stride(1),
        mask.stride(0), mask.stride(1), decay, charge, 1.0, vr,
        BLOCK_B=16, BLOCK_N=BN, BK=bk, L=L, SOFT=soft, FWD=0)
    gy = inp["gy"]
    gz, gr, dx = (torch.empty_like(x) for _ in range(3))
    ddst = torch.zeros(N)
    sid = 1 if surr == "atan" else 0
    ref_ax.recdel_bwd_kernel[(triton_cdiv(B, 16),)](
        gy, u, drop, W, mask, lag, y, gz, gr, dx, ddst, T, B, N,
        gy.stride(0), gy.stride(1), gy.stride(2), W.stride(0), W.stride(1),
        mask.stride(0), mask.stride(1), decay, 1.0, vr, 1.0, 2.0,
        BLOCK_B=16, BLOCK_N=BN, BK=bk, L=L, SOFT=soft, DETACH=bool(detach_reset), SURR=sid,
        APPROX=False)
    dW = gr.reshape(T * B, N).t() @ z.reshape(T * B, N)
    db = gr.reshape(T * B, N).sum(0)
    dmask = torch.zeros(N, L)
    for l in range(1, min(L, T)):
        dmask[:, l] = (gz[l:T] * y[0:T - l]).sum(dim=(0, 1))
    d_ = d.clone().requires_grad_(True)
    p_ = p.clone().requires_grad_(use_sig_p) if use_sig_p else None
    m2, _ = build_mask(d_, sigma, p_, use_sig_p)
    targets = [d_] + ([p_] if use_sig_p else [])
    grads = torch.autograd.grad(m2, targets, grad_outputs=dmask, allow_unused=True)
    out = dict(y=y, u=u, z=z, gz=gz, gr=gr, dx=dx, dW=dW, dbias=db, dmask=dmask, dd=grads[0])
    if use_sig_p:
        out["dp"] = grads[1]
    return out


def run_triton_axonal_hard(inp, sigma, use_sig_p, tau, v_reset, surr, detach_reset, mode):
    """The hard-tap variants of the reference's axonal scan (mode 1 / 2: ste_mode 1 / 2,
    mode 3: approx) on the interpreter, following AxonalRecdelTriton.forward / backward
    (recdel_base.py:350-445) and recdel_triton_backward's host reductions (:288-342)."""
    x, W, d, p = inp["x"], inp["W"], inp["d"], inp["p"]
    T, B, N = x.shape
    decay, charge, vr, soft = _lif_consts(tau, v_reset)
    frac = torch.zeros(N)
    if mode in (1, 2):
        mask, L = build_mask(d, sigma, p, use_sig_p)
        if mode == 1:
            lag = build_lag(d, L)
        else:
            lag, frac = build_lag_interp(d, L)
        fwd, approx = mode, False
    else:
        Lmax = int(torch.round(d).max().item()) + 2
        lag = build_lag(d, Lmax)
        mask, L = torch.zeros(N, 2), 2
        fwd, approx = 1, True
    keep = inp["keep"] if inp["keep"] is not None else torch.ones(B, N)
    drop = keep.unsqueeze(0).expand(T, B, N).contiguous()
    bias = inp["bias"] if inp["bias"] is not None else torch.zeros(N)
    Wt = W.t().contiguous()
    y, u, rec, z = (torch.empty_like(x) for _ in range(4))
    BN = 1 << (N - 1).bit_length()
    bk = min(64, BN)
    ref_ax.recdel_fwd_kernel[(triton_cdiv(B, 16),)](
        x, drop, Wt, bias, mask, lag, frac, y, u, rec, z, T, B, N,
        x.stride(0), x.stride(1), x.stride(2), Wt.stride(0), Wt.stride(1),
        mask.stride(0), mask.stride(1), decay, charge, 1.0, vr,
        BLOCK_B=16, BLOCK_N=BN, BK=bk, L=L, SOFT=soft, FWD=fwd)
    gy = inp["gy"]
    gz, gr, dx = (torch.empty_like(x) for _ in range(3))
    ddst = torch.zeros(N)
    sid = 1 if surr == "atan" else 0
    ref_ax.recdel_bwd_kernel[(triton_cdiv(B, 16),)](
        gy, u, drop, W, mask, lag, y, gz, gr, dx, ddst, T, B, N,
        gy.stride(0), gy.stride(1), gy.stride(2), W.stride(0), W.stride(1),
        mask.stride(0), mask.stride(1), decay, 1.0, vr, 1.0, 2.0,
        BLOCK_B=16, BLOCK_N=BN, BK=bk, L=L, SOFT=soft, DETACH=bool(detach_reset), SURR=sid,
        APPROX=approx)
    dW = gr.reshape(T * B, N).t() @ z.reshape(T * B, N)
    db = gr.reshape(T * B, N).sum(0)
    out = dict(y=y, u=u, z=z, gr=gr, dx=dx, dW=dW, dbias=db, lag=lag, frac=frac)
    if approx:
        out["dd"] = ddst
        return out
    dmask = torch.zeros(N, L)
    for l in range(1, min(L, T)):
        dmask[:, l] = (gz[l:T] * y[0:T - l]).sum(dim=(0, 1))
    d_ = d.clone().requires_grad_(True)
    p_ = p.clone().requires_grad_(use_sig_p) if use_sig_p else None
    m2, _ = build_mask(d_, sigma, p_, use_sig_p)
    targets = [d_] + ([p_] if use_sig_p else [])
    grads = torch.autograd.grad(m2, targets, grad_outputs=dmask, allow_unused=True)
    out["dd"] = grads[0]
    if use_sig_p:
        out["dp"] = grads[1]
    return out


def run_triton_synaptic(kind, inp, sigma, use_sig_p, tau, v_reset, surr, detach_reset):
    """Reference event-driven scatter + dense BPTT kernels (synaptic_eventdriven.py) on the
    interpreter, with the Cstack reductions of EventDrivenSyn / HybridSynDelay.backward."""
    x, W, p = inp["x"], inp["W"], inp["p"]
    d = inp["d"] + 0.0 + 1.0 * inp["offsets"] if kind == "hybrid" else inp["d"]
    T, B, N = x.shape
    decay, charge, vr, soft = _lif_consts(tau, v_reset)
    if use_sig_p:
        s_vec = 1.0 + 2.0 * float(sigma) * torch.sigmoid(p)
    else:
        s_vec = torch.full((N,), 1.0 + float(sigma))
    s_max = float(s_vec.max())
    L = int(math.ceil(1.0 + float(d.max()) + s_max)) + 1
    MAXR = int(math.ceil(s_max)) + 1
    Wt = W.t().contiguous()
    dt = d.t().contiguous()
    keep = inp["keep"] if inp["keep"] is not None else torch.ones(B, N)
    use_bias = inp["bias"] is not None
    bias = inp["bias"] if use_bias else torch.zeros(N)
    buf = torch.zeros(B, L, N)
    y = torch.empty(T, B, N)
    u = torch.empty(T, B, N)
    fired = torch.empty(B, N, dtype=torch.int32)
    BN = 1 << (N - 1).bit_length()
    ref_ed._ed_scatter_compact_kernel[(B,)](
        x, Wt, dt, s_vec, bias, keep, y, buf, fired, u, decay, charge, 1.0, vr, T, B,
        N=N, L=L, MAXR=MAXR, BLOCK_N=BN, USE_BIAS=use_bias, STORE_U=True, SOFT=soft)
    gy = inp["gy"]
    gr = torch.zeros(T, B, N)
    dx = torch.empty(T, B, N)
    sid = 1 if surr == "atan" else 0
    ref_ed._ed_bwd_kernel[(B,)](
        gy, u, keep, W.contiguous(), d.contiguous(), s_vec, gr, dx,
        decay, 1.0, vr, 1.0, 2.0, T, B,
        N=N, L=L, MAXR=MAXR, BLOCK_N=BN, SOFT=soft, DETACH=bool(detach_reset), SURR=sid)
    out = dict(y=y, u=u, gr=gr, dx=dx)
    if use_bias:
        out["dbias"] = gr.sum(dim=(0, 1))
    d_ = d.detach().clone().requires_grad_(True)
    p_ = p.clone().requires_grad_(use_sig_p) if use_sig_p else None
    mask3, Lm = build_syn_mask(d_, sigma, p_, use_sig_p)
    C = torch.zeros(N, N, Lm)
    for l in range(1, min(Lm, T)):
        M = T - l
        C[:, :, l] = gr[l:T].reshape(M * B, N).t() @ y[0:M].reshape(M * B, N)
    out["dW"] = (mask3.detach() * C).sum(-1)
    if kind == "hybrid" and not use_sig_p:
        dd_full = ref_delay_grad(C, W, d, sigma, Lm)
        out["dd_full"] = dd_full
        out["dd"] = dd_full.sum(0)          # the parametrization's broadcast-add backward
    else:
        # the event-driven Function's reductions; a hybrid layer with use_sig_p takes this
        # path too, because the hybrid kernel refuses per-source widths
        # (synaptic_hybrid.py:56, 140) and synaptic_recdel.forward falls back to it
        targets = [d_] + ([p_] if use_sig_p else [])
        grads = torch.autograd.grad(mask3, targets, grad_outputs=W.unsqueeze(-1) * C,
                                    allow_unused=True)
        out["dd"] = grads[0].sum(0) if kind == "hybrid" else grads[0]
        if use_sig_p:
            out["dp"] = grads[1]
    return out


def triton_cdiv(a, b):
    return (a + b - 1) // b


def ref_delay_grad(C, W, d, sigma, Lm):
    """synaptic_hybrid._delay_grad with the autotuner bypassed (the interpreter has no
    device to benchmark on): the same jitted kernel at one fixed tile."""
    N = W.shape[0]
    s = 1.0 + float(sigma)
    Ct = C.permute(1, 0, 2).contiguous()
    Wt = W.t().contiguous()
    dt = d.t().contiguous()
    dd_t = torch.empty(N, N)
    kern = ref_hy._hybrid_dd_kernel.fn
    kern[(triton_cdiv(N, 16),)](Ct, Wt, dt, dd_t, s, 1.0 / (s * s), N=N, LM=Lm, BLOCK_O=16)
    return dd_t.t().contiguous()


CASES = [
    # name, kind, seed, T, B, N, sigma, use_sig_p, bias, dropout, dmax, K, tau, v_reset, surr, detach
    ("ax_basic", "axonal", 1, 12, 3, 8, 0.0, False, False, False, 4.0, 0, 2.0, 0.0, "atan", False),
    ("ax_sigma_sigp", "axonal", 2, 14, 4, 12, 1.0, True, True, False, 5.0, 0, 2.0, None, "triangle", False),
    ("ax_odd_drop", "axonal", 3, 16, 5, 33, 0.5, False, True, True, 6.0, 0, 3.0, 0.0, "atan", True),
    ("ax_short_T", "axonal", 4, 5, 2, 7, 0.0, False, False, False, 9.0, 0, 2.0, 0.0, "atan", False),
    ("syn_basic", "synaptic", 5, 12, 3, 8, 0.0, False, False, False, 4.0, 0, 2.0, 0.0, "atan", False),
    ("syn_sigma_sigp", "synaptic", 6, 14, 3, 10, 1.5, True, True, False, 5.0, 0, 2.0, None, "triangle", False),
    ("syn_odd_drop", "synaptic", 7, 16, 4, 33, 0.7, False, True, True, 6.0, 0, 2.0, 0.0, "atan", True),
    ("hyb_basic", "hybrid", 8, 12, 3, 8, 0.0, False, False, False, 4.0, 3, 2.0, 0.0, "atan", False),
    ("hyb_sigma_bias", "hybrid", 9, 16, 4, 24, 0.5, False, True, False, 6.0, 4, 2.0, 0.0, "atan", False),
    ("hyb_soft_drop", "hybrid", 10, 14, 3, 17, 0.0, False, False, True, 5.0, 2, 2.0, None, "atan", False),
    # hard reset to a nonzero value: charge v - (v - v_reset)/tau + a, membrane starts at v_reset
    ("ax_vreset", "axonal", 15, 14, 4, 12, 0.5, False, True, False, 5.0, 0, 2.0, -0.5, "atan", False),
    ("syn_vreset", "synaptic", 16, 12, 3, 10, 0.5, False, False, False, 5.0, 0, 2.0, 0.3, "triangle", False),
    ("hyb_vreset", "hybrid", 17, 14, 3, 12, 0.0, False, True, False, 5.0, 3, 3.0, -0.5, "atan", True),
    # per-source triangle widths (use_sig_p) on the hybrid layer
    ("hyb_sigp", "hybrid", 18, 12, 3, 14, 1.0, True, True, False, 5.0, 3, 2.0, 0.0, "triangle", False),
]


# hard-tap axonal variants: name, seed, T, B, N, sigma, use_sig_p, bias, dropout, dmax,
# tau, v_reset, surr, detach, special delays (None: uniform in [0, dmax))
HARD_CASES = [
    ("hard_basic", 11, 12, 3, 8, 0.0, False, False, False, 4.0, 2.0, 0.0, "atan", False, None),
    ("hard_sigp_bias", 12, 14, 4, 12, 1.0, True, True, False, 5.0, 2.0, None, "triangle", False, None),
    ("hard_odd_drop", 13, 16, 5, 33, 0.5, False, True, True, 6.0, 3.0, 0.0, "atan", True, None),
    # ties of the rounding (half to even), integer delays and a negative delay
    ("hard_edges", 14, 15, 3, 10, 0.5, False, False, False, 4.0, 2.0, 0.0, "atan", False,
     [0.0, 0.5, 1.5, 2.5, 1.0, 3.0, -0.4, 2.25, 3.75, 0.99]),
]


def make_hard():
    out = []
    for (name, seed, T, B, N, sigma, sigp, bias, drop, dmax, tau, vr, surr, det, dspec) in HARD_CASES:
        inp = make_inputs(seed, T, B, N, "axonal", sigma, sigp, bias, drop, dmax)
        if dspec is not None:
            inp["d"] = torch.tensor(dspec)
        for mode in (1, 2, 3):
            res = run_triton_axonal_hard(inp, sigma, sigp, tau, vr, surr, det, mode)
            meta = dict(name=name, kind="axonal", mode=mode, T=T, B=B, N=N, sigma=sigma,
                        use_sig_p=sigp, tau=tau, v_reset=vr, surr=surr, detach_reset=det)
            out.append(dict(meta=meta, inputs=inp, triton=res))
            print(f"{name:16s} mode {mode}: spikes {int(res['y'].sum())}", flush=True)
    torch.save(out, os.path.join(HERE, "ax_hard.pt"))


def main():
    torch.set_num_threads(4)
    if "--hard-only" in sys.argv:
        make_hard()
        return
    only = sys.argv[sys.argv.index("--only") + 1].split(",") if "--only" in sys.argv else None
    for (name, kind, seed, T, B, N, sigma, sigp, bias, drop, dmax, K, tau, vr, surr,
         det) in CASES:
        if only is not None and name not in only:
            continue
        inp = make_inputs(seed, T, B, N, kind, sigma, sigp, bias, drop, dmax, K)
        v2 = run_v2(kind, inp, sigma, sigp, tau, vr, surr, det)
        if kind == "axonal":
            tri = run_triton_axonal(inp, sigma, sigp, tau, vr, surr, det)
        else:
            tri = run_triton_synaptic(kind, inp, sigma, sigp, tau, vr, surr, det)
        meta = dict(name=name, kind=kind, T=T, B=B, N=N, sigma=sigma, use_sig_p=sigp,
                    tau=tau, v_reset=vr, surr=surr, detach_reset=det, K=K)
        torch.save(dict(meta=meta, inputs=inp, v2=v2, triton=tri),
                   os.path.join(HERE, f"{name}.pt"))
        ydiff = (v2["y"] != tri["y"]).sum().item()
        gd = max(((v2[k] - tri[k]).abs().max() / (v2[k].abs().max() + 1e-12)).item()
                 for k in ("dx", "dW", "dd") if k in tri)
        print(f"{name:16s} L-case ok: spikes v2 vs triton differ at {ydiff}, "
              f"max rel grad diff {gd:.2e}", flush=True)
    if only is not None:
        return

    # closed-form hybrid delay gradient at integer / support-edge delays, through the
    # reference's fused kernel (tests/check_hybrid_kernel.py:131-154 values)
    dd_cases = []
    values = torch.tensor([0., 1., 2., 0.25, 1.5])
    for sigma in (0., 0.5, 1.):
        d = values.repeat(5, 1)
        W = torch.arange(1, 26).float().reshape(5, 5) / 25
        _, L = build_syn_mask(d, sigma, None, False)
        C = torch.arange(L).float().square().expand(5, 5, L).contiguous()
        dd = ref_delay_grad(C, W, d, sigma, L)
        dd_cases.append(dict(sigma=sigma, d=d, W=W, C=C, dd=dd))
    torch.save(dd_cases, os.path.join(HERE, "hybrid_dd_edges.pt"))
    print("hybrid_dd_edges ok")
    make_hard()


if __name__ == "__main__":
    main()
