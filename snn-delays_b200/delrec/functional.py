"""Autograd Functions of the delay-LIF hot path, backed by libdelrec_b200.so.

They keep the ``.apply`` argument lists of the reference's Triton Functions, so code
that called those keeps working:

* :class:`AxonalRecdelTriton`  src/delrec/triton_kernels/recdel_base.py:349-439
* :class:`EventDrivenSyn`      src/delrec/triton_kernels/synaptic_eventdriven.py:379-471
* :class:`HybridSynDelay`      src/delrec/triton_kernels/synaptic_hybrid.py:133-211
  (the (N,N) delay is materialised; its gradient is the per-synapse closed form)

plus :class:`HybridBaseDelay`, the hybrid path used by the modules: it takes the learned
(N,) base and the frozen (N,N) offsets directly and returns the base gradient without
materialising (N,N) delay gradients, and :class:`LIFMultiStep` / :class:`DclsConv1d`.
All of them run on CUDA only.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

# ---------------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------------


def half_widths(sigma, p_spread, use_sig_p, N, device):
    """s per source: 1 + 2 sigma sigmoid(p) under use_sig_p, else 1 + sigma
    (delay_layers_pytorch.py:135-141)."""
    if use_sig_p:
        return (1.0 + 2.0 * float(sigma) * torch.sigmoid(p_spread.detach().float())).contiguous()
    return torch.full((N,), 1.0 + float(sigma), device=device, dtype=torch.float32)


def ring_length(d_max, s_max) -> int:
    """L = ceil(1 + max d + s_max) + 1 (delay_layers_pytorch.py:145); one host sync."""
    return int(torch.ceil(1.0 + d_max + s_max).item()) + 1


# Host copies of device-side reductions that size the kernel launches (largest delay,
# widest triangle, smallest base, largest offset).  They are read back (one host
# synchronisation) only when a tensor they depend on changed since the last call: a
# tensor is identified by the object itself and its in-place version counter, which an
# optimizer step or a clamp_ advances, so a training step syncs once per layer and
# repeated forwards between two updates (evaluation, micro-batches) do not sync at all.
_STATS: dict = {}


def _cached_stats(tag, tensors, compute):
    import weakref
    key = (tag,) + tuple(id(t) if t is not None else None for t in tensors)
    try:
        vers = tuple(t._version if t is not None else None for t in tensors)
    except RuntimeError:   # inference-mode tensors carry no version counter
        return compute()
    hit = _STATS.get(key)
    if hit is not None:
        refs, v, vals = hit
        if v == vers and all((r() is t) if t is not None else r is None for r, t in zip(refs, tensors)):
            return vals
    vals = compute()
    if len(_STATS) > 512:
        _STATS.clear()
    _STATS[key] = (tuple(weakref.ref(t) if t is not None else None for t in tensors), vers, vals)
    return vals


def _s_max(sigma, p_spread, use_sig_p, s):
    """The widest half-width: a host value unless the widths are learned per source."""
    if use_sig_p:
        return None
    return 1.0 + float(sigma)


def surrogate_params(config):
    """(surrogate id, gamma, alpha) exactly as the reference's shims derive them from
    ``config.surrogate_function`` (delay_layers_triton.py:28-35, 58)."""
    from .utils import Triangle
    surr = config.surrogate_function
    gamma = float(getattr(config, "surrogate_gamma", 1.0))
    if surr is Triangle.apply:
        return _lib.SURR_TRIANGLE, gamma, 2.0
    if "ATan" in type(surr).__name__:
        return _lib.SURR_ATAN, gamma, float(getattr(surr, "alpha", 2.0))
    return _lib.SURR_TRIANGLE, gamma, 2.0


def lif_from_layer(layer) -> _lib.LIF:
    nm = layer.neuron_module
    sid, gamma, alpha = surrogate_params(layer.config)
    return _lib.lif_struct(nm.tau, nm.v_threshold, nm.v_reset, layer.config.detach_reset,
                           sid, gamma, alpha)


def _layer(kind, T, B, N, L, K, has_bias, has_keep, s_max, d_min=0.0):
    return _lib.Layer(kind, T, B, N, L, K, int(has_bias), int(has_keep), float(s_max), float(d_min))


# The library's factored hybrid backward takes base windows reaching at most one lag below
# lag 1; wider ones (bases near or below zero with a wide triangle) run the per-synapse path.
HYBRID_MM_MAX = 1


def hybrid_thresholds(base_min, s_max, K):
    """How far below lag 1 the learned base's triangle window reaches (the number of
    offset thresholds the hybrid backward tracks), in float32 exactly like the library."""
    import numpy as np
    onepd = np.float32(1.0) + np.float32(base_min)
    s = np.float32(s_max)
    l = int(np.floor(onepd - s)) - 1
    while not (s - np.abs(np.float32(l) - onepd) >= 0) and l < 1:
        l += 1
    return max(0, min(1 - l, int(K)))


def _keep2d(drop, B, N):
    if drop is None:
        return None
    if drop.dim() == 3:          # the reference passes the fixed mask expanded over T
        drop = drop[0]
    return drop.detach().float().contiguous()


def _run(fn, *args):
    _lib.check(getattr(_lib.lib(), fn)(*args), fn)


# ---------------------------------------------------------------------------------
# generic layer forward / backward through the C-ABI
# ---------------------------------------------------------------------------------


def layer_forward(kind, x, W, bias, d, offsets, s, keep, L, K, lif, s_max=None, d_min=0.0):
    x = x.detach().contiguous()
    T, B, N = x.shape
    W = W.detach().contiguous()
    d = d.detach().contiguous()
    _lib.require_cuda(x, W, d, s, bias, keep, offsets)
    s_max = float(s.max()) if s_max is None else float(s_max)
    desc = _layer(kind, T, B, N, L, K, bias is not None, keep is not None, s_max, d_min)
    y = torch.empty_like(x)
    u = torch.empty_like(x)
    wsfn = {_lib.AXONAL: "delrec_axonal_forward_workspace",
            _lib.SYNAPTIC: "delrec_synaptic_forward_workspace",
            _lib.HYBRID: "delrec_hybrid_forward_workspace"}[kind]
    nbytes = getattr(_lib.lib(), wsfn)(ctypes.byref(desc))
    ws = _lib.workspace(nbytes, x.device)
    st = _lib.stream_ptr(x.device)
    P = _lib.ptr
    if kind == _lib.HYBRID:
        _run("delrec_hybrid_forward", ctypes.byref(desc), ctypes.byref(lif), P(x), P(W), P(bias), P(d),
             P(offsets), P(s), P(keep), P(y), P(u), P(ws), ws.numel(), st)
    else:
        fn = "delrec_axonal_forward" if kind == _lib.AXONAL else "delrec_synaptic_forward"
        _run(fn, ctypes.byref(desc), ctypes.byref(lif), P(x), P(W), P(bias), P(d), P(s), P(keep),
             P(y), P(u), P(ws), ws.numel(), st)
    return y, u, desc


def layer_backward(kind, desc, lif, gy, u, y, W, d, offsets, s, keep, need, hard=None):
    """The layer's backward through the C-ABI; ``hard`` = (mode, d_hard) runs the axonal
    hard-tap backward (delrec_axonal_backward_hard) instead."""
    gy = gy.detach().contiguous()
    _lib.require_cuda(gy)
    T, B, N = gy.shape
    dev = gy.device
    dx = torch.empty_like(gy)
    dW = torch.empty(N, N, device=dev) if need.get("W") else None
    db = torch.empty(N, device=dev) if need.get("bias") else None
    dshape = (N, N) if kind == _lib.SYNAPTIC else (N,)
    dd = torch.empty(dshape, device=dev) if need.get("d") else None
    ds = torch.empty(N, device=dev) if need.get("s") else None
    P = _lib.ptr
    g = _lib.Grads(dx.data_ptr(), dW.data_ptr() if dW is not None else None,
                   db.data_ptr() if db is not None else None,
                   dd.data_ptr() if dd is not None else None,
                   ds.data_ptr() if ds is not None else None)
    wsfn = {_lib.AXONAL: "delrec_axonal_backward_workspace",
            _lib.SYNAPTIC: "delrec_synaptic_backward_workspace",
            _lib.HYBRID: "delrec_hybrid_backward_workspace"}[kind]
    if hard is not None:
        wsfn = "delrec_axonal_backward_hard_workspace"
    nbytes = getattr(_lib.lib(), wsfn)(ctypes.byref(desc))
    ws = _lib.workspace(nbytes, dev)
    st = _lib.stream_ptr(dev)
    if hard is not None:
        mode, d_hard = hard
        _run("delrec_axonal_backward_hard", ctypes.byref(desc), ctypes.byref(lif), mode, P(gy), P(u),
             P(y), P(W), P(d), P(s), P(d_hard), P(keep), ctypes.byref(g), P(ws), ws.numel(), st)
    elif kind == _lib.HYBRID:
        _run("delrec_hybrid_backward", ctypes.byref(desc), ctypes.byref(lif), P(gy), P(u), P(y), P(W),
             P(d), P(offsets), P(s), P(keep), ctypes.byref(g), P(ws), ws.numel(), st)
    else:
        fn = "delrec_axonal_backward" if kind == _lib.AXONAL else "delrec_synaptic_backward"
        _run(fn, ctypes.byref(desc), ctypes.byref(lif), P(gy), P(u), P(y), P(W), P(d), P(s), P(keep),
             ctypes.byref(g), P(ws), ws.numel(), st)
    return dx, dW, db, dd, ds


def _dp_from_ds(ds, p_spread, sigma):
    """chain rule of s = 1 + 2 sigma sigmoid(p)"""
    sg = torch.sigmoid(p_spread.detach().float())
    return ds * (2.0 * float(sigma)) * sg * (1.0 - sg)


# ---------------------------------------------------------------------------------
# axonal
# ---------------------------------------------------------------------------------


def hard_delays(d, dmax, L, mode):
    """The hard taps of the rounded / interpolated axonal forwards written as delays of a
    half-width-1 triangle (delays.py:33-47 build_lag / build_lag_interp, taken on the
    reference's own ring length L), and the largest of them as a host float.
    mode 1 (STE rounded) and 3 (approx): one tap at lag = clamp(round(d) + 1, 1, L - 1),
    delay lag - 1; mode 2 (STE interpolated): lag = clamp(floor(1 + d), 1, L - 1),
    f = clamp(1 + d - lag, 0, 1), delay (lag - 1) + f, whose triangle weighs lag by 1 - f
    and lag + 1 by f exactly."""
    import numpy as np
    dd = d.detach().float()
    hi = float(max(1, L - 1))
    if mode == 2:
        pos = 1.0 + dd
        lag = torch.floor(pos).clamp_(1.0, hi)
        d_hard = (lag - 1.0) + (pos - lag).clamp_(0.0, 1.0)
        p32 = np.float32(1.0) + np.float32(dmax)
        l32 = np.float32(min(max(np.floor(p32), 1.0), hi))
        dh_max = float((l32 - np.float32(1.0)) + np.float32(min(max(p32 - l32, 0.0), 1.0)))
    else:
        d_hard = (torch.round(dd) + 1.0).clamp_(1.0, hi) - 1.0
        dh_max = min(max(float(np.round(np.float32(dmax))) + 1.0, 1.0), hi) - 1.0
    return d_hard.contiguous(), dh_max


class AxonalRecdelTriton(torch.autograd.Function):
    """Axonal delay layer (per-source delay d (N,)).  Same arguments as the reference's
    ``AxonalRecdelTriton.apply`` (recdel_base.py:351-353); ``drop`` may be the (T,B,N)
    expanded fixed mask or the (B,N) mask itself.

    ``ste_mode`` 1 / 2 (forward_version 'triton_ste'): the forward runs on the hard taps
    (rounded lag, or the 2-tap interpolation), the backward is the soft triangle's except
    the weight gradient, which correlates with the forward's hard z (recdel_base.py:
    356-372, 401-412).  ``approx`` ('triton_approx'): the single rounded tap forward and
    its own backward, with the straight-through delay gradient
    dd = sum gz(t) (y(t-lag-1) - y(t-lag)) and no spread gradient (recdel_base.py:373-378,
    265-278, 416-419).  The hard forwards run the same kernels as the soft one, at
    half-width 1 with the taps written as delays (``hard_delays``)."""

    @staticmethod
    def forward(ctx, x, W, bias, d, p_spread, drop, sigma, tau, v_th, v_reset, use_sig_p,
                detach_reset, surr_id, gamma=1.0, approx=False, ste_mode=0, alpha=2.0):
        T, B, N = x.shape
        s = half_widths(sigma, p_spread, use_sig_p, N, x.device)
        sm = _s_max(sigma, p_spread, use_sig_p, s)
        if sm is None:
            dmax, sm = _cached_stats(("ax", float(sigma)), (d, p_spread),
                                     lambda: torch.stack([d.detach().max().float(), s.max()]).tolist())
        else:
            dmax = _cached_stats("ax", (d,), lambda: [float(d.detach().max())])[0]
        L = ring_length(torch.tensor(dmax, dtype=torch.float32), torch.tensor(sm, dtype=torch.float32))
        lif = _lib.lif_struct(tau, v_th, v_reset, detach_reset, surr_id, gamma, alpha)
        keep = _keep2d(drop, B, N)
        b = bias.detach().float().contiguous() if bias is not None else None
        ste_mode = int(ste_mode) if ste_mode else 0
        if ste_mode not in (0, 1, 2):
            raise ValueError(f"ste_mode must be 0, 1 or 2, got {ste_mode}")
        mode = ste_mode if ste_mode else (3 if approx else 0)
        if mode == 0:
            y, u, desc = layer_forward(_lib.AXONAL, x, W, b, d, None, s, keep, L, 0, lif, s_max=sm)
            d_hard = torch.empty(0)
        else:
            # approx sizes its taps on Lmax = round(max d) + 2 (recdel_base.py:374-375)
            Lh = L if mode != 3 else int(round(dmax)) + 2
            d_hard, dh_max = hard_delays(d, dmax, Lh, 2 if mode == 2 else 1)
            ones = torch.ones(N, device=x.device, dtype=torch.float32)
            Lf = ring_length(torch.tensor(dh_max, dtype=torch.float32), torch.tensor(1.0))
            y, u, desc = layer_forward(_lib.AXONAL, x, W, b, d_hard, None, ones, keep, Lf, 0, lif,
                                       s_max=1.0)
            if mode != 3:   # the STE backward runs on the soft triangle's ring
                desc = _layer(_lib.AXONAL, T, B, N, L, 0, b is not None, keep is not None, sm)
        ctx.save_for_backward(u, y, W, d, s, keep if keep is not None else torch.empty(0), p_spread,
                              d_hard)
        ctx.meta = (desc, lif, sigma, use_sig_p, keep is not None, mode)
        return y

    @staticmethod
    def backward(ctx, gy):
        u, y, W, d, s, keep, p_spread, d_hard = ctx.saved_tensors
        desc, lif, sigma, use_sig_p, has_keep, mode = ctx.meta
        need = dict(W=ctx.needs_input_grad[1], bias=ctx.needs_input_grad[2],
                    d=ctx.needs_input_grad[3], s=use_sig_p and ctx.needs_input_grad[4])
        Wc = W.detach().contiguous()
        kp = keep if has_keep else None
        if mode == 0:
            dx, dW, db, dd, ds = layer_backward(_lib.AXONAL, desc, lif, gy, u, y, Wc,
                                                d.detach().contiguous(), None, s, kp, need)
        elif mode == 3:
            need["s"] = False
            ones = torch.ones_like(d_hard)
            dx, dW, db, dd, ds = layer_backward(_lib.AXONAL, desc, lif, gy, u, y, Wc, d_hard, None,
                                                ones, kp, need, hard=(_lib.HARD_APPROX, None))
        else:
            dx, dW, db, dd, ds = layer_backward(_lib.AXONAL, desc, lif, gy, u, y, Wc,
                                                d.detach().contiguous(), None, s, kp, need,
                                                hard=(_lib.HARD_STE, d_hard))
        dp = _dp_from_ds(ds, p_spread, sigma) if ds is not None else None
        return (dx, dW, db, dd, dp) + (None,) * 12


# ---------------------------------------------------------------------------------
# synaptic (and the reference-signature hybrid)
# ---------------------------------------------------------------------------------


def _effective_d(d, layer):
    return d.detach().round() if getattr(layer, "round_delays", False) else d.detach()


class EventDrivenSyn(torch.autograd.Function):
    """Synaptic delay layer, d (N,N) with d[i,o] target i source o; same arguments as
    the reference (synaptic_eventdriven.py:386): (x, W, d, p_spread, bias, drop, layer)."""

    @staticmethod
    def forward(ctx, x, W, d, p_spread, bias, drop, layer):
        T, B, N = x.shape
        d_eff = _effective_d(d, layer).float().contiguous()
        s = half_widths(layer.sigma, p_spread, layer.use_sig_p, N, x.device)
        rnd = bool(getattr(layer, "round_delays", False))
        sm = _s_max(layer.sigma, p_spread, layer.use_sig_p, s)
        if sm is None:
            dmax, sm = _cached_stats(("syn", rnd, float(layer.sigma)), (d, p_spread),
                                     lambda: torch.stack([d_eff.max(), s.max()]).tolist())
        else:
            dmax = _cached_stats(("syn", rnd), (d,), lambda: [float(d_eff.max())])[0]
        L = ring_length(torch.tensor(dmax, dtype=torch.float32), torch.tensor(sm, dtype=torch.float32))
        lif = lif_from_layer(layer)
        keep = _keep2d(drop, B, N)
        b = bias.detach().float().contiguous() if bias is not None else None
        y, u, desc = layer_forward(_lib.SYNAPTIC, x, W, b, d_eff, None, s, keep, L, 0, lif, s_max=sm)
        ctx.save_for_backward(u, y, W, d_eff, s, keep if keep is not None else torch.empty(0), p_spread)
        ctx.meta = (desc, lif, float(layer.sigma), bool(layer.use_sig_p), keep is not None)
        return y

    @staticmethod
    def backward(ctx, gy):
        u, y, W, d_eff, s, keep, p_spread = ctx.saved_tensors
        desc, lif, sigma, use_sig_p, has_keep = ctx.meta
        need = dict(W=ctx.needs_input_grad[1], d=ctx.needs_input_grad[2],
                    s=use_sig_p and ctx.needs_input_grad[3], bias=ctx.needs_input_grad[4])
        dx, dW, db, dd, ds = layer_backward(_lib.SYNAPTIC, desc, lif, gy, u, y, W.detach().contiguous(),
                                            d_eff, None, s, keep if has_keep else None, need)
        dp = _dp_from_ds(ds, p_spread, sigma) if ds is not None else None
        return dx, dW, dd, dp, db, None, None


class HybridSynDelay(torch.autograd.Function):
    """Reference-signature hybrid path (synaptic_hybrid.py:139): ``d`` is the materialised
    (N,N) delay base[o] + offsets[i,o]; the gradient of ``d`` is the per-synapse
    closed form, reduced to the base by the caller's parametrization."""

    @staticmethod
    def forward(ctx, x, W, d, bias, drop, layer):
        if getattr(layer, "use_sig_p", False):
            raise ValueError("hybrid kernel: use_sig_p not supported (as in the reference)")
        T, B, N = x.shape
        d_eff = _effective_d(d, layer).float().contiguous()
        s = half_widths(layer.sigma, None, False, N, x.device)
        L = ring_length(d_eff.max(), s.max())
        lif = lif_from_layer(layer)
        keep = _keep2d(drop, B, N)
        b = bias.detach().float().contiguous() if bias is not None else None
        y, u, desc = layer_forward(_lib.SYNAPTIC, x, W, b, d_eff, None, s, keep, L, 0, lif)
        ctx.save_for_backward(u, y, W, d_eff, s, keep if keep is not None else torch.empty(0))
        ctx.meta = (desc, lif, keep is not None)
        return y

    @staticmethod
    def backward(ctx, gy):
        u, y, W, d_eff, s, keep = ctx.saved_tensors
        desc, lif, has_keep = ctx.meta
        need = dict(W=ctx.needs_input_grad[1], d=ctx.needs_input_grad[2], s=False,
                    bias=ctx.needs_input_grad[3])
        dx, dW, db, dd, _ = layer_backward(_lib.SYNAPTIC, desc, lif, gy, u, y, W.detach().contiguous(),
                                           d_eff, None, s, keep if has_keep else None, need)
        return dx, dW, dd, db, None, None


# ---------------------------------------------------------------------------------
# hybrid (module path): learned base (N,) + frozen integer offsets (N,N)
# ---------------------------------------------------------------------------------


class HybridBaseDelay(torch.autograd.Function):
    """(x, W, base, offsets, p_spread, bias, drop, layer) -> spikes.  Gradients for x, W,
    base (already summed over targets, as the parametrization would), p_spread, bias.

    The backward factors each synapse's delay into the learned base (axonal taps) and its
    frozen integer offset.  When the base's triangle reaches more than HYBRID_MM_MAX lags
    below lag 1 (very negative bases or wide sigma) it runs the per-synapse kernels on the
    materialised delay instead and sums the (N,N) delay gradient over the targets."""

    @staticmethod
    def forward(ctx, x, W, base, offsets, p_spread, bias, drop, layer):
        T, B, N = x.shape
        base_eff = _effective_d(base, layer).float().contiguous()
        off = offsets.detach().float().contiguous()
        s = half_widths(layer.sigma, p_spread, layer.use_sig_p, N, x.device)
        # every scalar the launch needs, read back once per update of base / p_spread
        rnd = bool(getattr(layer, "round_delays", False))
        stats = _cached_stats(("hyb", rnd, float(layer.sigma), bool(layer.use_sig_p)),
                              (base, offsets, p_spread if layer.use_sig_p else None),
                              lambda: torch.stack([base_eff.max() + off.max(), s.max(), base_eff.min(),
                                                   off.max()]).tolist())
        dmax, s_max, base_min, off_max = stats
        K = int(round(off_max)) if off.numel() else 0
        L = int(math.ceil(1.0 + dmax + s_max)) + 1
        Lt = ring_length(torch.tensor(dmax, dtype=torch.float32), torch.tensor(s_max, dtype=torch.float32))
        L = max(L, Lt)
        lif = lif_from_layer(layer)
        keep = _keep2d(drop, B, N)
        b = bias.detach().float().contiguous() if bias is not None else None
        mm = hybrid_thresholds(base_min, s_max, K)
        if mm <= HYBRID_MM_MAX:
            y, u, desc = layer_forward(_lib.HYBRID, x, W, b, base_eff, off, s, keep, L, K, lif,
                                       s_max=s_max, d_min=base_min)
            kind, dsave = _lib.HYBRID, base_eff
        else:
            d_full = (base_eff[None, :] + 0.0 + 1.0 * off).contiguous()
            y, u, desc = layer_forward(_lib.SYNAPTIC, x, W, b, d_full, None, s, keep, L, 0, lif,
                                       s_max=s_max)
            kind, dsave = _lib.SYNAPTIC, d_full
        ctx.save_for_backward(u, y, W, dsave, off, s, keep if keep is not None else torch.empty(0),
                              p_spread)
        ctx.meta = (desc, lif, float(layer.sigma), bool(layer.use_sig_p), keep is not None, kind)
        return y

    @staticmethod
    def backward(ctx, gy):
        u, y, W, dsave, off, s, keep, p_spread = ctx.saved_tensors
        desc, lif, sigma, use_sig_p, has_keep, kind = ctx.meta
        need = dict(W=ctx.needs_input_grad[1], d=ctx.needs_input_grad[2],
                    s=use_sig_p and ctx.needs_input_grad[4], bias=ctx.needs_input_grad[5])
        dx, dW, db, dd, ds = layer_backward(kind, desc, lif, gy, u, y, W.detach().contiguous(),
                                            dsave, off if kind == _lib.HYBRID else None, s,
                                            keep if has_keep else None, need)
        if kind == _lib.SYNAPTIC and dd is not None:
            dd = dd.sum(0)
        dp = _dp_from_ds(ds, p_spread, sigma) if ds is not None else None
        return dx, dW, dd, None, dp, db, None, None


def hybrid_delay_grad(C, W, d, sigma):
    """Closed-form per-synapse delay gradient (synaptic_hybrid.py:116-126)."""
    C = C.detach().float().contiguous()
    W = W.detach().float().contiguous()
    d = d.detach().float().contiguous()
    _lib.require_cuda(C, W, d)
    N, LM = W.shape[0], C.shape[-1]
    out = torch.empty(N, N, device=C.device)
    P = _lib.ptr
    _run("delrec_hybrid_delay_grad", N, LM, P(C), P(W), P(d), float(sigma), P(out),
         _lib.stream_ptr(C.device))
    return out


def build_mask(d, s, L):
    """Dense triangle mask (rows of d, lags 0..L-1); s per row (axonal) or per source
    column (synaptic (N,N) d)."""
    d = d.detach().float().contiguous()
    s = s.detach().float().contiguous()
    _lib.require_cuda(d, s)
    R = d.numel()
    period = s.numel()
    out = torch.empty(*d.shape, L, device=d.device)
    _run("delrec_build_mask", R, L, _lib.ptr(d), _lib.ptr(s), period, _lib.ptr(out),
         _lib.stream_ptr(d.device))
    return out


# ---------------------------------------------------------------------------------
# plain multi-step LIF
# ---------------------------------------------------------------------------------


class LIFMultiStep(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, lif_args):
        x = x.detach().contiguous()
        _lib.require_cuda(x)
        T = x.shape[0]
        M = x.numel() // T
        lif = _lib.lif_struct(*lif_args)
        y = torch.empty_like(x)
        u = torch.empty_like(x)
        P = _lib.ptr
        _run("delrec_lif_forward", T, M, ctypes.byref(lif), P(x), P(y), P(u), _lib.stream_ptr(x.device))
        ctx.save_for_backward(u)
        ctx.lif = lif
        ctx.TM = (T, M)
        return y

    @staticmethod
    def backward(ctx, gy):
        (u,) = ctx.saved_tensors
        gy = gy.contiguous()
        dx = torch.empty_like(gy)
        T, M = ctx.TM
        P = _lib.ptr
        _run("delrec_lif_backward", T, M, ctypes.byref(ctx.lif), P(gy), P(u), P(dx),
             _lib.stream_ptr(gy.device))
        return dx, None


# ---------------------------------------------------------------------------------
# DCLS feedforward delay convolution
# ---------------------------------------------------------------------------------


class DclsConv1d(torch.autograd.Function):
    """(T,B,Cin) -> (T,B,Cout) causal conv with Gaussian-interpolated learnable positions.
    weight (Cout, Cin/groups, 1); P, SIG (1, Cout, Cin/groups, 1)."""

    @staticmethod
    def forward(ctx, x, weight, P, SIG, bias, K, groups, lpad):
        x = x.detach().contiguous()
        T, B, Cin = x.shape
        Cout = weight.shape[0]
        w = weight.detach().float().reshape(Cout, -1)[:, :].contiguous()
        p = P.detach().float().reshape(Cout, -1).contiguous()
        sg = SIG.detach().float().reshape(Cout, -1).contiguous()
        b = bias.detach().float().contiguous() if bias is not None else None
        _lib.require_cuda(x, w, p, sg, b)
        ker = torch.empty(Cout, Cin // groups, K, device=x.device)
        out = torch.empty(T, B, Cout, device=x.device)
        Pp = _lib.ptr
        _run("delrec_dcls_forward", T, B, Cin, Cout, groups, K, lpad, Pp(x), Pp(w), Pp(p), Pp(sg), Pp(b),
             Pp(ker), Pp(out), _lib.stream_ptr(x.device))
        ctx.save_for_backward(x, w, p, sg)
        ctx.meta = (K, groups, lpad, bias is not None, weight.shape, P.shape, SIG.shape)
        return out

    @staticmethod
    def backward(ctx, gout):
        x, w, p, sg = ctx.saved_tensors
        K, groups, lpad, has_bias, wshape, pshape, sshape = ctx.meta
        gout = gout.contiguous()
        T, B, Cin = x.shape
        Cout = w.shape[0]
        dev = x.device
        dx = torch.empty_like(x) if ctx.needs_input_grad[0] else None
        dw = torch.empty_like(w) if ctx.needs_input_grad[1] else None
        dP = torch.empty_like(p) if ctx.needs_input_grad[2] else None
        dS = torch.empty_like(sg) if ctx.needs_input_grad[3] else None
        db = torch.empty(Cout, device=dev) if (has_bias and ctx.needs_input_grad[4]) else None
        nbytes = _lib.lib().delrec_dcls_backward_workspace(T, B, Cin, Cout, groups, K)
        ws = _lib.workspace(nbytes, dev)
        Pp = _lib.ptr
        _run("delrec_dcls_backward", T, B, Cin, Cout, groups, K, lpad, Pp(x), Pp(w), Pp(p), Pp(sg),
             Pp(gout), Pp(dx), Pp(dw), Pp(dP), Pp(dS), Pp(db), Pp(ws), ws.numel(),
             _lib.stream_ptr(dev))
        rs = lambda t, shp: None if t is None else t.reshape(shp)
        return dx, rs(dw, wshape), rs(dP, pshape), rs(dS, sshape), db, None, None, None
