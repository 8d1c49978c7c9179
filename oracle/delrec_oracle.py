"""CPU oracle for the DelRec delay-LIF hot path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference arm of
``bench.py`` may import this module.  The product path (``delrec`` under
``snn-delays_b200/``) never imports it and has no CPU fallback.

This is a plain-PyTorch (CPU, fp32 by default) restatement of the reference's canonical
``multi_step_forward_v2`` scans, with backpropagation-through-time obtained from torch
autograd over the unrolled graph, exactly as the reference computes its gradients on
CPU.  It is written from the reference's documented equations, not copied:

* triangular delay kernel  h(l; d) = max(0, s - |l - (1 + d)|) / s^2, s = 1 + sigma
  or s_j = 1 + 2 sigma sigmoid(p_j) under ``use_sig_p``; ring length
  L = ceil(1 + max d + s_max) + 1, usable lags 1..L-1
  (src/delrec/delay_layers_pytorch.py:135-151, 200-218; triton_kernels/delays.py:13-63)
* axonal step   z[b,j] = sum_l h_j(l) y[t-l,b,j];  rec[b,i] = sum_j W[i,j] z[b,j] (+ bias_i)
  (delay_layers_pytorch.py:166-179)
* synaptic step rec[b,i] = sum_o sum_l W[i,o] h_io(l) y[t-l,b,o] (+ bias_i),
  s indexed by the source o (delay_layers_pytorch.py:283-310)
* hybrid delay  d[i,o] = base[o] + offsets[i,o] (src/delrec/networks.py:823-829), scanned
  with the synaptic step
* LIF neuron, SpikingJelly ``LIFNode`` single-step semantics with decay_input=False
  (the neuron the v2 scans call at delay_layers_pytorch.py:179,310; the reference
  restates the same algebra in triton_kernels/lif.py:24-56):
    charge  v = v * (1 - 1/tau) + a                (v_reset None or 0)
            v = v - (v - v_reset) / tau + a        (other hard resets)
    fire    s = heaviside(v - v_th)   (>= 0 is a spike; surrogate gradient backward)
    reset   v = (1 - s) v + s v_reset  (hard)   |   v = v - s v_th  (soft, v_reset None)
  initial v = v_reset (0.0 when v_reset is None)
* surrogates  ATan(alpha): (alpha/2) / (1 + (pi/2 alpha x)^2);
              Triangle(gamma): (1/gamma)^2 max(0, gamma - |x|)
  (triton_kernels/surrogate.py:20-27, src/delrec/utils.py:23-41)
* recurrent dropout: one keep-mask (values 0 or 1/(1-p)) per forward, applied to
  (rec + bias) at every step (delay_layers_triton.py:37-48, delay_layers_pytorch.py:179)

The functions are device-agnostic torch code: the parity tests evaluate them in float64 on
the CPU for small cases and, for the full BASELINE-shaped cases (where the CPU would take
hours), in float64 on the GPU; either way they are the checker, never the product.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own v2 scans (imported
unmodified) and its own Triton kernels (under the Triton CPU interpreter) on seeded
inputs; ``tests/test_oracle_golden.py`` checks this oracle against those fixtures.
"""

from __future__ import annotations

import math

import torch


# ----------------------------------------------------------------------------------
# surrogate spike functions (forward: heaviside with ties firing; backward: surrogate)
# ----------------------------------------------------------------------------------

class _HeavisideATan(torch.autograd.Function):
    """Spike = [x >= 0]; d spike / dx = (alpha/2) / (1 + (pi/2 * alpha * x)^2)."""

    @staticmethod
    def forward(ctx, x, alpha):
        ctx.save_for_backward(x)
        ctx.alpha = float(alpha)
        return (x >= 0).to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        a = ctx.alpha
        t = (math.pi / 2 * a) * x
        return (a / 2) / (1 + t * t) * g, None


class _HeavisideTriangle(torch.autograd.Function):
    """Spike = [x >= 0]; d spike / dx = (1/gamma)^2 * max(0, gamma - |x|)."""

    @staticmethod
    def forward(ctx, x, gamma):
        ctx.save_for_backward(x)
        ctx.gamma = float(gamma)
        return (x >= 0).to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        gm = ctx.gamma
        return g * ((1 / gm) * (1 / gm) * (gm - x.abs()).clamp(min=0)), None


class ATanSpike:
    """Callable surrogate: ``ATanSpike(alpha)(x)``."""

    def __init__(self, alpha: float = 2.0):
        self.alpha = float(alpha)

    def __call__(self, x):
        return _HeavisideATan.apply(x, self.alpha)


class TriangleSpike:
    """Callable surrogate: ``TriangleSpike(gamma)(x)``."""

    def __init__(self, gamma: float = 1.0):
        self.gamma = float(gamma)

    def __call__(self, x):
        return _HeavisideTriangle.apply(x, self.gamma)


# ----------------------------------------------------------------------------------
# LIF neuron (SpikingJelly LIFNode, single step, decay_input=False)
# ----------------------------------------------------------------------------------

class OracleLIF:
    """Single-step LIF neuron with explicit state ``v`` (a float until the first step).

    The membrane starts at v_reset (0 for the soft reset), as SpikingJelly's LIFNode and
    the reference's v2 scans have it.  ``v_init`` overrides that start: the reference's
    Triton kernels begin every scan at 0 (recdel_base.py:53, the same in the synaptic
    kernels), which differs from v2 only for a hard reset to a nonzero value."""

    def __init__(self, tau=2.0, v_threshold=1.0, v_reset=0.0, surrogate=None,
                 detach_reset=False, v_init=None):
        self.tau = float(tau)
        self.v_threshold = float(v_threshold)
        self.v_reset = None if v_reset is None else float(v_reset)
        self.surrogate = surrogate if surrogate is not None else ATanSpike(2.0)
        self.detach_reset = bool(detach_reset)
        self.v_init = None if v_init is None else float(v_init)
        self.reset()

    def reset(self):
        if self.v_init is not None:
            self.v = self.v_init
        else:
            self.v = 0.0 if self.v_reset is None else self.v_reset

    def single_step_forward(self, a):
        if not torch.is_tensor(self.v):
            self.v = torch.full_like(a, self.v)
        if self.v_reset is None or self.v_reset == 0.0:
            u = self.v * (1.0 - 1.0 / self.tau) + a
        else:
            u = self.v - (self.v - self.v_reset) / self.tau + a
        s = self.surrogate(u - self.v_threshold)
        sd = s.detach() if self.detach_reset else s
        if self.v_reset is None:
            self.v = u - sd * self.v_threshold
        else:
            self.v = (1.0 - sd) * u + sd * self.v_reset
        self.u = u
        return s


# ----------------------------------------------------------------------------------
# triangular delay kernel
# ----------------------------------------------------------------------------------

def spread(sigma, p_spread, use_sig_p, dtype=torch.float32, device=None):
    """Half-width s of the triangle: a 0-d tensor, or (N,) per source under use_sig_p.

    Returns (s, s_max) with s_max a 0-d tensor."""
    if use_sig_p:
        s = 1.0 + 2.0 * sigma * torch.sigmoid(p_spread).to(dtype)
        return s, s.max()
    s = torch.tensor(1.0 + float(sigma), dtype=dtype, device=device)
    return s, s


def ring_length(d, s_max) -> int:
    """L = ceil(1 + max d + s_max) + 1 (delay_layers_pytorch.py:145)."""
    return int(torch.ceil(1.0 + torch.max(d) + s_max).item()) + 1


def triangle(d, s, L):
    """h[..., l] = max(0, s - |l - (1 + d)|) / s^2 for l = 0..L-1; ``s`` broadcasts
    against ``d`` (append the lag axis yourself for per-source widths)."""
    lags = torch.arange(L, dtype=d.dtype, device=d.device)
    return torch.clamp(s - torch.abs(lags - (1.0 + d)[..., None]), min=0.0) / (s * s)


# ----------------------------------------------------------------------------------
# scans
# ----------------------------------------------------------------------------------

def _prepare_d(d, round_delays):
    if round_delays:
        return d + (d.round() - d).detach()
    return d


def axonal_scan(x, W, d, lif: OracleLIF, sigma=0.0, p_spread=None, use_sig_p=False,
                bias=None, keep=None, round_delays=False, record_u=False):
    """Axonal delay layer over T steps.  x (T,B,N); W (N,N) with W[i,j] target i,
    source j; d (N,) per source.  Returns y (T,B,N) [, u (T,B,N)]."""
    T, B, N = x.shape
    d = _prepare_d(d.to(x.dtype), round_delays)
    s, s_max = spread(sigma, p_spread, use_sig_p, x.dtype, x.device)
    L = ring_length(d, s_max)
    sj = s[:, None] if use_sig_p else s
    h = triangle(d, sj, L)                       # (N, L), h[j, l]
    hist = x.new_zeros(L, B, N)                  # hist[l] = y[t - l], slot 0 unused
    ys, us = [], []
    for t in range(T):
        if L >= 2:
            # z[b, j] = sum_{l>=1} h[j, l] * y[t - l, b, j]
            z = (hist[1:].permute(1, 2, 0) * h[:, 1:]).sum(-1)
            rec = z @ W.t()
        else:
            rec = x.new_zeros(B, N)
        if bias is not None:
            rec = rec + bias
        if keep is not None:
            rec = rec * keep
        y = lif.single_step_forward(x[t] + rec)
        if L >= 2:
            hist = torch.cat([hist[:1], y[None], hist[1:-1]], 0)
        ys.append(y)
        us.append(lif.u)
    y = torch.stack(ys)
    return (y, torch.stack(us)) if record_u else y


def hard_lags(d, L, interp=False):
    """The reference's hard taps (triton_kernels/delays.py:33-47): lag = clamp(round(d)+1,
    1, L-1), or for the interpolation lag = clamp(floor(1+d), 1, L-1) with the fraction
    f = clamp(1+d-lag, 0, 1) weighing lag+1 (and 1-f lag).  Returns (lag long, f)."""
    hi = max(1, L - 1)
    if interp:
        pos = 1.0 + d
        lag = torch.floor(pos).long().clamp(1, hi)
        return lag, (pos - lag.to(d.dtype)).clamp(0.0, 1.0)
    return (torch.round(d).long() + 1).clamp(1, hi), torch.zeros_like(d)


def axonal_scan_hard(x, W, d, lif: OracleLIF, mode, sigma=0.0, p_spread=None, use_sig_p=False,
                     bias=None, keep=None, record_u=False):
    """The axonal layer's hard-tap variants (triton_kernels/recdel_base.py:350-445), their
    gradients expressed through autograd:

    * mode 1 / 2 ('triton_ste', rounded / interpolated): the forward reads the hard taps
      z_hard; autograd sees z = z_soft + (z_hard - z_soft).detach(), so the recurrence and
      the delay / spread gradients are the soft triangle's while the weight gradient
      correlates with z_hard (recdel_base.py:360-372, 401-412);
    * mode 3 ('triton_approx'): z = y[t-lag] + (d - d.detach()) (y[t-lag-1] - y[t-lag]).detach()
      with lag sized on Lmax = round(max d) + 2: the single tap's own backward plus the
      straight-through delay gradient sum gz (y[t-lag-1] - y[t-lag]) and no spread
      gradient (recdel_base.py:373-378, 265-278, 416-419)."""
    T, B, N = x.shape
    d = d.to(x.dtype)
    s, s_max = spread(sigma, p_spread, use_sig_p, x.dtype, x.device)
    L = ring_length(d, s_max)
    if mode == 3:
        lag, frac = hard_lags(d.detach(), int(torch.round(d.detach()).max().item()) + 2)
    else:
        lag, frac = hard_lags(d.detach(), L, interp=(mode == 2))
    R = max(L, int(lag.max().item()) + 2)
    h = triangle(d, s[:, None] if use_sig_p else s, R) if mode != 3 else None
    hist = x.new_zeros(R, B, N)                  # hist[l] = y[t - l]
    idx0 = lag.view(1, N, 1).expand(B, N, 1)
    ys, us = [], []
    for t in range(T):
        hp = hist.permute(1, 2, 0)               # (B, N, R)
        y0 = torch.gather(hp, 2, idx0).squeeze(-1)
        y1 = torch.gather(hp, 2, idx0 + 1).squeeze(-1)
        if mode == 3:
            z = y0 + (d - d.detach()) * (y1 - y0).detach()
        else:
            z_hard = (1.0 - frac) * y0 + frac * y1 if mode == 2 else y0
            z_soft = (hp[..., 1:] * h[:, 1:]).sum(-1)
            z = z_soft + (z_hard - z_soft).detach()
        rec = z @ W.t()
        if bias is not None:
            rec = rec + bias
        if keep is not None:
            rec = rec * keep
        y = lif.single_step_forward(x[t] + rec)
        hist = torch.cat([hist[:1], y[None], hist[1:-1]], 0)
        ys.append(y)
        us.append(lif.u)
    y = torch.stack(ys)
    return (y, torch.stack(us)) if record_u else y


def synaptic_scan(x, W, d, lif: OracleLIF, sigma=0.0, p_spread=None, use_sig_p=False,
                  bias=None, keep=None, round_delays=False, record_u=False):
    """Synaptic delay layer.  d (N,N) with d[i,o] target i, source o; the half-width is
    indexed by the source o."""
    T, B, N = x.shape
    d = _prepare_d(d.to(x.dtype), round_delays)
    s, s_max = spread(sigma, p_spread, use_sig_p, x.dtype, x.device)
    L = ring_length(d, s_max)
    so = s[None, :, None] if use_sig_p else s
    h = triangle(d, so, L)                       # (N, N, L), h[i, o, l]
    Wm = W[..., None] * h                        # (N, N, L)
    hist = x.new_zeros(L, B, N)
    ys, us = [], []
    for t in range(T):
        if L >= 2:
            # rec[b, i] = sum_{o, l>=1} Wm[i, o, l] * y[t - l, b, o]
            rec = torch.einsum('iol,lbo->bi', Wm[:, :, 1:], hist[1:])
        else:
            rec = x.new_zeros(B, N)
        if bias is not None:
            rec = rec + bias
        if keep is not None:
            rec = rec * keep
        y = lif.single_step_forward(x[t] + rec)
        if L >= 2:
            hist = torch.cat([hist[:1], y[None], hist[1:-1]], 0)
        ys.append(y)
        us.append(lif.u)
    y = torch.stack(ys)
    return (y, torch.stack(us)) if record_u else y


def hybrid_delays(base, offsets):
    """Effective per-synapse delay of the hybrid model (networks.py:823-829)."""
    return base + 0.0 + 1.0 * offsets


def vanilla_scan(x, W, lif: OracleLIF, keep=None):
    """Delay-free recurrent layer: rec = dropout(y[t-1]) @ W, W (N_in, N_out)
    (delay_layers_pytorch.py:18-47)."""
    T, B, N = x.shape
    ys, prev = [], None
    for t in range(T):
        if prev is None:
            rec = x.new_zeros(B, N)
        else:
            src = prev * keep if keep is not None else prev
            rec = src @ W
        prev = lif.single_step_forward(x[t] + rec)
        ys.append(prev)
    return torch.stack(ys)


def lif_multistep(x, lif: OracleLIF):
    """Plain (non-recurrent) multi-step LIF layer."""
    return torch.stack([lif.single_step_forward(x[t]) for t in range(x.shape[0])])


# ----------------------------------------------------------------------------------
# closed-form triangle derivative (mirrors the reference's fused dd kernel,
# triton_kernels/synaptic_hybrid.py:83-113, and its pure-torch mirror
# tests/test_hybrid_delay_invariance.py:135-142)
# ----------------------------------------------------------------------------------

def closed_form_delay_grad(C, W, d, sigma):
    """dd[i,o] = W[i,o] * sum_l C[i,o,l] * sign(l-1-d) / s^2 where |l-1-d| <= s."""
    s = 1.0 + float(sigma)
    lm = C.shape[-1]
    a = torch.arange(lm, dtype=d.dtype, device=d.device).view(1, 1, lm) - 1.0 - d.unsqueeze(-1)
    g = torch.sign(a) * (a.abs() <= s).to(d.dtype) / (s * s)
    return (W.unsqueeze(-1) * C * g).sum(-1)


# ----------------------------------------------------------------------------------
# DCLS-style feedforward delay (Gaussian-interpolated kernel + causal conv over time).
# The exact construction lives in the third-party DCLS 0.1.1 package, which is not in
# the reference tree: this restates its published method, and parity is UNPINNED.
# ----------------------------------------------------------------------------------

def dcls_gauss_kernel(weight, P, SIG, dilated_kernel_size):
    """weight (Cout, Cin_g, 1), P (1, Cout, Cin_g, 1), SIG same shape ->
    dense kernel (Cout, Cin_g, K): w * g(k) / (sum_k g(k) + eps),
    g(k) = exp(-0.5 ((k - (P + K//2)) / (|SIG| + eps))^2)."""
    K = int(dilated_kernel_size)
    k = torch.arange(K, dtype=weight.dtype, device=weight.device)
    c = P[0, :, :, 0] + K // 2                      # (Cout, Cin_g)
    sg = SIG[0, :, :, 0].abs() + 1e-7
    g = torch.exp(-0.5 * ((k - c[..., None]) / sg[..., None]) ** 2)
    g = g / (g.sum(-1, keepdim=True) + 1e-7)
    return weight[:, :, :1] * g


def dcls_conv(x, weight, P, SIG, K, groups, left_padding, bias=None):
    """(T,B,Cin) -> (T,B,Cout): causal left-padded conv1d with the constructed kernel."""
    ker = dcls_gauss_kernel(weight, P, SIG, K)
    xb = torch.nn.functional.pad(x.permute(1, 2, 0), (left_padding, 0))
    out = torch.nn.functional.conv1d(xb, ker, bias, groups=groups)
    return out.permute(2, 0, 1)
