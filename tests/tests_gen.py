"""Seeded synthetic cases in the golden-fixture format (used by GPU parity tests)."""

import math

import torch


def make_case(kind, seed, T, B, N, sigma, sigp, bias, drop, dmax, K, v_reset=0.0, surr="atan",
              gain=1.0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(T, B, N, generator=g) * 0.9 + 0.35) * gain
    W = torch.randn(N, N, generator=g) * (1.2 / math.sqrt(N))
    if kind == "synaptic":
        d = torch.rand(N, N, generator=g) * dmax
    else:
        d = torch.rand(N, generator=g) * dmax
    p = torch.randn(N, generator=g) if sigp else torch.zeros(N)
    b = torch.randn(N, generator=g) * 0.2 if bias else None
    keep = (torch.rand(B, N, generator=g) > 0.3).float() / 0.7 if drop else None
    gy = torch.randn(T, B, N, generator=g)
    off = torch.randint(K + 1, (N, N), generator=g).float() if kind == "hybrid" else None
    meta = dict(name=f"rand_{kind}_{N}", kind=kind, T=T, B=B, N=N, sigma=sigma, use_sig_p=sigp,
                tau=2.0, v_reset=v_reset, surr=surr, detach_reset=False, K=K)
    return dict(meta=meta, inputs=dict(x=x, W=W, d=d, p=p, bias=b, keep=keep, gy=gy, offsets=off))
