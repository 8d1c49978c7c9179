"""Comparison helpers shared by the GPU parity tests.

Contract (from the reference's own accuracy claims, tightened): spike trains identical
except where the oracle membrane is within 1e-5 of the threshold (a near-tie; counted and
reported); membranes within 1e-5 relative up to the first near-tie of a sample;
parameter gradients within 1e-4 relative to the gradient's max magnitude."""

import torch

U_RTOL = 1e-5
GRAD_RTOL = 1e-4
TIE = 1e-5


def rel_err(a, b):
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return ((a - b).abs().max() / (b.abs().max() + 1e-30)).item()


def compare_scan(y, u, y_ref, u_ref, v_th=1.0):
    """Returns (n_near_ties, clean) where clean means the spike trains are identical.
    Raises AssertionError on a real mismatch."""
    y = y.detach().cpu()
    u = u.detach().cpu()
    y_ref = y_ref.detach().cpu()
    u_ref = u_ref.detach().cpu()
    T, B, N = y.shape
    ties = 0
    for b in range(B):
        diff = (y[:, b] != y_ref[:, b])
        if diff.any():
            t0 = int(diff.any(1).nonzero()[0])
            bad = diff[t0].nonzero().flatten()
            gap = (u_ref[t0, b, bad] - v_th).abs()
            assert bool((gap < TIE).all()), (
                f"sample {b}: spike mismatch at t={t0} neurons {bad.tolist()[:8]} that are not "
                f"near-ties (|u-th| = {gap.tolist()[:8]})")
            ties += int(bad.numel())
            upto = t0 + 1
        else:
            upto = T
        ud, ur = u[:upto, b].double(), u_ref[:upto, b].double()
        tol = U_RTOL * torch.clamp(ur.abs(), min=1.0)
        err = (ud - ur).abs()
        assert bool((err <= tol).all()), (
            f"sample {b}: membrane mismatch, max |du| = {err.max().item():.3e}")
    return ties, ties == 0


def compare_grads(got: dict, ref: dict, keys, rtol=GRAD_RTOL):
    out = {}
    for k in keys:
        if k not in ref or ref[k] is None:
            continue
        assert got.get(k) is not None, f"missing gradient {k}"
        e = rel_err(got[k], ref[k])
        out[k] = e
        assert e < rtol, f"gradient {k}: relative error {e:.3e} >= {rtol}"
    return out


def mismatch_samples(y, y_ref):
    """Batch samples whose spike trains differ anywhere (after compare_scan has checked
    that every first difference is a near-tie)."""
    d = (y.detach().cpu() != y_ref.detach().cpu()).any(0).any(-1)
    return d.nonzero().flatten().tolist()


def grad_keys(meta, has_bias):
    # the straight-through single-tap variant (mode 3) has no spread gradient
    sig = meta["use_sig_p"] and meta.get("mode", 0) != 3
    return ["dx", "dW", "dd"] + (["dp"] if sig else []) + (["dbias"] if has_bias else [])
