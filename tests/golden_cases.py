"""Loader for the committed golden fixtures (tests/golden/*.pt) and a helper that
replays one case through the CPU oracle."""

import glob
import os

import torch

from oracle import delrec_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


# Fixtures that pin the oracle on the CPU but have not yet run through the library on a
# GPU: the hybrid kernels' route with per-source widths (use_sig_p with the base window at
# most one lag below lag 1; the random GPU case with use_sig_p takes the per-synapse route).
NOT_YET_ON_GPU = ("hyb_sigp",)


def case_names(gpu=False):
    other = ("hybrid_dd", "ax_hard", "ref_state_dicts")   # fixtures of other tests
    names = sorted(os.path.basename(p)[:-3] for p in glob.glob(os.path.join(GOLDEN, "*.pt"))
                   if not os.path.basename(p).startswith(other))
    return [n for n in names if not (gpu and n in NOT_YET_ON_GPU)]


def hard_cases():
    """The axonal hard-tap fixtures: a list of {meta (mode 1/2 = triton_ste rounded /
    interpolated, 3 = triton_approx), inputs, triton}."""
    return torch.load(os.path.join(GOLDEN, "ax_hard.pt"), weights_only=False)


def load(name):
    return torch.load(os.path.join(GOLDEN, name + ".pt"), weights_only=False)


def surrogate(meta):
    return O.ATanSpike(2.0) if meta["surr"] == "atan" else O.TriangleSpike(1.0)


def nonzero_hard_reset(meta):
    """A hard reset to a nonzero value: there the reference's Triton kernels start the
    membrane at 0 and its v2 scans (SpikingJelly) at v_reset; this library follows v2."""
    return meta["v_reset"] is not None and meta["v_reset"] != 0.0


def oracle_run(case, dtype=torch.float32, device="cpu", v_init=None):
    """Forward + BPTT of one golden case through the oracle; returns a dict like the
    fixture's ``v2`` entry (tensors on the CPU).  ``device``/``dtype`` choose where and in
    which precision the oracle's torch code is evaluated; ``v_init`` the initial membrane
    (default v_reset)."""
    if case["meta"].get("mode", 0):
        return oracle_run_hard(case, dtype, device)
    meta, inp = case["meta"], case["inputs"]
    c = lambda t: None if t is None else t.to(device=device, dtype=dtype).clone()
    x = c(inp["x"]).requires_grad_(True)
    W = c(inp["W"]).requires_grad_(True)
    base = c(inp["d"]).requires_grad_(True)
    p = c(inp["p"]).requires_grad_(meta["use_sig_p"])
    b = c(inp["bias"])
    if b is not None:
        b.requires_grad_(True)
    lif = O.OracleLIF(tau=meta["tau"], v_threshold=1.0, v_reset=meta["v_reset"],
                      surrogate=surrogate(meta), detach_reset=meta["detach_reset"], v_init=v_init)
    kw = dict(sigma=meta["sigma"], p_spread=p, use_sig_p=meta["use_sig_p"], bias=b,
              keep=c(inp["keep"]), record_u=True)
    if meta["kind"] == "axonal":
        y, u = O.axonal_scan(x, W, base, lif, **kw)
    else:
        d = O.hybrid_delays(base, c(inp["offsets"])) if meta["kind"] == "hybrid" else base
        y, u = O.synaptic_scan(x, W, d, lif, **kw)
    (y * c(inp["gy"])).sum().backward()
    out = dict(y=y.detach(), u=u.detach(), dx=x.grad, dW=W.grad, dd=base.grad)
    if meta["use_sig_p"]:
        out["dp"] = p.grad
    if b is not None:
        out["dbias"] = b.grad
    return {k: v.cpu() for k, v in out.items()}


def oracle_run_hard(case, dtype=torch.float32, device="cpu"):
    """Forward + BPTT of one hard-tap fixture through ``axonal_scan_hard``."""
    meta, inp = case["meta"], case["inputs"]
    c = lambda t: None if t is None else t.to(device=device, dtype=dtype).clone()
    x = c(inp["x"]).requires_grad_(True)
    W = c(inp["W"]).requires_grad_(True)
    d = c(inp["d"]).requires_grad_(True)
    p = c(inp["p"]).requires_grad_(meta["use_sig_p"])
    b = c(inp["bias"])
    if b is not None:
        b.requires_grad_(True)
    lif = O.OracleLIF(tau=meta["tau"], v_threshold=1.0, v_reset=meta["v_reset"],
                      surrogate=surrogate(meta), detach_reset=meta["detach_reset"])
    y, u = O.axonal_scan_hard(x, W, d, lif, meta["mode"], sigma=meta["sigma"], p_spread=p,
                              use_sig_p=meta["use_sig_p"], bias=b, keep=c(inp["keep"]),
                              record_u=True)
    (y * c(inp["gy"])).sum().backward()
    out = dict(y=y.detach(), u=u.detach(), dx=x.grad, dW=W.grad, dd=d.grad)
    if meta["use_sig_p"] and p.grad is not None:
        out["dp"] = p.grad
    if b is not None:
        out["dbias"] = b.grad
    return {k: v.cpu() for k, v in out.items() if v is not None}


def subset_case(case, samples):
    """The same case restricted to the given batch samples (samples are independent, so
    every per-sample quantity is unchanged and the parameter gradients are the sums over
    the kept samples)."""
    idx = torch.as_tensor(list(samples), dtype=torch.long)
    inp = dict(case["inputs"])
    inp["x"] = inp["x"][:, idx].contiguous()
    inp["gy"] = inp["gy"][:, idx].contiguous()
    if inp.get("keep") is not None:
        inp["keep"] = inp["keep"][idx].contiguous()
    meta = dict(case["meta"], B=int(idx.numel()))
    return dict(meta=meta, inputs=inp)
