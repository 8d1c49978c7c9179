"""Shared GPU-side driver of the parity tests: run one case through the library's C-ABI
(via the autograd Functions that mirror the reference's), run the oracle on the same
inputs, and compare spikes, membranes and gradients.

Gradients are always compared.  A near-tie (|u - threshold| < 1e-5 in the oracle) may
flip one spike, after which that sample's trajectory legitimately diverges; such samples
are dropped and both sides are re-run on the remaining samples (samples are independent,
so the kept samples' results are unchanged), and the gradients are compared there.  The
near-tie count and the maximum errors of every case can be written to a JSON report
(environment variable DELREC_PARITY_REPORT)."""

import json
import os
from types import SimpleNamespace

import torch

from golden_cases import oracle_run, subset_case
from parity import compare_grads, compare_scan, grad_keys, mismatch_samples, TIE

DEV = "cuda"
_REPORT = {}


def layer_ns(meta):
    from delrec.utils import Triangle
    from delrec.neuron import ATan
    surr = ATan(2.0) if meta["surr"] == "atan" else Triangle.apply
    cfg = SimpleNamespace(surrogate_function=surr, surrogate_gamma=1.0,
                          detach_reset=meta["detach_reset"])
    nm = SimpleNamespace(tau=meta["tau"], v_threshold=1.0, v_reset=meta["v_reset"], decay_input=False)
    return SimpleNamespace(config=cfg, neuron_module=nm, sigma=meta["sigma"],
                           use_sig_p=meta["use_sig_p"], round_delays=False)


def run_cuda(meta, inp):
    """Forward + backward of one case on the GPU; returns a dict like the oracle's."""
    from delrec import functional as Fn
    c = lambda t: None if t is None else t.detach().clone().to(DEV)
    x = c(inp["x"]).requires_grad_(True)
    W = c(inp["W"]).requires_grad_(True)
    base = c(inp["d"]).requires_grad_(True)
    p = c(inp["p"]).requires_grad_(meta["use_sig_p"])
    b = c(inp["bias"])
    if b is not None:
        b.requires_grad_(True)
    keep = c(inp["keep"])
    layer = layer_ns(meta)
    if meta["kind"] == "axonal":
        sid = 1 if meta["surr"] == "atan" else 0
        mode = meta.get("mode", 0)   # 1 / 2: triton_ste rounded / interpolated, 3: triton_approx
        y = Fn.AxonalRecdelTriton.apply(x, W, b, base, p if meta["use_sig_p"] else None, keep,
                                        meta["sigma"], meta["tau"], 1.0, meta["v_reset"],
                                        meta["use_sig_p"], meta["detach_reset"], sid, 1.0,
                                        mode == 3, mode if mode in (1, 2) else 0, 2.0)
    elif meta["kind"] == "synaptic":
        y = Fn.EventDrivenSyn.apply(x, W, base, p, b, keep, layer)
    else:
        y = Fn.HybridBaseDelay.apply(x, W, base, c(inp["offsets"]), p, b, keep, layer)
    # membranes: the Functions keep u for the backward
    u = y.grad_fn.saved_tensors[0]
    (y * c(inp["gy"])).sum().backward()
    out = dict(y=y.detach(), u=u.detach(), dx=x.grad, dW=W.grad, dd=base.grad)
    if meta["use_sig_p"]:
        out["dp"] = p.grad
    if b is not None:
        out["dbias"] = b.grad
    torch.cuda.synchronize()
    return {k: v.cpu() for k, v in out.items() if v is not None}


def membrane_err(u, u_ref, y, y_ref):
    """max |u - u_ref| / max(1, |u_ref|) over each sample's steps up to its first spike
    difference (after which the trajectories may legitimately diverge)."""
    u, u_ref = u.double(), u_ref.double()
    T, B, _ = u.shape
    worst = 0.0
    for b in range(B):
        diff = (y[:, b] != y_ref[:, b]).any(1)
        upto = int(diff.nonzero()[0]) + 1 if diff.any() else T
        e = ((u[:upto, b] - u_ref[:upto, b]).abs() / u_ref[:upto, b].abs().clamp(min=1.0)).max()
        worst = max(worst, float(e))
    return worst


def check_case(case, name=None, oracle_device="cpu", oracle_dtype=torch.float64, max_rounds=3):
    """Full comparison of one case; returns the report record."""
    meta, inp = case["meta"], case["inputs"]
    keys = grad_keys(meta, inp["bias"] is not None)
    ref = oracle_run(case, oracle_dtype, oracle_device)
    got = run_cuda(meta, inp)
    ties, _ = compare_scan(got["y"], got["u"], ref["y"], ref["u"])
    rec = dict(kind=meta["kind"], T=meta["T"], B=meta["B"], N=meta["N"], K=meta.get("K", 0),
               sigma=meta["sigma"], spike_rate=float(ref["y"].float().mean()),
               near_tie_neurons=ties, membrane_rel_err=membrane_err(got["u"], ref["u"], got["y"], ref["y"]),
               tie_threshold=TIE)
    dropped = sorted(mismatch_samples(got["y"], ref["y"]))
    kept = [b for b in range(meta["B"]) if b not in dropped]
    rounds = 0
    while dropped and rounds < max_rounds:
        assert kept, "every sample had a near-tie"
        sub = subset_case(case, kept)
        ref = oracle_run(sub, oracle_dtype, oracle_device)
        got = run_cuda(sub["meta"], sub["inputs"])
        compare_scan(got["y"], got["u"], ref["y"], ref["u"])
        again = mismatch_samples(got["y"], ref["y"])
        if not again:
            break
        kept = [kept[i] for i in range(len(kept)) if i not in set(again)]
        rounds += 1
    assert not mismatch_samples(got["y"], ref["y"]), "near-tie samples remained after re-runs"
    rec["tie_samples_dropped"] = meta["B"] - len(kept)
    rec["grad_samples"] = len(kept)
    rec["grad_rel_err"] = compare_grads(got, ref, keys)
    if name:
        record(name, rec)
    return rec


def record(name, rec):
    _REPORT[name] = rec
    path = os.environ.get("DELREC_PARITY_REPORT")
    if path:
        old = {}
        if os.path.exists(path):
            with open(path) as f:
                old = json.load(f)
        old.update(_REPORT)
        with open(path, "w") as f:
            json.dump(old, f, indent=1, sort_keys=True)
