"""The CPU oracle against the reference's own outputs (golden fixtures).

The fixtures hold, per case, the reference's v2 scan + autograd (``v2``) and its Triton
kernels run by the Triton CPU interpreter (``triton``).  The oracle must reproduce the
spikes exactly and membranes / gradients to float tolerance."""

import pytest
import torch

from golden_cases import case_names, load, nonzero_hard_reset, oracle_run
from oracle import delrec_oracle as O

GRAD_RTOL = 1e-4


def _rel(a, b):
    return ((a - b).abs().max() / (b.abs().max() + 1e-12)).item()


@pytest.mark.parametrize("name", case_names())
def test_oracle_matches_reference_v2(name):
    case = load(name)
    out = oracle_run(case)
    ref = case["v2"]
    assert torch.equal(out["y"], ref["y"]), "spike trains differ from the reference v2 scan"
    torch.testing.assert_close(out["u"], ref["u"], rtol=1e-5, atol=1e-6)
    for k in ("dx", "dW", "dd", "dp", "dbias"):
        if k in ref and k in out:
            assert _rel(out[k], ref[k]) < GRAD_RTOL, f"{k}: rel {_rel(out[k], ref[k]):.2e}"


@pytest.mark.parametrize("name", case_names())
def test_oracle_matches_reference_triton(name):
    """For a hard reset to a nonzero value the reference's Triton kernels start the
    membrane at 0 (recdel_base.py:53), its v2 scans at v_reset: with that one start changed
    the oracle reproduces the kernels, so the start is the only difference."""
    case = load(name)
    out = oracle_run(case, v_init=0.0 if nonzero_hard_reset(case["meta"]) else None)
    ref = case["triton"]
    assert torch.equal(out["y"], ref["y"]), "spike trains differ from the reference kernels"
    torch.testing.assert_close(out["u"], ref["u"], rtol=1e-5, atol=1e-5)
    for k in ("dx", "dW", "dd", "dp", "dbias"):
        if k in ref and k in out:
            assert _rel(out[k], ref[k]) < GRAD_RTOL, f"{k}: rel {_rel(out[k], ref[k]):.2e}"


@pytest.mark.parametrize("idx", range(12))
def test_oracle_hard_taps_match_reference_triton(idx):
    """The 'triton_ste' (rounded, interpolated) and 'triton_approx' axonal variants:
    oracle against the reference's kernels in those modes (recdel_base.py:350-445)."""
    from golden_cases import hard_cases, oracle_run_hard
    cases = hard_cases()
    assert len(cases) == 12
    case = cases[idx]
    out = oracle_run_hard(case)
    ref = case["triton"]
    assert torch.equal(out["y"], ref["y"]), "spike trains differ from the reference kernels"
    torch.testing.assert_close(out["u"], ref["u"], rtol=1e-5, atol=1e-5)
    for k in ("dx", "dW", "dd", "dp", "dbias"):
        if k in ref and (k != "dbias" or case["inputs"]["bias"] is not None):
            assert k in out, k
            assert _rel(out[k], ref[k]) < GRAD_RTOL, f"{k}: rel {_rel(out[k], ref[k]):.2e}"
    if case["meta"]["mode"] == 3:
        assert "dp" not in ref and "dp" not in out


def test_oracle_fp64_agrees_with_fp32():
    """Float64 replay of a case stays within the tolerance used for GPU parity."""
    case = load("hyb_sigma_bias")
    o32 = oracle_run(case)
    o64 = oracle_run(case, dtype=torch.float64)
    assert torch.equal(o32["y"], o64["y"].float())
    for k in ("dx", "dW", "dd"):
        assert _rel(o32[k].double(), o64[k]) < 1e-4


def test_hybrid_closed_form_dd_edges():
    """Closed-form triangle derivative at integer and support-edge delays equals the
    reference's fused delay-gradient kernel (synaptic_hybrid.py:83-126)."""
    import os
    from golden_cases import GOLDEN
    for c in torch.load(os.path.join(GOLDEN, "hybrid_dd_edges.pt")):
        dd = O.closed_form_delay_grad(c["C"], c["W"], c["d"], c["sigma"])
        torch.testing.assert_close(dd, c["dd"], atol=2e-5, rtol=2e-5)


@pytest.mark.parametrize("sigma", [0.0, 0.5, 1.3])
def test_closed_form_matches_autograd(sigma):
    """Port of tests/test_hybrid_delay_invariance.py:145-162 against the oracle."""
    torch.manual_seed(0)
    N, lm = 12, 6
    d = 0.3 + 3.0 * torch.rand(N, N)
    W = torch.randn(N, N)
    C = torch.randn(N, N, lm)
    C[:, :, 0] = 0.0
    d_ = d.clone().requires_grad_(True)
    mask = O.triangle(d_, torch.tensor(1.0 + sigma), lm)
    (ref,) = torch.autograd.grad(mask, d_, grad_outputs=W.unsqueeze(-1) * C)
    torch.testing.assert_close(O.closed_form_delay_grad(C, W, d, sigma), ref,
                               atol=1e-6, rtol=1e-5)
