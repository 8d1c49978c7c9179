"""Parity at the BASELINE configurations' own layer shapes (needs a B200).

Each case runs one delay layer through the library's C-ABI at the shape a benchmark
configuration uses and compares it with the oracle evaluated in float64 on the GPU (at
these sizes the CPU would take hours; the same oracle code is pinned against the
reference's fixtures on the CPU by test_oracle_golden.py):

* cfg4 (SSC-shaped, the north-star model): hybrid layer N=512, offsets {0..8}, base
  U[0,25], T=250, B=256 -- all four 64-sample tiles of the cooperative reverse scan;
* cfg3 (SHD-shaped): synaptic layer N=256, d U[0,25], T=250, B=256, at sigma 2 and 0;
* cfg5 (PS-MNIST-shaped): axonal layer d U[0,64] (ring L ~ 67, the 128-bit spike history
  of the source pass), T=784, at N=512 and, at reduced batch, N=1024 and 2048.

The cfg4 layer runs twice: with the default chunked reverse scan (long-lag synapses on
the tensor cores once per 8-step chunk) and with the step-by-step scan.

Tolerances are those of the other parity tests (membranes 1e-5 relative, spikes
identical except at near-ties, gradients 1e-4 relative to each tensor's max).  The
near-tie count and the errors of each case go to the JSON report named by the
environment variable DELREC_PARITY_REPORT."""

import pytest

from gpu_cases import check_case
from tests_gen import make_case

pytestmark = pytest.mark.gpu

CASES = {
    # name: kind, T, B, N, sigma, bias, drop, dmax, K[, reverse-scan variant]
    "cfg4_hybrid_N512_T250_B256": ("hybrid", 250, 256, 512, 0.0, False, False, 25.0, 8),
    "cfg4_hybrid_N512_T250_B256_stepwise": ("hybrid", 250, 256, 512, 0.0, False, False, 25.0, 8, 1),
    "cfg3_synaptic_N256_T250_B256_sigma2": ("synaptic", 250, 256, 256, 2.0, False, False, 25.0, 0),
    "cfg3_synaptic_N256_T250_B256_sigma0": ("synaptic", 250, 256, 256, 0.0, False, False, 25.0, 0),
    "cfg5_axonal_N512_T784_B128": ("axonal", 784, 128, 512, 0.0, False, False, 64.0, 0),
    "cfg5_axonal_N1024_T784_B32": ("axonal", 784, 32, 1024, 0.0, False, False, 64.0, 0),
    "cfg5_axonal_N2048_T784_B16": ("axonal", 784, 16, 2048, 0.0, False, False, 64.0, 0),
}


@pytest.mark.parametrize("name", list(CASES))
def test_config_shape_vs_oracle(name):
    from delrec import _lib
    kind, T, B, N, sigma, bias, drop, dmax, K = CASES[name][:9]
    variant = CASES[name][9] if len(CASES[name]) > 9 else _lib.REVERSE_SCAN_CHUNKED
    case = make_case(kind, 4000 + N, T, B, N, sigma, False, bias, drop, dmax, K)
    _lib.set_reverse_scan(variant)
    try:
        rec = check_case(case, name=name, oracle_device="cuda")
    finally:
        _lib.set_reverse_scan(_lib.REVERSE_SCAN_CHUNKED)
    rec["reverse_scan"] = "stepwise" if variant else "chunked"
    print(name, rec)
