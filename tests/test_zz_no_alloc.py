"""The allocation-free axonal forward (delrec_axonal_forward_noalloc).

It exists for callers that cannot allocate device memory while a layer runs; its
scratch is a fixed array inside the library instead of a caller workspace.  This test
calls it through the C-ABI twice in a row and checks both results against the regular
entry point (same spikes, membranes within the tolerance of the other parity tests),
so a second call that reuses the array's previous contents is covered too.  Widths
above 512 run the per-sample scan here while the workspace entry point runs those layers
step by step (a different summation order), so there spikes may differ only at near-ties
of the membrane, as in the oracle comparisons.  It lives in its own file, collected last."""

import ctypes

import pytest
import torch

from parity import U_RTOL, compare_scan

pytestmark = pytest.mark.gpu


def _call(fn_name, desc, lif, x, W, d, s, y, u, with_ws):
    from delrec import _lib
    P = _lib.ptr
    st = _lib.stream_ptr(x.device)
    lib = _lib.lib()
    if with_ws:
        nbytes = lib.delrec_axonal_forward_workspace(ctypes.byref(desc))
        ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=x.device)
        off = (-ws.data_ptr()) % 256
        ws = ws[off:off + nbytes]
        rc = lib.delrec_axonal_forward(ctypes.byref(desc), ctypes.byref(lif), P(x), P(W), None, P(d), P(s),
                                       None, P(y), P(u), P(ws), nbytes, st)
    else:
        rc = lib.delrec_axonal_forward_noalloc(ctypes.byref(desc), ctypes.byref(lif), P(x), P(W), None, P(d),
                                               P(s), None, P(y), P(u), st)
    _lib.check(rc, fn_name)


def _case(seed, T, B, N, dmax):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(T, B, N, generator=g) * 0.9 + 0.35).cuda()
    W = (torch.randn(N, N, generator=g) * (1.2 / N ** 0.5)).cuda()
    d = (torch.rand(N, generator=g) * dmax).cuda()
    return x, W, d


CASES = [
    # T, B, N, dmax: N <= 512 take the same per-sample kernels as the workspace entry point;
    # 768 runs the 4-neurons-per-thread scan, 1000 (not a multiple of 4) the generic one
    (40, 16, 96, 12.0),
    (30, 24, 256, 20.0),
    (24, 12, 768, 20.0),
    (20, 10, 1000, 16.0),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"N{c[2]}")
def test_noalloc_matches_workspace_entry_point_twice(case):
    from delrec import _lib
    T, B, N, dmax = case
    lif = _lib.lif_struct(2.0, 1.0, 0.0, False, _lib.SURR_ATAN, 1.0, 2.0)
    x, W, d = _case(N, T, B, N, dmax)
    s = torch.full((N,), 1.0, device="cuda")
    L = int(torch.ceil(1.0 + d.max() + 1.0).item()) + 1
    desc = _lib.Layer(_lib.AXONAL, T, B, N, L, 0, 0, 0, 1.0, 0.0)
    y_ref, u_ref = torch.empty_like(x), torch.empty_like(x)
    _call("delrec_axonal_forward", desc, lif, x, W, d, s, y_ref, u_ref, with_ws=True)
    for _ in range(2):  # the second call reuses the fixed scratch array
        y, u = torch.full_like(x, -7.0), torch.full_like(x, -7.0)
        _call("delrec_axonal_forward_noalloc", desc, lif, x, W, d, s, y, u, with_ws=False)
        torch.cuda.synchronize()
        if N <= 512:
            assert torch.equal(y, y_ref)
            torch.testing.assert_close(u, u_ref, rtol=U_RTOL, atol=U_RTOL)
        else:
            ties, _ = compare_scan(y, u, y_ref, u_ref)
            print(f"N={N}: {ties} near-ties between the two entry points")


@pytest.mark.parametrize("N", [1025, 2048])
def test_noalloc_rejects_layers_beyond_its_scratch(N):
    from delrec import _lib
    lif = _lib.lif_struct(2.0, 1.0, 0.0, False, _lib.SURR_ATAN, 1.0, 2.0)
    desc = _lib.Layer(_lib.AXONAL, 4, 2, N, 5, 0, 0, 0, 1.0, 0.0)
    dummy = torch.zeros(1, device="cuda")
    P = _lib.ptr
    rc = _lib.lib().delrec_axonal_forward_noalloc(ctypes.byref(desc), ctypes.byref(lif), P(dummy), P(dummy),
                                                  None, P(dummy), P(dummy), None, P(dummy), P(dummy),
                                                  _lib.stream_ptr())
    assert rc == 3  # DELREC_ERR_WORKSPACE, checked before any device work
