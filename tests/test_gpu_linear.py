"""Tensor-core feedforward projection (delrec_linear_forward/backward) against an fp64
torch reference: spike inputs (exact single piece) and real inputs (six piece products),
odd widths, no bias, the input-gradient-only and weight-gradient-only cases, and the
device check of a broken spike promise."""

import pytest
import torch

pytestmark = pytest.mark.gpu

# fp32 accuracy: the splits are exact, the accumulation is fp32 over K terms
RTOL = 1e-5


def _ref(x, W, b, g):
    x64, W64, g64 = x.double(), W.double(), g.double()
    out = x64 @ W64.t() + (b.double() if b is not None else 0.0)
    dx = g64 @ W64
    dW = g64.t() @ x64
    db = g64.sum(0)
    return out, dx, dW, db


def _close(a, ref, what):
    scale = ref.abs().max().item() + 1e-30
    err = (a.double() - ref).abs().max().item() / scale
    assert err < RTOL, f"{what}: max error {err:.3g} of max |ref|"


@pytest.mark.parametrize("M,K,N,binary,bias", [
    (4000, 700, 512, True, True),
    (3000, 512, 35, True, True),
    (2048, 9, 128, False, True),
    (777, 1, 10, False, False),
    (1500, 130, 70, False, True),
    (1000, 64, 64, True, False),
])
def test_linear_matches_fp64(M, K, N, binary, bias):
    from delrec.linear import LinearFn
    g = torch.Generator().manual_seed(M + K + N)
    if binary:
        x = (torch.rand(M, K, generator=g) < 0.05).float()
    else:
        x = torch.randn(M, K, generator=g)
    W = torch.randn(N, K, generator=g) * 0.1
    b = torch.randn(N, generator=g) if bias else None
    gout = torch.randn(M, N, generator=g)
    xd = x.cuda().requires_grad_(True)
    Wd = W.cuda().requires_grad_(True)
    bd = b.cuda().requires_grad_(True) if bias else None
    out = LinearFn.apply(xd, Wd, bd, binary)
    out.backward(gout.cuda())
    r_out, r_dx, r_dW, r_db = _ref(x, W, b, gout)
    _close(out.detach().cpu(), r_out, "out")
    _close(xd.grad.cpu(), r_dx, "dx")
    _close(Wd.grad.cpu(), r_dW, "dW")
    if bias:
        _close(bd.grad.cpu(), r_db, "dbias")


def test_linear_time_major_module_and_partial_grads():
    from delrec.linear import Linear
    torch.manual_seed(0)
    lin = Linear(40, 24, bias=True, binary_input=None).cuda()
    x = (torch.rand(7, 5, 40, device="cuda") < 0.2).float()          # detected as spikes
    y = lin(x)
    ref = x.double() @ lin.weight.double().t() + lin.bias.double()
    _close(y.detach().cpu(), ref.cpu(), "module out")
    y.sum().backward()                                               # x needs no grad
    _close(lin.weight.grad.cpu(), torch.ones(35, 24, dtype=torch.float64).t().cpu() @
           x.reshape(35, 40).double().cpu(), "module dW")


def test_broken_spike_promise_sets_status():
    from delrec import _lib
    from delrec.linear import LinearFn
    _lib.lib().delrec_clear_status()
    x = torch.full((64, 16), 0.5, device="cuda")
    W = torch.randn(8, 16, device="cuda")
    LinearFn.apply(x, W, None, True)
    torch.cuda.synchronize()
    assert _lib.status() != 0
    _lib.lib().delrec_clear_status()


def test_spike_input_check():
    """delrec_count_nonbinary: exact on 0/1 inputs, any other value (here one entry, in a
    ragged tail, and an unaligned view) is detected."""
    from delrec.linear import _is_binary
    g = torch.Generator().manual_seed(3)
    for n in (1, 7, 4096, 64001):
        x = (torch.rand(n, generator=g) < 0.3).float().cuda()
        assert _is_binary(x)
        y = x.clone()
        y[n - 1] = 0.5
        assert not _is_binary(y)
    z = (torch.rand(1001, generator=g) < 0.3).float().cuda()
    assert _is_binary(z[1:])
    z[500] = 2.0
    assert not _is_binary(z[1:])
