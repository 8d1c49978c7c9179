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


@pytest.mark.parametrize("T,B,N,C,bias", [(32, 64, 64, 4, True), (250, 20, 512, 35, False),
                                          (7, 3, 33, 10, True)])
def test_readout_time_sum_matches_fp64(T, B, N, C, bias):
    """The fused readout + time sum (delrec_readout_sum_forward / _backward): out, dy, dW and
    dbias against sum_t (y_t W^T + bias) in float64 through autograd."""
    from delrec.linear import readout_time_sum
    g = torch.Generator().manual_seed(T + N + C)
    y = (torch.rand(T, B, N, generator=g) < 0.1).float().cuda().requires_grad_(True)
    W = (torch.randn(C, N, generator=g) * 0.1).cuda().requires_grad_(True)
    b = torch.randn(C, generator=g).cuda().requires_grad_(True) if bias else None
    go = torch.randn(B, C, generator=g).cuda()
    out = readout_time_sum(y, W, b)
    (out * go).sum().backward()
    y64 = y.detach().double().requires_grad_(True)
    W64 = W.detach().double().requires_grad_(True)
    b64 = b.detach().double().requires_grad_(True) if bias else None
    ref = (y64 @ W64.t() + (b64 if bias else 0.0)).sum(0)
    (ref * go.double()).sum().backward()
    _close(out, ref.detach(), "out")
    _close(y.grad, y64.grad, "dy")
    _close(W.grad, W64.grad, "dW")
    if bias:
        _close(b.grad, b64.grad, "dbias")


def test_forward_time_summed_matches_the_unfused_model():
    """A hybrid-delay model's fused readout path (forward_time_summed) against forward()
    summed over time: the same loss and the same parameter gradients."""
    from delrec import networks
    from model_configs import mem_config
    cfg = mem_config(hidden=(64, 48), bias=True, T=40, B=32)
    cfg.hybrid_offset_scale = 3
    torch.manual_seed(0)
    model = networks.SNN_recurrent_hybrid_delays(cfg).cuda()
    g = torch.Generator().manual_seed(5)
    x = (torch.rand(40, 32, cfg.input_size, generator=g) < 0.2).float().cuda()
    labels = torch.randint(cfg.output_size, (32,), generator=g).cuda()
    grads = []
    for fused in (True, False):
        model.zero_grad(set_to_none=True)
        out = model.forward_time_summed(x) if fused else model(x).sum(0)
        loss = torch.nn.functional.cross_entropy(out, labels)
        loss.backward()
        grads.append((out.detach(), [p.grad.detach().clone() for p in model.parameters() if p.grad is not None]))
    (oa, ga), (ob, gb) = grads
    _close(oa, ob.double(), "out")
    assert len(ga) == len(gb)
    for a, b in zip(ga, gb):
        scale = b.abs().max().item() + 1e-30
        assert (a - b).abs().max().item() / scale < 1e-4
