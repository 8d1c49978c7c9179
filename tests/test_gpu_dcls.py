"""DCLS feedforward delay layer (row A11) on the GPU against the oracle (needs a B200).

The kernel construction belongs to the third-party DCLS 0.1.1 package, which is not in
the reference tree, so this parity is UNPINNED against DCLS itself: the oracle restates
DCLS's published Gaussian method (oracle.dcls_gauss_kernel / dcls_conv), and these tests
check the CUDA kernels against that restatement (forward 1e-5, every gradient through
autograd of the float64 oracle 1e-4, both relative to the tensor's max), plus central
finite differences of the CUDA forward itself for the positions P and widths SIG.

Shapes: cfg2 (HAR-shaped) 9 -> 128 channels, T=128, B=64 with the HAR kernel width 31
(dense), the same widened by 2*4 for the hybrid reparametrisation (networks.py:936-962),
and a depthwise layer (groups = channels) as in the axonal feedforward variant
(networks.py:565-586)."""

import pytest
import torch

from oracle import delrec_oracle as O
from parity import rel_err

pytestmark = pytest.mark.gpu

CASES = {
    # name: T, B, Cin, Cout, groups, K
    "cfg2_dense_K31": (128, 64, 9, 128, 1, 31),
    "cfg2_hybrid_widened_K39": (128, 64, 9, 128, 1, 39),
    "depthwise_K9": (64, 16, 24, 24, 24, 9),
}


def _params(T, B, Cin, Cout, groups, K, seed):
    g = torch.Generator().manual_seed(seed)
    cin_g = Cin // groups
    x = torch.randn(T, B, Cin, generator=g)
    w = torch.randn(Cout, cin_g, 1, generator=g) * 0.3
    lim = K // 2
    P = (torch.rand(1, Cout, cin_g, 1, generator=g) * 2 - 1) * lim
    SIG = 0.5 + torch.rand(1, Cout, cin_g, 1, generator=g) * 0.23 * lim
    SIG[0, ::5] *= -1.0          # |SIG| is used: negative widths take the sign branch
    bias = torch.randn(Cout, generator=g) * 0.1
    gout = torch.randn(T, B, Cout, generator=g)
    return x, w, P, SIG, bias, gout


def _cuda(x, w, P, SIG, bias, gout, K, groups):
    from delrec import functional as Fn
    leaf = [t.clone().cuda().requires_grad_(True) for t in (x, w, P, SIG, bias)]
    out = Fn.DclsConv1d.apply(*leaf, K, groups, K - 1)
    (out * gout.cuda()).sum().backward()
    torch.cuda.synchronize()
    return out.detach().cpu(), [t.grad.cpu() for t in leaf]


def _oracle(x, w, P, SIG, bias, gout, K, groups):
    leaf = [t.double().clone().requires_grad_(True) for t in (x, w, P, SIG, bias)]
    out = O.dcls_conv(leaf[0], leaf[1], leaf[2], leaf[3], K, groups, K - 1, bias=leaf[4])
    (out * gout.double()).sum().backward()
    return out.detach(), [t.grad for t in leaf]


@pytest.mark.parametrize("name", list(CASES))
def test_dcls_matches_oracle(name):
    T, B, Cin, Cout, groups, K = CASES[name]
    args = _params(T, B, Cin, Cout, groups, K, seed=K + Cin)
    out, grads = _cuda(*args, K, groups)
    ref, rgrads = _oracle(*args, K, groups)
    assert rel_err(out, ref) < 1e-5, f"forward {rel_err(out, ref):.2e}"
    for nm, a, b in zip(("dx", "dweight", "dP", "dSIG", "dbias"), grads, rgrads):
        e = rel_err(a, b)
        assert e < 1e-4, f"{nm}: relative error {e:.2e}"


def test_dcls_position_and_width_gradients_match_finite_differences():
    """d(loss)/dP and d(loss)/dSIG of the CUDA backward against central differences of
    the CUDA forward, loss = sum(gout * out) accumulated in float64, at the cfg2 shape."""
    from delrec import functional as Fn
    T, B, Cin, Cout, groups, K = CASES["cfg2_dense_K31"]
    x, w, P, SIG, bias, gout = _params(T, B, Cin, Cout, groups, K, seed=3)
    _, grads = _cuda(x, w, P, SIG, bias, gout, K, groups)
    dP, dSIG = grads[2], grads[3]
    xc, wc, bc, gc = x.cuda(), w.cuda(), bias.cuda(), gout.cuda().double()

    def loss(Pv, Sv):
        with torch.no_grad():
            out = Fn.DclsConv1d.apply(xc, wc, Pv.cuda(), Sv.cuda(), bc, K, groups, K - 1)
        return float((out.double() * gc).sum())

    eps = 1e-2
    g = torch.Generator().manual_seed(11)
    picks = torch.randint(Cout * Cin, (6,), generator=g).tolist()
    for flat in picks:
        co, ci = divmod(flat, Cin)
        for which, grad in (("P", dP), ("SIG", dSIG)):
            hi_P, lo_P, hi_S, lo_S = P.clone(), P.clone(), SIG.clone(), SIG.clone()
            if which == "P":
                hi_P[0, co, ci, 0] += eps
                lo_P[0, co, ci, 0] -= eps
            else:
                hi_S[0, co, ci, 0] += eps
                lo_S[0, co, ci, 0] -= eps
            fd = (loss(hi_P, hi_S) - loss(lo_P, lo_S)) / (2 * eps)
            an = float(grad[0, co, ci, 0])
            scale = max(abs(fd), float(grad.abs().max()) * 1e-2, 1e-6)
            assert abs(fd - an) / scale < 2e-2, f"{which}[{co},{ci}]: analytic {an:.5g} vs finite difference {fd:.5g}"
