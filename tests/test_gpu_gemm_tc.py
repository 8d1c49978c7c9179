"""The library's tcgen05 tensor-core GEMM (delrec_tc_gemm) against float64 matmuls
(needs a B200).  It carries the weight gradients, the lag-correlation stack and the
projections, so it is checked on its own first: exact bf16 operands (one product),
fp32 operands split into hi + lo bf16 pieces (three products, fp32-level accuracy),
ragged shapes and a reduction length that is not a multiple of the 64-wide stage,
accumulation into D, and split reductions over a training step's T*B rows."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _pieces(x, n):
    """Exact-as-possible bf16 pieces of an fp32 matrix: x ~ p0 + p1 (+ p2)."""
    out, r = [], x.clone()
    for _ in range(n):
        p = r.to(torch.bfloat16)
        out.append(p)
        r = r - p.float()
    return out


def _padded(p, ld):
    """bf16 rows padded to a row stride of ld elements (16-byte multiple)."""
    M, K = p.shape
    buf = torch.zeros(M, ld, dtype=torch.bfloat16, device=p.device)
    buf[:, :K] = p
    return buf


def _gemm(A, B, prods, K, ksplit=1, block_n=128, D=None, accumulate=False, layout=0):
    """layout bit 0: A pieces stored (K, M); bit 1: B pieces stored (K, N)."""
    from delrec import _lib
    M = A[0].shape[1] if layout & 1 else A[0].shape[0]
    N = B[0].shape[1] if layout & 2 else B[0].shape[0]
    lda, ldb = A[0].shape[1], B[0].shape[1]
    if D is None:
        D = torch.full((M, N), float("nan"), device="cuda")
    pa = (ctypes.c_int * len(prods))(*[p[0] for p in prods])
    pb = (ctypes.c_int * len(prods))(*[p[1] for p in prods])
    Ap = (ctypes.c_void_p * len(A))(*[t.data_ptr() for t in A])
    Bp = (ctypes.c_void_p * len(B))(*[t.data_ptr() for t in B])
    lib = _lib.lib()
    nbytes = lib.delrec_tc_gemm_workspace(M, N, ksplit)
    ws = _lib.workspace(nbytes, "cuda")
    rc = lib.delrec_tc_gemm(M, N, K, layout, len(A), Ap, lda, len(B), Bp, ldb, len(prods), pa, pb, ksplit, block_n,
                            _lib.ptr(D), D.shape[1], int(accumulate), _lib.ptr(ws), ws.numel(), _lib.stream_ptr())
    _lib.check(rc, "delrec_tc_gemm")
    torch.cuda.synchronize()
    return D


def _err(D, ref):
    return ((D.double() - ref).abs().max() / ref.abs().max()).item()


@pytest.mark.parametrize("M,N,K,block_n", [(256, 256, 512, 128), (128, 64, 64, 64), (512, 512, 1024, 256)])
def test_exact_bf16_single_product(M, N, K, block_n):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    D = _gemm([a], [b], [(0, 0)], K, block_n=block_n)
    ref = a.double() @ b.double().t()
    assert _err(D, ref) < 2e-6


def test_ragged_shapes_and_partial_stage():
    M, N, K, ld = 300, 200, 777, 784
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    for bn in (64, 128, 256):
        D = _gemm([_padded(a, ld)], [_padded(b, ld)], [(0, 0)], K, block_n=bn)
        assert _err(D, a.double() @ b.double().t()) < 2e-6, bn


def test_three_product_split_reaches_fp32_accuracy_and_accumulates():
    M, N, K = 384, 320, 2048
    g = torch.Generator(device="cuda").manual_seed(9)
    a = torch.randn(M, K, device="cuda", generator=g)
    b = torch.randn(N, K, device="cuda", generator=g)
    A, B = _pieces(a, 2), _pieces(b, 2)
    ref = a.double() @ b.double().t()
    D = _gemm(A, B, [(0, 0), (0, 1), (1, 0)], K)
    assert _err(D, ref) < 2e-5
    D0 = torch.randn(M, N, device="cuda", generator=g)
    D1 = _gemm(A, B, [(0, 0), (0, 1), (1, 0)], K, D=D0.clone(), accumulate=True)
    assert _err(D1, ref + D0.double()) < 2e-5


@pytest.mark.parametrize("ksplit", [1, 8])
def test_training_step_length_reduction(ksplit):
    """dW-shaped: 512 x 512 outputs over 64000 reduction rows (T=250, B=256).  The tensor
    core's fp32 accumulator drifts over a sum this long (~1e-4 of the result's max in one
    piece), which is why the library splits such reductions into parts of at most ~24K
    and adds the parts in IEEE fp32: split eight ways it is within 1e-5."""
    M = N = 512
    K = 64000
    g = torch.Generator(device="cuda").manual_seed(ksplit)
    a = torch.randn(M, K, device="cuda", generator=g) * 1e-3
    b = (torch.rand(N, K, device="cuda", generator=g) < 0.05).float()     # spike-like operand
    A, B = _pieces(a, 2), _pieces(b, 1)
    ref = a.double() @ b.double().t()
    D = _gemm(A, B, [(0, 0), (1, 0)], K, ksplit=ksplit, block_n=256)
    assert _err(D, ref) < (1e-5 if ksplit >= 8 else 2e-4)


@pytest.mark.parametrize("layout", [1, 2, 3])
def test_mn_major_operands(layout):
    """Operands stored with the M / N index contiguous (reductions over the rows of a
    (T*B, N) activation), ragged sizes, one- and three-product forms."""
    M, N, K = 320, 192, 1000
    g = torch.Generator(device="cuda").manual_seed(20 + layout)
    a = torch.randn(M, K, device="cuda", generator=g)
    b = torch.randn(N, K, device="cuda", generator=g)
    A, B = _pieces(a, 2), _pieces(b, 2)
    if layout & 1:
        A = [p.t().contiguous() for p in A]
    if layout & 2:
        B = [p.t().contiguous() for p in B]
    ref = a.double() @ b.double().t()
    for bn in (64, 128, 256):
        D = _gemm(A, B, [(0, 0), (0, 1), (1, 0)], K, block_n=bn, layout=layout)
        assert _err(D, ref) < 2e-5, bn
    ref1 = A[0].double().t() @ B[0].double() if layout == 3 else None
    if ref1 is not None:
        D = _gemm(A, B, [(0, 0)], K, ksplit=3, layout=layout)
        assert _err(D, ref1) < 2e-6
