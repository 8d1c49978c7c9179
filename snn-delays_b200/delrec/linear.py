"""Feedforward projections of the model zoo (the torch.nn.Linear layers of
src/delrec/networks.py:84-96, 140-181) on the library's tensor-core path.

``Linear`` is a ``torch.nn.Linear`` (same parameters, same state_dict keys) whose forward
runs ``delrec_linear_forward`` / ``delrec_linear_backward``: bf16 tensor-core GEMMs on
exact three-piece bf16 splits of the fp32 operands, fp32 accumulation.  When the input
is a spike train (every value 0 or 1) one piece carries it exactly and the GEMMs are
half as long; ``binary_input`` says so (True: promised, checked on the device through the
status word; None: tested on each call).  CUDA tensors only.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib


def _is_binary(x):
    """True when every entry of the CUDA tensor x is 0 or 1: one counting kernel
    (delrec_count_nonbinary) and one read of its result (a synchronisation)."""
    if x.data_ptr() % 16 != 0:
        x = x.clone()
    count = torch.empty(1, dtype=torch.int32, device=x.device)
    _lib.check(_lib.lib().delrec_count_nonbinary(_lib.ptr(x), x.numel(), _lib.ptr(count),
                                                 _lib.stream_ptr(x.device)), "delrec_count_nonbinary")
    return int(count.item()) == 0


class LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, binary_input):
        _lib.require_cuda(x, weight, bias)
        K = x.shape[-1]
        N = weight.shape[0]
        x2 = x.detach().reshape(-1, K)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        M = x2.shape[0]
        binary = _is_binary(x2) if binary_input is None else bool(binary_input)
        dev = x.device
        out = torch.empty(M, N, device=dev, dtype=torch.float32)
        w = weight.detach()
        b = bias.detach() if bias is not None else None
        if M > 0:
            lib = _lib.lib()
            ws = _lib.workspace(lib.delrec_linear_forward_workspace(M, K, N, int(binary)), dev)
            P = _lib.ptr
            _lib.check(lib.delrec_linear_forward(M, K, N, P(x2), P(w), P(b), int(binary), P(out), P(ws),
                                                 ws.numel(), _lib.stream_ptr(dev)), "delrec_linear_forward")
        ctx.save_for_backward(x2, w)
        ctx.binary = binary
        ctx.has_bias = bias is not None
        ctx.xshape = x.shape
        return out.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, gout):
        x2, w = ctx.saved_tensors
        M, K = x2.shape
        N = w.shape[0]
        g = gout.reshape(M, N)
        if not g.is_contiguous() or g.dtype != torch.float32:
            g = g.float().contiguous()
        need_dx, need_dw, need_db = ctx.needs_input_grad[0], ctx.needs_input_grad[1], \
            ctx.has_bias and ctx.needs_input_grad[2]
        dev = g.device
        dx = torch.empty(M, K, device=dev) if need_dx else None
        dw = torch.empty(N, K, device=dev) if need_dw else None
        db = torch.empty(N, device=dev) if need_db else None
        if M == 0:
            dw = dw.zero_() if dw is not None else None
            db = db.zero_() if db is not None else None
        elif need_dx or need_dw or need_db:
            lib = _lib.lib()
            ws = _lib.workspace(lib.delrec_linear_backward_workspace(M, K, N, int(ctx.binary)), dev)
            P = _lib.ptr
            _lib.check(lib.delrec_linear_backward(M, K, N, P(x2), P(w), P(g), int(ctx.binary), P(dx), P(dw),
                                                  P(db), P(ws), ws.numel(), _lib.stream_ptr(dev)),
                       "delrec_linear_backward")
        return (dx.view(ctx.xshape) if dx is not None else None), dw, db, None


class ReadoutTimeSum(torch.autograd.Function):
    """sum_t (y_t W^T + bias): the readout Linear of the model zoo (networks.py:140-181)
    summed over time as the SSC / PS-MNIST loss does (utils.py:188-200), fused in the
    library (delrec_readout_sum_forward / _backward) without forming the (T,B,C) readout.
    y (T,B,N), weight (C,N), bias (C) or None -> (B,C)."""

    @staticmethod
    def forward(ctx, y, weight, bias):
        _lib.require_cuda(y, weight, bias)
        T, B, N = y.shape
        C = weight.shape[0]
        y = y.detach().contiguous()
        w = weight.detach().contiguous()
        b = bias.detach().contiguous() if bias is not None else None
        ysum = torch.empty(B, N, device=y.device, dtype=torch.float32)
        out = torch.empty(B, C, device=y.device, dtype=torch.float32)
        P = _lib.ptr
        _lib.check(_lib.lib().delrec_readout_sum_forward(T, B, N, C, P(y), P(w), P(b), P(ysum), P(out),
                                                         _lib.stream_ptr(y.device)),
                   "delrec_readout_sum_forward")
        ctx.save_for_backward(ysum, w)
        ctx.T = T
        ctx.has_bias = bias is not None
        return out

    @staticmethod
    def backward(ctx, g):
        ysum, w = ctx.saved_tensors
        T = ctx.T
        B, N = ysum.shape
        C = w.shape[0]
        g = g.detach().contiguous()
        dev = g.device
        dy = torch.empty(T, B, N, device=dev, dtype=torch.float32) if ctx.needs_input_grad[0] else None
        dW = torch.empty(C, N, device=dev, dtype=torch.float32) if ctx.needs_input_grad[1] else None
        db = (torch.empty(C, device=dev, dtype=torch.float32)
              if ctx.has_bias and ctx.needs_input_grad[2] else None)
        P = _lib.ptr
        _lib.check(_lib.lib().delrec_readout_sum_backward(T, B, N, C, P(ysum), P(w), P(g), P(dy), P(dW), P(db),
                                                          _lib.stream_ptr(dev)),
                   "delrec_readout_sum_backward")
        return dy, dW, db


def readout_time_sum(y, weight, bias=None):
    """sum over time of the readout y_t W^T + bias, fused (see ReadoutTimeSum)."""
    return ReadoutTimeSum.apply(y, weight, bias)


class Linear(torch.nn.Linear):
    """torch.nn.Linear with the tensor-core fp32-accurate projection of this library."""

    def __init__(self, in_features, out_features, bias=True, binary_input=None, device=None, dtype=None):
        super().__init__(in_features, out_features, bias=bias, device=device, dtype=dtype)
        self.binary_input = binary_input

    def forward(self, x):
        if not x.is_cuda:
            raise RuntimeError("delrec_b200 runs on CUDA tensors only (there is no CPU path)")
        return LinearFn.apply(x, self.weight, self.bias, self.binary_input)

    def extra_repr(self):
        return super().extra_repr() + f", binary_input={self.binary_input}"
