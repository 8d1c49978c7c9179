"""Neuron, surrogate and dropout modules with SpikingJelly's public behaviour
(``activation_based.neuron.LIFNode``, ``surrogate.ATan``, ``layer.Dropout``,
``base.MemoryModule``), which the reference builds its layers from
(src/delrec/delay_layers.py:21-31, networks.py:84-96).

The delay layers only read the LIF constants from ``neuron_module``; the multi-step
``LIFNode.forward`` (used between projections in the model zoo) runs the CUDA LIF kernel.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import functional as Fn


class MemoryModule(torch.nn.Module):
    """Module with resettable state registered through ``register_memory``."""

    def __init__(self):
        super().__init__()
        self._memories = {}
        self._memories_rv = {}

    def register_memory(self, name, value):
        self._memories[name] = value
        self._memories_rv[name] = value

    def reset(self):
        for k in self._memories:
            self._memories[k] = self._memories_rv[k]

    def __getattr__(self, name):
        mem = self.__dict__.get("_memories")
        if mem is not None and name in mem:
            return mem[name]
        return super().__getattr__(name)

    def __setattr__(self, name, value):
        mem = self.__dict__.get("_memories")
        if mem is not None and name in mem:
            mem[name] = value
        else:
            super().__setattr__(name, value)


class _ATanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, alpha):
        ctx.save_for_backward(x)
        ctx.alpha = alpha
        return (x >= 0).to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        a = ctx.alpha
        return a / 2 / (1 + (math.pi / 2 * a * x).pow(2)) * g, None


class ATan(torch.nn.Module):
    """Heaviside spike with the arctangent surrogate gradient."""

    def __init__(self, alpha: float = 2.0, spiking: bool = True):
        super().__init__()
        self.alpha = alpha
        self.spiking = spiking

    def forward(self, x):
        return _ATanFn.apply(x, self.alpha)


class LIFNode(MemoryModule):
    """Leaky integrate-and-fire neuron (tau, v_threshold, v_reset (None = soft reset),
    surrogate_function, detach_reset).  Multi-step mode runs the CUDA kernel; only
    ``decay_input=False`` is supported (the reference's fused kernels assume it too)."""

    def __init__(self, tau: float = 2.0, decay_input: bool = True, v_threshold: float = 1.0,
                 v_reset=0.0, surrogate_function=None, detach_reset: bool = False,
                 step_mode: str = "s", backend: str = "torch", store_v_seq: bool = False):
        super().__init__()
        self.tau = tau
        self.decay_input = decay_input
        self.v_threshold = v_threshold
        self.v_reset = v_reset
        self.surrogate_function = surrogate_function if surrogate_function is not None else ATan()
        self.detach_reset = detach_reset
        self.step_mode = step_mode
        self.backend = backend
        self.store_v_seq = store_v_seq
        self.register_memory("v", 0.0 if v_reset is None else v_reset)

    def _lif_args(self):
        surr = self.surrogate_function
        from .utils import Triangle
        if "ATan" in type(surr).__name__:
            sid, alpha = 1, float(getattr(surr, "alpha", 2.0))
        else:
            sid, alpha = 0, 2.0
        gamma = 1.0
        if surr is not Triangle.apply and hasattr(surr, "gamma"):
            gamma = float(surr.gamma)
        return (self.tau, self.v_threshold, self.v_reset, self.detach_reset, sid, gamma, alpha)

    def forward(self, x):
        if self.step_mode != "m":
            raise NotImplementedError("delrec_b200 LIFNode runs in multi-step mode ('m') only")
        if self.decay_input:
            raise NotImplementedError("decay_input=True is not supported by the CUDA kernels")
        return Fn.LIFMultiStep.apply(x, self._lif_args())

    def extra_repr(self):
        return (f"tau={self.tau}, v_threshold={self.v_threshold}, v_reset={self.v_reset}, "
                f"detach_reset={self.detach_reset}, step_mode={self.step_mode}")


class Dropout(MemoryModule):
    """Dropout whose mask is drawn once (on the first call after ``reset``) and reused,
    so a recurrent layer sees the same mask at every time step."""

    def __init__(self, p: float = 0.5, step_mode: str = "s"):
        super().__init__()
        self.p = p
        self.step_mode = step_mode
        self.register_memory("mask", None)

    def create_mask(self, x):
        self.mask = F.dropout(torch.ones_like(x), self.p, training=True)

    def forward(self, x):
        if not self.training or self.p <= 0:
            return x
        if self.step_mode == "m":
            if self.mask is None:
                self.create_mask(x[0])
            return x * self.mask
        if self.mask is None:
            self.create_mask(x)
        return x * self.mask

    def extra_repr(self):
        return f"p={self.p}, step_mode={self.step_mode}"


class BatchNorm1d(torch.nn.BatchNorm1d):
    """Multi-step batch norm over (T, B, N, 1) inputs flattened on (T*B)."""

    def __init__(self, num_features, step_mode="m", **kw):
        super().__init__(num_features, **kw)
        self.step_mode = step_mode

    def forward(self, x):
        if self.step_mode == "m" and x.dim() >= 3:
            shp = x.shape
            y = super().forward(x.flatten(0, 1))
            return y.view(shp)
        return super().forward(x)
