"""Helpers used by the model zoo: the Triangle surrogate and ``reset_states``
(src/delrec/utils.py:23-46)."""

import torch


class Triangle(torch.autograd.Function):
    """Spike = [x >= 0]; surrogate gradient (1/gamma)^2 * max(0, gamma - |x|)."""

    @staticmethod
    def forward(ctx, input, gamma=1.0):
        ctx.save_for_backward(input)
        ctx.gamma = float(gamma)
        return input.ge(0.).float()

    @staticmethod
    def backward(ctx, grad_output):
        (input,) = ctx.saved_tensors
        g = ctx.gamma
        return grad_output * ((1 / g) * (1 / g) * (g - input.abs()).clamp(min=0)), None


def reset_states(model):
    """Reset every stateful module (LIF membranes, dropout masks) before a forward."""
    for m in model.modules():
        if hasattr(m, "reset"):
            m.reset()
