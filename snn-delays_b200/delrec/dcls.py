"""A Dcls1d-compatible module (learnable-position dilated convolution, the DCLS 0.1.1
``construct.modules.Dcls1d`` the reference builds ``dcls_module`` on,
networks.py:18-50) running on the CUDA DCLS kernels of this package.

Parameters keep DCLS's layout: weight (C_out, C_in/groups, kernel_count),
P and SIG (1, C_out, C_in/groups, kernel_count), bias (C_out).  Only the Gaussian
('gauss') construction with kernel_count == 1 is provided.  DCLS itself is not part of
the reference tree, so its numerics are restated from its published method and are not
pinned to DCLS outputs.
"""

from __future__ import annotations

import math

import torch

from . import functional as Fn


class Dcls1d(torch.nn.Module):
    def __init__(self, in_channels, out_channels, kernel_count=1, stride=1, padding=0,
                 dilated_kernel_size=1, groups=1, bias=True, padding_mode="zeros", version="gauss"):
        super().__init__()
        if version != "gauss" or kernel_count != 1:
            raise NotImplementedError("Dcls1d: only version='gauss' with kernel_count=1 is provided")
        if in_channels % groups or out_channels % groups:
            raise ValueError("in_channels and out_channels must be divisible by groups")
        self.in_channels, self.out_channels = in_channels, out_channels
        self.kernel_count, self.groups, self.version = kernel_count, groups, version
        self.dilated_kernel_size = (dilated_kernel_size,) if isinstance(dilated_kernel_size, int) \
            else tuple(dilated_kernel_size)
        cin_g = in_channels // groups
        self.weight = torch.nn.Parameter(torch.empty(out_channels, cin_g, kernel_count))
        self.P = torch.nn.Parameter(torch.empty(1, out_channels, cin_g, kernel_count))
        self.SIG = torch.nn.Parameter(torch.empty(1, out_channels, cin_g, kernel_count))
        self.bias = torch.nn.Parameter(torch.empty(out_channels)) if bias else None
        self.reset_parameters()

    def reset_parameters(self):
        torch.nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        lim = self.dilated_kernel_size[0] // 2
        with torch.no_grad():
            self.P.uniform_(-lim, lim)
            self.SIG.fill_(0.23 * max(lim, 1))
        if self.bias is not None:
            fan_in = (self.in_channels // self.groups) * self.kernel_count
            bound = 1.0 / math.sqrt(fan_in)
            torch.nn.init.uniform_(self.bias, -bound, bound)

    def clamp_parameters(self):
        lim = self.dilated_kernel_size[0] // 2
        from .networks import learned_delay_parameter
        with torch.no_grad():
            learned_delay_parameter(self, "P").clamp_(-lim, lim)

    def conv_time_major(self, x, left_padding, right_padding):
        K = self.dilated_kernel_size[0]
        if left_padding + right_padding != K - 1:
            raise NotImplementedError("Dcls1d: only the length-preserving causal padding "
                                      "(left + right == kernel size - 1) is provided")
        return Fn.DclsConv1d.apply(x, self.weight, self.P, self.SIG, self.bias, K, self.groups,
                                   left_padding)

    def forward(self, x):
        """(B, C_in, T) -> (B, C_out, T) with symmetric 'same' padding."""
        K = self.dilated_kernel_size[0]
        y = self.conv_time_major(x.permute(2, 0, 1).contiguous(), (K - 1) // 2, K - 1 - (K - 1) // 2)
        return y.permute(1, 2, 0)
