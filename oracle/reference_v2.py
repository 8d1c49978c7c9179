"""The reference's own CPU path, loaded unmodified for the benchmark's reference arm.

TEST / MEASUREMENT INFRASTRUCTURE ONLY -- nothing in the product package imports this
module.  It loads ``delay_layers_pytorch.py`` (the reference's pure-PyTorch scans,
src/delrec/delay_layers_pytorch.py:121-194 axonal and :271-325 synaptic
``multi_step_forward_v2``, the CPU default of the reference) from an installed copy of the
reference package -- ``baseline/_ref`` made by

    python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
        --target baseline/_ref <copy of the reference checkout> --no-deps

-- under a private module name (the file imports only torch, and the reference package is
also called ``delrec``, like this repository's package), and drives the scans with the
host object their mixins expect (the attributes delay_layers.py:100-143 sets) and the
oracle's SpikingJelly-equivalent LIF neuron (that dependency is not installed here).
"""

import importlib.util
import os

import torch

from oracle.delrec_oracle import OracleLIF

_MOD = None


def load(root):
    """The reference's delay_layers_pytorch module from ``root`` (a pip --target
    directory), or None when it is not installed there."""
    global _MOD
    if _MOD is not None:
        return _MOD
    path = os.path.join(root, "delrec", "delay_layers_pytorch.py")
    if not os.path.exists(path):
        return None
    spec = importlib.util.spec_from_file_location("reference_delay_layers_pytorch", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    _MOD = mod
    return mod


class _Host:
    """The attributes the reference's v2 scan mixins read."""

    def __init__(self, W, d, sigma, lif, bias=None, keep=None):
        self.recurrent_weights = W
        self.recurrent_delays = d
        self.sigma = sigma
        self.neuron_module = lif
        self.use_sig_p = False
        self.p_spread = torch.zeros(W.shape[0])
        self.round_delays = False
        self.use_rec_bias = bias is not None
        self.recurrent_bias = bias
        self.store_v_seq = False
        self.neurons = W.shape[0]
        self._keep = keep

    def dropout(self, r):
        return r if self._keep is None else r * self._keep


def scan(mod, kind, x, W, d, lif: OracleLIF, sigma=0.0, bias=None):
    """One recurrent delay layer through the reference's multi_step_forward_v2:
    ``kind`` "axonal" (d (N,)) or "synaptic" (d (N,N); the hybrid model passes its
    materialised base + offsets, as the reference's hybrid layer does)."""
    base = mod.AxonalTorchScans if kind == "axonal" else mod.SynapticTorchScans
    host_cls = type("ReferenceHost", (_Host, base), {})
    lif.reset()
    host = host_cls(W, d, sigma, lif, bias)
    return host.multi_step_forward_v2(x)
