"""Recurrent spiking layers with learnable transmission delays — the drop-in modules.

    vanilla_recurrent   recurrent LIF without delays
    axonal_recdel       one delay per source neuron        d_j   (N,)
    synaptic_recdel     one delay per connection           d_ij  (N, N)
    common_recdel       one delay shared by the whole layer      (1,)

Same constructors, parameter names, ``state_dict`` layout, ``sigma`` attribute (not a
buffer), ``update_sigma(epoch)`` annealing and ``forward(x_seq (T,B,N)) -> spikes``
as src/delrec/delay_layers.py:34-304.  ``forward`` always runs the CUDA kernels of
libdelrec_b200.so; CPU tensors raise (the reference's pure-PyTorch scans are not part
of this package).  A hybrid layer (``_hybrid_delay`` tag set by the model zoo's
reparametrization) routes to the hybrid kernels with the learned (N,) base and the
frozen (N,N) offsets, instead of materialising the (N,N) delay.
"""

from __future__ import annotations

import torch

from . import functional as Fn
from .neuron import Dropout, LIFNode, MemoryModule

# forward_version values that select the CUDA kernels; the pure-PyTorch reference scans
# ('v1', 'v2') are not shipped with this package.
_CUDA_VERSIONS = (None, "triton_exact", "triton_approx", "triton_ste", "eventdriven", "hybrid_triton",
                  "cuda")
AXONAL_CUDA_DEFAULT = "triton_exact"
SYNAPTIC_CUDA_DEFAULT = "eventdriven"


def _make_recurrent_dropout(config):
    return Dropout(config.recurrent_dropout_rate, step_mode="s")


def _check_cuda(x_seq, layer):
    if not x_seq.is_cuda:
        raise RuntimeError(
            f"{type(layer).__name__}: delrec_b200 runs on CUDA only; move the model and "
            "inputs to a CUDA device (there is no CPU fallback)")
    fv = getattr(layer, "forward_version", None)
    if fv in ("v1", "v2", "eventdriven_torch"):
        raise NotImplementedError(
            f"forward_version={fv!r} is the reference's pure-PyTorch scan, which this package "
            "does not ship; leave forward_version unset to run the CUDA kernels")
    if fv not in _CUDA_VERSIONS:
        raise ValueError(f"unknown forward_version {fv!r}")
    if getattr(layer.neuron_module, "decay_input", False):
        raise NotImplementedError("decay_input=True is not supported by the CUDA kernels")


def _axonal_variant(layer):
    """forward_version -> the axonal scan's (approx, ste_mode) (delay_layers.py:204-211,
    delay_layers_triton.py:60-61): 'triton_approx' is the straight-through single-tap
    scan, 'triton_ste' the hard-tap forward with the soft backward -- rounded taps, or
    the 2-tap interpolation when config.ste_round_forward is False."""
    fv = getattr(layer, "forward_version", None)
    if fv == "triton_approx":
        return dict(approx=True, ste_mode=0)
    if fv == "triton_ste":
        return dict(approx=False, ste_mode=1 if getattr(layer.config, "ste_round_forward", True) else 2)
    return dict(approx=False, ste_mode=0)


def _keep_mask(layer, B, N, x_seq):
    """One fixed recurrent-dropout mask per forward, drawn from the layer's own dropout
    module exactly as the reference does (delay_layers_triton.py:43-48)."""
    if layer.training and layer.config.recurrent_dropout_rate > 0:
        ones = torch.ones(B, N, device=x_seq.device, dtype=x_seq.dtype)
        return layer.dropout(ones)
    return None


class vanilla_recurrent(MemoryModule):
    """Delay-free recurrent LIF layer: rec = dropout(y[t-1]) @ W with W (N_in, N_out)
    (delay_layers.py:34-74).  Runs as an axonal layer with d = 0, sigma = 0 and W^T."""

    def __init__(self, config, neurons: int, neuron_module=LIFNode):
        super().__init__()
        self.config = config
        self.step_mode = config.step_mode
        self.store_v_seq = config.store_v_seq
        self.neuron_module = neuron_module(
            tau=config.tau, decay_input=config.decay_input, v_reset=config.v_reset,
            v_threshold=config.v_threshold, surrogate_function=config.surrogate_function,
            detach_reset=config.detach_reset, step_mode="s", backend=config.backend)
        self.neurons = neurons
        self.recurrent_weights = torch.nn.Parameter(torch.zeros(neurons, neurons), requires_grad=True)
        self.dropout = _make_recurrent_dropout(config)
        self.init_recurrent_weights()

    def init_recurrent_weights(self):
        torch.nn.init.orthogonal_(self.recurrent_weights, gain=1.0)

    def forward(self, x_seq: torch.Tensor):
        if self.step_mode == "s":
            raise NotImplementedError("single-step mode is not supported")
        _check_cuda(x_seq, self)
        T, B, N = x_seq.shape
        if self.training and self.config.recurrent_dropout_rate > 0:
            raise NotImplementedError("vanilla_recurrent with recurrent dropout (dropout on the "
                                      "presynaptic spikes) is not supported")
        sid, gamma, alpha = Fn.surrogate_params(self.config)
        nm = self.neuron_module
        d = torch.zeros(N, device=x_seq.device)
        y = Fn.AxonalRecdelTriton.apply(
            x_seq, self.recurrent_weights.t(), None, d, None, None, 0.0, nm.tau, nm.v_threshold,
            nm.v_reset, False, self.config.detach_reset, sid, gamma, False, 0, alpha)
        self.x_seq = x_seq
        if self.store_v_seq:
            self.v_seq = None
        return y


class axonal_recdel(MemoryModule):
    """Per-neuron (axonal) delays d (N,), W (N,N) with W[i,j] target i, source j
    (delay_layers.py:86-216)."""

    def __init__(self, config, neurons: int, neuron_module=LIFNode):
        super().__init__()
        self.config = config
        self.step_mode = config.step_mode
        self.store_v_seq = config.store_v_seq
        self.neuron_module = neuron_module(
            tau=config.tau, decay_input=config.decay_input, v_reset=config.v_reset,
            v_threshold=config.v_threshold, surrogate_function=config.surrogate_function,
            detach_reset=config.detach_reset, step_mode="s", backend=config.backend)
        self.neurons = neurons
        self.sigma = float(self.config.sigma_init)
        self.round_delays = getattr(config, "round_delays", False)
        self.recurrent_weights = torch.nn.Parameter(torch.zeros(neurons, neurons), requires_grad=True)
        self.recurrent_delays = torch.nn.Parameter(torch.zeros(neurons), requires_grad=True)
        self.dropout = _make_recurrent_dropout(config)
        self.use_sig_p = config.use_sig_p
        if self.use_sig_p:
            self.p_spread = torch.nn.Parameter(torch.zeros(neurons), requires_grad=True)
        self.use_rec_bias = getattr(config, "use_rec_bias", False)
        if self.use_rec_bias:
            self.recurrent_bias = torch.nn.Parameter(torch.zeros(neurons), requires_grad=True)
        self.init_recurrent_weights()
        self.init_recurrent_delays()

    def init_recurrent_weights(self):
        init_mode = getattr(self.config, "init_rec_weights", "orthogonal")
        if init_mode == "orthogonal":
            torch.nn.init.orthogonal_(self.recurrent_weights, gain=self.config.rec_delay_init_gain)
        elif init_mode == "kaiming_uniform":
            torch.nn.init.kaiming_uniform_(self.recurrent_weights, a=5 ** 0.5)
        else:
            raise ValueError(f"Unknown init_rec_weights '{init_mode}' "
                             "(expected 'orthogonal' or 'kaiming_uniform').")
        if getattr(self, "use_rec_bias", False):
            bound = 1.0 / (self.recurrent_weights.shape[1] ** 0.5)
            torch.nn.init.uniform_(self.recurrent_bias, -bound, bound)

    def init_recurrent_delays(self):
        with torch.no_grad():
            mode = self.config.init_rec_delay
            if mode == "half_normal":
                hn = torch.abs(torch.randn_like(self.recurrent_delays) * self.config.delay_std_init)
                self.recurrent_delays.copy_(hn)
                self.recurrent_delays.clamp_(min=0.0)
            elif mode == "uniform_integer":
                maximum = self.config.hybrid_offset_scale
                if int(maximum) != maximum or maximum < 0:
                    raise ValueError("hybrid_offset_scale must be a nonnegative integer")
                self.recurrent_delays.copy_(torch.randint(
                    0, int(maximum) + 1, self.recurrent_delays.shape,
                    device=self.recurrent_delays.device))
            elif mode == "uniform":
                torch.nn.init.uniform_(self.recurrent_delays, a=self.config.init_recdel_offset,
                                       b=self.config.max_rec_delay)
                self.recurrent_delays.clamp_(min=0.0)

    def update_sigma(self, current_epoch):
        """sigma_epoch = sigma_init * (sigma_decay^(100/epochs))^epoch (Eq. 13).  ``sigma``
        is a plain attribute, not in the state_dict."""
        decay_per_epoch = self.config.sigma_decay ** (100 / self.config.epochs)
        self.sigma = self.config.sigma_init * (decay_per_epoch ** current_epoch)

    def clamp_recurrent_delays(self):
        with torch.no_grad():
            self.recurrent_delays.clamp_(min=0)

    # -- CUDA path ------------------------------------------------------------------
    def multi_step_forward_triton(self, x_seq: torch.Tensor, approx: bool = False, ste_mode: int = 0):
        T, B, N = x_seq.shape
        sid, gamma, alpha = Fn.surrogate_params(self.config)
        keep = _keep_mask(self, B, N, x_seq)
        p_spread = self.p_spread if self.use_sig_p else None
        bias = self.recurrent_bias if self.use_rec_bias else None
        d_in = self.recurrent_delays
        if self.round_delays:
            d_in = d_in + (d_in.round() - d_in).detach()
        nm = self.neuron_module
        y = Fn.AxonalRecdelTriton.apply(
            x_seq, self.recurrent_weights, bias, d_in, p_spread, keep, float(self.sigma),
            nm.tau, nm.v_threshold, nm.v_reset, self.use_sig_p, self.config.detach_reset,
            sid, gamma, approx, ste_mode, alpha)
        self.x_seq = x_seq
        self.rec_now_seq = None
        if self.store_v_seq:
            self.v_seq = None
        return y

    def forward(self, x_seq: torch.Tensor):
        if self.step_mode == "s":
            raise NotImplementedError("single-step mode is not supported")
        _check_cuda(x_seq, self)
        return self.multi_step_forward_triton(x_seq, **_axonal_variant(self))


class synaptic_recdel(axonal_recdel):
    """Per-connection delays d (N,N) (delay_layers.py:219-284).  A hybrid layer (tagged
    ``_hybrid_delay`` with ``recurrent_delays`` parametrized as base + frozen offsets)
    runs the hybrid kernels."""

    def __init__(self, config, neurons: int, neuron_module=LIFNode):
        super().__init__(config=config, neurons=neurons, neuron_module=neuron_module)
        self.recurrent_delays = torch.nn.Parameter(torch.zeros(neurons, neurons), requires_grad=True)
        self.init_recurrent_delays()

    def multi_step_forward_eventdriven(self, x_seq: torch.Tensor):
        T, B, N = x_seq.shape
        keep = _keep_mask(self, B, N, x_seq)
        bias = self.recurrent_bias if self.use_rec_bias else None
        p_spread = self.p_spread if self.use_sig_p else torch.zeros(N, device=x_seq.device)
        y = Fn.EventDrivenSyn.apply(x_seq, self.recurrent_weights, self.recurrent_delays,
                                    p_spread, bias, keep, self)
        self.x_seq = x_seq
        self.rec_now_seq = None
        if self.store_v_seq:
            self.v_seq = None
        return y

    def multi_step_forward_hybrid_triton(self, x_seq: torch.Tensor):
        from torch.nn.utils import parametrize
        T, B, N = x_seq.shape
        keep = _keep_mask(self, B, N, x_seq)
        bias = self.recurrent_bias if self.use_rec_bias else None
        if parametrize.is_parametrized(self, "recurrent_delays"):
            par = self.parametrizations.recurrent_delays
            rep = par[0]
            base = par.original
            if tuple(base.shape) == (N,) and getattr(rep, "position_shift", 0.0) == 0.0 \
                    and getattr(rep, "position_sign", 1.0) == 1.0:
                p_spread = self.p_spread if self.use_sig_p else torch.zeros(N, device=x_seq.device)
                y = Fn.HybridBaseDelay.apply(x_seq, self.recurrent_weights, base, rep.offsets,
                                             p_spread, bias, keep, self)
                self.x_seq = x_seq
                self.rec_now_seq = None
                if self.store_v_seq:
                    self.v_seq = None
                return y
        y = Fn.HybridSynDelay.apply(x_seq, self.recurrent_weights, self.recurrent_delays,
                                    bias, keep, self)
        self.x_seq = x_seq
        self.rec_now_seq = None
        if self.store_v_seq:
            self.v_seq = None
        return y

    def forward(self, x_seq: torch.Tensor):
        if self.step_mode == "s":
            raise NotImplementedError("single-step mode is not supported")
        _check_cuda(x_seq, self)
        fv = getattr(self, "forward_version", None)
        if fv == "hybrid_triton" or (fv is None and getattr(self, "_hybrid_delay", False)):
            return self.multi_step_forward_hybrid_triton(x_seq)
        return self.multi_step_forward_eventdriven(x_seq)


class common_recdel(axonal_recdel):
    """One learnable delay shared by every neuron of the layer, recurrent_delays (1,)
    (delay_layers.py:287-304)."""

    def __init__(self, config, neurons: int, neuron_module=LIFNode):
        super().__init__(config=config, neurons=neurons, neuron_module=neuron_module)
        self.recurrent_delays = torch.nn.Parameter(torch.zeros(1), requires_grad=True)
        self.init_recurrent_delays()

    def multi_step_forward_triton(self, x_seq, approx=False, ste_mode=0):
        T, B, N = x_seq.shape
        sid, gamma, alpha = Fn.surrogate_params(self.config)
        keep = _keep_mask(self, B, N, x_seq)
        p_spread = self.p_spread if self.use_sig_p else None
        bias = self.recurrent_bias if self.use_rec_bias else None
        d_in = self.recurrent_delays
        if self.round_delays:
            d_in = d_in + (d_in.round() - d_in).detach()
        d_in = d_in.expand(N).contiguous()
        nm = self.neuron_module
        y = Fn.AxonalRecdelTriton.apply(
            x_seq, self.recurrent_weights, bias, d_in, p_spread, keep, float(self.sigma),
            nm.tau, nm.v_threshold, nm.v_reset, self.use_sig_p, self.config.detach_reset,
            sid, gamma, approx, ste_mode, alpha)
        self.x_seq = x_seq
        self.rec_now_seq = None
        return y

    def forward(self, x_seq):
        if self.step_mode == "s":
            raise NotImplementedError("single-step mode is not supported")
        _check_cuda(x_seq, self)
        return self.multi_step_forward_triton(x_seq, **_axonal_variant(self))
