"""Network zoo around the delay layers (the constructors and state_dict layout of
src/delrec/networks.py), running on the CUDA kernels of this package.

A hidden block is  projection -> Dropout -> [recurrent delay layer | LIF] ->
spike_registrator -> [BatchNorm]; the network ends in a Linear readout.  Hybrid
delays tie a (N, N) delay tensor to one learned (N,) leaf plus frozen integer offsets
through ``torch.nn.utils.parametrize`` exactly as networks.py:802-984 does, so the
parameter names (``parametrizations.recurrent_delays.original``) and offset buffers
(``parametrizations.recurrent_delays.0.offsets``) are unchanged.
"""

from __future__ import annotations

import math
from copy import copy

import torch

from .dcls import Dcls1d
from .delay_layers import axonal_recdel, common_recdel, synaptic_recdel
from .linear import Linear, readout_time_sum
from .neuron import BatchNorm1d, Dropout


def _lif(config, step_mode=None):
    return config.neuron_module(
        tau=config.tau, decay_input=config.decay_input, v_reset=config.v_reset,
        v_threshold=config.v_threshold, surrogate_function=config.surrogate_function,
        detach_reset=config.detach_reset, step_mode=step_mode or config.step_mode,
        backend=config.backend, store_v_seq=config.store_v_seq)


class dcls_module(Dcls1d):
    """Causal (left-padded) DCLS convolution over time: (T,B,N_in) -> (T,B,N_out)
    (networks.py:22-50)."""

    def __init__(self, config, in_channels, out_channels, groups):
        super().__init__(in_channels=in_channels, out_channels=out_channels,
                         kernel_count=config.kernel_count, groups=groups,
                         dilated_kernel_size=config.max_feedforward_delay, bias=config.bias,
                         version=config.DCLSversion)
        self.config = config
        self.left_padding, self.right_padding = config.left_padding, config.right_padding

    def forward(self, x):
        assert x.dim() == 3  # (T, B, N)
        return self.conv_time_major(x, self.left_padding, self.right_padding)


class modified_batchnorm(BatchNorm1d):
    def __init__(self, num_features, step_mode="m"):
        super().__init__(num_features, step_mode=step_mode)


class spike_registrator(torch.nn.Module):
    """Pass-through that keeps a copy of the spike trains (firing-rate penalties)."""

    def __init__(self):
        super().__init__()
        self.spikes = None

    def forward(self, x):
        assert x.dim() == 3
        self.spikes = x.clone()
        return x


def _spike_input(config, idx):
    """The input of the idx-th projection is a spike train (0/1) when a spiking layer
    feeds it directly.  The first projection's data is tested on every call (None), which
    costs a read of the test's result (a synchronisation) per forward, unless the optional
    ``config.input_spikes`` declares it: True for datasets of 0/1 spike trains (checked on
    the device through the status word), False for real-valued inputs."""
    if idx == 0:
        v = getattr(config, "input_spikes", None)
        return None if v is None else bool(v)
    return False if config.use_batch_norm else True


def _init_ff(m, config):
    if isinstance(m, torch.nn.Linear):
        if config.init_ff_weights == "kaiming":
            torch.nn.init.kaiming_uniform_(m.weight, nonlinearity="relu")
        elif config.init_ff_weights == "normal":
            torch.nn.init.normal_(m.weight, mean=0.0, std=0.1)


class SNN(torch.nn.Module):
    """Feedforward LIF network: Linear -> Dropout -> LIF -> spike_registrator per layer."""

    def __init__(self, config):
        super().__init__()
        assert config.dataset in ["SSC", "PSMNIST", "HAR", "AL", "MG", "MEM"], "Unsupported SNN dataset."
        self.config = config
        layers, dim = [], config.input_size
        for idx, width in enumerate(config.hidden_layers):
            layers.append(Linear(dim, width, bias=config.bias, binary_input=_spike_input(config, idx)))
            dim = width
            layers.append(Dropout(config.feedforward_dropout_rate, step_mode="m"))
            layers.append(_lif(config))
            layers.append(spike_registrator())
            if config.use_batch_norm:
                layers.append(modified_batchnorm(width, step_mode="m"))
        layers.append(Linear(dim, config.output_size, bias=config.bias,
                             binary_input=_spike_input(config, len(config.hidden_layers))))
        self.layers = torch.nn.Sequential(*layers)
        self.init_weights()

    def forward(self, x):
        assert x.dim() == 3
        return self.layers(x)

    def forward_time_summed(self, x):
        """sum_t forward(x)[t], (B, output_size): what the SSC / PS-MNIST loss feeds to the
        cross-entropy (utils.py:188-200, calc_loss_SSC).  With a Linear readout the
        projection and the time sum run fused in the library, and the (T,B,C) readout is
        never formed; with a DCLS readout it is forward(x).sum(0)."""
        assert x.dim() == 3
        last = self.layers[-1]
        if type(last) is not Linear:
            return self.forward(x).sum(0)
        h = x
        for m in self.layers[:-1]:
            h = m(h)
        return readout_time_sum(h, last.weight, last.bias)

    def init_weights(self):
        for m in self.layers:
            _init_ff(m, self.config)


def _recurrent_stack(config, recurrent_cls):
    layers, dim = [], config.input_size
    for idx, width in enumerate(config.hidden_layers):
        layers.append(Linear(dim, width, bias=config.bias, binary_input=_spike_input(config, idx)))
        dim = width
        layers.append(Dropout(config.feedforward_dropout_rate, step_mode="m"))
        last = idx == len(config.hidden_layers) - 1
        if last and getattr(config, "no_recurrence_in_last_layer", False):
            layers.append(_lif(config))
        else:
            layers.append(recurrent_cls(config, width, config.neuron_module))
        layers.append(spike_registrator())
        if config.use_batch_norm:
            layers.append(modified_batchnorm(width, step_mode="m"))
    layers.append(Linear(dim, config.output_size, bias=config.bias,
                         binary_input=_spike_input(config, len(config.hidden_layers))))
    return torch.nn.Sequential(*layers)


class SNN_axonal_recurrent_delays(SNN):
    """Recurrent layers with learned axonal delays (networks.py:140-231)."""

    def __init__(self, config, _recurrent_cls=axonal_recdel):
        super().__init__(config)
        self.config = config
        self.layers = _recurrent_stack(config, _recurrent_cls)
        self.init_weights()

    def clamp_delays(self):
        for m in self.layers:
            if isinstance(m, axonal_recdel):
                m.clamp_recurrent_delays()

    def round_pos(self):
        stochastic = getattr(self.config, "round_mode", "nearest") == "stochastic"
        with torch.no_grad():
            for m in self.layers:
                if isinstance(m, axonal_recdel):
                    d = m.recurrent_delays
                    if stochastic:
                        d.copy_(torch.floor(d + torch.rand_like(d)))
                    else:
                        d.round_()
                    m.clamp_recurrent_delays()

    def log_params(self):
        logs = {}
        for idx, layer in enumerate(self.layers):
            if isinstance(layer, axonal_recdel):
                logs[f"sigma_rec{idx}"] = layer.sigma
                logs[f"pos_rec{idx}"] = float(learned_delay_parameter(layer, "recurrent_delays").detach().mean())
        return logs


class SNN_synaptic_recurrent_delays(SNN_axonal_recurrent_delays):
    """Per-connection learned delays (networks.py:234-280)."""

    def __init__(self, config):
        SNN_axonal_recurrent_delays.__init__(self, config, synaptic_recdel)


class SNN_common_recurrent_delays(SNN_axonal_recurrent_delays):
    """One shared learned delay per recurrent layer (networks.py:283-324)."""

    def __init__(self, config):
        SNN_axonal_recurrent_delays.__init__(self, config, common_recdel)


def _freeze_delays(model, round_first):
    for layer in model.layers:
        if isinstance(layer, axonal_recdel):
            with torch.no_grad():
                if round_first:
                    layer.recurrent_delays.round_()
                    layer.clamp_recurrent_delays()
                else:
                    layer.recurrent_delays.fill_(0.0)
            layer.recurrent_delays.requires_grad = False
            layer.sigma = 0.0
            layer.config.sigma_init = 0.0
            layer.use_sig_p = False
            if hasattr(layer, "p_spread"):
                del layer.p_spread


class SNN_vanilla_recurrent(SNN_axonal_recurrent_delays):
    """Recurrent layers with every delay frozen at 0 (lag 1) (networks.py:327-347)."""

    def __init__(self, config):
        super().__init__(config)
        _freeze_delays(self, round_first=False)


class SNN_fixed_recurrent_delays(SNN_axonal_recurrent_delays):
    """Axonal delays frozen at their rounded initial values (networks.py:349-371)."""

    def __init__(self, config):
        super().__init__(config)
        _freeze_delays(self, round_first=True)


class SNN_fixed_synaptic_recurrent_delays(SNN_synaptic_recurrent_delays):
    """Synaptic delays frozen at their rounded initial values (networks.py:373-400)."""

    def __init__(self, config):
        super().__init__(config)
        _freeze_delays(self, round_first=True)


# ----------------------------------------------------------------------------------
# feedforward (DCLS) delays
# ----------------------------------------------------------------------------------


def _init_dcls(m, config, mode):
    if mode == "kaiming":
        torch.nn.init.kaiming_uniform_(m.weight, nonlinearity="relu")
    elif mode == "normal":
        torch.nn.init.normal_(m.weight, mean=0.0, std=0.1)
    elif mode == "default":
        torch.nn.init.kaiming_uniform_(m.weight, a=math.sqrt(5))
    torch.nn.init.uniform_(m.P, a=config.init_pos_a, b=config.init_pos_b)
    m.clamp_parameters()


class SNN_synaptic_feedforward_delays(SNN):
    """Dense DCLS projections with one learned delay per synapse (networks.py:402-519)."""

    def __init__(self, config):
        super().__init__(config)
        self.config = config
        layers, dim = [], config.input_size
        for idx, width in enumerate(config.hidden_layers):
            if config.no_delay_in_first_layer and idx == 0:
                layers.append(Linear(dim, width, bias=config.bias))
            else:
                layers.append(dcls_module(config, dim, width, groups=1))
            dim = width
            layers.append(Dropout(config.feedforward_dropout_rate, step_mode="m"))
            layers.append(_lif(config))
            layers.append(spike_registrator())
            if config.use_batch_norm:
                layers.append(modified_batchnorm(width, step_mode="m"))
        if config.no_delay_in_last_layer:
            layers.append(Linear(dim, config.output_size, bias=config.bias))
        else:
            layers.append(dcls_module(config, dim, config.output_size, groups=1))
        self.layers = torch.nn.Sequential(*layers)
        self.init_weights()

    def init_weights(self):
        for m in self.layers:
            _init_ff(m, self.config)
            if isinstance(m, dcls_module):
                _init_dcls(m, self.config, self.config.init_dcls_weights)

    def clamp_delays(self, train=True):
        for m in self.layers:
            if isinstance(m, dcls_module):
                m.clamp_parameters()

    def round_pos(self):
        with torch.no_grad():
            for m in self.layers:
                if isinstance(m, dcls_module):
                    m.P.round_()
                    m.clamp_parameters()


class SNN_axonal_feedforward_delays(SNN_synaptic_feedforward_delays):
    """Depthwise unit-weight DCLS time shifts followed by a trainable Linear
    (networks.py:521-641)."""

    def __init__(self, config):
        SNN.__init__(self, config)
        self.config = config
        layers, dim = [], config.input_size
        for idx, width in enumerate(config.hidden_layers):
            layers.extend(self._delay_stage(dim, width, delayed=not (config.no_delay_in_first_layer and idx == 0)))
            dim = width
            if config.use_batch_norm:
                layers.append(modified_batchnorm(width, step_mode="m"))
            layers.append(_lif(config))
            layers.append(spike_registrator())
            layers.append(Dropout(config.feedforward_dropout_rate, step_mode="m"))
        layers.extend(self._delay_stage(dim, config.output_size, delayed=not config.no_delay_in_last_layer))
        self.layers = torch.nn.Sequential(*layers)
        self.init_weights()

    def _delay_stage(self, in_dim, out_dim, delayed):
        if not delayed:
            return [Linear(in_dim, out_dim, bias=self.config.bias)]
        dc = copy(self.config)
        dc.bias = False
        return [dcls_module(dc, in_channels=in_dim, out_channels=in_dim, groups=in_dim),
                Linear(in_dim, out_dim, bias=self.config.bias)]

    def init_weights(self):
        for m in self.layers:
            _init_ff(m, self.config)
            if isinstance(m, dcls_module):
                torch.nn.init.constant_(m.weight, 1.0)
                m.weight.requires_grad = False
                torch.nn.init.uniform_(m.P, a=self.config.init_pos_a, b=self.config.init_pos_b)
                m.clamp_parameters()
                if self.config.DCLSversion == "gauss":
                    torch.nn.init.constant_(m.SIG, self.config.siginit)
                    m.SIG.requires_grad = False


class SNN_recurrent_and_feedforward_delays(SNN_synaptic_feedforward_delays, SNN_axonal_recurrent_delays):
    """Dense DCLS projections + axonal recurrent delays (networks.py:643-750)."""

    def __init__(self, config):
        SNN.__init__(self, config)
        self.config = config
        layers, dim = [], config.input_size
        for idx, width in enumerate(config.hidden_layers):
            if config.no_delay_in_first_layer and idx == 0:
                layers.append(Linear(dim, width, bias=config.bias))
            else:
                layers.append(dcls_module(config, dim, width, groups=1))
            dim = width
            layers.append(Dropout(config.feedforward_dropout_rate, step_mode="m"))
            layers.append(axonal_recdel(config, width, config.neuron_module))
            layers.append(spike_registrator())
            if config.use_batch_norm:
                layers.append(modified_batchnorm(width, step_mode="m"))
        if config.no_delay_in_last_layer:
            layers.append(Linear(dim, config.output_size, bias=config.bias))
        else:
            layers.append(dcls_module(config, dim, config.output_size, groups=1))
        self.layers = torch.nn.Sequential(*layers)
        SNN_synaptic_feedforward_delays.init_weights(self)

    def forward(self, x):
        return SNN.forward(self, x)

    def clamp_delays(self):
        SNN_synaptic_feedforward_delays.clamp_delays(self)
        SNN_axonal_recurrent_delays.clamp_delays(self)

    def round_pos(self):
        SNN_synaptic_feedforward_delays.round_pos(self)
        SNN_axonal_recurrent_delays.round_pos(self)


class SNN_axonal_recurrent_and_feedforward_delays(SNN_recurrent_and_feedforward_delays):
    """Axonal delays on both pathways (networks.py:753-799); kernel_count must be 1."""

    recurrent_module = axonal_recdel
    axonal_feedforward = True

    def __init__(self, config):
        torch.nn.Module.__init__(self)
        if config.kernel_count != 1:
            raise ValueError("These paired models require kernel_count=1 (one delay per axon/synapse).")
        self.config = config
        mods, dim = [], config.input_size
        for idx, width in enumerate(config.hidden_layers):
            mods.extend(self._projection(dim, width, not (idx == 0 and config.no_delay_in_first_layer)))
            mods.append(Dropout(config.feedforward_dropout_rate, step_mode="m"))
            last = idx == len(config.hidden_layers) - 1
            if last and getattr(config, "no_recurrence_in_last_layer", False):
                mods.append(_lif(config))
            else:
                mods.append(self.recurrent_module(config, width, config.neuron_module))
            mods.append(spike_registrator())
            if config.use_batch_norm:
                mods.append(modified_batchnorm(width, step_mode="m"))
            dim = width
        mods.extend(self._projection(dim, config.output_size, not config.no_delay_in_last_layer))
        self.layers = torch.nn.Sequential(*mods)
        self.init_weights()

    def _projection(self, inputs, outputs, delayed):
        if not delayed:
            return [Linear(inputs, outputs, bias=self.config.bias)]
        if not self.axonal_feedforward:
            return [dcls_module(self.config, inputs, outputs, groups=1)]
        dc = copy(self.config)
        dc.bias = False
        return [dcls_module(dc, inputs, inputs, groups=inputs),
                Linear(inputs, outputs, bias=self.config.bias)]

    def init_weights(self):
        SNN_synaptic_feedforward_delays.init_weights(self)
        if self.axonal_feedforward:
            for m in self.layers:
                if isinstance(m, dcls_module):
                    torch.nn.init.ones_(m.weight)
                    m.weight.requires_grad_(False)


class SNN_synaptic_recurrent_and_feedforward_delays(SNN_axonal_recurrent_and_feedforward_delays):
    """Per-synapse delays on both pathways (networks.py:802-807)."""

    recurrent_module = synaptic_recdel
    axonal_feedforward = False


# ----------------------------------------------------------------------------------
# hybrid delays: learned axonal base + frozen integer per-synapse offsets
# ----------------------------------------------------------------------------------


class _AxonalWithFixedOffsets(torch.nn.Module):
    """delay = axonal + position_shift + position_sign * offsets (offsets: frozen buffer)."""

    def __init__(self, offsets, position_shift=0.0, position_sign=1.0):
        super().__init__()
        self.register_buffer("offsets", offsets)
        self.position_shift = position_shift
        self.position_sign = position_sign

    def forward(self, axonal):
        assert torch.broadcast_shapes(axonal.shape, self.offsets.shape) == self.offsets.shape, (
            f"axonal {tuple(axonal.shape)} does not broadcast into offsets {tuple(self.offsets.shape)}")
        return axonal + self.position_shift + self.position_sign * self.offsets


def learned_delay_parameter(module, name):
    """The leaf parameter of a (possibly parametrized) delay tensor."""
    from torch.nn.utils import parametrize
    if parametrize.is_parametrized(module, name):
        return getattr(module.parametrizations, name).original
    return getattr(module, name)


_HYBRID_OFFSET_DISTRIBUTIONS = ("uniform", "gaussian", "triangular")


def _hybrid_params(config):
    maximum = getattr(config, "hybrid_offset_scale", 4)
    if int(maximum) != maximum or maximum < 0:
        raise ValueError("hybrid_offset_scale must be a nonnegative integer")
    if config.kernel_count != 1:
        raise ValueError("hybrid delay models require kernel_count=1 (one delay per axon/synapse).")
    distribution = getattr(config, "hybrid_offset_distribution", "uniform")
    if distribution not in _HYBRID_OFFSET_DISTRIBUTIONS:
        raise ValueError(f"hybrid_offset_distribution must be one of {_HYBRID_OFFSET_DISTRIBUTIONS}, "
                         f"got {distribution!r}")
    sigma = getattr(config, "hybrid_offset_sigma", None)
    if distribution == "gaussian" and not (sigma is not None and sigma > 0):
        raise ValueError("distribution 'gaussian' requires a positive hybrid_offset_sigma")
    return int(maximum), getattr(config, "hybrid_delay_seed", 123), distribution, sigma


def _draw_offsets(shape, maximum, generator, distribution="uniform", sigma=None):
    """Frozen integer offsets in [0, maximum] (networks.py:873-907)."""
    if maximum == 0:
        return torch.zeros(shape)
    if distribution == "uniform":
        return torch.randint(maximum + 1, shape, generator=generator).float()
    if distribution == "gaussian":
        draws = torch.normal(maximum / 2.0, float(sigma), size=shape, generator=generator)
        return draws.round().clamp_(0, maximum)
    if distribution == "triangular":
        u = torch.rand(shape, generator=generator)
        draws = torch.where(u < 0.5, maximum * torch.sqrt(u / 2.0),
                            maximum * (1.0 - torch.sqrt((1.0 - u) / 2.0)))
        return draws.round().clamp_(0, maximum)
    raise ValueError(f"Unknown distribution {distribution!r} (expected one of {_HYBRID_OFFSET_DISTRIBUTIONS}).")


def hybrid_centered_base(base, config, *, pathway):
    """Shift the base so the mean effective delay equals the base ('centered')."""
    if getattr(config, "hybrid_base_centering", "normal") != "centered":
        return base
    half = getattr(config, "hybrid_offset_scale", 4) / 2.0
    return base + half if pathway == "feedforward" else base - half


def _reparametrize_feedforward_delay(module, maximum, generator, config, *, freeze_sig,
                                     distribution="uniform", sigma=None):
    """Widen a dense dcls_module by 2*maximum and tie P to one learned delay per source
    plus frozen offsets (networks.py:936-962)."""
    from torch.nn.utils import parametrize
    offsets = _draw_offsets(module.P.shape, maximum, generator, distribution, sigma)
    base = hybrid_centered_base(module.P[:, :1].detach().clone(), config, pathway="feedforward")
    module.dilated_kernel_size = (config.max_feedforward_delay + 2 * maximum,)
    module.left_padding += 2 * maximum
    parametrize.register_parametrization(module, "P", _AxonalWithFixedOffsets(offsets, maximum, -1.0),
                                         unsafe=True)
    module.parametrizations.P.original = torch.nn.Parameter(base)
    if freeze_sig and config.DCLSversion == "gauss":
        torch.nn.init.constant_(module.SIG, config.siginit)
        module.SIG.requires_grad = False


def _reparametrize_recurrent_delay(module, maximum, generator, config, distribution="uniform", sigma=None):
    """Tie a synaptic_recdel's (N,N) recurrent_delays to one learned (N,) leaf plus frozen
    (N,N) offsets (networks.py:965-984)."""
    from torch.nn.utils import parametrize
    offsets = _draw_offsets(module.recurrent_delays.shape, maximum, generator, distribution, sigma)
    base = hybrid_centered_base(module.recurrent_delays[0].detach().clone(), config, pathway="recurrent")
    parametrize.register_parametrization(module, "recurrent_delays", _AxonalWithFixedOffsets(offsets),
                                         unsafe=True)
    module.parametrizations.recurrent_delays.original = torch.nn.Parameter(base)
    module._hybrid_delay = True
    module.forward_version = None


class SNN_hybrid_recurrent_and_feedforward_delays(SNN_synaptic_recurrent_and_feedforward_delays):
    """Hybrid delays on both pathways (networks.py:987-1042)."""

    def __init__(self, config):
        maximum, seed, distribution, sigma = _hybrid_params(config)
        self._hybrid_max = maximum
        self.recurrent_module, self.axonal_feedforward = synaptic_recdel, False
        SNN_axonal_recurrent_and_feedforward_delays.__init__(self, config)
        generator = torch.Generator().manual_seed(seed)
        self.base_position_bound = config.max_feedforward_delay // 2
        for module in self.layers:
            if isinstance(module, dcls_module):
                _reparametrize_feedforward_delay(module, maximum, generator, config, freeze_sig=False,
                                                 distribution=distribution, sigma=sigma)
            elif isinstance(module, axonal_recdel):
                _reparametrize_recurrent_delay(module, maximum, generator, config, distribution, sigma)

    def clamp_delays(self):
        with torch.no_grad():
            for module in self.layers:
                if isinstance(module, dcls_module):
                    learned_delay_parameter(module, "P").clamp_(-self.base_position_bound, self.base_position_bound)
                elif isinstance(module, axonal_recdel):
                    learned_delay_parameter(module, "recurrent_delays").clamp_(min=0)

    def round_pos(self):
        with torch.no_grad():
            for module in self.layers:
                if isinstance(module, dcls_module):
                    learned_delay_parameter(module, "P").round_()
                elif isinstance(module, axonal_recdel):
                    learned_delay_parameter(module, "recurrent_delays").round_()
        self.clamp_delays()


class SNN_hybrid_feedforward_delays(SNN_axonal_feedforward_delays):
    """Feedforward-only hybrid delays (networks.py:1045-1125)."""

    def __init__(self, config):
        self._hybrid_max, seed, distribution, sigma = _hybrid_params(config)
        super().__init__(config)
        maximum = self._hybrid_max
        generator = torch.Generator().manual_seed(seed)
        self.base_position_bound = config.max_feedforward_delay // 2
        for module in self.layers:
            if isinstance(module, dcls_module):
                _reparametrize_feedforward_delay(module, maximum, generator, config, freeze_sig=True,
                                                 distribution=distribution, sigma=sigma)

    def _delay_stage(self, in_dim, out_dim, delayed):
        if not delayed:
            return super()._delay_stage(in_dim, out_dim, delayed)
        return [dcls_module(self.config, in_channels=in_dim, out_channels=out_dim, groups=1)]

    def init_weights(self):
        for m in self.layers:
            _init_ff(m, self.config)
            if isinstance(m, dcls_module):
                torch.nn.init.kaiming_uniform_(m.weight, a=math.sqrt(5))
                torch.nn.init.uniform_(m.P, a=self.config.init_pos_a, b=self.config.init_pos_b)
                m.clamp_parameters()
                if self.config.DCLSversion == "gauss":
                    torch.nn.init.constant_(m.SIG, self.config.siginit)
                    m.SIG.requires_grad = False

    def clamp_delays(self, train=True):
        with torch.no_grad():
            for module in self.layers:
                if isinstance(module, dcls_module):
                    learned_delay_parameter(module, "P").clamp_(-self.base_position_bound, self.base_position_bound)

    def round_pos(self):
        with torch.no_grad():
            for module in self.layers:
                if isinstance(module, dcls_module):
                    learned_delay_parameter(module, "P").round_()
        self.clamp_delays()


class SNN_recurrent_hybrid_delays(SNN_axonal_recurrent_delays):
    """Recurrent-only hybrid delays d(i,j) = d_j + delta_ij (networks.py:1128-1183).
    At hybrid_offset_scale == 0 this is exactly SNN_axonal_recurrent_delays."""

    def __init__(self, config):
        maximum, seed, distribution, sigma = _hybrid_params(config)
        self._hybrid_max = maximum
        if maximum == 0:
            super().__init__(config)
            return
        SNN_synaptic_recurrent_delays.__init__(self, config)
        generator = torch.Generator().manual_seed(seed)
        for module in self.layers:
            if isinstance(module, axonal_recdel):
                _reparametrize_recurrent_delay(module, maximum, generator, config, distribution, sigma)

    def clamp_delays(self):
        if self._hybrid_max == 0:
            return super().clamp_delays()
        with torch.no_grad():
            for module in self.layers:
                if isinstance(module, axonal_recdel):
                    learned_delay_parameter(module, "recurrent_delays").clamp_(min=0)

    def round_pos(self):
        if self._hybrid_max == 0:
            return super().round_pos()
        with torch.no_grad():
            for module in self.layers:
                if isinstance(module, axonal_recdel):
                    learned_delay_parameter(module, "recurrent_delays").round_()
        self.clamp_delays()


class SNN_fixed_hybrid_recurrent_delays(SNN_recurrent_hybrid_delays):
    """Hybrid with the rounded axonal base frozen (networks.py:1186-1204)."""

    def __init__(self, config):
        super().__init__(config)
        self.round_pos()
        for layer in self.layers:
            if isinstance(layer, axonal_recdel):
                learned_delay_parameter(layer, "recurrent_delays").requires_grad_(False)
                layer.sigma = 0.0
                layer.config.sigma_init = 0.0
                layer.use_sig_p = False
                if hasattr(layer, "p_spread"):
                    del layer.p_spread
