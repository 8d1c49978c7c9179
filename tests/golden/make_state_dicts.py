"""Generate tests/golden/ref_state_dicts.pt: the reference's own model zoo, built.

Run here (it needs the read-only reference checkout; the GPU box never runs it):

    python tests/golden/make_state_dicts.py <path of the reference checkout>

It imports the reference's ``delrec.networks`` / ``delrec.delay_layers`` unmodified from
the checkout's ``src/`` and builds every model class of networks.py for a few MEM-shaped
configs (tests/model_configs.py) under fixed seeds, recording each state_dict (keys,
shapes, initial values) and, for the hybrid models, the offsets buffer.

SpikingJelly and DCLS are not installed in this container, so minimal stand-ins with
their documented module structure are registered in ``sys.modules`` first:
  * ``spikingjelly.activation_based``: ``base.MemoryModule`` (an ``nn.Module``),
    ``neuron.LIFNode`` (no parameters or buffers), ``layer.Dropout`` (none),
    ``layer.BatchNorm1d`` (``torch.nn.BatchNorm1d`` with a ``step_mode``),
    ``surrogate.ATan`` (a parameter-free module);
  * ``DCLS.construct.modules.Dcls1d`` (0.1.1, version 'gauss'): weight
    (out, in/groups, kernel_count), bias (out), P and SIG (1, out, in/groups,
    kernel_count), its parameter-free kernel builder ``DCK``, ``clamp_parameters()``.
The stand-in Dcls1d does not restate DCLS's own parameter initialisation, so for models
with a DCLS layer only the keys and shapes are meaningful (the fixture marks them).
"""

import os
import sys
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
TESTS = os.path.dirname(HERE)


class _MemoryModule(torch.nn.Module):
    def reset(self):
        pass


class _ATan(torch.nn.Module):
    def __init__(self, alpha=2.0, spiking=True):
        super().__init__()
        self.alpha = alpha
        self.spiking = spiking


class _LIFNode(_MemoryModule):
    def __init__(self, tau=2.0, decay_input=True, v_threshold=1.0, v_reset=0.0,
                 surrogate_function=None, detach_reset=False, step_mode="s", backend="torch",
                 store_v_seq=False):
        super().__init__()
        self.tau, self.decay_input = tau, decay_input
        self.v_threshold, self.v_reset = v_threshold, v_reset
        self.surrogate_function = surrogate_function if surrogate_function is not None else _ATan()
        self.detach_reset, self.step_mode = detach_reset, step_mode
        self.backend, self.store_v_seq = backend, store_v_seq


class _Dropout(_MemoryModule):
    def __init__(self, p=0.5, step_mode="s"):
        super().__init__()
        self.p, self.step_mode = p, step_mode


class _BatchNorm1d(torch.nn.BatchNorm1d):
    def __init__(self, num_features, eps=1e-5, momentum=0.1, affine=True,
                 track_running_stats=True, step_mode="s"):
        super().__init__(num_features, eps, momentum, affine, track_running_stats)
        self.step_mode = step_mode


class _ConstructKernel1d(torch.nn.Module):
    """DCLS's parameter-free kernel builder held as ``Dcls1d.DCK``."""

    def __init__(self, out_channels, in_channels, groups, kernel_count, dilated_kernel_size,
                 version="gauss"):
        super().__init__()
        self.args = (out_channels, in_channels, groups, kernel_count, dilated_kernel_size, version)


class _Dcls1d(torch.nn.Module):
    def __init__(self, in_channels, out_channels, kernel_count, stride=1, dilated_kernel_size=1,
                 padding=0, dilation=1, groups=1, bias=True, padding_mode="zeros", scaling=1,
                 version="gauss"):
        super().__init__()
        self.in_channels, self.out_channels = in_channels, out_channels
        self.kernel_count, self.groups = kernel_count, groups
        self.dilated_kernel_size = (dilated_kernel_size,)
        self.version = version
        shape = (out_channels, in_channels // groups, kernel_count)
        self.weight = torch.nn.Parameter(torch.zeros(shape))
        self.bias = torch.nn.Parameter(torch.zeros(out_channels)) if bias else None
        self.P = torch.nn.Parameter(torch.zeros((1,) + shape))
        self.SIG = torch.nn.Parameter(torch.ones((1,) + shape))
        self.DCK = _ConstructKernel1d(out_channels, in_channels, groups, kernel_count,
                                      self.dilated_kernel_size, version)

    def clamp_parameters(self):
        lim = self.dilated_kernel_size[0] // 2
        with torch.no_grad():
            self.P.clamp_(-lim, lim)


def install_standins():
    sj = types.ModuleType("spikingjelly")
    ab = types.ModuleType("spikingjelly.activation_based")
    base = types.ModuleType("spikingjelly.activation_based.base")
    neuron = types.ModuleType("spikingjelly.activation_based.neuron")
    layer = types.ModuleType("spikingjelly.activation_based.layer")
    surrogate = types.ModuleType("spikingjelly.activation_based.surrogate")
    functional = types.ModuleType("spikingjelly.activation_based.functional")
    base.MemoryModule = _MemoryModule
    neuron.LIFNode = _LIFNode
    layer.Dropout = _Dropout
    layer.BatchNorm1d = _BatchNorm1d
    layer.Linear = torch.nn.Linear
    surrogate.ATan = _ATan
    functional.reset_net = lambda net: None
    for name, m in (("base", base), ("neuron", neuron), ("layer", layer),
                    ("surrogate", surrogate), ("functional", functional)):
        setattr(ab, name, m)
        sys.modules["spikingjelly.activation_based." + name] = m
    sj.activation_based = ab
    sys.modules["spikingjelly"] = sj
    sys.modules["spikingjelly.activation_based"] = ab
    dcls = types.ModuleType("DCLS")
    construct = types.ModuleType("DCLS.construct")
    modules = types.ModuleType("DCLS.construct.modules")
    modules.Dcls1d = _Dcls1d
    construct.modules = modules
    dcls.construct = construct
    sys.modules.update({"DCLS": dcls, "DCLS.construct": construct,
                        "DCLS.construct.modules": modules})


# (class name, config overrides, seed); hidden / bias are mem_config arguments
CASES = [
    ("SNN", dict(hidden=(16, 12)), 1),
    ("SNN_axonal_recurrent_delays", dict(hidden=(16, 12)), 2),
    ("SNN_axonal_recurrent_delays", dict(hidden=(16,), bias=True, use_rec_bias=True,
                                         use_sig_p=True, sigma_init=1.0, use_batch_norm=True,
                                         init_rec_delay="half_normal"), 3),
    ("SNN_synaptic_recurrent_delays", dict(hidden=(16, 12)), 4),
    ("SNN_synaptic_recurrent_delays", dict(hidden=(12,), use_sig_p=True, sigma_init=0.5,
                                           use_rec_bias=True), 5),
    ("SNN_common_recurrent_delays", dict(hidden=(16, 12)), 6),
    ("SNN_vanilla_recurrent", dict(hidden=(16, 12)), 7),
    ("SNN_fixed_recurrent_delays", dict(hidden=(16, 12)), 8),
    ("SNN_fixed_synaptic_recurrent_delays", dict(hidden=(16,)), 9),
    ("SNN_recurrent_hybrid_delays", dict(hidden=(16, 12)), 10),
    ("SNN_recurrent_hybrid_delays", dict(hidden=(16,), hybrid_offset_scale=0), 11),
    ("SNN_fixed_hybrid_recurrent_delays", dict(hidden=(16,)), 12),
    ("SNN_synaptic_feedforward_delays", dict(hidden=(16, 12)), 13),
    ("SNN_axonal_feedforward_delays", dict(hidden=(16, 12)), 14),
    ("SNN_recurrent_and_feedforward_delays", dict(hidden=(16,)), 15),
    ("SNN_axonal_recurrent_and_feedforward_delays", dict(hidden=(16, 12)), 16),
    ("SNN_synaptic_recurrent_and_feedforward_delays", dict(hidden=(16,)), 17),
    ("SNN_hybrid_recurrent_and_feedforward_delays", dict(hidden=(16,)), 18),
    ("SNN_hybrid_feedforward_delays", dict(hidden=(16, 12)), 19),
]


def build(networks, mem_config, name, overrides, seed, neuron_module=None, surrogate=None):
    """One model of the named class for the case's config, built under the case's seed."""
    ov = dict(overrides)
    kw = dict(hidden=ov.pop("hidden"), bias=ov.pop("bias", False))
    if neuron_module is not None:
        kw.update(neuron_module=neuron_module, surrogate=surrogate)
    cfg = mem_config(**kw)
    for k, v in ov.items():
        setattr(cfg, k, v)
    torch.manual_seed(seed)
    return getattr(networks, name)(cfg)


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_state_dicts.py <path of the reference checkout>")
    install_standins()
    sys.path.insert(0, os.path.join(sys.argv[1], "src"))
    sys.path.insert(0, TESTS)
    from delrec import networks  # the reference's
    from model_configs import mem_config
    assert os.path.realpath(networks.__file__).startswith(os.path.realpath(sys.argv[1]))
    out = []
    for name, ov, seed in CASES:
        m = build(networks, mem_config, name, ov, seed, _LIFNode, _ATan(2.0))
        sd = {k: v.detach().clone() for k, v in m.state_dict().items()}
        has_dcls = any(isinstance(x, _Dcls1d) for x in m.modules())
        out.append(dict(name=name, overrides=ov, seed=seed, state=sd, dcls=has_dcls))
        print(f"{name:48s} {len(sd):3d} entries{'  (DCLS: keys and shapes)' if has_dcls else ''}")
    torch.save(out, os.path.join(HERE, "ref_state_dicts.pt"))


if __name__ == "__main__":
    main()
