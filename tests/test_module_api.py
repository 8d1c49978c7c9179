"""Module-level drop-in contract checked on CPU: constructors, parameter names and
state_dict layout, the hybrid reparametrization, sigma annealing, the ValueError paths
of the reference, and that a CPU forward raises instead of falling back."""

import copy
import math

import pytest
import torch

from model_configs import mem_config


def _nw():
    from delrec import networks
    return networks


def test_axonal_state_dict_layout():
    nw = _nw()
    cfg = mem_config(hidden=[16], bias=False)
    torch.manual_seed(0)
    m = nw.SNN_axonal_recurrent_delays(cfg)
    keys = set(m.state_dict())
    assert keys == {"layers.0.weight", "layers.2.recurrent_weights", "layers.2.recurrent_delays",
                    "layers.4.weight"}, keys
    rec = m.layers[2]
    assert rec.recurrent_weights.shape == (16, 16) and rec.recurrent_delays.shape == (16,)
    assert isinstance(rec.sigma, float) and "sigma" not in m.state_dict()


def test_optional_parameters():
    nw = _nw()
    cfg = mem_config(hidden=[8], bias=True)
    cfg.use_sig_p = True
    cfg.use_rec_bias = True
    m = nw.SNN_synaptic_recurrent_delays(cfg)
    keys = set(m.state_dict())
    for k in ("layers.2.recurrent_weights", "layers.2.recurrent_delays", "layers.2.p_spread",
              "layers.2.recurrent_bias", "layers.0.bias", "layers.4.bias"):
        assert k in keys
    assert m.layers[2].recurrent_delays.shape == (8, 8)


@pytest.mark.parametrize("maximum", [0, 4])
def test_hybrid_layout(maximum):
    nw = _nw()
    cfg = mem_config(hidden=[16], bias=False)
    cfg.hybrid_offset_scale = maximum
    torch.manual_seed(0)
    h = nw.SNN_recurrent_hybrid_delays(cfg)
    if maximum == 0:
        torch.manual_seed(0)
        a = nw.SNN_axonal_recurrent_delays(cfg)
        hs, as_ = h.state_dict(), a.state_dict()
        assert set(hs) == set(as_)
        for k in as_:
            assert torch.equal(hs[k], as_[k]), k
        return
    keys = set(h.state_dict())
    assert "layers.2.parametrizations.recurrent_delays.original" in keys
    assert "layers.2.parametrizations.recurrent_delays.0.offsets" in keys
    leaf = nw.learned_delay_parameter(h.layers[2], "recurrent_delays")
    assert leaf.shape == (16,) and leaf.requires_grad
    off = h.layers[2].parametrizations.recurrent_delays[0].offsets
    assert not off.requires_grad and off.min() >= 0 and off.max() <= maximum
    assert torch.equal(off, off.round())
    # the effective (N, N) delay is base[o] + offsets[i, o]
    d = h.layers[2].recurrent_delays
    assert torch.allclose(d, leaf[None, :] + off)
    assert getattr(h.layers[2], "_hybrid_delay", False)


def test_hybrid_offsets_follow_the_seeded_generator():
    nw = _nw()
    cfg = mem_config(hidden=[12], bias=False)
    cfg.hybrid_offset_scale = 3
    a = nw.SNN_recurrent_hybrid_delays(cfg)
    b = nw.SNN_recurrent_hybrid_delays(cfg)
    oa = a.layers[2].parametrizations.recurrent_delays[0].offsets
    ob = b.layers[2].parametrizations.recurrent_delays[0].offsets
    assert torch.equal(oa, ob)
    g = torch.Generator().manual_seed(cfg.hybrid_delay_seed)
    assert torch.equal(oa, torch.randint(4, (12, 12), generator=g).float())


def test_value_errors():
    nw = _nw()
    for bad in (-1, 1.5):
        cfg = mem_config(hidden=[8])
        cfg.hybrid_offset_scale = bad
        with pytest.raises(ValueError):
            nw.SNN_recurrent_hybrid_delays(cfg)
    cfg = mem_config(hidden=[8])
    cfg.kernel_count = 2
    with pytest.raises(ValueError):
        nw.SNN_recurrent_hybrid_delays(cfg)


def test_update_sigma_schedule():
    nw = _nw()
    cfg = mem_config(hidden=[8])
    cfg.sigma_init, cfg.sigma_decay, cfg.epochs = 2.0, 0.95, 50
    m = nw.SNN_axonal_recurrent_delays(cfg)
    layer = m.layers[2]
    layer.update_sigma(10)
    assert math.isclose(layer.sigma, 2.0 * (0.95 ** (100 / 50)) ** 10)


def test_clamp_and_round():
    nw = _nw()
    cfg = mem_config(hidden=[8])
    cfg.hybrid_offset_scale = 2
    m = nw.SNN_recurrent_hybrid_delays(cfg)
    leaf = nw.learned_delay_parameter(m.layers[2], "recurrent_delays")
    with torch.no_grad():
        leaf.copy_(torch.linspace(-2, 3.4, 8))
    m.round_pos()
    assert torch.equal(leaf, leaf.round()) and leaf.min() >= 0


def test_cpu_forward_raises_no_fallback():
    nw = _nw()
    cfg = mem_config(hidden=[8])
    m = nw.SNN_axonal_recurrent_delays(cfg)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(4, 2, cfg.input_size))


def test_reference_forward_versions_are_not_shipped():
    nw = _nw()
    cfg = mem_config(hidden=[8])
    m = nw.SNN_axonal_recurrent_delays(cfg)
    m.layers[2].forward_version = "v2"
    from delrec.delay_layers import _check_cuda
    x = torch.zeros(2, 2, 8)
    with pytest.raises(RuntimeError):
        m(torch.zeros(4, 2, cfg.input_size))


def test_hard_tap_forward_versions_select_the_variant():
    """forward_version 'triton_approx' / 'triton_ste' (with config.ste_round_forward)
    choose the axonal scan's (approx, ste_mode) as delay_layers.py:204-211 and
    delay_layers_triton.py:60-61 do; other versions run the soft scan."""
    from types import SimpleNamespace
    from delrec.delay_layers import _axonal_variant
    lay = SimpleNamespace(config=SimpleNamespace(), forward_version=None)
    assert _axonal_variant(lay) == dict(approx=False, ste_mode=0)
    lay.forward_version = "triton_exact"
    assert _axonal_variant(lay) == dict(approx=False, ste_mode=0)
    lay.forward_version = "triton_approx"
    assert _axonal_variant(lay) == dict(approx=True, ste_mode=0)
    lay.forward_version = "triton_ste"
    assert _axonal_variant(lay) == dict(approx=False, ste_mode=1)
    lay.config.ste_round_forward = False
    assert _axonal_variant(lay) == dict(approx=False, ste_mode=2)


def test_hard_delays_follow_build_lag():
    """The hard taps as half-width-1 delays: round(d) (ties to even) clamped at 0, or the
    interpolation position max(d, 0); the host maximum equals the device one."""
    from delrec.functional import hard_delays
    d = torch.tensor([0.0, 0.5, 1.5, 2.5, 1.0, -0.7, 3.7, 2.49999])
    dh, mx = hard_delays(d, float(d.max()), 7, 1)
    assert dh.tolist() == [0.0, 0.0, 2.0, 2.0, 1.0, 0.0, 4.0, 2.0] and mx == 4.0
    dh, mx = hard_delays(d, float(d.max()), 7, 2)
    pos = 1.0 + d
    lag = torch.floor(pos).clamp(1, 6)
    assert torch.equal(dh, (lag - 1.0) + (pos - lag).clamp(0, 1))
    assert mx == float(dh.max())
    assert torch.equal((1.0 + dh)[d >= 0], pos[d >= 0])


def test_feedforward_models_build():
    nw = _nw()
    cfg = mem_config(hidden=[16])
    for name in ("SNN_axonal_feedforward_delays", "SNN_synaptic_feedforward_delays",
                 "SNN_hybrid_feedforward_delays", "SNN_recurrent_and_feedforward_delays",
                 "SNN_hybrid_recurrent_and_feedforward_delays"):
        m = getattr(nw, name)(cfg)
        assert sum(p.numel() for p in m.parameters()) > 0
    h = nw.SNN_hybrid_feedforward_delays(cfg)
    dc = [m for m in h.layers if isinstance(m, nw.dcls_module)][0]
    assert nw.learned_delay_parameter(dc, "P").shape[:3] == (1, 1, cfg.input_size)


@pytest.mark.parametrize("hybrid_name,axonal_name", [
    ("SNN_hybrid_feedforward_delays", "SNN_axonal_feedforward_delays"),
    ("SNN_recurrent_hybrid_delays", "SNN_axonal_recurrent_delays"),
])
def test_maximum_positive_keeps_axonal_delay_budget(hybrid_name, axonal_name):
    """tests/test_hybrid_delay_invariance.py:81-109 of the reference (construction part):
    one learned delay per source, as many delay leaves as the axonal model, frozen
    integer offsets in [0, 4] stored as buffers."""
    nw = _nw()
    from delrec.delay_layers import axonal_recdel

    def leaves(model, name):
        kind = nw.dcls_module if name == "P" else axonal_recdel
        return [nw.learned_delay_parameter(m, name) for m in model.layers if isinstance(m, kind)]

    cfg = mem_config(hidden=[16], bias=True, T=10, B=4, C=8, K=3)
    cfg.kernel_count = 1
    cfg.hybrid_offset_scale = 4
    torch.manual_seed(0)
    h = getattr(nw, hybrid_name)(cfg)
    cfg0 = mem_config(hidden=[16], bias=True, T=10, B=4, C=8, K=3)
    cfg0.kernel_count = 1
    cfg0.hybrid_offset_scale = 0
    torch.manual_seed(0)
    a = getattr(nw, axonal_name)(cfg0)
    for name in ("P", "recurrent_delays"):
        hl, al = leaves(h, name), leaves(a, name)
        assert len(hl) == len(al)
        for x, y in zip(hl, al):
            assert x.requires_grad and x.numel() == y.numel()
    offsets = [b for n, b in h.named_buffers() if n.endswith(".offsets")]
    assert offsets and all(not b.requires_grad for b in offsets)
    assert all(int(b.max()) <= 4 and int(b.min()) >= 0 for b in offsets)


def test_declared_input_spikes_reach_the_first_projection():
    """config.input_spikes (optional) sets the first projection's binary_input: unset ->
    tested per call (None), True -> spike path, False -> real-valued path; the later
    projections read spikes from a spiking layer either way."""
    from delrec import networks
    for flag, want in ((None, None), (True, True), (False, False)):
        cfg = mem_config(hidden=[16, 8], bias=False)
        if flag is not None:
            cfg.input_spikes = flag
        model = networks.SNN_axonal_recurrent_delays(cfg)
        lins = [m for m in model.layers if type(m).__name__ == "Linear"]
        assert lins[0].binary_input == want
        assert all(m.binary_input is True for m in lins[1:])


def _ref_state_dict_cases():
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_state_dicts.pt")
    return torch.load(path, weights_only=False)


@pytest.mark.parametrize("idx", range(19))
def test_state_dict_matches_the_reference_model_zoo(idx):
    """Every model class of the reference's networks.py, built by the reference's own code
    (tests/golden/make_state_dicts.py) and by this package for the same config and seed:
    the same state_dict keys and shapes, and -- for models without a DCLS layer, whose
    initial values the reference's own code and torch's RNG fully determine -- the same
    initial values (weights, delays, spreads, biases, BatchNorm, hybrid offsets)."""
    import sys, os
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    from make_state_dicts import build
    case = _ref_state_dict_cases()[idx]
    m = build(_nw(), mem_config, case["name"], case["overrides"], case["seed"])
    ours, ref = m.state_dict(), case["state"]
    assert list(ours) == list(ref), (sorted(set(ours) ^ set(ref)), case["name"])
    for k, v in ref.items():
        assert ours[k].shape == v.shape and ours[k].dtype == v.dtype, k
        if not case["dcls"]:
            assert torch.equal(ours[k], v), f"{case['name']}: {k} differs"
