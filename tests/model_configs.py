"""Config objects shaped like the reference's configs/perf_*.py flag classes."""

class _Cfg:
    pass


def mem_config(hidden=(64,), bias=False, T=32, B=64, C=8, K=4, neuron_module=None, surrogate=None):
    """MEM toy (configs/perf_MEM.py) with the SpikingJelly-equivalent
    neuron of this package (or the given neuron class and surrogate)."""
    if neuron_module is None:
        from delrec.neuron import ATan, LIFNode
        neuron_module, surrogate = LIFNode, ATan(alpha=2.0)
    c = _Cfg()
    c.dataset = "MEM"
    c.input_size, c.output_size = C, K
    c.time_window, c.batch_size = T, B
    c.hidden_layers = list(hidden)
    c.bias = bias
    c.use_batch_norm = False
    c.feedforward_dropout_rate = 0.0
    c.recurrent_dropout_rate = 0.0
    c.init_ff_weights = "default"
    c.init_dcls_weights = "default"
    c.no_delay_in_first_layer = False
    c.no_delay_in_last_layer = False
    c.no_recurrence_in_last_layer = False
    c.neuron_module = neuron_module
    c.surrogate_function = surrogate
    c.tau, c.decay_input, c.v_threshold, c.v_reset = 2.0, False, 1.0, 0.0
    c.detach_reset = False
    c.step_mode, c.backend, c.store_v_seq = "m", "torch", False
    c.init_rec_weights = "kaiming_uniform"
    c.rec_delay_init_gain = 0.5
    c.use_rec_bias = False
    c.init_rec_delay = "uniform"
    c.init_recdel_offset = 0.0
    c.max_rec_delay = 16.0
    c.delay_std_init = 2.0
    c.use_sig_p = False
    c.sigma_init, c.sigma_decay, c.epochs = 0.0, 0.95, 200
    c.hybrid_offset_scale = 4
    c.hybrid_delay_seed = 123
    c.hybrid_offset_distribution = "uniform"
    c.hybrid_offset_sigma = 2.0
    c.hybrid_base_centering = "normal"
    c.round_delays = False
    c.DCLSversion = "gauss"
    c.kernel_count = 1
    c.max_feedforward_delay = 9
    c.left_padding = c.max_feedforward_delay - 1
    c.right_padding = 0
    c.init_pos_a = -(c.max_feedforward_delay // 2)
    c.init_pos_b = c.max_feedforward_delay // 2
    c.siginit = 1.0
    return c
