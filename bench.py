"""Training-throughput benchmark of the delay-LIF hot path (samples x timesteps / s).

Workload (the north-star model): SNN_recurrent_hybrid_delays with two
recurrent hybrid-delay LIF layers of 512 neurons (learned axonal base U[0,25] + frozen
integer offsets U{0..8}, sigma = 0), 700 input channels of Bernoulli spikes with
per-channel rates U[0, 5%], T = 250, 35 classes, batch 256 per GPU.  One step = forward,
time-summed cross-entropy, backward with the gradient all-reduce of N > 1 ranks
(bucketed, launched during the backward) and an Adam update.
Synthetic data stands in for the SSC-shaped dataset (not available offline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's CPU path on
this host's cores on a bounded sample of the same workload: its own pure-PyTorch v2 scans
(delay_layers_pytorch.py) loaded unmodified from the baseline/_ref install, or, when that
install is absent, their restatement in ``oracle/``; autograd BPTT either way.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "snn-delays_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402

METRIC = "train samples*timesteps/s (fwd+bwd) per B200"
UNIT = "samples*timesteps/s"

CONFIGS = {
    # name: (hidden, C, K, T, B, kind, dmax, offset_scale, rate_max)
    "cfg4_ssc_hybrid_2x512": dict(hidden=[512, 512], C=700, K=35, T=250, B=256, model="SNN_recurrent_hybrid_delays",
                                  dmax=25.0, offsets=8, rate=0.05),
    "cfg1_mem_axonal_64": dict(hidden=[64], C=8, K=4, T=32, B=64, model="SNN_axonal_recurrent_delays",
                               dmax=16.0, offsets=0, rate=0.1),
    "cfg3_shd_synaptic_2x256": dict(hidden=[256, 256], C=700, K=20, T=250, B=256,
                                    model="SNN_synaptic_recurrent_delays", dmax=25.0, offsets=0, rate=0.05),
    "cfg5_psmnist_axonal_512": dict(hidden=[512], C=1, K=10, T=784, B=256, model="SNN_axonal_recurrent_delays",
                                    dmax=64.0, offsets=0, rate=None),
    "cfg2_har_dcls_hybrid_128": dict(hidden=[128], C=9, K=6, T=128, B=64,
                                     model="SNN_hybrid_recurrent_and_feedforward_delays", dmax=8.0, offsets=4,
                                     rate=None, input="normal"),
}


def make_config(spec, B):
    from model_configs import mem_config
    cfg = mem_config(hidden=spec["hidden"], bias=True, T=spec["T"], B=B, C=spec["C"], K=spec["K"])
    cfg.dataset = "SSC"
    cfg.init_rec_weights = "kaiming_uniform"
    # N(0, 0.1) projections (the reference's init_ff_weights='normal' option): with the
    # sparse Bernoulli inputs this puts the first hidden layer at a few percent firing,
    # the regime of the reference's SSC runs (1.8 %); kaiming/default inits stay silent
    cfg.init_ff_weights = "normal"
    cfg.max_rec_delay = spec["dmax"]
    cfg.hybrid_offset_scale = spec["offsets"]
    cfg.hybrid_base_centering = "normal"
    cfg.sigma_init = 0.0
    # the synthetic inputs' kind is known: Bernoulli spike trains or real values, so the
    # first projection needs no per-call 0/1 test (and no host synchronisation per step)
    cfg.input_spikes = spec["rate"] is not None and spec.get("input") != "normal"
    return cfg


def make_inputs(spec, B, seed=1, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    T, C = spec["T"], spec["C"]
    if spec.get("input") == "normal":   # HAR-shaped: real-valued N(0,1) input currents
        x = torch.randn(T, B, C, generator=g)
    elif spec["rate"] is None:   # PS-MNIST-shaped: one channel of intensities, permuted in time
        x = torch.rand(B, T, generator=g)[:, torch.randperm(T, generator=g)].t().unsqueeze(-1)
    else:
        rates = torch.rand(C, generator=g) * spec["rate"]
        x = (torch.rand(T, B, C, generator=g) < rates).float()
    labels = torch.randint(spec["K"], (B,), generator=g)
    return x.contiguous(), labels


def build_model(spec, B, device):
    from delrec import networks
    cfg = make_config(spec, B)
    torch.manual_seed(0)
    model = getattr(networks, spec["model"])(cfg)
    return model.to(device), cfg


def loss_fn(out, labels):
    return torch.nn.functional.cross_entropy(out.sum(0), labels)


def model_loss(model, x, labels):
    """The same loss as loss_fn(model(x), labels): the readout summed over time, fused in
    the library (forward_time_summed) instead of forming the (T,B,C) readout."""
    return torch.nn.functional.cross_entropy(model.forward_time_summed(x), labels)


# ----------------------------------------------------------------------------------
# clocks sampled during the timed region
# ----------------------------------------------------------------------------------
class ClockSampler:
    """``nvidia-smi -lms 100`` running for the life of the ``with`` block; the summary
    keeps the samples stamped inside [begin(), end()] (the timed region), or the one
    nearest to it when the region is shorter than the sampling period."""
    QUERY = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index):
        self.index = index
        self.samples = []          # (wall time, [fields])
        self._proc = None
        self._t = None
        self._t0 = self._t1 = None

    def _read(self):
        for line in self._proc.stdout:
            f = [v.strip() for v in line.strip().split(",")]
            if len(f) >= 7:
                self.samples.append((time.time(), f))

    def __enter__(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            t_wait = time.time() + 5.0
            while not self.samples and time.time() < t_wait:   # sampler is live
                time.sleep(0.02)
        except OSError:
            self._proc = None
        return self

    def begin(self):
        self._t0 = time.time()

    def end(self):
        self._t1 = time.time()

    def __exit__(self, *a):
        if self._proc is not None:
            time.sleep(0.15)
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
            self._t.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        t0 = self._t0 if self._t0 is not None else self.samples[0][0]
        t1 = self._t1 if self._t1 is not None else self.samples[-1][0]
        inside = [f for (ts, f) in self.samples if t0 <= ts <= t1]
        if not inside:
            inside = [min(self.samples, key=lambda s: abs(s[0] - 0.5 * (t0 + t1)))[1]]

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [x for x in (num(f[0]) for f in inside) if x is not None]
        mx = [x for x in (num(f[1]) for f in inside) if x is not None]
        reasons = sorted({self.NAMES[i] for f in inside for i in range(4) if f[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(inside)}


# ----------------------------------------------------------------------------------
# distributed helpers
# ----------------------------------------------------------------------------------
def dist_setup(n_gpus):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        rank = int(os.environ["RANK"])
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        os.environ.setdefault("NCCL_DEBUG", "WARN")   # keep stdout to the one JSON line
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        return rank, ws, local
    return 0, 1, 0


def make_allreduce(params, ws):
    """The gradient averaging of N > 1 ranks: bucketed all-reduces launched from the
    gradient hooks during the backward (they overlap the earlier layers' backward)."""
    if ws == 1:
        return None
    from delrec.data_parallel import OverlappedAllReduce
    return OverlappedAllReduce(params, bucket_bytes=2 << 20)


def finish_allreduce(ar, params, ws):
    if ws > 1:
        ar.finish()


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, ws):
    if ws == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------------
# CPU side (reference algorithm restated in oracle/)
# ----------------------------------------------------------------------------------
REF_ROOT = os.path.join(ROOT, "baseline", "_ref")


def reference_scans():
    """The reference's own pure-PyTorch scans (delay_layers_pytorch.py, loaded unmodified
    from the baseline/_ref install) or None when that install is absent."""
    from oracle import reference_v2
    try:
        return reference_v2.load(REF_ROOT)
    except Exception:
        return None


def cpu_step_fn(model, spec, cfg, ref_mod=None):
    """A callable running one fwd+bwd of the model on CPU for a batch x (T,b,C).  The
    recurrent delay layers run the reference's own multi_step_forward_v2 when ``ref_mod``
    (reference_scans()) is given, else the oracle's restatement of it."""
    from oracle import delrec_oracle as O
    from oracle import reference_v2
    from delrec import networks
    params = []
    layers = []
    for m in model.layers:
        if isinstance(m, torch.nn.Linear):
            w = m.weight.detach().cpu().clone().requires_grad_(True)
            b = m.bias.detach().cpu().clone().requires_grad_(True) if m.bias is not None else None
            layers.append(("lin", w, b))
            params += [w] + ([b] if b is not None else [])
        elif isinstance(m, networks.dcls_module):
            w = m.weight.detach().cpu().clone().requires_grad_(True)
            b = m.bias.detach().cpu().clone().requires_grad_(True) if m.bias is not None else None
            P = m.P.detach().cpu().clone()          # effective positions (offsets included)
            S = m.SIG.detach().cpu().clone()
            layers.append(("dcls", w, b, P, S, m.dilated_kernel_size[0], m.groups, m.left_padding))
            params += [w] + ([b] if b is not None else [])
        elif not isinstance(m, (torch.nn.Dropout, networks.spike_registrator)) and \
                type(m).__name__ not in ("Dropout",) and not hasattr(m, "recurrent_weights"):
            raise NotImplementedError(f"oracle replay: unsupported module {type(m).__name__}")
        elif hasattr(m, "recurrent_weights"):
            W = m.recurrent_weights.detach().cpu().clone().requires_grad_(True)
            leaf = networks.learned_delay_parameter(m, "recurrent_delays")
            base = leaf.detach().cpu().clone().requires_grad_(True)
            off = None
            if getattr(m, "_hybrid_delay", False):
                off = m.parametrizations.recurrent_delays[0].offsets.detach().cpu()
            layers.append(("rec", W, base, off, m.recurrent_weights.shape[0] == base.numel() and off is None
                           and base.dim() == 1))
            params += [W, base]

    def step(x, labels):
        h = x
        for L in layers:
            if L[0] == "lin":
                h = h @ L[1].t() + (L[2] if L[2] is not None else 0.0)
            elif L[0] == "dcls":
                _, w, b, P, S, K, groups, lpad = L
                h = O.dcls_conv(h, w, P, S, K, groups, lpad, b)
            else:
                _, W, base, off, axonal = L
                lif = O.OracleLIF(tau=cfg.tau, v_threshold=cfg.v_threshold, v_reset=cfg.v_reset,
                                  surrogate=O.ATanSpike(2.0))
                if ref_mod is not None:
                    d = O.hybrid_delays(base, off) if off is not None else base
                    h = reference_v2.scan(ref_mod, "axonal" if axonal else "synaptic", h, W, d, lif)
                elif off is not None:
                    h = O.synaptic_scan(h, W, O.hybrid_delays(base, off), lif, sigma=0.0)
                elif axonal:
                    h = O.axonal_scan(h, W, base, lif, sigma=0.0)
                else:
                    h = O.synaptic_scan(h, W, base, lif, sigma=0.0)
        loss = loss_fn(h, labels)
        for p in params:
            p.grad = None
        loss.backward()
        return loss
    return step


def _cpu_timed_steps(step, x, labels, warmup, steps, budget_s):
    """Median seconds per oracle step.  Warm-up steps run on the first tenth of the
    timesteps (they only warm the allocator and thread pool); timed steps run the full
    sample and stop early once ``budget_s`` is spent (at least one step always runs)."""
    T = x.shape[0]
    xw = x[: max(1, T // 10)].contiguous()
    for _ in range(warmup):
        step(xw, labels)
    times = []
    t_start = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        step(x, labels)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    return statistics.median(times), len(times)


def time_cpu(model, spec, cfg, sample_b, steps, threads, warmup=1, budget_s=60.0):
    torch.set_num_threads(threads)
    ref_mod = reference_scans()
    step = cpu_step_fn(model, spec, cfg, ref_mod)
    x, labels = make_inputs(spec, sample_b, seed=2)
    med, done = _cpu_timed_steps(step, x, labels, warmup, steps, budget_s)
    return sample_b * spec["T"] / med, med, done, ("reference" if ref_mod is not None else "port")


def run_reference_arm(args, spec):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    model, cfg = build_model(spec, args.cpu_sample_b, "cpu")
    x, labels = make_inputs(spec, args.cpu_sample_b, seed=2)
    ref_mod = reference_scans()
    kind = "reference" if ref_mod is not None else "port"
    step = cpu_step_fn(model, spec, cfg, ref_mod)
    med, done = _cpu_timed_steps(step, x, labels, args.warmup, args.steps, args.cpu_budget)
    value = args.cpu_sample_b * spec["T"] / med
    what = ("the reference's own multi_step_forward_v2 (delay_layers_pytorch.py, from the baseline/_ref "
            "install) with autograd BPTT" if ref_mod is not None else
            "the oracle's restatement of the reference's v2 scan with autograd BPTT")
    sample = (f"{args.cpu_sample_b} sample(s) x T={spec['T']} of {args.config} per step through {what}, "
              f"median of {done} step(s) ({med:.1f} s/step; the full per-GPU batch is {spec['B']})")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "steps_timed": done, "warmup": args.warmup, "ms_per_step": med * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": args.config, "model": spec["model"], "hidden": spec["hidden"],
                       "T": spec["T"], "batch_per_step": args.cpu_sample_b},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------------
def firing_rates(model):
    from delrec.networks import spike_registrator
    return [round(float(m.spikes.detach().mean()), 4) for m in model.layers
            if isinstance(m, spike_registrator) and m.spikes is not None]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="cfg4_ssc_hybrid_2x512", choices=list(CONFIGS))
    ap.add_argument("--cpu-sample-b", type=int, default=64)
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--cpu-budget", type=float, default=150.0,
                    help="seconds of timed CPU steps after which the reference arm stops early")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-strong", action="store_true", help="skip the fixed-global-batch record (N > 1)")
    ap.add_argument("--T", type=int, default=None, help="override T (profiling of small cases)")
    ap.add_argument("--B", type=int, default=None, help="override the per-GPU batch")
    ap.add_argument("--hidden", type=int, default=None,
                    help="override the width of every recurrent layer (BASELINE config 5 sweeps it)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    spec = dict(CONFIGS[args.config])
    if args.T:
        spec["T"] = args.T
    if args.B:
        spec["B"] = args.B
    if args.hidden:
        spec["hidden"] = [args.hidden] * len(spec["hidden"])

    if args.impl == "reference":
        run_reference_arm(args, spec)
        return

    rank, ws, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from delrec import _lib
    B = spec["B"]
    model, cfg = build_model(spec, B, dev)
    params = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.Adam(params, lr=1e-3)
    ar = make_allreduce(params, ws)
    x_cpu, labels_cpu = make_inputs(spec, B, seed=1 + rank)
    x = x_cpu.to(dev)
    labels = labels_cpu.to(dev)

    def step(xb, lb):
        opt.zero_grad(set_to_none=True)
        loss = model_loss(model, xb, lb)
        loss.backward()
        finish_allreduce(ar, params, ws)
        opt.step()
        model.clamp_delays()
        return loss

    for _ in range(args.warmup):
        step(x, labels)
    torch.cuda.synchronize()
    rates = firing_rates(model)

    # ---- device-resident timed region
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.launch_count()
    barrier(ws)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        clk.begin()
        start.record()
        for _ in range(args.steps):
            step(x, labels)
        end.record()
        torch.cuda.synchronize()
        clk.end()
    barrier(ws)
    launches = _lib.launch_count() - launches0
    ms = max_over_ranks(start.elapsed_time(end), ws) / args.steps
    units = B * spec["T"] * ws
    value = units / (ms / 1e3)

    # ---- end to end through the public API: every step's batch is copied from pinned
    #      host memory (on a side stream, one step ahead, double-buffered, as a data
    #      loader prefetches) and every step's loss is read back; the timed region spans
    #      all copies and all steps
    e2e = None
    if not args.no_e2e:
        xh = x_cpu.pin_memory()
        lh = labels_cpu.pin_memory()
        out_h = torch.empty(1, pin_memory=True)
        compute = torch.cuda.current_stream(dev)
        copier = torch.cuda.Stream(dev)
        bufs = [(torch.empty(x_cpu.shape, device=dev), torch.empty(labels_cpu.shape, dtype=labels_cpu.dtype,
                                                                   device=dev)) for _ in range(2)]
        ready = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]

        def fetch(slot, wait_free):
            with torch.cuda.stream(copier):
                if wait_free:
                    copier.wait_event(freed[slot])
                bufs[slot][0].copy_(xh, non_blocking=True)
                bufs[slot][1].copy_(lh, non_blocking=True)
                ready[slot].record(copier)

        barrier(ws)
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(compute)
        copier.wait_event(s2)
        fetch(0, False)
        for i in range(args.steps):
            cur = i % 2
            if i + 1 < args.steps:
                fetch((i + 1) % 2, i >= 1)
            compute.wait_event(ready[cur])
            loss = step(bufs[cur][0], bufs[cur][1])
            freed[cur].record(compute)
            out_h.copy_(loss.detach().reshape(1), non_blocking=True)
        e2.record(compute)
        torch.cuda.synchronize()
        ms2 = max_over_ranks(s2.elapsed_time(e2), ws) / args.steps
        e2e = {"value": units / (ms2 / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int(xh.numel() * 4 + lh.numel() * 8), "d2h_bytes_per_step": 4,
               "input_prefetch": "side stream, one step ahead"}

    # ---- dominant kernel roofline: the reverse-scan launches of two more training
    #      steps, each bracketed by CUDA events on its own stream inside the library
    #      (every rank runs the steps: they contain the gradient all-reduce)
    roof = roofline_probe(model, step, x, labels, spec, B)
    if roof is not None and "chunk_gemm" not in roof:
        smem = scan_smem_roofline(model, spec, B, roof["ms_per_launch"], clk.summary().get("sm_mhz"))
        if smem is not None:
            roof["smem"] = smem
    step_roof = step_roofline(spec, B, ms)
    floor = latency_floor(model, spec, B)

    # ---- strong scaling (BASELINE config 4 is quoted at a fixed global batch of 256):
    #      the same step with 256 / N samples per GPU, in the same invocation
    strong = None
    if ws > 1 and spec["B"] % ws == 0 and not args.no_strong:
        Bs = spec["B"] // ws
        model_s, _ = build_model(spec, Bs, dev)
        params_s = [p for p in model_s.parameters() if p.requires_grad]
        opt_s = torch.optim.Adam(params_s, lr=1e-3)
        ar_s = make_allreduce(params_s, ws)
        xs = x[:, :Bs].contiguous()
        ls = labels[:Bs].contiguous()

        def step_s(xb, lb):
            opt_s.zero_grad(set_to_none=True)
            loss = model_loss(model_s, xb, lb)
            loss.backward()
            finish_allreduce(ar_s, params_s, ws)
            opt_s.step()
            model_s.clamp_delays()
            return loss

        for _ in range(3):
            step_s(xs, ls)
        ks = max(3, min(args.steps, 10))
        barrier(ws)
        torch.cuda.synchronize()
        a3, b3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a3.record()
        for _ in range(ks):
            step_s(xs, ls)
        b3.record()
        torch.cuda.synchronize()
        barrier(ws)
        ms_s = max_over_ranks(a3.elapsed_time(b3), ws) / ks
        strong = {"global_batch": spec["B"], "batch_per_gpu": Bs, "steps": ks, "ms_per_step": ms_s,
                  "value": spec["B"] * spec["T"] / (ms_s / 1e3), "unit": UNIT, "scaling": "strong"}
    elif ws == 1:
        strong = {"global_batch": B, "batch_per_gpu": B, "steps": args.steps, "ms_per_step": ms,
                  "value": value, "unit": UNIT, "scaling": "strong",
                  "note": "one GPU: the main measurement (global batch = per-GPU batch)"}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        model_cpu, cfg_cpu = build_model(spec, args.cpu_sample_b, "cpu")
        v, med, done, kind = time_cpu(model_cpu, spec, cfg_cpu, args.cpu_sample_b, args.cpu_steps, threads)
        what = "the reference's own v2 scan" if kind == "reference" else "the oracle's v2 restatement"
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": kind,
               "sample": f"{args.cpu_sample_b} sample(s) x T={spec['T']} of the same model per step "
                         f"({what} fwd + autograd BPTT), median of {done} ({med:.1f} s/step)"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": args.config, "model": spec["model"], "hidden": spec["hidden"],
                           "input_channels": spec["C"], "classes": spec["K"], "T": spec["T"],
                           "batch_per_gpu": B, "global_batch": B * ws, "parallelism": f"dp{ws}",
                           "l2": "inputs larger than L2 (x is T*B*C*4 bytes per step)",
                           "firing_rates": rates},
                "gpu_launches": launches, "clocks": clk.summary(), "e2e": e2e,
                "roofline": roof, "step_roofline": step_roof, "latency_floor": floor,
                "strong_scaling": strong, "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _profiled_traffic(kernel):
    """DRAM bytes per sample-timestep of ``kernel`` from the committed ncu summary
    (profiles/<kernel>.txt, line ``dram_bytes_per_sample_step: <x>``), or None."""
    path = os.path.join(ROOT, "profiles", f"{kernel}.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_sample_step:"):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


def chunk_gemm_executed_flops(B, N, T, KP1):
    """Tensor-core flops the chunk GEMMs (k_chunk_gz) of one layer's reverse scan execute:
    per chunk of 8 steps, 128-row tiles (16 samples) x (source, offset) columns -- 256 per
    full column block of (256 // KP1) & ~3 sources, the last block its used columns rounded
    up to 16 -- over the N-target reduction padded to blocks of 32, three bf16 products."""
    ntg = (256 // KP1) & ~3
    ntiles = math.ceil(N / ntg)
    ncl = min(256, ((N - (ntiles - 1) * ntg) * KP1 + 15) // 16 * 16)
    cols = math.ceil(B / 16) * ((ntiles - 1) * 256 + ncl)
    return cols * 2.0 * 128 * (math.ceil(N / 32) * 32) * 3 * math.ceil(T / 8)


def roofline_probe(model, step, x, labels, spec, B):
    """Average duration of the reverse-scan kernel (the dominant kernel of the step) over
    the launches of two training steps, timed with CUDA events recorded on the stream
    each launch is issued on, and its algorithmic throughput: the recurrent contraction
    gz = W^T gr of the backward scan, 2*N^2 flops per sample-timestep, 2*N^2*B*T per
    launch.  Peak: the measured sustained bf16 tensor rate (the kernel runs inside a
    seconds-long training step)."""
    from delrec import _lib
    rec = [m for m in model.layers if hasattr(m, "recurrent_weights")]
    if not rec:
        return None
    _lib.scan_timing(True)
    try:
        for _ in range(2):
            step(x, labels)
        torch.cuda.synchronize()
        total_ms, n = _lib.scan_time(0)
        steps_ms, n_steps = _lib.scan_time(1)
        gemm_ms, n_gemm = _lib.scan_time(2)
    finally:
        _lib.scan_timing(False)
    if n == 0:
        return None
    N = rec[0].neurons
    T = spec["T"]
    ms = total_ms / n
    flops = 2.0 * N * N * B * T
    peaks, src = _peaks()
    # fp32-accurate tensor rate: a 3-product bf16 split carries an fp32 contraction
    peak = peaks["bf16_tflops_sustained"] / 3.0
    achieved = flops / (ms / 1e3) / 1e12
    chunked = n_gemm > 0
    per_unit = _profiled_traffic("k_bwd_chunk_cfg4" if chunked else "k_bwd_hybrid64") \
        if spec["model"].endswith("hybrid_delays") else None
    kern = {"hybrid": "k_bwd_chunk steps + k_chunk_gz tensor-core chunk GEMMs" if chunked else "k_bwd_hybrid64",
            "synaptic": "k_bwd_hybrid64 (synaptic buckets)", "axonal": "k_bwd_axonal_mma or k_bwd (by size)"}
    kind = "hybrid" if "hybrid" in spec["model"] else ("synaptic" if "synaptic" in spec["model"] else "axonal")
    out = {"bound": "tensor", "kernel": f"{kern[kind]}: reverse scan of one recurrent layer",
           "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
           "traffic": per_unit * B * T if per_unit else None,
           "ms_per_launch": ms, "launches_timed": n, "flops_per_launch": flops,
           "flops_definition": "2*N^2*B*T: the recurrent contraction gz = W^T gr, each synapse once",
           "peak_source": f"bf16_tflops_sustained / 3 ({src}; fp32-accurate 3-product bf16 rate)",
           "traffic_source": "ncu dram bytes per sample-timestep of a T=64 capture of the same kernels "
                             "(profiles/), scaled to B*T" if per_unit else None}
    if chunked:
        # the chunk GEMMs: executed tensor-core work against the measured sustained bf16 rate
        exec_flops = chunk_gemm_executed_flops(B, N, T, spec["offsets"] + 1)
        layers = n
        g_ms = gemm_ms / layers
        out["chunk_gemm"] = {"kernel": "k_chunk_gz", "ms_per_layer": g_ms, "launches_per_layer": n_gemm / layers,
                             "executed_tflops": exec_flops / (g_ms / 1e3) / 1e12,
                             "peak_tflops": peaks["bf16_tflops_sustained"],
                             "frac": exec_flops / (g_ms / 1e3) / 1e12 / peaks["bf16_tflops_sustained"],
                             "executed_flops_per_layer": exec_flops}
        out["chunk_steps"] = {"kernel": "k_bwd_chunk", "ms_per_layer": steps_ms / layers,
                              "launches_per_layer": n_steps / layers,
                              "us_per_timestep": steps_ms / layers * 1e3 / T}
    return out


SMEM_BYTES_PER_CLK_SM = 128   # shared-memory bandwidth per SM (32 banks x 4 bytes)
N_SMS = 148


def scan_smem_roofline(model, spec, B, ms, sm_mhz):
    """Second roofline of the hybrid / synaptic reverse scan, whose per-step synapse sums
    run on the CUDA cores from shared memory: every synapse reads its target's gr value
    (4 bytes) once per sample-timestep, N^2*4*B*T algorithmic shared-memory bytes per
    launch, against 128 bytes/clock/SM x 148 SMs at the median SM clock sampled during
    the timed region (the record loads, the per-step restage and the ring traffic are
    overhead on top)."""
    if "hybrid" not in spec["model"] and "synaptic" not in spec["model"]:
        return None
    rec = [m for m in model.layers if hasattr(m, "recurrent_weights")]
    if not rec or not sm_mhz or not ms:
        return None
    N = rec[0].neurons
    nbytes = 4.0 * N * N * B * spec["T"]
    achieved = nbytes / (ms / 1e3) / 1e12
    peak = SMEM_BYTES_PER_CLK_SM * N_SMS * sm_mhz * 1e6 / 1e12
    return {"bound": "smem", "achieved": achieved, "peak": peak, "unit": "TB/s", "frac": achieved / peak,
            "bytes_per_launch": nbytes,
            "peak_source": f"128 B/clk/SM x {N_SMS} SMs at the sampled median {sm_mhz:.0f} MHz"}


def latency_floor(model, spec, B):
    """The reverse scans' per-step exchange alone (delrec_exchange_floor: publish gr to L2,
    meet the batch tile, restage gr into shared memory; no LIF, no synapse sums) over T
    steps on the tiling the layer's scan uses, times the number of recurrent layers: the
    latency floor of the step-by-step part of the backward."""
    from delrec import _lib
    rec = [m for m in model.layers if hasattr(m, "recurrent_weights")]
    if not rec:
        return None
    N, T = rec[0].neurons, spec["T"]
    try:
        f_ms = _lib.exchange_floor_ms(T, B, N)
    except RuntimeError:
        return None
    return {"ms_per_layer": f_ms, "layers": len(rec), "ms_per_step": f_ms * len(rec),
            "us_per_timestep": f_ms * 1e3 / T,
            "what": "T steps of the per-step gr exchange (L2 publish, tile arrival counter, "
                    "shared-memory restage) on the scan's grid, no compute"}


def step_algorithmic(spec, B):
    """Algorithmic flops and HBM bytes of one training step (per GPU), per unit (one
    sample x one timestep) times B*T.
    Flops (dense-equivalent, 2 per multiply-add): each recurrent delay layer 6*N^2 (forward
    contraction, backward contraction gz = W^T gr, weight gradient); each Linear in->out
    6*in*out (forward, input gradient, weight gradient), 4*in*out for the first one (its
    input needs no gradient).
    Bytes (fp32 tensors at op boundaries): each delay layer 28*N (forward reads x, writes
    y and the saved state; backward reads gy, the state and the spikes, writes dx); each
    Linear 4*(in+out) forward plus 4*(2*out+in) backward, 4*(out+in) for the first."""
    T, C, K = spec["T"], spec["C"], spec["K"]
    hid = spec["hidden"]
    flops = 0.0
    nbytes = 0.0
    dims = [C] + list(hid)
    for j, N in enumerate(hid):
        fin = dims[j]
        first = j == 0
        flops += (4.0 if first else 6.0) * fin * N + 6.0 * N * N
        nbytes += 4.0 * (fin + N) + (4.0 * (N + fin) if first else 4.0 * (2 * N + fin)) + 28.0 * N
    flops += 6.0 * hid[-1] * K
    nbytes += 4.0 * (hid[-1] + K) + 4.0 * (2 * K + hid[-1])
    units = T * B
    return flops * units, nbytes * units


def step_roofline(spec, B, ms):
    """The step's floor time: the slower of its algorithmic flops at the fp32-accurate
    tensor rate (the measured sustained bf16 rate / 3: a 3-product bf16 split carries an
    fp32 contraction) and its algorithmic bytes at the measured HBM bandwidth; frac =
    floor / measured step time."""
    flops, nbytes = step_algorithmic(spec, B)
    peaks, src = _peaks()
    p_fp32acc = peaks["bf16_tflops_sustained"] / 3.0
    t_flops = flops / (p_fp32acc * 1e12)
    t_bytes = nbytes / (peaks["hbm_gbs"] * 1e9)
    floor_ms = max(t_flops, t_bytes) * 1e3
    # the same floor with the fp32 CUDA-core rate (148 SMs x 128 FMA/clk x 2 at the max
    # SM clock): the fraction a SIMT-only implementation could reach
    p_simt = 148 * 128 * 2 * peaks.get("sm_max_mhz", 1965.0) * 1e6 / 1e12
    simt_ms = max(flops / (p_simt * 1e12), t_bytes) * 1e3
    return {"flops": flops, "bytes": nbytes, "floor_ms": floor_ms,
            "bound": "tensor" if t_flops >= t_bytes else "hbm", "frac": floor_ms / ms,
            "peak_tflops_fp32acc": p_fp32acc, "peak_hbm_gbs": peaks["hbm_gbs"],
            "peak_source": f"bf16_tflops_sustained/3 and hbm_gbs ({src})",
            "simt_floor_ms": simt_ms, "simt_frac": simt_ms / ms, "peak_tflops_fp32_simt": p_simt}


if __name__ == "__main__":
    main()
