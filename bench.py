"""Training-throughput benchmark of the delay-LIF hot path (samples x timesteps / s).

Workload (the north-star model): SNN_recurrent_hybrid_delays with two
recurrent hybrid-delay LIF layers of 512 neurons (learned axonal base U[0,25] + frozen
integer offsets U{0..8}, sigma = 0), 700 input channels of Bernoulli spikes with
per-channel rates U[0, 5%], T = 250, 35 classes, batch 256 per GPU.  One step = forward,
time-summed cross-entropy, backward, gradient all-reduce (N > 1) and an Adam update.
Synthetic data stands in for the SSC-shaped dataset (not available offline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the reference algorithm's CPU
path (the pure-PyTorch v2 scan restated in ``oracle/``, autograd BPTT) on this host's
cores on a bounded sample of the same workload.
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
    return cfg


def make_inputs(spec, B, seed=1, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    T, C = spec["T"], spec["C"]
    if spec["rate"] is None:   # PS-MNIST-shaped: one channel of intensities, permuted in time
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


# ----------------------------------------------------------------------------------
# clocks sampled during the timed region
# ----------------------------------------------------------------------------------
class ClockSampler:
    def __init__(self, index):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([v.strip() for v in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 4 + i and s[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        return rank, ws, local
    return 0, 1, 0


def allreduce_grads(params, ws):
    if ws == 1:
        return
    import torch.distributed as dist
    grads = [p.grad for p in params if p.grad is not None]
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat)
    flat.div_(ws)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n


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
def cpu_step_fn(model, spec, cfg):
    """A callable running one fwd+bwd of the oracle model on CPU for a batch x (T,b,C)."""
    from oracle import delrec_oracle as O
    from delrec import networks
    params = []
    layers = []
    for m in model.layers:
        if isinstance(m, torch.nn.Linear):
            w = m.weight.detach().cpu().clone().requires_grad_(True)
            b = m.bias.detach().cpu().clone().requires_grad_(True) if m.bias is not None else None
            layers.append(("lin", w, b))
            params += [w] + ([b] if b is not None else [])
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
            else:
                _, W, base, off, axonal = L
                lif = O.OracleLIF(tau=cfg.tau, v_threshold=cfg.v_threshold, v_reset=cfg.v_reset,
                                  surrogate=O.ATanSpike(2.0))
                if off is not None:
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


def time_cpu(model, spec, cfg, sample_b, steps, threads):
    torch.set_num_threads(threads)
    step = cpu_step_fn(model, spec, cfg)
    x, labels = make_inputs(spec, sample_b, seed=2)
    step(x, labels)  # warm
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step(x, labels)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    units = sample_b * spec["T"]
    return units / med, med


def run_reference_arm(args, spec):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    model, cfg = build_model(spec, args.cpu_sample_b, "cpu")
    x, labels = make_inputs(spec, args.cpu_sample_b, seed=2)
    step = cpu_step_fn(model, spec, cfg)
    torch.set_num_threads(threads)
    for _ in range(args.warmup):
        step(x, labels)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step(x, labels)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    value = args.cpu_sample_b * spec["T"] / med
    sample = (f"{args.cpu_sample_b} samples x T={spec['T']} of {args.config} per step "
              f"(the full per-GPU batch is {spec['B']})")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": med * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.config, "model": spec["model"], "hidden": spec["hidden"],
                       "T": spec["T"], "batch_per_step": args.cpu_sample_b},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
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
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="cfg4_ssc_hybrid_2x512", choices=list(CONFIGS))
    ap.add_argument("--cpu-sample-b", type=int, default=2)
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--T", type=int, default=None, help="override T (profiling of small cases)")
    ap.add_argument("--B", type=int, default=None, help="override the per-GPU batch")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    spec = dict(CONFIGS[args.config])
    if args.T:
        spec["T"] = args.T
    if args.B:
        spec["B"] = args.B

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
    x_cpu, labels_cpu = make_inputs(spec, B, seed=1 + rank)
    x = x_cpu.to(dev)
    labels = labels_cpu.to(dev)

    def step(xb, lb):
        opt.zero_grad(set_to_none=True)
        out = model(xb)
        loss = loss_fn(out, lb)
        loss.backward()
        allreduce_grads(params, ws)
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
        start.record()
        for _ in range(args.steps):
            step(x, labels)
        end.record()
        torch.cuda.synchronize()
    barrier(ws)
    launches = _lib.launch_count() - launches0
    ms = max_over_ranks(start.elapsed_time(end), ws) / args.steps
    units = B * spec["T"] * ws
    value = units / (ms / 1e3)

    # ---- end to end through the public API: pinned host input -> device each step,
    #      loss read back each step
    e2e = None
    if not args.no_e2e:
        xh = x_cpu.pin_memory()
        lh = labels_cpu.pin_memory()
        out_h = torch.empty(1, pin_memory=True)
        barrier(ws)
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            xd = xh.to(dev, non_blocking=True)
            ld = lh.to(dev, non_blocking=True)
            loss = step(xd, ld)
            out_h.copy_(loss.detach().reshape(1), non_blocking=True)
        e2.record()
        torch.cuda.synchronize()
        ms2 = max_over_ranks(s2.elapsed_time(e2), ws) / args.steps
        e2e = {"value": units / (ms2 / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int(xh.numel() * 4 + lh.numel() * 8), "d2h_bytes_per_step": 4}

    # ---- dominant kernel roofline: the reverse scan of one hybrid layer, timed alone
    roof = roofline_probe(model, x, labels, dev) if rank == 0 else None

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        model_cpu, cfg_cpu = build_model(spec, args.cpu_sample_b, "cpu")
        v, med = time_cpu(model_cpu, spec, cfg_cpu, args.cpu_sample_b, args.cpu_steps, threads)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{args.cpu_sample_b} samples x T={spec['T']} of the same model per step, "
                         f"median of {args.cpu_steps} ({med:.1f} s/step)"}

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
                "roofline": roof, "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def roofline_probe(model, x, labels, dev):
    """Times the hybrid layer's reverse scan (the dominant kernel) on its own with CUDA
    events on the launching stream, and converts its algorithmic flops to TFLOP/s.
    Algorithmic work per launch: the recurrent contraction of the backward,
    2*N^2 flops per sample-timestep (gz = W^T gr with the per-synapse shift)."""
    from delrec import functional as Fn
    from delrec import networks
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    rec = [m for m in model.layers if hasattr(m, "recurrent_weights")]
    if not rec:
        return None
    layer = rec[0]
    T, B = x.shape[0], x.shape[1]
    N = layer.neurons
    with torch.no_grad():
        h = model.layers[0](x)
    h = h.detach().requires_grad_(True)
    y = layer(h)
    gy = torch.randn_like(y)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    s.record()
    for _ in range(reps):
        torch.autograd.grad(y, [h], gy, retain_graph=True)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / reps
    flops = 2.0 * N * N * B * T
    peak = peaks.get("bf16_tflops")
    achieved = flops / (ms / 1e3) / 1e12
    return {"bound": "tensor", "kernel": "layer backward (reverse scan + gradient reductions)",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": (achieved / peak) if peak else None, "traffic": None,
            "ms_per_launch": ms, "flops_per_launch": flops,
            "peak_source": "MEASURED_PEAKS.json bf16_tflops (measured)" if peak else "absent"}


if __name__ == "__main__":
    main()
