"""Batch-parallel gradient averaging on world_size 2 with gloo (CPU), including a rank
that fails: the survivor's collective must end with an error, not hang."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, ws, port, out, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=10))
    from delrec.data_parallel import allreduce_gradients, shard_batch
    torch.manual_seed(0)
    lin = torch.nn.Linear(6, 3)
    x = torch.arange(4 * 8 * 6, dtype=torch.float32).reshape(4, 8, 6) / 100.0
    y = torch.arange(8) % 3
    xs, ys = shard_batch(x, y, rank, ws)
    loss = torch.nn.functional.cross_entropy(lin(xs).sum(0), ys, reduction="sum")
    loss.backward()
    if rank == fail_rank:
        raise SystemExit(3)           # leaves before the collective
    try:
        allreduce_gradients(list(lin.parameters()), average=False)
        out[rank] = lin.weight.grad.clone()
    except Exception as e:            # the peer vanished: the collective errors out
        out[rank] = str(type(e).__name__)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(fail_rank=-1):
    ws = 2
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, ws, port, out, fail_rank)) for r in range(ws)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank hung")
    return dict(out), [p.exitcode for p in procs]


def test_allreduce_matches_full_batch_gradient():
    out, codes = _run()
    assert codes == [0, 0]
    torch.manual_seed(0)
    lin = torch.nn.Linear(6, 3)
    x = torch.arange(4 * 8 * 6, dtype=torch.float32).reshape(4, 8, 6) / 100.0
    y = torch.arange(8) % 3
    torch.nn.functional.cross_entropy(lin(x).sum(0), y, reduction="sum").backward()
    for r in range(2):
        torch.testing.assert_close(out[r], lin.weight.grad, rtol=1e-5, atol=1e-6)


def test_failed_rank_does_not_hang_the_survivor():
    out, codes = _run(fail_rank=1)
    assert codes[1] == 3
    assert 0 in out and isinstance(out[0], str)   # an error was raised, not a hang


def _delay_model_worker(rank, ws, port, out, overlapped):
    """One rank: the hybrid delay model's real parameters, the rank's batch shard run through
    the oracle replay of the model on those very parameter tensors (so autograd's
    gradient hooks fire as in training), then the gradient averaging."""
    import sys
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    here = os.path.dirname(os.path.abspath(__file__))
    for p in (os.path.dirname(here), here):
        if p not in sys.path:
            sys.path.insert(0, p)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=20))
    from delrec.data_parallel import OverlappedAllReduce, allreduce_gradients, shard_batch
    x, y, model, step = _delay_model_case()
    params = [p for p in model.parameters() if p.requires_grad]
    ar = OverlappedAllReduce(params, bucket_bytes=4096, average=False) if overlapped else None
    xs, ys = shard_batch(x, y, rank, ws)
    step(xs, ys)
    if overlapped:
        ar.finish()
        ar.remove()
    else:
        allreduce_gradients(params, average=False)
    out[rank] = {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}
    dist.destroy_process_group()


def _delay_model_case():
    """A small SNN_recurrent_hybrid_delays (hidden 12, offsets <= 3) and a step that runs
    its forward + loss + backward through the oracle on the model's own parameters."""
    from delrec import networks
    from model_configs import mem_config
    from oracle import delrec_oracle as O
    cfg = mem_config(hidden=[12], bias=False, T=10, B=8, C=5, K=3)
    cfg.hybrid_offset_scale = 3
    torch.manual_seed(0)
    model = networks.SNN_recurrent_hybrid_delays(cfg)
    g = torch.Generator().manual_seed(7)
    x = (torch.rand(10, 8, 5, generator=g) < 0.4).float() * 2.0
    y = torch.arange(8) % 3
    lay = model.layers
    rec = lay[2]

    def step(xb, yb):
        base = networks.learned_delay_parameter(rec, "recurrent_delays")
        off = rec.parametrizations.recurrent_delays[0].offsets
        lif = O.OracleLIF(tau=2.0, v_threshold=1.0, v_reset=0.0, surrogate=O.ATanSpike(2.0))
        h = xb @ lay[0].weight.t()
        s = O.synaptic_scan(h, rec.recurrent_weights, O.hybrid_delays(base, off), lif)
        out = s @ lay[4].weight.t()
        torch.nn.functional.cross_entropy(out.sum(0), yb, reduction="sum").backward()
    return x, y, model, step


@pytest.mark.parametrize("overlapped", [False, True])
def test_delay_model_gradients_match_full_batch(overlapped):
    """World size 2 over the hybrid delay model's parameter set (recurrent weights, the
    parametrized base, the projections): the summed shard gradients equal the full-batch
    gradient, with one flat all-reduce and with the bucketed all-reduce launched from the
    gradient hooks during the backward."""
    ws = 2
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_delay_model_worker, args=(r, ws, port, out, overlapped)) for r in range(ws)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank hung")
    assert [p.exitcode for p in procs] == [0, 0]
    x, y, model, step = _delay_model_case()
    step(x, y)
    full = {n: p.grad for n, p in model.named_parameters() if p.grad is not None}
    assert len(full) >= 3
    for r in range(ws):
        assert out[r].keys() == full.keys()
        for n in full:
            torch.testing.assert_close(out[r][n], full[n], rtol=1e-5, atol=1e-6)
