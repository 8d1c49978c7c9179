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
