"""Data-parallel semantics on CPU ranks (gloo, world size 2), with the oracle as the replica.

The GPU path shards the global batch contiguously across ranks, each rank backpropagates
the mean loss of its shard, the flat gradient buffer is summed across ranks and scaled by
1/world inside AdamW.  For equal shards this equals the reference's row-weighted mean
(scripts/train-gpt.ts:105-123, 200-219) and hence the full-batch gradient
(tests/scripts/checkpoint.test.ts:83-107).  These tests run that exact host logic with
torch.distributed on gloo, plus the failure paths: a rank that raises, and a rank that
never joins a collective (bounded by the process-group timeout).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank, world, port, q):
    import torch

    from oracle.oracle import Oracle
    _init(rank, world, port)
    o = Oracle()
    cfg = o.cfg(32, 8, 2, 2, 16, "modern")
    p = o.init(cfg, 8)
    b, t = 4, 8
    ids = o.uniform_ints(b * t, 5, 32)
    tgt = o.uniform_ints(b * t, 6, 32)
    per = b // world
    sl = slice(rank * per * t, (rank + 1) * per * t)
    loss, g = o.loss_grad(cfg, p, ids[sl], tgt[sl], per, t)
    gt = torch.from_numpy(g.astype(np.float64))
    dist.all_reduce(gt)
    lt = torch.tensor([loss], dtype=torch.float64)
    dist.all_reduce(lt)
    if rank == 0:
        full_loss, full_g = o.loss_grad(cfg, p, ids, tgt, b, t)
        q.put((float(lt.item() / world), full_loss, (gt.numpy() / world), full_g))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_mean_equals_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    loss, full_loss, g, full_g = q.get(timeout=120)
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    assert abs(loss - full_loss) < 1e-5
    np.testing.assert_allclose(g, full_g, atol=5e-6)


def _failing_worker(rank, world, port, q, mode):
    import torch
    _init(rank, world, port, timeout_s=5)
    try:
        if rank == 1:
            if mode == "raise":
                raise RuntimeError("injected rank failure")
            if mode == "absent":
                dist.barrier()
                return  # leaves without joining the next collective
        dist.barrier()
        x = torch.ones(4)
        dist.all_reduce(x)
        q.put((rank, "ok"))
    except RuntimeError as e:
        q.put((rank, "error:" + str(e)[:80]))


@pytest.mark.parametrize("mode", ["raise", "absent"])
def test_rank_failure_is_detected_on_the_host(mode):
    """A failing or departed rank ends the surviving rank's next collective with an error
    within the process-group timeout instead of hanging it."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for pr in procs:
        pr.start()
    results = {}
    for _ in range(2):
        try:
            r, msg = q.get(timeout=60)
            results[r] = msg
        except Exception:
            break
    for pr in procs:
        pr.join(timeout=60)
        if pr.is_alive():
            pr.kill()
    assert 0 in results and results[0].startswith("error"), results
