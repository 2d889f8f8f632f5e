"""Data parallel on real GPUs: two ranks, one GPU each, NCCL all-reduce inside the backward.

The sum of the two ranks' shard-mean gradients divided by 2 must equal the full-batch gradient
(the reference's row-weighted mean, scripts/train-gpt.ts:209-217; checkpoint.test.ts:83-107):
checked against the CPU oracle with maxRelErr <= 2e-3, and both ranks must hold identical
gradients afterwards.  Skipped when fewer than 2 GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from oracle.oracle import Oracle
    from turt_b200.runtime import Context, Model, make_config
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        orc = Oracle()
        V, T, L, H, E, b, t = 512, 64, 2, 2, 64, 4, 64
        cfg = orc.cfg(V, T, L, H, E, "modern")
        params = orc.init(cfg, 7)
        st = orc.rng(99)
        ids = np.array([int(orc.rng_next(st) * V) for _ in range(b * t)], np.int32)
        tgt = np.array([int(orc.rng_next(st) * V) for _ in range(b * t)], np.int32)
        ctx = Context(rank)
        model = Model(ctx, make_config(V, T, L, H, E, "modern"))
        model.load_flat(params)
        uid = [Model.dp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        model.dp_init(rank, world, uid[0])
        per = b // world
        sl = slice(rank * per * t, (rank + 1) * per * t)
        model.zero_grad()
        loss = model.forward_backward(ids[sl], tgt[sl], per, t)
        model.dp_wait(30000)
        g = model.grads_flat() / world
        model.close()
        ctx.close()
        if rank == 0:
            ref_loss, ref_g = orc.loss_grad(cfg, params, ids, tgt, b, t)
            q.put(("ok", g, ref_g))
        else:
            q.put(("ok1", g, None))
    except Exception as e:  # surface the failure to the parent
        q.put(("error", repr(e), None))
    finally:
        dist.destroy_process_group()


def test_two_gpu_dp_equals_full_batch():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from oracle.oracle import max_rel_err
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[0] != "error", r[1]
    g0 = [r for r in res if r[0] == "ok"][0]
    g1 = [r for r in res if r[0] == "ok1"][0]
    np.testing.assert_array_equal(g0[1], g1[1])
    assert max_rel_err(g0[1], g0[2]) <= 2e-3
