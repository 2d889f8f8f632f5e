"""One process driving several GPUs (turt_group_*): the reference's in-process data-parallel
worker pool (scripts/train-gpt.ts:66-123,200-219) with one replica per device.

The batch is split into contiguous shards of floor(b/n) (+1 for the first b mod n) sequences,
each shard's mean-loss gradient weighted by rows_i / b and summed over NCCL: every replica must
then hold the full-batch mean gradient (checked against the CPU oracle, maxRelErr <= 2e-3, loss
1e-4), the loss must be the row-weighted mean, replicas must agree bit for bit, and a clip +
AdamW step must leave them identical.  On one GPU the group is a single replica (no NCCL); the
multi-GPU cases run when the box has 2 or more GPUs.
"""
import numpy as np
import pytest

from oracle.oracle import Oracle, max_rel_err

pytestmark = pytest.mark.gpu


def _ngpu():
    import torch
    return torch.cuda.device_count()


def _case(orc, b, t, V=512, T=64, L=2, H=2, E=64, arch="modern"):
    cfg = orc.cfg(V, T, L, H, E, arch)
    params = orc.init(cfg, 7)
    st = orc.rng(99)
    ids = np.array([int(orc.rng_next(st) * V) for _ in range(b * t)], np.int32)
    tgt = np.array([int(orc.rng_next(st) * V) for _ in range(b * t)], np.int32)
    return cfg, params, ids, tgt


@pytest.mark.parametrize("ndev,b", [(1, 4), (2, 4), (2, 5), (4, 7), (8, 8)])
@pytest.mark.parametrize("arch", ["modern", "gpt2"])
def test_group_matches_full_batch(ndev, b, arch):
    if _ngpu() < ndev:
        pytest.skip(f"needs {ndev} GPUs")
    import os
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from turt_b200.runtime import Group, make_config
    orc = Oracle()
    V, T, L, H, E, t = 512, 64, 2, 2, 64, 64
    cfg, params, ids, tgt = _case(orc, b, t, V, T, L, H, E, arch)
    ref_loss, ref_g = orc.loss_grad(cfg, params, ids, tgt, b, t)
    g = Group(list(range(ndev)), make_config(V, T, L, H, E, arch))
    try:
        g.load_flat(params)
        # the first call of a shape reduces after the whole backward, later ones per layer
        for _ in range(2):
            g.zero_grad()
            loss = g.forward_backward(ids, tgt, b, t)
            grads = [g.grads_flat(r) for r in range(ndev)]
            assert max_rel_err([loss], [ref_loss]) <= 1e-4, (loss, ref_loss)
            assert max_rel_err(grads[0], ref_g) <= 2e-3
        g.adamw_step(3e-4, 0.9, 0.95, 1e-8, 0.1, 0.1, 0.05, clip=1.0)
        g.synchronize()
        new = [g.params_flat(r) for r in range(ndev)]
    finally:
        g.close()
    assert max_rel_err([loss], [ref_loss]) <= 1e-4, (loss, ref_loss)
    assert max_rel_err(grads[0], ref_g) <= 2e-3
    for r in range(1, ndev):
        np.testing.assert_array_equal(grads[r], grads[0])
        np.testing.assert_array_equal(new[r], new[0])
    assert not np.array_equal(new[0], params)


def test_group_micro_batches_accumulate():
    """Two deferred-then-reducing micro-batches equal one step over their union."""
    ndev = min(2, _ngpu())
    from turt_b200.runtime import Group, make_config
    orc = Oracle()
    V, T, L, H, E, t, b = 512, 64, 2, 2, 64, 64, 8
    cfg, params, ids, tgt = _case(orc, b, t, V, T, L, H, E)
    ref_loss, ref_g = orc.loss_grad(cfg, params, ids, tgt, b, t)
    g = Group(list(range(ndev)), make_config(V, T, L, H, E))
    try:
        g.load_flat(params)
        g.zero_grad()
        half = b // 2 * t
        g.defer(True)
        g.forward_backward(ids[:half], tgt[:half], b // 2, t, loss_scale=0.5, want_loss=False)
        g.defer(False)
        g.forward_backward(ids[half:], tgt[half:], b // 2, t, loss_scale=0.5)
        grads = g.grads_flat()
    finally:
        g.close()
    assert max_rel_err(grads, ref_g) <= 2e-3


def test_group_rejects_bad_arguments():
    from turt_b200._lib import ERR_INVALID, ERR_RANGE, TurtError
    from turt_b200.runtime import Group, make_config
    with pytest.raises(TurtError) as ei:
        Group([0, 0], make_config(48, 16, 1, 2, 32))
    assert ei.value.code == ERR_INVALID
    g = Group([0], make_config(48, 16, 1, 2, 32))
    try:
        with pytest.raises(TurtError) as ei:
            g.forward_backward(np.array([1, 2, 48, 3], np.uint32), np.array([1, 2, 3, 4], np.uint32), 1, 4)
        assert ei.value.code == ERR_RANGE
        assert np.isfinite(g.forward_backward(np.array([1, 2, 3, 4], np.uint32), np.array([1, 2, 3, 4], np.uint32), 1, 4))
    finally:
        g.close()
