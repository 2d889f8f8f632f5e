"""Parity at the shapes the throughput numbers are quoted on.

* The headline train step itself: 6 layers, 6 heads, d 384, SwiGLU 1024, RMSNorm, RoPE, tied
  8192 vocab, 32 sequences of 256 tokens (N = 8192 rows, so the GEMM tile planner and the
  fused attention kernels make exactly the choices they make in the timed step).
* The attention shape of the 12-layer / 768-d gpt2 workload: head dim 64, T = 512 (LayerNorm,
  GELU, learned positions, biases), on a 2-layer model.
* The attention shape of the 12-layer / 768-d data-parallel workload: modern, head dim 64,
  T = 1024, on a 2-layer model.

Procedure of scripts/gpu-gpt-validate.ts:52-91: CPU model seed mulberry32(7), tokens then
targets from one mulberry32(99) stream, every parameter gradient compared with maxRelErr
(denominator floor 1e-3).  The oracle runs as the reference's CPU data-parallel pool
(scripts/train-gpt.ts:200-219: contiguous shards, row-weighted gradient mean) on the host's
cores, which is the full-batch mean gradient.  Tolerances: loss 1e-4 relative, gradients 2e-3.
"""
import os

import numpy as np
import pytest

from oracle.oracle import Oracle, max_rel_err

pytestmark = pytest.mark.gpu

LOSS_TOL = 1e-4
GRAD_TOL = 2e-3


@pytest.fixture(scope="module")
def ctx():
    from turt_b200.runtime import Context
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def _tokens(orc, n, vocab, seed=99):
    st = orc.rng(seed)
    ids = np.array([int(orc.rng_next(st) * vocab) for _ in range(n)], dtype=np.int32)
    tgt = np.array([int(orc.rng_next(st) * vocab) for _ in range(n)], dtype=np.int32)
    return ids, tgt


def _parity(ctx, orc, V, T, L, H, E, arch, b, t, hidden=0, attn=0):
    from turt_b200.runtime import Model, make_config
    cfg = orc.cfg(V, T, L, H, E, arch, hidden)
    params = orc.init(cfg, 7)
    ids, tgt = _tokens(orc, b * t, V)
    workers = max(1, min(b, os.cpu_count() or 1))
    ref_loss, ref_g = orc.dp_grads(cfg, params, ids, tgt, b, t, workers)
    model = Model(ctx, make_config(V, T, L, H, E, arch, hidden))
    try:
        model.set_attention(attn)
        model.load_flat(params)
        loss = model.forward_backward(ids, tgt, b, t)
        g = model.grads_flat()
        names, shapes = model.names, model.shapes
    finally:
        model.close()
    worst, worst_name, off = 0.0, "", 0
    for name, shp in zip(names, shapes):
        n = int(np.prod(shp))
        e = max_rel_err(g[off:off + n], ref_g[off:off + n])
        if e > worst:
            worst, worst_name = e, name
        off += n
    return max_rel_err([loss], [ref_loss]), worst, worst_name, (loss, ref_loss)


def test_headline_6L_384d_batch32x256(ctx, orc):
    """The benchmarked train step, full size: modern 6L/6H/384d, h 1024, V 8192, 32 x 256."""
    le, ge, name, losses = _parity(ctx, orc, 8192, 256, 6, 6, 384, "modern", 32, 256, hidden=1024)
    assert le <= LOSS_TOL, losses
    assert ge <= GRAD_TOL, (ge, name)


@pytest.mark.parametrize("attn", [pytest.param(0, id="auto"), pytest.param(2, id="cuda-core")])
def test_gpt2_head_dim64_T512(ctx, orc, attn):
    """gpt2 arch, 4 heads of 64, T 512 (the 12L-768d gpt2 workload's attention shape), b 2."""
    le, ge, name, losses = _parity(ctx, orc, 1024, 512, 2, 4, 256, "gpt2", 2, 512, attn=attn)
    assert le <= LOSS_TOL, losses
    assert ge <= GRAD_TOL, (ge, name)


@pytest.mark.parametrize("attn", [pytest.param(0, id="auto"), pytest.param(2, id="cuda-core")])
@pytest.mark.parametrize("t", [1024, 777])
def test_modern_head_dim64_T1024(ctx, orc, attn, t):
    """modern arch, 2 heads of 64, block 1024 (the 12L-768d data-parallel workload's attention
    shape), full and ragged sequence lengths, b 2."""
    le, ge, name, losses = _parity(ctx, orc, 512, 1024, 2, 2, 128, "modern", 2, t, attn=attn)
    assert le <= LOSS_TOL, losses
    assert ge <= GRAD_TOL, (ge, name)
