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


@pytest.mark.parametrize("arch", ["modern", "gpt2"])
def test_width_768(ctx, orc, arch):
    """Rows of 768 (the 12-layer / 768-d workloads' width): the norm backwards run one row per
    warp iteration with one block per SM, 12 heads of 64; 1 layer, b 4 x 64."""
    le, ge, name, losses = _parity(ctx, orc, 512, 64, 1, 12, 768, arch, 4, 64)
    assert le <= LOSS_TOL, losses
    assert ge <= GRAD_TOL, (ge, name)


@pytest.mark.parametrize("arch", ["modern", "gpt2", "modern-T1024"])
def test_gradients_bit_identical_across_runs(ctx, orc, arch):
    """Two identical train steps give bit-identical losses and gradients: the embedding
    backward adds each vocab row's positions in a fixed order (the reference's GATHER_BWD is a
    sequential scan, src/infer/webgpu/autograd.ts:428-438) and split-K GEMMs add their partial
    sums in split order, so nothing depends on thread scheduling.  Full headline shape (the
    weight-gradient GEMMs split K there); gpt2 adds the learned-position gradient; T = 1024 runs
    the long-sequence attention kernels (dQ and dK / dV each summed by one CTA, no atomics)."""
    from turt_b200.runtime import Model, make_config
    if arch == "modern":
        V, T, L, H, E, hidden, b, t = 8192, 256, 6, 6, 384, 1024, 32, 256
    elif arch == "gpt2":
        V, T, L, H, E, hidden, b, t = 8192, 256, 2, 6, 384, 0, 32, 256
    else:  # long sequences: the online-softmax attention kernels
        arch = "modern"
        V, T, L, H, E, hidden, b, t = 2048, 1024, 2, 4, 256, 0, 4, 1024
    cfg = orc.cfg(V, T, L, H, E, arch, hidden)
    params = orc.init(cfg, 7)
    ids, tgt = _tokens(orc, b * t, V, seed=5)
    model = Model(ctx, make_config(V, T, L, H, E, arch, hidden))
    try:
        model.load_flat(params)
        runs = []
        for _ in range(3):
            model.zero_grad()
            loss = model.forward_backward(ids, tgt, b, t)
            runs.append((loss, model.grads_flat()))
    finally:
        model.close()
    for loss, g in runs[1:]:
        assert loss == runs[0][0]
        np.testing.assert_array_equal(g, runs[0][1])
