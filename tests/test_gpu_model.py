"""Full-model parity: CUDA train step vs the CPU oracle on identical seeded weights/tokens.

Procedure of scripts/gpu-gpt-validate.ts:52-91 (CPU model seed mulberry32(7), tokens then
targets from one mulberry32(99) stream, every parameter gradient compared with maxRelErr,
denominator floor 1e-3).  Tolerances: loss 1e-4 relative, gradients 2e-3 relative (TF32
tensor-core GEMMs with fp32 accumulation).
"""
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


def _run_parity(ctx, orc, V, T, L, H, E, arch, b, t, hidden=0, attn=0):
    from turt_b200.runtime import Model, make_config
    cfg = orc.cfg(V, T, L, H, E, arch, hidden)
    params = orc.init(cfg, 7)
    ids, tgt = _tokens(orc, b * t, V)
    ref_loss, ref_g = orc.loss_grad(cfg, params, ids, tgt, b, t)
    model = Model(ctx, make_config(V, T, L, H, E, arch, hidden))
    try:
        model.set_attention(attn)
        assert model.num_params() == orc.num_params(cfg)
        assert model.shapes == orc.param_shapes(cfg)
        model.load_flat(params)
        np.testing.assert_array_equal(model.params_flat(), params)
        loss = model.forward_backward(ids, tgt, b, t)
        g = model.grads_flat()
    finally:
        model.close()
    loss_err = max_rel_err([loss], [ref_loss])
    worst, worst_name = 0.0, ""
    off = 0
    for name, shp in zip(model.names, model.shapes):
        n = int(np.prod(shp))
        e = max_rel_err(g[off:off + n], ref_g[off:off + n])
        if e > worst:
            worst, worst_name = e, name
        off += n
    return loss, ref_loss, loss_err, worst, worst_name


ATTN = [pytest.param(1, id="tensor-attn"), pytest.param(2, id="flash-attn")]


@pytest.mark.parametrize("attn", ATTN)
@pytest.mark.parametrize("arch", ["gpt2", "modern"])
def test_validate_config(ctx, orc, arch, attn):
    """The reference's own validation config: V 48, block 16, 2 layers, 2 heads, E 32, b 2, t 8."""
    loss, ref, le, ge, name = _run_parity(ctx, orc, 48, 16, 2, 2, 32, arch, 2, 8, attn=attn)
    assert le <= LOSS_TOL, (loss, ref)
    assert ge <= GRAD_TOL, (ge, name)


@pytest.mark.parametrize("attn", ATTN)
@pytest.mark.parametrize("hidden", [320, 352])
def test_tiny_modern_8x128(ctx, orc, hidden, attn):
    """Tiny modern GPT (4 layers, 4 heads, d 128, vocab 8192, batch 8 x 128), SwiGLU 320 and 352."""
    loss, ref, le, ge, name = _run_parity(ctx, orc, 8192, 128, 4, 4, 128, "modern", 8, 128, hidden, attn)
    assert le <= LOSS_TOL, (loss, ref)
    assert ge <= GRAD_TOL, (ge, name)


@pytest.mark.parametrize("attn", ATTN)
def test_gpt2_hd64(ctx, orc, attn):
    """gpt2 arch with head dim 64 and a ragged sequence length (t not a multiple of 64)."""
    loss, ref, le, ge, name = _run_parity(ctx, orc, 512, 96, 2, 2, 128, "gpt2", 3, 80, attn=attn)
    assert le <= LOSS_TOL, (loss, ref)
    assert ge <= GRAD_TOL, (ge, name)


def test_adamw_clip_step(ctx, orc):
    """One full step (fwd+bwd+clip+AdamW, scripts/train-gpt.ts:241-242): the GPU's clip + AdamW
    pass applied to its own gradients must match the oracle's clipGradNorm + AdamW on the same
    gradients (src/optim/clip.ts:7-24, src/optim/adam.ts:35-54)."""
    from turt_b200.runtime import Model, make_config
    V, T, L, H, E, b, t = 256, 32, 2, 2, 64, 4, 32
    cfg = orc.cfg(V, T, L, H, E, "modern")
    params = orc.init(cfg, 7)
    ids, tgt = _tokens(orc, b * t, V)
    lr, b1, b2, eps, wd, clip = 3e-4, 0.9, 0.95, 1e-8, 0.1, 1.0
    model = Model(ctx, make_config(V, T, L, H, E, "modern"))
    try:
        model.load_flat(params)
        model.zero_grad()
        loss = model.forward_backward(ids, tgt, b, t)
        g = model.grads_flat()
        model.adamw_step(lr, b1, b2, eps, wd, 1 - b1, 1 - b2, clip=clip)
        p_gpu = model.params_flat()
    finally:
        model.close()
    ref_loss, ref_g = orc.loss_grad(cfg, params, ids, tgt, b, t)
    assert max_rel_err([loss], [ref_loss]) <= LOSS_TOL
    assert max_rel_err(g, ref_g) <= GRAD_TOL
    gc = g.copy()
    norm = orc.clip(gc, clip)
    assert norm > clip  # the clip is active at init
    p_ref = params.copy()
    orc.adamw(p_ref, gc, np.zeros_like(p_ref), np.zeros_like(p_ref), lr, b1, b2, eps, wd, 1)
    np.testing.assert_allclose(p_gpu, p_ref, rtol=0, atol=1e-6)


def test_out_of_range_token_rejected(ctx, orc):
    from turt_b200._lib import ERR_RANGE, TurtError
    from turt_b200.runtime import Model, make_config
    model = Model(ctx, make_config(48, 16, 1, 2, 32, "modern"))
    try:
        ids = np.array([1, 2, 48, 3], dtype=np.uint32)
        tgt = np.array([1, 2, 3, 4], dtype=np.uint32)
        with pytest.raises(TurtError) as ei:
            model.forward_backward(ids, tgt, 1, 4)
        assert ei.value.code == ERR_RANGE
        with pytest.raises(TurtError) as ei:
            model.forward_backward(tgt, np.array([1, 2, 3, 4096], dtype=np.uint32), 1, 4)
        assert ei.value.code == ERR_RANGE
        # the context stays usable after the error
        loss = model.forward_backward(tgt, tgt, 1, 4)
        assert np.isfinite(loss)
    finally:
        model.close()


def test_sequence_longer_than_block_rejected(ctx):
    from turt_b200._lib import ERR_INVALID, TurtError
    from turt_b200.runtime import Model, make_config
    model = Model(ctx, make_config(48, 8, 1, 2, 32, "modern"))
    try:
        with pytest.raises(TurtError) as ei:
            model.forward_backward(np.zeros(16, np.uint32), np.zeros(16, np.uint32), 1, 16)
        assert ei.value.code == ERR_INVALID
    finally:
        model.close()


@pytest.mark.parametrize("pair", [0, 1, 2])
@pytest.mark.parametrize("bn", [64, 128, 192, 256])
@pytest.mark.parametrize("arch", ["gpt2", "modern"])
def test_fused_epilogues_every_tile_width(ctx, orc, arch, bn, pair):
    """Bias / GELU / SwiGLU / residual epilogues and the attention GEMMs (two-level batch,
    causal skips) under each forced GEMM tile width and kernel (single CTA / CTA pair)."""
    from turt_b200._lib import check, lib
    if pair == 2 and bn > 128:
        pytest.skip("two CTAs per SM exist for tile widths 64 and 128")
    check(lib().turt_gemm_set_tile(bn, pair))
    try:
        loss, ref, le, ge, name = _run_parity(ctx, orc, 512, 96, 2, 2, 128, arch, 3, 80, 352 if arch == "modern" else 0)
    finally:
        check(lib().turt_gemm_set_tile(0, -1))
    assert le <= LOSS_TOL, (loss, ref)
    assert ge <= GRAD_TOL, (ge, name)


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
@pytest.mark.parametrize("t", [7, 130, 200, 301])
def test_tensor_attention_ragged(ctx, orc, arch, t):
    """Tensor-core attention with sequence lengths that are not multiples of 4 (padded score
    pitch), of the 128-row tile (diagonal tiles split), above one tile, and above 256; head dim
    16 (the three-launch chain: score GEMM, softmax rows, P.V GEMM)."""
    loss, ref, le, ge, name = _run_parity(ctx, orc, 256, 320, 2, 4, 64, arch, 2, t, attn=1)
    assert le <= LOSS_TOL, (loss, ref)
    assert ge <= GRAD_TOL, (ge, name)


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
@pytest.mark.parametrize("E,H", [(64, 2), (128, 2)])
@pytest.mark.parametrize("t", [7, 64, 130, 200, 256])
def test_fused_attention_forward(ctx, orc, arch, E, H, t):
    """The single-kernel attention forward (T <= 256, head dims 32 and 64): one or two query
    tiles, key counts that are not whole 64-key chunks, a ragged last tile and a row pitch that
    is not a multiple of 32 (P zero-filled past the causal block); the backward reads its P."""
    loss, ref, le, ge, name = _run_parity(ctx, orc, 256, 256, 2, H, E, arch, 2, t, attn=1)
    assert le <= LOSS_TOL, (loss, ref)
    assert ge <= GRAD_TOL, (ge, name)


def test_bounded_wait_times_out_and_context_survives(ctx, orc):
    """A device wait that nothing completes gives up after its limit (1 ms here), the call
    reports TURT_ERR_TIMEOUT, and the same context then runs a full train step correctly
    (the reference only notices a failed step by a zero loss, scripts/gpu-pretrain.ts:232-238)."""
    import time

    from turt_b200._lib import ERR_TIMEOUT, lib, last_error
    t0 = time.perf_counter()
    rc = lib().turt_wait_selftest(ctx.handle, 1000)
    elapsed = time.perf_counter() - t0
    assert rc == ERR_TIMEOUT
    assert "timed out" in last_error()
    assert elapsed < 5.0
    ctx.synchronize()  # the flag was cleared by the report
    loss, ref, le, ge, name = _run_parity(ctx, orc, 48, 16, 2, 2, 32, "modern", 2, 8)
    assert le <= LOSS_TOL, (loss, ref)
    assert ge <= GRAD_TOL, (ge, name)


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
@pytest.mark.parametrize("E,H", [(64, 2), (128, 2)])
@pytest.mark.parametrize("t", [7, 64, 130, 256, 301])
def test_online_attention_any_length(ctx, orc, arch, E, H, t):
    """The tensor-core online-softmax attention (forward, dQ and dK / dV kernels, no [T][T]
    buffers) forced at every length, head dims 32 and 64: one block of keys, a ragged last
    block, several 128-row query tiles and key tiles, and the lengths the default takes it at."""
    loss, ref, le, ge, name = _run_parity(ctx, orc, 256, 320, 2, H, E, arch, 2, t, attn=3)
    assert le <= LOSS_TOL, (loss, ref)
    assert ge <= GRAD_TOL, (ge, name)
