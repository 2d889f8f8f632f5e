"""The train step's fused memory-bound kernels, standalone (turt_fused_*), against the oracle.

RMSNorm backward (RMS_DX + RMS_DG, autograd.ts:331-365, with the residual gradient added),
SwiGLU backward (SILU_BWD and the gate*up product rule), fused softmax cross-entropy
(CE_FWD + CE_BWD, autograd.ts:441-471) and AdamW with global-norm clipping (adam.ts:31-54,
clip.ts:7-24).  The first case of each test is the standalone backward-op benchmark's full
shape: RMSNorm [8192,384], SwiGLU [8192,1024], softmax-CE [8192,8192], AdamW over 10M.  The kernels compute in fp32; the oracle, like the reference's JavaScript, in
doubles.  Two bounds: max|got - ref| / max|ref| <= 1e-5 (fp32 rounding of the tensor's scale)
and the reference validator's maxRelErr (denominator max(1e-3, |a|, |b|)) <= 1e-3, which is
what fp32 rounding of O(1) terms leaves on entries that cancel to ~1e-3 (an fp32 emulation of
AdamW's m update gives 1e-4 there); the model's gradient bar is 2e-3.
"""
import numpy as np
import pytest

from oracle.oracle import Oracle, max_rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3     # maxRelErr
NORM_TOL = 1e-5


def _ok(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    norm = float(np.max(np.abs(got - ref)) / max(1e-30, np.max(np.abs(ref))))
    return max_rel_err(got, ref) < TOL and norm < NORM_TOL


def _ok_terms(got, ref, abs_terms, coef=1e-5):
    """Entries that are sums of a few fp32 terms (RMSNorm's dx = rs*g*dy - k*x + dres): each within
    1e-5 of the sum of its terms' magnitudes.  The oracle restates the reference's autograd chain
    with an fp32 rounding after every operation, a different path from the kernel's one-pass
    formula; an fp32 emulation of the kernel at [8192,768] sits 3.7e-6 of sum|terms| from it and
    reaches maxRelErr 1.4e-3 on entries the residual add cancels to ~1e-3."""
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return bool(np.all(np.abs(got - ref) <= coef * np.asarray(abs_terms, np.float64) + 1e-7))


def _ok_sum(got, ref, abs_terms):
    """For a column sum over many rows computed in fp32: each entry within 1e-6 of the sum of
    its terms' magnitudes (about 16 fp32 ulps of that sum; a plain blocked fp32 sum of 8192
    rows already leaves maxRelErr ~1.1e-3 on entries that cancel to ~0.1)."""
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return bool(np.all(np.abs(got - ref) <= 1e-6 * np.asarray(abs_terms, np.float64) + 1e-7))


@pytest.fixture(scope="module")
def ctx():
    from turt_b200.runtime import Context
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def _dev(ctx, a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    p = ctx.buffer(a.size)
    ctx.upload(p, a)
    return p


@pytest.mark.parametrize("rows,E", [(8192, 384), (1024, 384), (1000, 384), (100, 32), (37, 768), (8192, 768),
                                    (2500, 640)])
@pytest.mark.parametrize("with_res", [False, True])
def test_rms_bwd(ctx, orc, rows, E, with_res):
    """RMSNorm backward (residual gradient optional) and its dgamma column sum.  Called twice:
    dgamma accumulates both calls and dx is rewritten identically.  1000 rows leave the last block
    short; E 640 / 768 run one row per warp iteration with one block per SM."""
    from turt_b200._lib import check, lib
    rng = np.random.default_rng(rows + E)
    x = rng.standard_normal((rows, E)).astype(np.float32)
    gam = (1 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    dy = rng.standard_normal((rows, E)).astype(np.float32)
    dres = rng.standard_normal((rows, E)).astype(np.float32) if with_res else None
    rstd = (1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1) + 1e-5)).astype(np.float32)
    _, ref_dx, ref_dg = orc.rmsnorm(x, gam, dy)
    if with_res:
        ref_dx = ref_dx + dres
    dg0 = rng.standard_normal(E).astype(np.float32)  # dg accumulates
    bufs = [_dev(ctx, a) for a in (x, dy, gam, rstd, dg0)]
    dx = ctx.buffer(rows * E)
    dr = _dev(ctx, dres) if with_res else None
    for _ in range(2):
        check(lib().turt_fused_rms_bwd(ctx.handle, bufs[0], bufs[1], bufs[2], bufs[3], dr, dx, bufs[4], rows, E))
    got_dx = ctx.download(dx, rows * E).reshape(rows, E)
    got_dg = ctx.download(bufs[4], E)
    x64, rs64 = x.astype(np.float64), rstd.astype(np.float64)
    k64 = rs64 ** 3 * (dy.astype(np.float64) * gam * x64).sum(axis=1) / E
    dx_terms = np.abs(rs64[:, None] * dy * gam) + np.abs(k64[:, None] * x64) + (np.abs(dres) if with_res else 0.0)
    assert _ok_terms(got_dx, ref_dx, dx_terms)
    assert max_rel_err(got_dx, ref_dx) < 2e-3  # the model's gradient bar
    assert np.max(np.abs(got_dx - ref_dx)) / np.max(np.abs(ref_dx)) < NORM_TOL
    abs_terms = 2 * np.abs(dy.astype(np.float64) * x * rstd[:, None]).sum(axis=0) + np.abs(dg0)
    assert _ok_sum(got_dg, 2 * ref_dg.astype(np.float64) + dg0, abs_terms)


@pytest.mark.parametrize("n", [8192 * 1024, 8192 * 1024 // 64, 1003])
def test_swiglu_bwd(ctx, orc, n):
    from turt_b200._lib import check, lib
    rng = np.random.default_rng(n)
    a, u, d = (rng.standard_normal(n).astype(np.float32) for _ in range(3))
    ref_du = d * orc.silu(a)
    ref_da = orc.silu_bwd(a, d * u)
    pa, pu, pd = (_dev(ctx, t) for t in (a, u, d))
    da, du = ctx.buffer(n), ctx.buffer(n)
    check(lib().turt_fused_swiglu_bwd(ctx.handle, pa, pu, pd, da, du, n))
    assert _ok(ctx.download(da, n), ref_da)
    assert _ok(ctx.download(du, n), ref_du)


@pytest.mark.parametrize("N,V", [(8192, 8192), (256, 8192), (33, 48)])
def test_ce_fused(ctx, orc, N, V):
    from turt_b200._lib import check, lib, u32
    rng = np.random.default_rng(N + V)
    logits = (3 * rng.standard_normal((N, V))).astype(np.float32)
    tgt = rng.integers(0, V, N).astype(np.uint32)
    ref_loss, ref_g = orc.cross_entropy(logits, tgt)
    pl = _dev(ctx, logits)
    pt = ctx.index_buffer(u32(tgt))
    rows = ctx.buffer(N)
    check(lib().turt_fused_ce(ctx.handle, pl, pt, rows, N, V, 1.0 / N))
    got_g = ctx.download(pl, N * V).reshape(N, V)
    got_loss = float(ctx.download(rows, N).astype(np.float64).mean())
    assert abs(got_loss - ref_loss) / abs(ref_loss) < 1e-6
    assert _ok(got_g, ref_g)


@pytest.mark.parametrize("n", [10_000_000, 100_003])
@pytest.mark.parametrize("clip", [0.0, 1.0])
def test_adamw_clip(ctx, orc, clip, n):
    from turt_b200._lib import check, lib
    import ctypes as C
    rng = np.random.default_rng(5)
    p, g, m = (rng.standard_normal(n).astype(np.float32) for _ in range(3))
    v = np.abs(rng.standard_normal(n)).astype(np.float32)
    lr, b1, b2, eps, wd, k = 3e-4, 0.9, 0.95, 1e-8, 0.1, 3
    bc1, bc2 = 1 - b1 ** k, 1 - b2 ** k
    rp, rg, rm, rv = p.copy(), g.copy(), m.copy(), v.copy()
    ref_norm = float(np.sqrt((g.astype(np.float64) ** 2).sum()))
    if clip > 0:
        orc.clip(rg, clip)
    orc.adamw_bc(rp, rg, rm, rv, lr, b1, b2, eps, wd, bc1, bc2)
    bufs = [_dev(ctx, t) for t in (p, g, m, v)]
    norm = C.c_double()
    check(lib().turt_fused_adamw_clip(ctx.handle, bufs[0], bufs[1], bufs[2], bufs[3], n, lr, b1, b2, eps, wd, bc1,
                                      bc2, clip, C.byref(norm)))
    assert abs(norm.value - ref_norm) / ref_norm < 1e-9
    for buf, ref in zip((bufs[0], bufs[2], bufs[3]), (rp, rm, rv)):
        assert _ok(ctx.download(buf, n), ref)
    np.testing.assert_array_equal(ctx.download(bufs[1], n), g)  # the gradient is not modified
