"""TF32 tensor-core GEMM (tcgen05) against a float64 reference, through the C ABI.

Covers every operand layout the train step uses (K-major / MN-major A and B), batching,
accumulate, tile residues (M, N, K not multiples of the tile), the host-array entry point
(GpuCompute.matmul, scripts/gpu-bench.ts cases incl. [17,33,9]) and the CUDA-core path.
Tolerances (normalised error max|C - C_ref| / max|C_ref|): plain TF32 keeps 10 mantissa
bits per operand -> 4e-3; error-compensated 3xTF32 -> 2e-5 (fp32 accumulation level).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = {1: 4e-3, 3: 2e-5}


def _tol(prec, K):
    """3xTF32 products are fp32-exact to ~2^-21; what remains is the tensor core's fp32
    accumulation, whose error grows with the length of one output's K chain (5.4e-5 measured
    at K = 8192 in one chain), so the bound scales with K beyond 1024."""
    return TOL[prec] * (max(1.0, K / 1024) if prec == 3 else 1.0)


@pytest.fixture(scope="module")
def ctx():
    from turt_b200.runtime import Context
    c = Context(0)
    yield c
    c.close()


def _norm_err(got, ref):
    return float(np.max(np.abs(got - ref)) / max(1e-30, np.max(np.abs(ref))))


@pytest.mark.parametrize("M,K,N", [(128, 32, 128), (256, 384, 384), (200, 96, 72), (1024, 384, 1152),
                                   (16, 32, 96), (384, 1000, 128), (8192, 384, 64)])
@pytest.mark.parametrize("transA,transB", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("prec", [1, 3])
def test_matmul_into_layouts(ctx, M, K, N, transA, transB, prec):
    from turt_b200._lib import check, lib
    check(lib().turt_set_precision(ctx.handle, prec))
    rng = np.random.default_rng(M * 7 + K * 3 + N + transA * 2 + transB)
    a = rng.uniform(-1, 1, (K, M) if transA else (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (N, K) if transB else (K, N)).astype(np.float32)
    ref = (a.T if transA else a).astype(np.float64) @ (b.T if transB else b).astype(np.float64)
    da, db, dc = ctx.buffer(a.size), ctx.buffer(b.size), ctx.buffer(M * N)
    ctx.upload(da, a)
    ctx.upload(db, b)
    check(lib().turt_matmul_into(ctx.handle, da, db, dc, M, K, N, 1, transA, transB, 0))
    got = ctx.download(dc, M * N).reshape(M, N)
    assert _norm_err(got, ref) < TOL[prec]
    # accumulate into the existing output
    check(lib().turt_matmul_into(ctx.handle, da, db, dc, M, K, N, 1, transA, transB, 1))
    got2 = ctx.download(dc, M * N).reshape(M, N)
    assert _norm_err(got2, 2 * ref) < TOL[prec]
    check(lib().turt_set_precision(ctx.handle, 3))
    for p in (da, db, dc):
        ctx.free(p)
    ctx.reclaim()


@pytest.mark.parametrize("prec", [1, 3])
def test_matmul_batched(ctx, prec):
    from turt_b200._lib import check, lib
    check(lib().turt_set_precision(ctx.handle, prec))
    G, M, K, N = 12, 64, 64, 64
    rng = np.random.default_rng(1)
    a = rng.standard_normal((G, M, K)).astype(np.float32)
    b = rng.standard_normal((G, N, K)).astype(np.float32)  # transB
    ref = np.einsum("gmk,gnk->gmn", a.astype(np.float64), b.astype(np.float64))
    da, db, dc = ctx.buffer(a.size), ctx.buffer(b.size), ctx.buffer(G * M * N)
    ctx.upload(da, a)
    ctx.upload(db, b)
    check(lib().turt_matmul_into(ctx.handle, da, db, dc, M, K, N, G, 0, 1, 0))
    got = ctx.download(dc, G * M * N).reshape(G, M, N)
    assert _norm_err(got, ref) < TOL[prec]
    check(lib().turt_set_precision(ctx.handle, 3))


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (16, 16, 16), (17, 33, 9), (64, 128, 384), (256, 160, 1024)])
def test_host_matmul(ctx, m, k, n):
    """scripts/gpu-bench.ts:67-84 correctness cases through the host-array entry point."""
    from turt_b200._lib import check, lib, ptr
    rng = np.random.default_rng(m * 7 + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    out = np.empty((m, n), dtype=np.float32)
    check(lib().turt_host_matmul(ctx.handle, ptr(a), m, k, ptr(b), n, ptr(out)))
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert _norm_err(out, ref) < TOL[3]


def test_simt_fallback_odd_pitch(ctx):
    """Pitches that are not multiples of 16 bytes take the fp32 CUDA-core kernel."""
    from turt_b200._lib import check, lib
    M, K, N = 17, 33, 9
    rng = np.random.default_rng(3)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    da, db, dc = ctx.buffer(a.size), ctx.buffer(b.size), ctx.buffer(M * N)
    ctx.upload(da, a)
    ctx.upload(db, b)
    check(lib().turt_matmul_into(ctx.handle, da, db, dc, M, K, N, 1, 0, 0, 0))
    got = ctx.download(dc, M * N).reshape(M, N)
    np.testing.assert_allclose(got, a.astype(np.float64) @ b, rtol=1e-5, atol=1e-5)


@pytest.fixture
def tile():
    """Forces the GEMM tile width for one test and restores automatic selection after it."""
    from turt_b200._lib import check, lib
    yield lambda bn, pair=-1: check(lib().turt_gemm_set_tile(bn, pair))
    check(lib().turt_gemm_set_tile(0, -1))


KERNELS = [pytest.param(1, 0, id="tf32-single"), pytest.param(3, 0, id="x3-single"),
           pytest.param(3, 1, id="x3-pair"), pytest.param(3, 2, id="x3-dual")]


@pytest.mark.parametrize("bn", [64, 128, 192, 256])
@pytest.mark.parametrize("M,K,N", [(1000, 200, 520), (2048, 384, 1152), (384, 8192, 384), (130, 72, 100)])
@pytest.mark.parametrize("transA,transB", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("prec,pair", KERNELS)
def test_tile_widths(ctx, tile, bn, M, K, N, transA, transB, prec, pair):
    """Every tile width on every layout and kernel (single CTA, CTA pair): ragged edges
    (a pair tile whose second CTA holds only rows beyond M), several work units per
    persistent CTA (both TMEM accumulator buffers, ring phases wrapping), and split-K
    (K 8192 output 384^2, single-CTA kernel)."""
    from turt_b200._lib import check, lib
    if pair == 2 and bn > 128:
        pytest.skip("two CTAs per SM exist for tile widths 64 and 128")
    tile(bn, pair)
    check(lib().turt_set_precision(ctx.handle, prec))
    rng = np.random.default_rng(bn + M + K + N + 10 * transA + transB + prec + 7 * pair)
    a = rng.uniform(-1, 1, (K, M) if transA else (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (N, K) if transB else (K, N)).astype(np.float32)
    ref = (a.T if transA else a).astype(np.float64) @ (b.T if transB else b).astype(np.float64)
    da, db, dc = ctx.buffer(a.size), ctx.buffer(b.size), ctx.buffer(M * N)
    try:
        ctx.upload(da, a)
        ctx.upload(db, b)
        check(lib().turt_matmul_into(ctx.handle, da, db, dc, M, K, N, 1, transA, transB, 0))
        assert _norm_err(ctx.download(dc, M * N).reshape(M, N), ref) < _tol(prec, K)
        check(lib().turt_matmul_into(ctx.handle, da, db, dc, M, K, N, 1, transA, transB, 1))
        assert _norm_err(ctx.download(dc, M * N).reshape(M, N), 2 * ref) < _tol(prec, K)
    finally:
        check(lib().turt_set_precision(ctx.handle, 3))
        for p in (da, db, dc):
            ctx.free(p)
        ctx.reclaim()
