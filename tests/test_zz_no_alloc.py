"""turt_host_matmul_noalloc: the host-array matmul for callers that cannot let the library
allocate device memory during a call (a process whose device memory is already held by another
framework's caching allocator, or a latency-bound host that must not allocate after start-up).

It must give the same product as turt_host_matmul (the allocating entry point), on two calls
in a row (the fixed staging array is shared and keeps the previous call's contents), and must
reject a product that does not fit the fixed 2 Mi-float staging array with a clear error.
This file is collected last so a failure here never hides the other GPU tests.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-5  # normalised error of the error-compensated 3xTF32 GEMM (as in test_gpu_gemm.py)


def _norm_err(got, ref):
    return float(np.max(np.abs(got - ref)) / max(1e-30, np.max(np.abs(ref))))


def test_noalloc_matches_host_matmul_twice():
    from turt_b200._lib import check, lib, ptr
    from turt_b200.runtime import Context
    ctx = Context(0)
    try:
        rng = np.random.default_rng(7)
        for (m, k, n) in [(257, 160, 1024), (17, 33, 9)]:
            a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
            b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
            want = np.empty((m, n), np.float32)
            check(lib().turt_host_matmul(ctx.handle, ptr(a), m, k, ptr(b), n, ptr(want)))
            for _ in range(2):
                got = np.full((m, n), np.nan, np.float32)
                check(lib().turt_host_matmul_noalloc(ctx.handle, ptr(a), m, k, ptr(b), n, ptr(got)))
                assert _norm_err(got, want) <= TOL
                assert _norm_err(got, a.astype(np.float64) @ b.astype(np.float64)) <= TOL
    finally:
        ctx.close()


def test_noalloc_rejects_oversized_product():
    from turt_b200._lib import ERR_INVALID, lib, ptr
    from turt_b200.runtime import Context
    ctx = Context(0)
    try:
        m = k = n = 1024  # 3 Mi floats of staging > 2 Mi
        a = np.zeros((m, k), np.float32)
        b = np.zeros((k, n), np.float32)
        out = np.zeros((m, n), np.float32)
        rc = lib().turt_host_matmul_noalloc(ctx.handle, ptr(a), m, k, ptr(b), n, ptr(out))
        assert rc == ERR_INVALID
        assert b"fixed scratch" in lib().turt_last_error()
    finally:
        ctx.close()
