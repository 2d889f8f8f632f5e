"""turt_host_matmul_noalloc: the host-array matmul for callers that cannot let the library
allocate device memory during a call (a process whose device memory is already held by another
framework's caching allocator, or a latency-bound host that must not allocate after start-up).

It must give the same product as turt_host_matmul (the allocating entry point) at every
precision the context can be set to, on two calls in a row (the fixed staging array is shared
and keeps the previous call's contents); it must accept a product that fills the fixed
2 Mi-float staging array exactly, return zeros for k = 0, reject a product that does not fit
with a clear error, and leave the library's buffer count and the device's free memory unchanged.
This file is collected last so a failure here never hides the other GPU tests.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# Normalised error bound per precision: the CUDA-core fp32 kernel and one TF32 pass run the same
# kernel as turt_host_matmul on the same staged operands; 3xTF32 as in test_gpu_gemm.py.
TOL = {0: 1e-6, 1: 2e-3, 3: 2e-5}


def _norm_err(got, ref):
    return float(np.max(np.abs(got - ref)) / max(1e-30, np.max(np.abs(ref))))


def _live(ctx):
    from turt_b200._lib import check, lib
    live, peak = C.c_int(), C.c_int()
    check(lib().turt_live_buffers(ctx.handle, C.byref(live), C.byref(peak)))
    return live.value


@pytest.mark.parametrize("precision", [3, 1, 0])
def test_noalloc_matches_host_matmul_twice(precision):
    from turt_b200._lib import check, lib, ptr
    from turt_b200.runtime import Context
    ctx = Context(0)
    try:
        ctx.set_precision(precision)
        rng = np.random.default_rng(7)
        for (m, k, n) in [(257, 160, 1024), (17, 33, 9), (64, 128, 384)]:
            a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
            b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
            want = np.empty((m, n), np.float32)
            check(lib().turt_host_matmul(ctx.handle, ptr(a), m, k, ptr(b), n, ptr(want)))
            exact = a.astype(np.float64) @ b.astype(np.float64)
            for _ in range(2):
                got = np.full((m, n), np.nan, np.float32)
                check(lib().turt_host_matmul_noalloc(ctx.handle, ptr(a), m, k, ptr(b), n, ptr(got)))
                assert _norm_err(got, want) <= TOL[precision], (m, k, n, precision)
                assert _norm_err(got, exact) <= TOL[precision], (m, k, n, precision)
    finally:
        ctx.close()


def test_noalloc_at_the_size_limit_and_k0():
    from turt_b200._lib import check, lib, ptr
    from turt_b200.runtime import Context
    ctx = Context(0)
    try:
        rng = np.random.default_rng(11)
        # 1024*1024 + 1024*512 + 1024*512 = 2 Mi floats: fills the staging array exactly.
        m, k, n = 1024, 1024, 512
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        want = np.empty((m, n), np.float32)
        check(lib().turt_host_matmul(ctx.handle, ptr(a), m, k, ptr(b), n, ptr(want)))
        got = np.full((m, n), np.nan, np.float32)
        check(lib().turt_host_matmul_noalloc(ctx.handle, ptr(a), m, k, ptr(b), n, ptr(got)))
        assert _norm_err(got, want) <= TOL[3]
        # k = 0: the product is all zeros even though the array holds the previous call's data.
        z = np.full((33, 17), np.nan, np.float32)
        ea = np.zeros((33, 0), np.float32)
        eb = np.zeros((0, 17), np.float32)
        check(lib().turt_host_matmul_noalloc(ctx.handle, ptr(ea), 33, 0, ptr(eb), 17, ptr(z)))
        assert np.all(z == 0.0)
    finally:
        ctx.close()


def test_noalloc_allocates_nothing():
    import torch
    from turt_b200._lib import check, lib, ptr
    from turt_b200.runtime import Context
    ctx = Context(0)
    try:
        rng = np.random.default_rng(5)
        m, k, n = 300, 200, 500
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        out = np.empty((m, n), np.float32)
        check(lib().turt_host_matmul_noalloc(ctx.handle, ptr(a), m, k, ptr(b), n, ptr(out)))  # warm-up
        torch.cuda.synchronize(0)
        live0 = _live(ctx)
        free0, _ = torch.cuda.mem_get_info(0)
        for _ in range(3):
            check(lib().turt_host_matmul_noalloc(ctx.handle, ptr(a), m, k, ptr(b), n, ptr(out)))
        torch.cuda.synchronize(0)
        free1, _ = torch.cuda.mem_get_info(0)
        assert _live(ctx) == live0
        assert free1 == free0
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
