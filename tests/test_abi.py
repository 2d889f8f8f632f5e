"""The C ABI without a GPU: the library loads and exports every symbol include/turt_cuda.h
declares, the header parses into ctypes signatures, and entry points reject bad arguments
before touching a device."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "turt_b200", "libturt_cuda.so")
HEADER = os.path.join(ROOT, "include", "turt_cuda.h")


def declared():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    return sorted(set(re.findall(r"\b(turt_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def built():
    if not os.path.exists(LIB):
        from turt_b200.build import build
        build()
    return LIB


def test_header_declares_the_boundary():
    names = declared()
    # model level, op level, host matmul and DP groups of the boundary
    for n in ["turt_init", "turt_model_create", "turt_forward_backward", "turt_adamw_step", "turt_clip_grad_norm",
              "turt_param_upload", "turt_grad_download", "turt_matmul_into", "turt_host_matmul", "turt_ce_bwd",
              "turt_rope", "turt_permute4", "turt_adamw", "turt_dp_init", "turt_dp_allreduce_grads"]:
        assert n in names


def test_library_exports_every_declared_symbol(built):
    out = subprocess.run(["nm", "-D", "--defined-only", built], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (turt_\w+)", out))
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing


def test_ctypes_signatures_cover_the_header(built):
    from turt_b200._lib import parse_header
    sigs = parse_header()
    assert sorted(sigs) == declared()
    lib = C.CDLL(built)
    for name in sigs:
        assert hasattr(lib, name)


def test_no_gpu_calls_fail_cleanly(built):
    """Without a GPU, turt_init reports an error instead of crashing; null handles are rejected."""
    from turt_b200._lib import lib
    L = lib()
    h = C.c_void_p()
    rc = L.turt_init(0, C.byref(h))
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if not has_gpu:
        assert rc != 0
        assert L.turt_last_error()
    else:
        assert rc == 0
        L.turt_ctx_destroy(h)
    assert L.turt_model_destroy(None) != 0
    assert L.turt_zero_grad(None) != 0
    assert L.turt_dp_defer(None, 1) != 0
    n = C.c_uint64()
    assert L.turt_launch_count(C.byref(n)) == 0
