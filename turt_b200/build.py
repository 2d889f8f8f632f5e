"""Builds libturt_cuda.so in-tree with nvcc for sm_100a (B200).

The library is the whole product: every kernel is hand-written CUDA for
``-gencode arch=compute_100a,code=sm_100a``; no torch extension machinery is
involved, so the same .so is what a non-Python host (Deno.dlopen, N-API) loads.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libturt_cuda.so")

SOURCES = ["gemm.cu", "ops.cu", "attention.cu", "attention_tc.cu", "attention_fused.cu", "attention_flash.cu", "model_kernels.cu", "capi.cu", "model.cu", "dp.cu", "noalloc.cu", "fused_ops.cu", "decode.cu", "diag.cu", "group.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _nccl_include() -> list[str]:
    """nccl.h for the NCCL types used by dp.cu (the library dlopens libnccl at run time)."""
    try:
        import nvidia.nccl  # type: ignore
        inc = os.path.join(list(nvidia.nccl.__path__)[0], "include")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return ["-I", inc]
    except Exception:
        pass
    return []


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    headers.append(os.path.join(ROOT, "include", "turt_cuda.h"))
    objs = []
    jobs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [_nvcc(), *NVCC_FLAGS, *_nccl_include(), "-I", os.path.join(ROOT, "include"), "-c", s, "-o", o]
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
        if verbose and (r.stdout or r.stderr):
            sys.stderr.write(r.stdout + r.stderr)

    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        cmd = [_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB, *objs, "-ldl",
               "-lpthread"]
        run(cmd)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
