"""ctypes binding of libturt_cuda.so.

Argument and return types are read from include/turt_cuda.h, so the header stays the
single description of the C ABI.  Loading fails loudly when the library is missing or
no B200 is present: there is no CPU fallback behind this module.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libturt_cuda.so")
HEADER = os.path.join(ROOT, "include", "turt_cuda.h")

OK = 0
ERR_INVALID = 1
ERR_CUDA = 2
ERR_RANGE = 3
ERR_TIMEOUT = 4
ERR_NCCL = 5
ERR_NONFINITE = 6
ERR_UNSUPPORTED = 7

ARCH_GPT2 = 0
ARCH_MODERN = 1


class TurtError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[turt {code}] {msg}")
        self.code = code


class TurtConfig(C.Structure):
    _fields_ = [("vocab_size", C.c_int), ("block_size", C.c_int), ("n_layer", C.c_int), ("n_head", C.c_int),
                ("n_embd", C.c_int), ("arch", C.c_int), ("hidden", C.c_int)]


_SCALARS = {"int": C.c_int, "size_t": C.c_size_t, "float": C.c_float, "double": C.c_double,
            "uint16_t": C.c_uint16, "uint32_t": C.c_uint32, "uint64_t": C.c_uint64}


def _ctype(decl: str):
    decl = decl.replace("const ", "").strip()
    if "*" in decl:
        return C.c_void_p
    base = decl.split()[0]
    return _SCALARS[base]


def parse_header(path: str = HEADER) -> dict:
    """Returns {name: (restype, [argtypes])} for every function declared in the header."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    sigs = {}
    for m in re.finditer(r"^\s*((?:const\s+)?[A-Za-z_][\w]*\s*\**)\s*(turt_\w+)\s*\(([^)]*)\)\s*;", text, re.M):
        ret, name, args = m.group(1).strip(), m.group(2), m.group(3).strip()
        if ret.startswith("const char") or ret.startswith("char"):
            rt = C.c_char_p
        elif "*" in ret:
            rt = C.c_void_p
        else:
            rt = _SCALARS[ret.split()[0]]
        argt = []
        if args and args != "void":
            for a in args.split(","):
                a = a.strip()
                # drop the parameter name
                mm = re.match(r"(.*?)([A-Za-z_]\w*)$", a)
                argt.append(_ctype(mm.group(1) if mm and mm.group(1).strip() else a))
        sigs[name] = (rt, argt)
    return sigs


_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library with every header-declared function typed."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise TurtError(ERR_CUDA, f"{LIB_PATH} is not built (run __graft_entry__.build())")
            L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
            for name, (rt, at) in parse_header().items():
                fn = getattr(L, name)
                fn.restype = rt
                fn.argtypes = at
            _lib = L
    return _lib


def last_error() -> str:
    s = lib().turt_last_error()
    return s.decode() if s else ""


def check(rc: int) -> None:
    if rc != OK:
        raise TurtError(rc, last_error())


def ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32)
