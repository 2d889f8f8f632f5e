"""ctypes wrapper for the C oracle (oracle/turt_oracle.c).

TEST INFRASTRUCTURE ONLY: the oracle is the checker for the CUDA library and the
timed CPU baseline.  Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference legs use this module; the product path never does.

Two builds of the same source exist: ``f32`` (faithful: f32 storage with the
reference's JavaScript-double intermediates, src/math/tensor.ts) and ``f64``
(all double; used for central-difference gradient checks only).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
SRC = os.path.join(HERE, "turt_oracle.c")

ARCH_GPT2 = 0
ARCH_MODERN = 1


def build(force: bool = False) -> None:
    """Compile both oracle variants with gcc into oracle/_build/."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    for name, extra in (("libturt_oracle.so", ["-O3", "-mavx2", "-mfma"]),
                        ("libturt_oracle64.so", ["-O3", "-mavx2", "-mfma", "-DORACLE_F64"])):
        out = os.path.join(BUILD_DIR, name)
        if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(SRC):
            continue
        cmd = ["gcc", *extra, "-fPIC", "-shared", "-fvisibility=hidden", "-o", out, SRC, "-lm", "-lpthread"]
        subprocess.run(cmd, check=True)


def _f(a):
    return a.ctypes.data_as(C.c_void_p)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


class Oracle:
    """Numpy-facing handle on one oracle build."""

    def __init__(self, f64: bool = False):
        name = "libturt_oracle64.so" if f64 else "libturt_oracle.so"
        path = os.path.join(BUILD_DIR, name)
        if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(SRC):
            build()
        self.lib = C.CDLL(path)
        self.dt = np.float64 if f64 else np.float32
        L = self.lib
        vp, i, d, sz = C.c_void_p, C.c_int, C.c_double, C.c_size_t
        L.oc_rng_next.restype = d
        L.oc_rng_next.argtypes = [vp]
        L.oc_gaussian.restype = d
        L.oc_gaussian.argtypes = [vp]
        L.oc_randn.argtypes = [vp, sz, vp, d]
        L.oc_mm_fwd.argtypes = [vp, vp, vp, i, i, i]
        L.oc_mm_bwd_a.argtypes = [vp, vp, vp, i, i, i]
        L.oc_mm_bwd_b.argtypes = [vp, vp, vp, i, i, i]
        L.oc_bmm_fwd.argtypes = [vp, vp, vp, i, i, i, i]
        L.oc_bmm_bwd.argtypes = [vp, vp, vp, vp, vp, i, i, i, i]
        L.oc_softmax_fwd.argtypes = [vp, vp, i, i]
        L.oc_softmax_bwd.argtypes = [vp, vp, vp, i, i]
        L.oc_mask_fwd.argtypes = [vp, vp, i, i]
        L.oc_mask_bwd.argtypes = [vp, vp, i, i]
        L.oc_gelu_fwd.argtypes = [vp, vp, sz]
        L.oc_gelu_bwd.argtypes = [vp, vp, vp, sz]
        L.oc_silu_fwd.argtypes = [vp, vp, sz]
        L.oc_silu_bwd.argtypes = [vp, vp, vp, vp, sz]
        L.oc_rope_fwd.argtypes = [vp, vp, i, i, i, d]
        L.oc_rope_bwd.argtypes = [vp, vp, i, i, i, d]
        L.oc_gather_fwd.restype = i
        L.oc_gather_fwd.argtypes = [vp, vp, vp, i, i, i]
        L.oc_gather_bwd.argtypes = [vp, vp, vp, i, i]
        L.oc_ce_fwd.restype = d
        L.oc_ce_fwd.argtypes = [vp, vp, vp, i, i, vp]
        L.oc_ce_bwd.argtypes = [vp, vp, d, vp, i, i]
        L.oc_permute_fwd.argtypes = [vp, vp, vp, vp, i]
        L.oc_permute_bwd.argtypes = [vp, vp, vp, vp, i]
        L.oc_rmsnorm.argtypes = [vp, vp, vp, vp, vp, vp, i, i, d]
        L.oc_layernorm.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i, i, d]
        L.oc_hidden.restype = i
        L.oc_hidden.argtypes = [vp]
        L.oc_num_params.restype = sz
        L.oc_num_params.argtypes = [vp]
        L.oc_param_shapes.restype = i
        L.oc_param_shapes.argtypes = [vp, vp]
        L.oc_init.argtypes = [vp, C.c_uint32, vp]
        L.oc_init_state.argtypes = [vp, vp, vp]
        L.oc_loss_grad.restype = d
        L.oc_loss_grad.argtypes = [vp, vp, vp, vp, vp, i, i, vp]
        L.oc_logits.restype = i
        L.oc_logits.argtypes = [vp, vp, vp, i, i, vp]
        L.oc_generate.restype = i
        L.oc_generate.argtypes = [vp, vp, vp, i, i, d, i, vp, vp]
        L.oc_clip.restype = d
        L.oc_clip.argtypes = [vp, sz, d]
        L.oc_adamw.argtypes = [vp, vp, vp, vp, sz, d, d, d, d, d, i]
        L.oc_adamw_bc.argtypes = [vp, vp, vp, vp, sz, d, d, d, d, d, d, d]
        L.oc_dp_grads.restype = d
        L.oc_dp_grads.argtypes = [vp, vp, vp, vp, vp, i, i, i, vp]
        L.oc_dp_step.restype = d
        L.oc_dp_step.argtypes = [vp, vp, vp, vp, vp, i, vp, vp, i, i, i, d, d, d, d, d, d, vp, vp]

    # ------------------------------------------------------------- helpers
    def arr(self, x):
        return np.ascontiguousarray(x, dtype=self.dt)

    def zeros(self, *shape):
        return np.zeros(shape, dtype=self.dt)

    # ----------------------------------------------------------------- RNG
    @staticmethod
    def rng(seed: int) -> np.ndarray:
        """A mulberry32 state cell (src/math/random.ts:8-17)."""
        return np.array([seed & 0xFFFFFFFF], dtype=np.uint32)

    def rng_next(self, state) -> float:
        return self.lib.oc_rng_next(_f(state))

    def randn(self, n: int, seed: int, std: float = 1.0) -> np.ndarray:
        """randn(n, seed, std) as in scripts/gpu-ops-validate.ts:17-22."""
        st = self.rng(seed)
        out = np.empty(n, dtype=self.dt)
        self.lib.oc_randn(_f(out), n, _f(st), std)
        return out

    def uniform_ints(self, n: int, seed: int, hi: int, state=None) -> np.ndarray:
        """floor(rng() * hi) draws (scripts/gpu-gpt-validate.ts:61-63)."""
        st = self.rng(seed) if state is None else state
        return np.array([int(self.lib.oc_rng_next(_f(st)) * hi) for _ in range(n)], dtype=np.int32)

    # --------------------------------------------------------------- ops
    def matmul(self, a, b):
        a, b = self.arr(a), self.arr(b)
        M, K = a.shape
        N = b.shape[1]
        y = self.zeros(M, N)
        self.lib.oc_mm_fwd(_f(a), _f(b), _f(y), M, K, N)
        return y

    def matmul_bwd(self, a, b, g):
        a, b, g = self.arr(a), self.arr(b), self.arr(g)
        M, K = a.shape
        N = b.shape[1]
        da, db = self.zeros(M, K), self.zeros(K, N)
        self.lib.oc_mm_bwd_a(_f(g), _f(b), _f(da), M, K, N)
        self.lib.oc_mm_bwd_b(_f(a), _f(g), _f(db), M, K, N)
        return da, db

    def bmm(self, a, b):
        a, b = self.arr(a), self.arr(b)
        G, M, K = a.shape
        N = b.shape[2]
        y = self.zeros(G, M, N)
        self.lib.oc_bmm_fwd(_f(a), _f(b), _f(y), G, M, K, N)
        return y

    def bmm_bwd(self, a, b, g):
        a, b, g = self.arr(a), self.arr(b), self.arr(g)
        G, M, K = a.shape
        N = b.shape[2]
        da, db = self.zeros(G, M, K), self.zeros(G, K, N)
        self.lib.oc_bmm_bwd(_f(a), _f(b), _f(g), _f(da), _f(db), G, M, K, N)
        return da, db

    def softmax(self, x):
        x = self.arr(x)
        d = x.shape[-1]
        y = np.empty_like(x)
        self.lib.oc_softmax_fwd(_f(x), _f(y), x.size // d, d)
        return y

    def softmax_bwd(self, y, g):
        y, g = self.arr(y), self.arr(g)
        d = y.shape[-1]
        gx = np.zeros_like(y)
        self.lib.oc_softmax_bwd(_f(y), _f(g), _f(gx), y.size // d, d)
        return gx

    def mask(self, x):
        x = self.arr(x)
        t = x.shape[-1]
        y = np.empty_like(x)
        self.lib.oc_mask_fwd(_f(x), _f(y), x.size // (t * t), t)
        return y

    def mask_bwd(self, g):
        g = self.arr(g)
        t = g.shape[-1]
        gx = np.zeros_like(g)
        self.lib.oc_mask_bwd(_f(g), _f(gx), g.size // (t * t), t)
        return gx

    def gelu(self, x):
        x = self.arr(x)
        y = np.empty_like(x)
        self.lib.oc_gelu_fwd(_f(x), _f(y), x.size)
        return y

    def gelu_bwd(self, x, g):
        x, g = self.arr(x), self.arr(g)
        gx = np.zeros_like(x)
        self.lib.oc_gelu_bwd(_f(x), _f(g), _f(gx), x.size)
        return gx

    def silu(self, x):
        x = self.arr(x)
        y = np.empty_like(x)
        self.lib.oc_silu_fwd(_f(x), _f(y), x.size)
        return y

    def silu_bwd(self, x, g):
        x, g = self.arr(x), self.arr(g)
        y = self.silu(x)
        gx = np.zeros_like(x)
        self.lib.oc_silu_bwd(_f(x), _f(y), _f(g), _f(gx), x.size)
        return gx

    def rope(self, x, base: float = 10000.0):
        x = self.arr(x)
        G, T, hd = x.shape
        if hd % 2:
            raise ValueError(f"rope requires an even headDim, got {hd}")
        y = np.empty_like(x)
        self.lib.oc_rope_fwd(_f(x), _f(y), G, T, hd, base)
        return y

    def rope_bwd(self, g, base: float = 10000.0):
        g = self.arr(g)
        G, T, hd = g.shape
        gx = np.zeros_like(g)
        self.lib.oc_rope_bwd(_f(g), _f(gx), G, T, hd, base)
        return gx

    def gather(self, table, idx):
        table = self.arr(table)
        idx = _i32(idx)
        V, D = table.shape
        out = self.zeros(len(idx), D)
        if self.lib.oc_gather_fwd(_f(table), _f(idx), _f(out), len(idx), V, D) != 0:
            raise IndexError("gatherRows index out of range")
        return out

    def gather_bwd(self, idx, g, vocab):
        idx, g = _i32(idx), self.arr(g)
        D = g.shape[1]
        gt = self.zeros(vocab, D)
        self.lib.oc_gather_bwd(_f(idx), _f(g), _f(gt), len(idx), D)
        return gt

    def cross_entropy(self, logits, tgt):
        """Returns (loss, dlogits) for loss = mean CE (tensor.ts:708-745)."""
        logits, tgt = self.arr(logits), _i32(tgt)
        n, V = logits.shape
        probs = np.empty_like(logits)
        err = np.zeros(1, dtype=np.int32)
        loss = self.lib.oc_ce_fwd(_f(logits), _f(tgt), _f(probs), n, V, _f(err))
        if err[0]:
            raise IndexError("target out of range")
        g = np.zeros_like(logits)
        self.lib.oc_ce_bwd(_f(probs), _f(tgt), 1.0, _f(g), n, V)
        return loss, g

    def permute(self, x, perm):
        x = self.arr(x)
        shape = np.array(x.shape, dtype=np.int32)
        p = np.array(perm, dtype=np.int32)
        y = np.empty(tuple(x.shape[q] for q in perm), dtype=self.dt)
        self.lib.oc_permute_fwd(_f(x), _f(y), _f(shape), _f(p), x.ndim)
        return y

    def permute_bwd(self, g, in_shape, perm):
        g = self.arr(g)
        shape = np.array(in_shape, dtype=np.int32)
        p = np.array(perm, dtype=np.int32)
        gx = np.zeros(in_shape, dtype=self.dt)
        self.lib.oc_permute_bwd(_f(g), _f(gx), _f(shape), _f(p), len(in_shape))
        return gx

    def rmsnorm(self, x, gamma, gy=None, eps=1e-5):
        x, gamma = self.arr(x), self.arr(gamma)
        d = x.shape[-1]
        rows = x.size // d
        y = np.empty_like(x)
        dx = np.zeros_like(x)
        dg = np.zeros_like(gamma)
        gyp = None if gy is None else self.arr(gy)
        self.lib.oc_rmsnorm(_f(x), _f(gamma), _f(y), None if gyp is None else _f(gyp), _f(dx), _f(dg),
                            rows, d, eps)
        return (y, dx, dg) if gy is not None else y

    def layernorm(self, x, gamma, beta, gy=None, eps=1e-5):
        x, gamma, beta = self.arr(x), self.arr(gamma), self.arr(beta)
        d = x.shape[-1]
        rows = x.size // d
        y = np.empty_like(x)
        dx, dg, db = np.zeros_like(x), np.zeros_like(gamma), np.zeros_like(beta)
        gyp = None if gy is None else self.arr(gy)
        self.lib.oc_layernorm(_f(x), _f(gamma), _f(beta), _f(y), None if gyp is None else _f(gyp), _f(dx),
                              _f(dg), _f(db), rows, d, eps)
        return (y, dx, dg, db) if gy is not None else y

    # ------------------------------------------------------------- model
    @staticmethod
    def cfg(vocab, block, n_layer, n_head, n_embd, arch="modern", hidden=0) -> np.ndarray:
        a = ARCH_MODERN if arch == "modern" else ARCH_GPT2
        return np.array([vocab, block, n_layer, n_head, n_embd, a, hidden], dtype=np.int32)

    def hidden(self, cfg) -> int:
        return self.lib.oc_hidden(_f(cfg))

    def num_params(self, cfg) -> int:
        return self.lib.oc_num_params(_f(cfg))

    def param_shapes(self, cfg):
        buf = np.zeros(2 * 4096, dtype=np.int32)
        n = self.lib.oc_param_shapes(_f(cfg), _f(buf))
        out = []
        for k in range(n):
            r, c = int(buf[2 * k]), int(buf[2 * k + 1])
            out.append((r, c) if c else (r,))
        return out

    def init(self, cfg, seed: int) -> np.ndarray:
        p = np.zeros(self.num_params(cfg), dtype=self.dt)
        self.lib.oc_init(_f(cfg), seed, _f(p))
        return p

    def init_state(self, cfg, state) -> np.ndarray:
        """GPT init drawing from (and advancing) a mulberry32 state cell."""
        p = np.zeros(self.num_params(cfg), dtype=self.dt)
        self.lib.oc_init_state(_f(cfg), _f(state), _f(p))
        return p

    def split(self, cfg, flat):
        """Split a flat parameter/gradient vector into per-tensor views (parameters() order)."""
        out, off = [], 0
        for shp in self.param_shapes(cfg):
            n = int(np.prod(shp))
            out.append(flat[off:off + n].reshape(shp))
            off += n
        return out

    def loss_grad(self, cfg, params, ids, tgt, b, t, grads=True):
        params = self.arr(params)
        ids, tgt = _i32(ids), _i32(tgt)
        g = np.zeros_like(params) if grads else None
        err = np.zeros(1, dtype=np.int32)
        loss = self.lib.oc_loss_grad(_f(cfg), _f(params), None if g is None else _f(g), _f(ids), _f(tgt), b, t,
                                     _f(err))
        if err[0]:
            raise ValueError(f"oracle forward rejected its input (code {err[0]})")
        return (loss, g) if grads else loss

    def logits(self, cfg, params, ids, b, t):
        params, ids = self.arr(params), _i32(ids)
        out = np.zeros((b * t, int(cfg[0])), dtype=self.dt)
        if self.lib.oc_logits(_f(cfg), _f(params), _f(ids), b, t, _f(out)):
            raise ValueError("oracle forward rejected its input")
        return out

    def generate(self, cfg, params, prompt, max_new, temperature=1.0, topk=0, rng_state=None):
        params = self.arr(params)
        prompt = _i32(prompt)
        st = rng_state if rng_state is not None else self.rng(42)
        out = np.zeros(len(prompt) + max_new, dtype=np.int32)
        n = self.lib.oc_generate(_f(cfg), _f(params), _f(prompt), len(prompt), max_new, temperature, topk,
                                 _f(st), _f(out))
        return out[:n].tolist()

    def clip(self, grads, max_norm):
        return self.lib.oc_clip(_f(grads), grads.size, max_norm)

    def adamw(self, p, g, m, v, lr, b1, b2, eps, wd, t):
        self.lib.oc_adamw(_f(p), _f(g), _f(m), _f(v), p.size, lr, b1, b2, eps, wd, t)

    def adamw_bc(self, p, g, m, v, lr, b1, b2, eps, wd, bc1, bc2):
        self.lib.oc_adamw_bc(_f(p), _f(g), _f(m), _f(v), p.size, lr, b1, b2, eps, wd, bc1, bc2)

    def dp_grads(self, cfg, params, ids, tgt, batch, t, workers):
        params = self.arr(params)
        ids, tgt = _i32(ids), _i32(tgt)
        g = np.zeros_like(params)
        err = np.zeros(1, dtype=np.int32)
        loss = self.lib.oc_dp_grads(_f(cfg), _f(params), _f(g), _f(ids), _f(tgt), batch, t, workers, _f(err))
        if err[0]:
            raise ValueError("oracle forward rejected its input")
        return loss, g

    def dp_step(self, cfg, params, m, v, step, ids, tgt, batch, t, workers, lr, b1, b2, eps, wd, clip):
        """One reference CPU data-parallel step (scripts/train-gpt.ts:234-242); updates params, m, v."""
        ids, tgt = _i32(ids), _i32(tgt)
        g = np.zeros_like(params)
        norm = np.zeros(1, dtype=np.float64)
        err = np.zeros(1, dtype=np.int32)
        loss = self.lib.oc_dp_step(_f(cfg), _f(params), _f(g), _f(m), _f(v), step, _f(ids), _f(tgt), batch, t,
                                   workers, lr, b1, b2, eps, wd, clip, _f(norm), _f(err))
        if err[0]:
            raise ValueError("oracle forward rejected its input")
        return loss, float(norm[0])


def max_rel_err(a, b) -> float:
    """maxRelErr of scripts/gpu-gpt-validate.ts:19-26 (denominator floor 1e-3)."""
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    if a.size == 0:
        return 0.0
    denom = np.maximum(1e-3, np.maximum(np.abs(a), np.abs(b)))
    return float(np.max(np.abs(a - b) / denom))
