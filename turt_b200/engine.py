"""Mirror of the reference's GPU engine interfaces over libturt_cuda.so.

The names, argument order and semantics follow turt's TypeScript classes so code written
against them ports line for line:

* ``GpuEngine`` -- src/infer/webgpu/autograd.ts:542-815: device buffers (raw device
  pointers here), deferred free + reclaim, and one method per kernel wrapper
  (``matmulInto``, ``ewise``, ... ``adamw``), each a call into the C ABI.
* ``GpuTensor`` -- autograd.ts:817-1210: a tape of GPU ops whose backward closures
  *accumulate* into ``ensureGrad()`` buffers, replayed in reverse topological order.
* ``GpuGPT`` -- src/models/gpu-gpt.ts:54-202: both architectures built from ``GpuTensor`` ops
  (``fused=False``, the reference's op-by-op graph) or backed by the library's fused train
  step (``fused=True``: one call for forward + backward, same parameters() order and values).
* ``GpuCompute`` / ``CudaBackend`` -- src/infer/webgpu/gpu.ts:59-141 and
  src/infer/backend.ts:11-16: host-array matmul.

Errors raise ``TurtError`` (the reference throws ``Error``); shape mismatches raise
``ValueError`` with the reference's messages.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from ._lib import TurtError, check, f32, lib, ptr, u32
from .runtime import Context, Model, make_config


class GpuEngine:
    """Device context + kernel wrappers (autograd.ts:542-815)."""

    def __init__(self, ctx: Context):
        self.ctx = ctx
        self.h = ctx.handle
        self.L = lib()
        self.sizes = {}

    @staticmethod
    def create(device: int = 0) -> "GpuEngine":
        return GpuEngine(Context(device))

    # ------------------------------------------------------------ buffers
    @property
    def liveBuffers(self) -> int:
        live, peak = C.c_int(), C.c_int()
        check(self.L.turt_live_buffers(self.h, C.byref(live), C.byref(peak)))
        return live.value

    @property
    def peakLiveBuffers(self) -> int:
        live, peak = C.c_int(), C.c_int()
        check(self.L.turt_live_buffers(self.h, C.byref(live), C.byref(peak)))
        return peak.value

    def buffer(self, elems: int) -> int:
        p = self.ctx.buffer(max(1, int(elems)))
        self.sizes[p] = int(elems)
        return p

    def indexBuffer(self, data) -> int:
        a = u32(data)
        p = self.ctx.index_buffer(a)
        self.sizes[p] = a.size
        return p

    def free(self, buf: int) -> None:
        if buf:
            self.ctx.free(buf)
            self.sizes.pop(buf, None)

    def reclaim(self) -> None:
        self.ctx.reclaim()

    def read(self, buf: int, elems: int) -> np.ndarray:
        return self.ctx.download(buf, int(elems))

    def fill(self, buf: int, value: float, elems: int) -> None:
        check(self.L.turt_fill(self.h, buf, value, int(elems)))

    def write(self, buf: int, data) -> None:
        self.ctx.upload(buf, f32(data))

    def tensor(self, data, shape, requiresGrad: bool = False) -> "GpuTensor":
        d = f32(data).ravel()
        buf = self.buffer(d.size)
        self.ctx.upload(buf, d)
        return GpuTensor(self, buf, list(shape), requiresGrad)

    def zeros(self, shape, requiresGrad: bool = False) -> "GpuTensor":
        return GpuTensor(self, self.buffer(int(np.prod(shape))), list(shape), requiresGrad)

    # ------------------------------------------------------------ kernels
    def matmulInto(self, a, b, out, M, K, N, batch, transA, transB, accum):
        check(self.L.turt_matmul_into(self.h, a, b, out, M, K, N, batch, int(transA), int(transB), int(accum)))

    def ewise(self, a, b, out, n, bLen, op, accum):
        check(self.L.turt_ewise(self.h, a, b, out, n, bLen, op, int(accum)))

    def scale(self, a, out, n, s, accum):
        check(self.L.turt_scale(self.h, a, out, n, s, int(accum)))

    def bcastAcc(self, src, out, n, bLen, s):
        check(self.L.turt_bcast_acc(self.h, src, out, n, bLen, s))

    def segsum(self, g, out, n, bLen, s, accum):
        check(self.L.turt_segsum(self.h, g, out, n, bLen, s, int(accum)))

    def total(self, a, out, n):
        check(self.L.turt_total(self.h, a, out, n))

    def reluInto(self, x, out, n):
        check(self.L.turt_relu(self.h, x, out, n))

    def reluBwd(self, x, gOut, gIn, n):
        check(self.L.turt_relu_bwd(self.h, x, gOut, gIn, n))

    def sgd(self, grad, param, n, lr):
        check(self.L.turt_sgd(self.h, grad, param, n, lr))

    def geluInto(self, x, out, n):
        check(self.L.turt_gelu(self.h, x, out, n))

    def geluBwd(self, x, gOut, gIn, n):
        check(self.L.turt_gelu_bwd(self.h, x, gOut, gIn, n))

    def siluInto(self, x, out, n):
        check(self.L.turt_silu(self.h, x, out, n))

    def siluBwd(self, x, gOut, gIn, n):
        check(self.L.turt_silu_bwd(self.h, x, gOut, gIn, n))

    def rmsFwd(self, x, gamma, out, rstd, rows, d, eps):
        check(self.L.turt_rms_fwd(self.h, x, gamma, out, rstd, rows, d, eps))

    def rmsDx(self, x, gOut, gamma, rstd, gIn, rows, d, eps):
        check(self.L.turt_rms_dx(self.h, x, gOut, gamma, rstd, gIn, rows, d, eps))

    def rmsDg(self, x, gOut, rstd, dgamma, rows, d):
        check(self.L.turt_rms_dg(self.h, x, gOut, rstd, dgamma, rows, d))

    def ropeInto(self, x, out, groups, t, hd, base):
        check(self.L.turt_rope(self.h, x, out, groups, t, hd, base))

    def ropeBwd(self, gOut, gIn, groups, t, hd, base):
        check(self.L.turt_rope_bwd(self.h, gOut, gIn, groups, t, hd, base))

    def softmaxInto(self, x, out, rows, d):
        check(self.L.turt_softmax(self.h, x, out, rows, d))

    def softmaxBwd(self, y, gOut, gIn, rows, d):
        check(self.L.turt_softmax_bwd(self.h, y, gOut, gIn, rows, d))

    def lnFwd(self, x, gamma, beta, out, mean, rstd, rows, d, eps):
        check(self.L.turt_ln_fwd(self.h, x, gamma, beta, out, mean, rstd, rows, d, eps))

    def lnDx(self, x, gOut, gamma, mean, rstd, gIn, rows, d, eps):
        check(self.L.turt_ln_dx(self.h, x, gOut, gamma, mean, rstd, gIn, rows, d, eps))

    def lnDgb(self, x, gOut, mean, rstd, dgamma, dbeta, rows, d):
        check(self.L.turt_ln_dgb(self.h, x, gOut, mean, rstd, dgamma, dbeta, rows, d))

    def gatherInto(self, table, idx, out, n, d, vocab=None):
        vocab = self.sizes.get(table, 0) // d if vocab is None else vocab
        check(self.L.turt_gather(self.h, table, idx, out, n, d, vocab))

    def gatherBwd(self, idx, gOut, dTable, n, d, vocab):
        check(self.L.turt_gather_bwd(self.h, idx, gOut, dTable, n, d, vocab))

    def ceFwd(self, logits, targets, perRow, rows, vocab):
        check(self.L.turt_ce_fwd(self.h, logits, targets, perRow, rows, vocab))

    def ceBwd(self, logits, targets, gLoss, dLogits, rows, vocab):
        check(self.L.turt_ce_bwd(self.h, logits, targets, gLoss, dLogits, rows, vocab))

    def maskInto(self, x, out, groups, t):
        check(self.L.turt_mask(self.h, x, out, groups, t))

    def maskBwd(self, gOut, gIn, groups, t):
        check(self.L.turt_mask_bwd(self.h, gOut, gIn, groups, t))

    def permute4(self, inp, out, inShape, perm, n, accum):
        s = (C.c_int * 4)(*[int(v) for v in inShape])
        p = (C.c_int * 4)(*[int(v) for v in perm])
        check(self.L.turt_permute4(self.h, inp, out, s, p, n, int(accum)))

    def adamw(self, grad, param, m, v, n, lr, b1, b2, eps, wd, bc1, bc2):
        check(self.L.turt_adamw(self.h, grad, param, m, v, n, lr, b1, b2, eps, wd, bc1, bc2))


class GpuTensor:
    """GPU-resident autograd tensor (autograd.ts:817-1210)."""

    def __init__(self, engine: GpuEngine, buffer: int, shape, requiresGrad: bool = False):
        self.engine = engine
        self.buffer = buffer
        self.shape = list(shape)
        self.requiresGrad = requiresGrad
        self.grad = None
        self.ctx = None  # (parents, backward closure, scratch buffers)

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    @property
    def ndim(self) -> int:
        return len(self.shape)

    def ensureGrad(self) -> int:
        if self.grad is None:
            self.grad = self.engine.buffer(self.size)
        return self.grad

    def zeroGrad(self) -> None:
        if self.grad is not None:
            self.engine.free(self.grad)
        self.grad = None

    def freeGraph(self) -> None:
        stack, seen = [self], set()
        while stack:
            t = stack.pop()
            if id(t) in seen or t.ctx is None:
                continue
            seen.add(id(t))
            parents, _, scratch = t.ctx
            stack.extend(parents)
            for b in scratch:
                self.engine.free(b)
            t.ctx = None
            self.engine.free(t.buffer)
            if t.grad is not None:
                self.engine.free(t.grad)
                t.grad = None

    def _out(self, buffer, shape, parents, backward, scratch=()) -> "GpuTensor":
        t = GpuTensor(self.engine, buffer, shape, any(p.requiresGrad for p in parents))
        if t.requiresGrad:
            t.ctx = (parents, lambda: backward(t), list(scratch))
        return t

    def read(self) -> np.ndarray:
        return self.engine.read(self.buffer, self.size).reshape(self.shape)

    # ------------------------------------------------------------------ ops
    def matmul(self, b: "GpuTensor") -> "GpuTensor":
        M, K = self.shape
        K2, N = b.shape
        if K != K2:
            raise ValueError(f"matmul shape mismatch: [{self.shape}] @ [{b.shape}]")
        e, a = self.engine, self
        out = e.buffer(M * N)
        e.matmulInto(a.buffer, b.buffer, out, M, K, N, 1, False, False, False)

        def bwd(t):
            if a.requiresGrad:
                e.matmulInto(t.grad, b.buffer, a.ensureGrad(), M, N, K, 1, False, True, True)
            if b.requiresGrad:
                e.matmulInto(a.buffer, t.grad, b.ensureGrad(), K, M, N, 1, True, False, True)
        return self._out(out, [M, N], [a, b], bwd)

    def _binary(self, b: "GpuTensor", op: int) -> "GpuTensor":
        e, a = self.engine, self
        n, bLen = a.size, b.size
        out = e.buffer(n)
        e.ewise(a.buffer, b.buffer, out, n, bLen, op, False)

        def bwd(t):
            g = t.grad
            if a.requiresGrad:
                if op == 2:
                    e.ewise(g, b.buffer, a.ensureGrad(), n, bLen, 2, True)
                else:
                    e.scale(g, a.ensureGrad(), n, 1, True)
            if b.requiresGrad:
                if op == 2:
                    if bLen == n:
                        e.ewise(g, a.buffer, b.ensureGrad(), n, n, 2, True)
                    else:
                        tmp = e.buffer(n)
                        e.ewise(g, a.buffer, tmp, n, n, 2, False)
                        e.segsum(tmp, b.ensureGrad(), n, bLen, 1, True)
                        e.free(tmp)
                else:
                    e.segsum(g, b.ensureGrad(), n, bLen, -1 if op == 1 else 1, True)
        return self._out(out, list(a.shape), [a, b], bwd)

    def add(self, b):
        return self._binary(b, 0)

    def sub(self, b):
        return self._binary(b, 1)

    def mul(self, b):
        return self._binary(b, 2)

    def scale(self, s: float) -> "GpuTensor":
        e, a, n = self.engine, self, self.size
        out = e.buffer(n)
        e.scale(a.buffer, out, n, s, False)

        def bwd(t):
            if a.requiresGrad:
                e.scale(t.grad, a.ensureGrad(), n, s, True)
        return self._out(out, list(a.shape), [a], bwd)

    def relu(self) -> "GpuTensor":
        e, a, n = self.engine, self, self.size
        out = e.buffer(n)
        e.reluInto(a.buffer, out, n)

        def bwd(t):
            if a.requiresGrad:
                e.reluBwd(a.buffer, t.grad, a.ensureGrad(), n)
        return self._out(out, list(a.shape), [a], bwd)

    def sum(self) -> "GpuTensor":
        e, a, n = self.engine, self, self.size
        out = e.buffer(1)
        e.total(a.buffer, out, n)

        def bwd(t):
            if a.requiresGrad:
                e.bcastAcc(t.grad, a.ensureGrad(), n, 1, 1)
        return self._out(out, [1], [a], bwd)

    def mean(self) -> "GpuTensor":
        return self.sum().scale(1 / self.size)

    def bmm(self, b: "GpuTensor") -> "GpuTensor":
        G, M, K = self.shape
        G2, K2, N = b.shape
        if G != G2 or K != K2:
            raise ValueError(f"bmm shape mismatch: [{self.shape}] @ [{b.shape}]")
        e, a = self.engine, self
        out = e.buffer(G * M * N)
        e.matmulInto(a.buffer, b.buffer, out, M, K, N, G, False, False, False)

        def bwd(t):
            if a.requiresGrad:
                e.matmulInto(t.grad, b.buffer, a.ensureGrad(), M, N, K, G, False, True, True)
            if b.requiresGrad:
                e.matmulInto(a.buffer, t.grad, b.ensureGrad(), K, M, N, G, True, False, True)
        return self._out(out, [G, M, N], [a, b], bwd)

    def bmmBT(self, k: "GpuTensor") -> "GpuTensor":
        G, M, K = self.shape
        G2, N, K2 = k.shape
        if G != G2 or K != K2:
            raise ValueError(f"bmmBT shape mismatch: [{self.shape}] @ [{k.shape}]^T")
        e, a = self.engine, self
        out = e.buffer(G * M * N)
        e.matmulInto(a.buffer, k.buffer, out, M, K, N, G, False, True, False)

        def bwd(t):
            if a.requiresGrad:
                e.matmulInto(t.grad, k.buffer, a.ensureGrad(), M, N, K, G, False, False, True)
            if k.requiresGrad:
                e.matmulInto(t.grad, a.buffer, k.ensureGrad(), N, M, K, G, True, False, True)
        return self._out(out, [G, M, N], [a, k], bwd)

    def matmulBT(self, b: "GpuTensor") -> "GpuTensor":
        Nr, D = self.shape
        V, D2 = b.shape
        if D != D2:
            raise ValueError(f"matmulBT shape mismatch: [{self.shape}] @ [{b.shape}]^T")
        e, a = self.engine, self
        out = e.buffer(Nr * V)
        e.matmulInto(a.buffer, b.buffer, out, Nr, D, V, 1, False, True, False)

        def bwd(t):
            if a.requiresGrad:
                e.matmulInto(t.grad, b.buffer, a.ensureGrad(), Nr, V, D, 1, False, False, True)
            if b.requiresGrad:
                e.matmulInto(t.grad, a.buffer, b.ensureGrad(), V, Nr, D, 1, True, False, True)
        return self._out(out, [Nr, V], [a, b], bwd)

    def reshape(self, shape) -> "GpuTensor":
        e, a = self.engine, self
        t = GpuTensor(e, a.buffer, list(shape), a.requiresGrad)
        if a.requiresGrad:
            t.ctx = ([a], lambda: e.scale(t.grad, a.ensureGrad(), a.size, 1, True), [])
        return t

    def gelu(self) -> "GpuTensor":
        e, a, n = self.engine, self, self.size
        out = e.buffer(n)
        e.geluInto(a.buffer, out, n)

        def bwd(t):
            if a.requiresGrad:
                e.geluBwd(a.buffer, t.grad, a.ensureGrad(), n)
        return self._out(out, list(a.shape), [a], bwd)

    def silu(self) -> "GpuTensor":
        e, a, n = self.engine, self, self.size
        out = e.buffer(n)
        e.siluInto(a.buffer, out, n)

        def bwd(t):
            if a.requiresGrad:
                e.siluBwd(a.buffer, t.grad, a.ensureGrad(), n)
        return self._out(out, list(a.shape), [a], bwd)

    def rmsNorm(self, gamma: "GpuTensor", eps: float = 1e-5) -> "GpuTensor":
        e, a = self.engine, self
        d = a.shape[-1]
        rows = a.size // d
        out = e.buffer(a.size)
        rstd = e.buffer(rows)
        e.rmsFwd(a.buffer, gamma.buffer, out, rstd, rows, d, eps)

        def bwd(t):
            if a.requiresGrad:
                e.rmsDx(a.buffer, t.grad, gamma.buffer, rstd, a.ensureGrad(), rows, d, eps)
            if gamma.requiresGrad:
                e.rmsDg(a.buffer, t.grad, rstd, gamma.ensureGrad(), rows, d)
        t = self._out(out, list(a.shape), [a, gamma], bwd, [rstd])
        if t.ctx is None:
            e.free(rstd)
        return t

    def rope(self, base: float = 10000.0) -> "GpuTensor":
        if self.ndim != 3:
            raise ValueError(f"rope expects a [groups, time, headDim] tensor, got {self.ndim}-D")
        groups, tt, hd = self.shape
        if hd % 2:
            raise ValueError(f"rope requires an even headDim, got {hd}")
        e, a = self.engine, self
        out = e.buffer(a.size)
        e.ropeInto(a.buffer, out, groups, tt, hd, base)

        def bwd(t):
            if a.requiresGrad:
                e.ropeBwd(t.grad, a.ensureGrad(), groups, tt, hd, base)
        return self._out(out, list(a.shape), [a], bwd)

    def softmax(self) -> "GpuTensor":
        e, a = self.engine, self
        d = a.shape[-1]
        rows = a.size // d
        out = e.buffer(a.size)
        e.softmaxInto(a.buffer, out, rows, d)

        def bwd(t):
            if a.requiresGrad:
                e.softmaxBwd(out, t.grad, a.ensureGrad(), rows, d)
        return self._out(out, list(a.shape), [a], bwd)

    def maskedFillCausal(self) -> "GpuTensor":
        e, a = self.engine, self
        t2 = a.shape[-1]
        groups = a.size // (t2 * t2)
        out = e.buffer(a.size)
        e.maskInto(a.buffer, out, groups, t2)

        def bwd(t):
            if a.requiresGrad:
                e.maskBwd(t.grad, a.ensureGrad(), groups, t2)
        return self._out(out, list(a.shape), [a], bwd)

    def permute(self, perm) -> "GpuTensor":
        if self.ndim != 4:
            raise ValueError("GpuTensor.permute currently supports 4-D tensors")
        e, a = self.engine, self
        in_shape = list(a.shape)
        out_shape = [in_shape[p] for p in perm]
        n = a.size
        out = e.buffer(n)
        e.permute4(a.buffer, out, in_shape, perm, n, False)

        def bwd(t):
            if a.requiresGrad:
                e.permute4(t.grad, a.ensureGrad(), in_shape, perm, n, True)
        return self._out(out, out_shape, [a], bwd)

    def layerNorm(self, gamma: "GpuTensor", beta: "GpuTensor", eps: float = 1e-5) -> "GpuTensor":
        e, a = self.engine, self
        d = a.shape[-1]
        rows = a.size // d
        out = e.buffer(a.size)
        mean, rstd = e.buffer(rows), e.buffer(rows)
        e.lnFwd(a.buffer, gamma.buffer, beta.buffer, out, mean, rstd, rows, d, eps)

        def bwd(t):
            if a.requiresGrad:
                e.lnDx(a.buffer, t.grad, gamma.buffer, mean, rstd, a.ensureGrad(), rows, d, eps)
            if gamma.requiresGrad:
                e.lnDgb(a.buffer, t.grad, mean, rstd, gamma.ensureGrad(), beta.ensureGrad(), rows, d)
        t = self._out(out, list(a.shape), [a, gamma, beta], bwd, [mean, rstd])
        if t.ctx is None:
            e.free(mean)
            e.free(rstd)
        return t

    def gatherRows(self, indices) -> "GpuTensor":
        e, a = self.engine, self
        vocab, d = a.shape
        idx = u32(indices)
        n = idx.size
        idx_buf = e.indexBuffer(idx)
        out = e.buffer(n * d)
        e.gatherInto(a.buffer, idx_buf, out, n, d, vocab)

        def bwd(t):
            if a.requiresGrad:
                e.gatherBwd(idx_buf, t.grad, a.ensureGrad(), n, d, vocab)
        t = self._out(out, [n, d], [a], bwd, [idx_buf])
        if t.ctx is None:
            e.free(idx_buf)
        return t

    def crossEntropyLogits(self, targets) -> "GpuTensor":
        e, a = self.engine, self
        rows, vocab = a.shape
        tgt = u32(targets)
        if tgt.size != rows:
            raise ValueError(f"Expected {rows} targets, got {tgt.size}")
        tgt_buf = e.indexBuffer(tgt)
        per_row = e.buffer(rows)
        e.ceFwd(a.buffer, tgt_buf, per_row, rows, vocab)
        sum_buf = e.buffer(1)
        e.total(per_row, sum_buf, rows)
        loss_buf = e.buffer(1)
        e.scale(sum_buf, loss_buf, 1, 1 / rows, False)
        e.free(per_row)
        e.free(sum_buf)

        def bwd(t):
            if a.requiresGrad:
                e.ceBwd(a.buffer, tgt_buf, t.grad, a.ensureGrad(), rows, vocab)
        t = self._out(loss_buf, [1], [a], bwd, [tgt_buf])
        if t.ctx is None:
            e.free(tgt_buf)
        return t

    def backward(self) -> None:
        if self.size != 1:
            raise ValueError("backward() requires a scalar")
        topo, seen = [], set()
        stack = [(self, False)]
        while stack:  # iterative post-order (same order as the recursive visit)
            t, expanded = stack.pop()
            if expanded:
                topo.append(t)
                continue
            if id(t) in seen:
                continue
            seen.add(id(t))
            stack.append((t, True))
            if t.ctx is not None:
                for p in reversed(t.ctx[0]):
                    if id(p) not in seen:
                        stack.append((p, False))
        self.engine.fill(self.ensureGrad(), 1, 1)
        for t in reversed(topo):
            if t.ctx is not None:
                t.ctx[1]()


class GpuGPT:
    """GPT on the GPU (src/models/gpu-gpt.ts:54-202), both architectures.

    fused=False builds the reference's op-by-op tape from GpuTensor ops; fused=True keeps
    the parameters in the library's fused model (one call per forward+backward, gradients
    accumulated exactly like the tape's ensureGrad buffers)."""

    def __init__(self, engine: GpuEngine, config: dict, skipInit: bool = False, fused: bool = False, seed=1):
        self.engine = engine
        self.config = dict(config)
        V, T, E, L, H = (config["vocabSize"], config["blockSize"], config["nEmbd"], config["nLayer"],
                         config["nHead"])
        if E % H:
            raise ValueError("nEmbd must be divisible by nHead")
        self.modern = config.get("arch", "gpt2") == "modern"
        self.headScale = 1 / math.sqrt(E / H)
        self.hidden = config.get("hidden") or (4 * E if not self.modern else max(64, round(8 * E / 3 / 64) * 64))
        self.fused = fused
        self._model = None
        if fused:
            self._model = Model(engine.ctx, make_config(V, T, L, H, E, "modern" if self.modern else "gpt2",
                                                        self.hidden))
            self.names, self.shapes = self._model.names, self._model.shapes
            if not skipInit:
                self._model.load_flat(self._init_flat(seed))
            return
        rng = np.random.default_rng(seed)
        res = 0.02 / math.sqrt(2 * L)

        def param(shape, std):
            data = np.zeros(int(np.prod(shape)), np.float32) if skipInit else rng.standard_normal(
                int(np.prod(shape))).astype(np.float32) * std
            return engine.tensor(data, shape, True)

        def const(shape, v):
            return engine.tensor(np.full(int(np.prod(shape)), v, np.float32), shape, True)
        h = self.hidden
        self.wte = param([V, E], 0.02)
        self.wpe = None if self.modern else param([T, E], 0.02)
        self.blocks = []
        for _ in range(L):
            blk = {"ln1g": const([E], 1), "qW": param([E, E], 0.02), "kW": param([E, E], 0.02),
                   "vW": param([E, E], 0.02), "projW": param([E, E], res), "ln2g": const([E], 1)}
            if self.modern:
                blk.update(gateW=param([E, h], 0.02), upW=param([E, h], 0.02), downW=param([h, E], res))
            else:
                blk.update(ln1b=const([E], 0), qb=const([E], 0), kb=const([E], 0), vb=const([E], 0),
                           projb=const([E], 0), ln2b=const([E], 0), fcW=param([E, h], 0.02), fcb=const([h], 0),
                           mpW=param([h, E], res), mpb=const([E], 0))
            self.blocks.append(blk)
        self.lnfg = const([E], 1)
        self.lnfb = None if self.modern else const([E], 0)

    def _init_flat(self, seed):
        rng = np.random.default_rng(seed)
        res = 0.02 / math.sqrt(2 * self.config["nLayer"])
        parts = []
        for name, shp in zip(self.names, self.shapes):
            n = int(np.prod(shp))
            base = name.split(".")[-1]
            if len(shp) == 1:
                parts.append(np.ones(n, np.float32) if base.endswith("g") else np.zeros(n, np.float32))
            else:
                parts.append((rng.standard_normal(n) * (res if base in ("projW", "downW", "mpW") else 0.02)).astype(
                    np.float32))
        return np.concatenate(parts)

    # parameters() order, gpu-gpt.ts:118-132
    def parameters(self):
        if self.fused:
            raise TypeError("fused GpuGPT keeps parameters in the library: use loadFlat / paramsFlat / gradsFlat")
        ps = [self.wte]
        if self.wpe is not None:
            ps.append(self.wpe)
        keys = (["ln1g", "qW", "kW", "vW", "projW", "ln2g", "gateW", "upW", "downW"] if self.modern else
                ["ln1g", "ln1b", "qW", "qb", "kW", "kb", "vW", "vb", "projW", "projb", "ln2g", "ln2b", "fcW", "fcb",
                 "mpW", "mpb"])
        for b in self.blocks:
            ps.extend(b[k] for k in keys)
        ps.append(self.lnfg)
        if self.lnfb is not None:
            ps.append(self.lnfb)
        return ps

    def numParams(self) -> int:
        if self.fused:
            return self._model.num_params()
        return sum(p.size for p in self.parameters())

    def loadFlat(self, flat) -> None:
        if self.fused:
            self._model.load_flat(flat)
            return
        off = 0
        for p in self.parameters():
            self.engine.write(p.buffer, flat[off:off + p.size])
            off += p.size

    def paramsFlat(self) -> np.ndarray:
        if self.fused:
            return self._model.params_flat()
        return np.concatenate([self.engine.read(p.buffer, p.size) for p in self.parameters()])

    def gradsFlat(self) -> np.ndarray:
        if self.fused:
            return self._model.grads_flat()
        return np.concatenate([self.engine.read(p.grad, p.size) if p.grad is not None else np.zeros(p.size, np.float32)
                               for p in self.parameters()])

    def zeroGrad(self) -> None:
        if self.fused:
            self._model.zero_grad()
        else:
            for p in self.parameters():
                p.zeroGrad()

    def _norm(self, x, g, b=None):
        return x.rmsNorm(g) if self.modern else x.layerNorm(g, b)

    def _attention(self, xln, blk, b, t):
        E, H = self.config["nEmbd"], self.config["nHead"]
        hd = E // H

        def split(p):
            return p.reshape([b, t, H, hd]).permute([0, 2, 1, 3]).reshape([b * H, t, hd])

        def lin(w, bias=None):
            y = xln.matmul(w)
            return y.add(bias) if bias is not None else y
        q = split(lin(blk["qW"], blk.get("qb")))
        k = split(lin(blk["kW"], blk.get("kb")))
        v = split(lin(blk["vW"], blk.get("vb")))
        if self.modern:
            q = q.rope()
            k = k.rope()
        scores = q.bmmBT(k).scale(self.headScale).maskedFillCausal().softmax()
        att = scores.bmm(v).reshape([b, H, t, hd]).permute([0, 2, 1, 3]).reshape([b * t, E])
        out = att.matmul(blk["projW"])
        return out.add(blk["projb"]) if "projb" in blk else out

    def _mlp(self, hln, blk):
        if self.modern:
            return hln.matmul(blk["gateW"]).silu().mul(hln.matmul(blk["upW"])).matmul(blk["downW"])
        return hln.matmul(blk["fcW"]).add(blk["fcb"]).gelu().matmul(blk["mpW"]).add(blk["mpb"])

    def loss(self, tokenIds, targets, b: int, t: int):
        """Forward pass returning the scalar loss (gpu-gpt.ts:185-201).

        fused=True runs forward and backward in one library call and returns the loss value
        (a float); the gradients are already accumulated, as after the tape's backward()."""
        if t > self.config["blockSize"]:
            raise ValueError(f"Sequence length {t} exceeds block size {self.config['blockSize']}")
        if self.fused:
            return self._model.forward_backward(tokenIds, targets, b, t)
        x = self.wte.gatherRows(tokenIds)
        if self.wpe is not None:
            x = x.add(self.wpe.gatherRows(np.arange(b * t, dtype=np.uint32) % t))
        for blk in self.blocks:
            h = x.add(self._attention(self._norm(x, blk["ln1g"], blk.get("ln1b")), blk, b, t))
            x = h.add(self._mlp(self._norm(h, blk["ln2g"], blk.get("ln2b")), blk))
        xf = self._norm(x, self.lnfg, self.lnfb)
        return xf.matmulBT(self.wte).crossEntropyLogits(targets)


class AdamW:
    """AdamW (src/optim/adam.ts:16-61) over GpuTensor parameters or a fused GpuGPT, with
    optional global-norm clipping (src/optim/clip.ts:7-24) folded into the update."""

    def __init__(self, model: GpuGPT, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weightDecay=0.01, clip=0.0):
        self.model, self.lr, self.beta1, self.beta2 = model, lr, beta1, beta2
        self.eps, self.weightDecay, self.clip, self.t = eps, weightDecay, clip, 0
        self._mv = None

    def step(self, grad_scale: float = 1.0) -> None:
        self.t += 1
        bc1 = 1 - self.beta1 ** self.t
        bc2 = 1 - self.beta2 ** self.t
        if self.model.fused:
            self.model._model.adamw_step(self.lr, self.beta1, self.beta2, self.eps, self.weightDecay, bc1, bc2,
                                         clip=self.clip, grad_scale=grad_scale)
            return
        e = self.model.engine
        ps = self.model.parameters()
        if self._mv is None:
            self._mv = [(e.buffer(p.size), e.buffer(p.size)) for p in ps]
        if self.clip > 0:
            g = np.concatenate([e.read(p.ensureGrad(), p.size) for p in ps]).astype(np.float64)
            norm = float(np.sqrt((g * g).sum()))
            if norm > self.clip:
                for p in ps:
                    e.scale(p.grad, p.grad, p.size, self.clip / norm, False)
        for p, (m, v) in zip(ps, self._mv):
            e.adamw(p.ensureGrad(), p.buffer, m, v, p.size, self.lr, self.beta1, self.beta2, self.eps,
                    self.weightDecay, bc1, bc2)


class GpuCompute:
    """Host-array matmul (src/infer/webgpu/gpu.ts:59-141).

    Defaults to FP32 CUDA-core arithmetic (precision 0), what the reference's WGSL matmul
    computes, so results meet scripts/gpu-bench.ts's check (5e-3 with a 1e-4 floor); pass
    precision=3 for the 3xTF32 tensor-core path."""

    def __init__(self, ctx: Context, precision: int = 0):
        self.ctx = ctx
        ctx.set_precision(precision)

    @staticmethod
    def create(device: int = 0, precision: int = 0) -> "GpuCompute":
        return GpuCompute(Context(device), precision)

    def matmul(self, a, m: int, k: int, b, n: int) -> np.ndarray:
        return self.bmm(a, 1, m, k, b, n)

    def bmm(self, a, batch: int, m: int, k: int, b, n: int) -> np.ndarray:
        a, b = f32(a).ravel(), f32(b).ravel()
        if a.size != batch * m * k:
            raise ValueError(f"A has {a.size} elems, expected {batch * m * k}")
        if b.size != batch * k * n:
            raise ValueError(f"B has {b.size} elems, expected {batch * k * n}")
        out = np.empty(batch * m * n, np.float32)
        check(lib().turt_host_bmm(self.ctx.handle, ptr(a), batch, m, k, ptr(b), n, ptr(out)))
        return out


class CudaBackend:
    """Backend (src/infer/backend.ts:11-16): name, isAvailable(), matmul(a, b) on 2-D arrays."""

    name = "cuda-b200"

    def __init__(self, device: int = 0):
        self.compute = GpuCompute.create(device)

    @staticmethod
    def available() -> bool:
        try:
            c = Context(0)
            c.close()
            return True
        except TurtError:
            return False

    def isAvailable(self) -> bool:
        return self.compute is not None

    def matmul(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        if a.ndim != 2 or b.ndim != 2:
            raise ValueError(f"CudaBackend.matmul requires 2-D tensors, got {a.ndim}-D and {b.ndim}-D")
        m, k = a.shape
        k2, n = b.shape
        if k != k2:
            raise ValueError(f"matmul shape mismatch: [{list(a.shape)}] @ [{list(b.shape)}]")
        return self.compute.matmul(a, m, k, b, n).reshape(m, n)
