"""Thin Python handles over the C ABI: a device context and a fused-step GPT model.

`Context` owns a turt_ctx (device, stream, error flags); `Model` owns a turt_model (flat
parameter / gradient / AdamW buffers in the library's internal layout) and exchanges
tensors with the host in the reference's parameters() order and [in, out] layout.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import ARCH_GPT2, ARCH_MODERN, TurtConfig, check, f32, lib, ptr, u32


class Context:
    def __init__(self, device: int = 0):
        self._h = C.c_void_p()
        check(lib().turt_init(device, C.byref(self._h)))
        self.device = device

    @property
    def handle(self):
        return self._h

    def synchronize(self) -> None:
        check(lib().turt_synchronize(self._h))

    def set_stream(self, stream_ptr: int) -> None:
        check(lib().turt_ctx_set_stream(self._h, stream_ptr))

    def set_precision(self, precision: int) -> None:
        """0 = fp32 CUDA cores (op level only), 1 = plain TF32, 3 = error-compensated 3xTF32 (default)."""
        check(lib().turt_set_precision(self._h, precision))

    @staticmethod
    def launch_count() -> int:
        n = C.c_uint64()
        check(lib().turt_launch_count(C.byref(n)))
        return n.value

    @property
    def stream(self) -> int:
        return lib().turt_ctx_stream(self._h) or 0

    # device buffers (raw pointers)
    def buffer(self, elems: int) -> int:
        p = C.c_void_p()
        check(lib().turt_buffer(self._h, elems, C.byref(p)))
        return p.value

    def index_buffer(self, data) -> int:
        a = u32(data)
        p = C.c_void_p()
        check(lib().turt_index_buffer(self._h, ptr(a), a.size, C.byref(p)))
        return p.value

    def free(self, p: int) -> None:
        check(lib().turt_free(self._h, p))

    def reclaim(self) -> None:
        check(lib().turt_reclaim(self._h))

    def upload(self, dst: int, host: np.ndarray) -> None:
        h = np.ascontiguousarray(host)
        check(lib().turt_upload(self._h, dst, ptr(h), h.nbytes))

    def download(self, src: int, n: int, dtype=np.float32) -> np.ndarray:
        out = np.empty(n, dtype=dtype)
        check(lib().turt_download(self._h, ptr(out), src, out.nbytes))
        return out

    def close(self) -> None:
        if self._h:
            lib().turt_ctx_destroy(self._h)
            self._h = C.c_void_p()


def make_config(vocab_size, block_size, n_layer, n_head, n_embd, arch="modern", hidden=0) -> TurtConfig:
    return TurtConfig(vocab_size, block_size, n_layer, n_head, n_embd,
                      ARCH_MODERN if arch == "modern" else ARCH_GPT2, hidden)


class Model:
    """Fused GPU train step for one GPT (both turt architectures)."""

    def __init__(self, ctx: Context, cfg: TurtConfig):
        self.ctx = ctx
        self.cfg = cfg
        self._h = C.c_void_p()
        check(lib().turt_model_create(ctx.handle, C.byref(cfg), C.byref(self._h)))
        n = C.c_int()
        check(lib().turt_param_count(self._h, C.byref(n)))
        self.names, self.shapes = [], []
        buf = C.create_string_buffer(64)
        shp = (C.c_int * 2)()
        nd = C.c_int()
        for i in range(n.value):
            check(lib().turt_param_info(self._h, i, buf, 64, shp, C.byref(nd)))
            self.names.append(buf.value.decode())
            self.shapes.append((shp[0], shp[1]) if nd.value == 2 else (shp[0],))

    @property
    def handle(self):
        return self._h

    ATTN_AUTO, ATTN_TENSOR, ATTN_FLASH, ATTN_TENSOR_ONLINE = 0, 1, 2, 3

    def set_attention(self, mode: int) -> None:
        """Attention implementation: ATTN_AUTO, ATTN_TENSOR (tensor-core, probabilities kept for
        the backward pass), ATTN_FLASH (fused CUDA-core online softmax) or ATTN_TENSOR_ONLINE
        (tensor-core online softmax, probabilities recomputed in the backward pass)."""
        check(lib().turt_model_set_attention(self._h, mode))

    def num_params(self) -> int:
        t = C.c_size_t()
        check(lib().turt_num_params(self._h, C.byref(t)))
        return t.value

    def sizes(self):
        return [int(np.prod(s)) for s in self.shapes]

    def load_flat(self, flat: np.ndarray) -> None:
        """Uploads a flat vector in parameters() order (scripts/params.ts layout)."""
        flat = f32(flat)
        off = 0
        for i, n in enumerate(self.sizes()):
            seg = np.ascontiguousarray(flat[off:off + n])
            check(lib().turt_param_upload(self._h, i, ptr(seg), n))
            off += n

    def _download_flat(self, fn) -> np.ndarray:
        out = np.empty(sum(self.sizes()), dtype=np.float32)
        off = 0
        for i, n in enumerate(self.sizes()):
            seg = np.empty(n, dtype=np.float32)
            check(fn(self._h, i, ptr(seg), n))
            out[off:off + n] = seg
            off += n
        return out

    def params_flat(self) -> np.ndarray:
        return self._download_flat(lib().turt_param_download)

    def init_reference(self, seed: int) -> None:
        """Weights exactly as the reference's CPU GPT(config, mulberry32(seed)) draws them."""
        check(lib().turt_model_init(self._h, seed & 0xFFFFFFFF))

    def param_list(self):
        """Every parameter, in parameters() order, as arrays of the reference's shapes."""
        out = []
        for i, shp in enumerate(self.shapes):
            a = np.empty(int(np.prod(shp)), dtype=np.float32)
            check(lib().turt_param_download(self._h, i, ptr(a), a.size))
            out.append(a.reshape(shp))
        return out

    def load_param_list(self, arrays) -> None:
        for i, (a, shp) in enumerate(zip(arrays, self.shapes)):
            a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
            if a.size != int(np.prod(shp)):
                raise ValueError(f"param {i} has {a.size} values, the model expects shape {shp}")
            check(lib().turt_param_upload(self._h, i, ptr(a), a.size))

    def adam_state(self):
        """AdamW first and second moments per parameter ([m...], [v...])."""
        ms, vs = [], []
        for i, shp in enumerate(self.shapes):
            m = np.empty(int(np.prod(shp)), dtype=np.float32)
            v = np.empty_like(m)
            check(lib().turt_adam_state_download(self._h, i, ptr(m), ptr(v), m.size))
            ms.append(m.reshape(shp))
            vs.append(v.reshape(shp))
        return ms, vs

    def load_adam_state(self, ms, vs) -> None:
        for i, (m, v) in enumerate(zip(ms, vs)):
            m = np.ascontiguousarray(m, dtype=np.float32).reshape(-1)
            v = np.ascontiguousarray(v, dtype=np.float32).reshape(-1)
            check(lib().turt_adam_state_upload(self._h, i, ptr(m), ptr(v), m.size))

    def grads_flat(self) -> np.ndarray:
        return self._download_flat(lib().turt_grad_download)

    def zero_grad(self) -> None:
        check(lib().turt_zero_grad(self._h))

    def forward_backward(self, ids, targets, b: int, t: int, loss_scale: float = 1.0, want_loss=True):
        ids, targets = u32(ids), u32(targets)
        if ids.size != b * t or targets.size != b * t:
            raise ValueError(f"expected {b * t} ids and targets")
        loss = C.c_float()
        check(lib().turt_forward_backward(self._h, ptr(ids), ptr(targets), b, t, loss_scale,
                                          C.byref(loss) if want_loss else None))
        return loss.value if want_loss else None

    def forward_backward_device(self, d_ids: int, d_targets: int, b: int, t: int, loss_scale: float = 1.0) -> None:
        """Step on ids/targets already in device memory (no host copies, no synchronization)."""
        check(lib().turt_forward_backward_device(self._h, d_ids, d_targets, b, t, loss_scale))

    def read_loss(self) -> float:
        loss = C.c_float()
        check(lib().turt_read_loss(self._h, C.byref(loss)))
        return loss.value

    def forward_device(self, d_ids: int, d_targets: int, b: int, t: int) -> float:
        """Mean loss of a forward pass on device-resident ids / targets (synchronizes)."""
        loss = C.c_float()
        check(lib().turt_forward_device(self._h, d_ids, d_targets, b, t, C.byref(loss)))
        return loss.value

    def forward(self, ids, targets, b: int, t: int) -> float:
        ids, targets = u32(ids), u32(targets)
        loss = C.c_float()
        check(lib().turt_forward(self._h, ptr(ids), ptr(targets), b, t, C.byref(loss)))
        return loss.value

    def generate_prefill(self, ids) -> np.ndarray:
        """Forward over one context of <= block_size token ids; refills the KV cache and returns
        the last position's logits (float32 [vocab])."""
        ids = u32(ids)
        out = np.empty(self.cfg.vocab_size, dtype=np.float32)
        check(lib().turt_generate_prefill(self._h, ptr(ids), len(ids), ptr(out)))
        return out

    def generate_step(self, token: int, pos: int) -> np.ndarray:
        """Appends `token` at `pos` (= the cached length) and returns its logits."""
        out = np.empty(self.cfg.vocab_size, dtype=np.float32)
        check(lib().turt_generate_step(self._h, int(token), int(pos), ptr(out)))
        return out

    def clip_grad_norm(self, max_norm: float) -> float:
        n = C.c_double()
        check(lib().turt_clip_grad_norm(self._h, max_norm, C.byref(n)))
        return n.value

    def adamw_step(self, lr, b1, b2, eps, wd, bc1, bc2, clip=0.0, grad_scale=1.0) -> None:
        check(lib().turt_adamw_step(self._h, lr, b1, b2, eps, wd, bc1, bc2, clip, grad_scale))

    # data parallel
    @staticmethod
    def dp_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        check(lib().turt_dp_unique_id(buf))
        return buf.raw

    def dp_init(self, rank: int, world: int, uid: bytes) -> None:
        check(lib().turt_dp_init(self._h, rank, world, C.create_string_buffer(uid, 128)))

    def dp_defer(self, defer: bool) -> None:
        check(lib().turt_dp_defer(self._h, 1 if defer else 0))

    def dp_wait(self, timeout_ms: int = 60000) -> None:
        check(lib().turt_dp_wait(self._h, timeout_ms))

    def dp_allreduce(self) -> None:
        check(lib().turt_dp_allreduce_grads(self._h))

    def close(self) -> None:
        if self._h:
            lib().turt_model_destroy(self._h)
            self._h = C.c_void_p()


class Group:
    """Several GPUs driven from this one process: one model replica per device, the batch split
    into contiguous shards and the gradients summed over NCCL inside the backward pass (the
    reference's in-process worker pool, scripts/train-gpt.ts:66-123,200-219)."""

    def __init__(self, devices, cfg: TurtConfig):
        devs = (C.c_int * len(devices))(*devices)
        self.cfg = cfg
        self.devices = list(devices)
        self._h = C.c_void_p()
        check(lib().turt_group_create(len(devices), devs, C.byref(cfg), C.byref(self._h)))
        rep = C.c_void_p()
        check(lib().turt_group_model(self._h, 0, C.byref(rep)))
        n = C.c_int()
        check(lib().turt_param_count(rep, C.byref(n)))
        self.names, self.shapes = [], []
        buf = C.create_string_buffer(64)
        shp = (C.c_int * 2)()
        nd = C.c_int()
        for i in range(n.value):
            check(lib().turt_param_info(rep, i, buf, 64, shp, C.byref(nd)))
            self.names.append(buf.value.decode())
            self.shapes.append((shp[0], shp[1]) if nd.value == 2 else (shp[0],))

    def sizes(self):
        return [int(np.prod(s)) for s in self.shapes]

    def replica(self, i: int) -> int:
        """turt_model handle of replica i (for per-device reads)."""
        rep = C.c_void_p()
        check(lib().turt_group_model(self._h, i, C.byref(rep)))
        return rep

    def load_flat(self, flat: np.ndarray) -> None:
        flat = f32(flat)
        off = 0
        for i, n in enumerate(self.sizes()):
            seg = np.ascontiguousarray(flat[off:off + n])
            check(lib().turt_group_param_upload(self._h, i, ptr(seg), n))
            off += n

    def _download_flat(self, fn, handle) -> np.ndarray:
        out = np.empty(sum(self.sizes()), dtype=np.float32)
        off = 0
        for i, n in enumerate(self.sizes()):
            seg = np.empty(n, dtype=np.float32)
            check(fn(handle, i, ptr(seg), n))
            out[off:off + n] = seg
            off += n
        return out

    def grads_flat(self, replica=None) -> np.ndarray:
        if replica is None:
            return self._download_flat(lib().turt_group_grad_download, self._h)
        return self._download_flat(lib().turt_grad_download, self.replica(replica))

    def params_flat(self, replica=None) -> np.ndarray:
        if replica is None:
            return self._download_flat(lib().turt_group_param_download, self._h)
        return self._download_flat(lib().turt_param_download, self.replica(replica))

    def zero_grad(self) -> None:
        check(lib().turt_group_zero_grad(self._h))

    def defer(self, defer: bool) -> None:
        check(lib().turt_group_defer(self._h, 1 if defer else 0))

    def forward_backward(self, ids, targets, b: int, t: int, loss_scale: float = 1.0, want_loss=True):
        ids, targets = u32(ids), u32(targets)
        if ids.size != b * t or targets.size != b * t:
            raise ValueError(f"expected {b * t} ids and targets")
        loss = C.c_float()
        check(lib().turt_group_forward_backward(self._h, ptr(ids), ptr(targets), b, t, loss_scale,
                                                C.byref(loss) if want_loss else None))
        return loss.value if want_loss else None

    def adamw_step(self, lr, b1, b2, eps, wd, bc1, bc2, clip=0.0) -> None:
        check(lib().turt_group_adamw_step(self._h, lr, b1, b2, eps, wd, bc1, bc2, clip))

    def synchronize(self) -> None:
        check(lib().turt_group_synchronize(self._h))

    def close(self) -> None:
        if self._h:
            lib().turt_group_destroy(self._h)
            self._h = C.c_void_p()
