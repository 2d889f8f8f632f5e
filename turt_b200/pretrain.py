"""Pretraining driver: the data feed and step schedule of scripts/gpu-pretrain.ts on the fused
train step.

* Corpus: a flat uint16 token file (train.bin / val.bin of the reference's data directory,
  gpu-pretrain.ts:51-54), uploaded once to device memory.
* Batches: random contiguous windows and their next-token targets (sampleBatch,
  gpu-pretrain.ts:57-68): window i starts at floor(rng() * (len - t - 1)) with the reference's
  mulberry32 stream (training batches from mulberry32(42 + startStep), eval batch i from
  mulberry32(90000 + i)); the starts are drawn on the host and the windows gathered on the
  device (turt_sample_windows), so no token batch crosses PCIe.
* Step: zeroGrad, `accum` micro-batches whose gradients accumulate (each micro-batch's mean
  loss, gpu-pretrain.ts:203-214), then one AdamW update over all parameters with lr from the
  warmup + cosine schedule (lrAt, :182-186), betas (0.9, 0.999), eps 1e-8, weight decay 0.1 and
  bias corrections 1 - beta^t (:218-224).
* Eval every `eval_every` steps and at the end: the mean loss of 16 validation micro-batches
  (evalLoss, :188-200); the best value is tracked and the model is checkpointed in the
  reference's TURTCKPT format (:239-245), with the AdamW moments in a sidecar file so that a
  resumed run continues the same optimizer trajectory.
"""
from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass

import numpy as np

from . import checkpoint as ckpt
from ._lib import check, lib


class Mulberry32:
    """mulberry32 (src/math/random.ts:8-17): floats in [0, 1) from a uint32 state."""

    def __init__(self, seed: int):
        self.state = seed & 0xFFFFFFFF

    def __call__(self) -> float:
        self.state = (self.state + 0x6D2B79F5) & 0xFFFFFFFF
        t = self.state
        t = ((t ^ (t >> 15)) * (t | 1)) & 0xFFFFFFFF
        t ^= (t + ((t ^ (t >> 7)) * (t | 61) & 0xFFFFFFFF)) & 0xFFFFFFFF
        return ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296.0


def load_tokens(path: str) -> np.ndarray:
    """A flat little-endian uint16 token file (prepare-data output)."""
    return np.fromfile(path, dtype="<u2")


def sample_starts(n_tokens: int, b: int, t: int, rng: Mulberry32) -> np.ndarray:
    """Window starts of one sampleBatch call: floor(rng() * (n_tokens - t - 1)) per sequence."""
    span = n_tokens - t - 1
    if span <= 0:
        raise ValueError(f"corpus of {n_tokens} tokens is shorter than one window of {t + 1}")
    return np.array([math.floor(rng() * span) for _ in range(b)], dtype=np.uint64)


def sample_batch(tokens: np.ndarray, b: int, t: int, rng: Mulberry32):
    """Host version of sampleBatch: (ids, targets) as uint32[b*t]."""
    starts = sample_starts(len(tokens), b, t, rng)
    idx = starts[:, None].astype(np.int64) + np.arange(t)[None, :]
    return tokens[idx].astype(np.uint32).reshape(-1), tokens[idx + 1].astype(np.uint32).reshape(-1)


def lr_at(step: int, warmup: int, steps: int, peak_lr: float, min_lr_frac: float = 0.1) -> float:
    """Linear warmup to peak_lr, then cosine decay to min_lr_frac * peak_lr (lrAt)."""
    if step < warmup:
        return peak_lr * (step + 1) / warmup
    p = min(1.0, (step - warmup) / max(1, steps - warmup))
    return peak_lr * (min_lr_frac + (1 - min_lr_frac) * 0.5 * (1 + math.cos(math.pi * p)))


class DeviceCorpus:
    """A token corpus resident in device memory, sampled into device id / target buffers."""

    def __init__(self, ctx, tokens: np.ndarray, max_b: int, t: int):
        import torch
        self.ctx, self.n, self.t = ctx, int(len(tokens)), t
        if self.n <= t + 1:
            raise ValueError(f"corpus of {self.n} tokens is shorter than one window of {t + 1}")
        self.tokens = torch.from_numpy(np.ascontiguousarray(tokens, dtype=np.uint16).view(np.int16)).cuda()
        torch.cuda.synchronize()  # the corpus is in place before the library's stream reads it
        self.ids = torch.empty(max_b * t, dtype=torch.int32, device="cuda")
        self.tgt = torch.empty(max_b * t, dtype=torch.int32, device="cuda")
        self.max_b = max_b

    def sample(self, b: int, rng: Mulberry32):
        """Draws b windows (host RNG, reference order) and gathers them on the device; returns
        device pointers (ids, targets) valid until the next call."""
        if b > self.max_b:
            raise ValueError(f"batch {b} exceeds the corpus buffers' {self.max_b}")
        starts = sample_starts(self.n, b, self.t, rng)
        check(lib().turt_sample_windows(self.ctx.handle, self.tokens.data_ptr(), self.n,
                                        starts.ctypes.data, b, self.t, self.ids.data_ptr(), self.tgt.data_ptr()))
        return self.ids.data_ptr(), self.tgt.data_ptr()


@dataclass
class Schedule:
    steps: int = 20000
    batch: int = 16
    micro: int = 16
    warmup: int = 200
    peak_lr: float = 6e-4
    min_lr_frac: float = 0.1
    eval_every: int = 500
    eval_batches: int = 16
    betas: tuple = (0.9, 0.999)
    eps: float = 1e-8
    weight_decay: float = 0.1


class Pretrainer:
    """gpu-pretrain.ts's loop on a turt_b200 Model (see the module docstring)."""

    def __init__(self, model, train_tokens: np.ndarray, val_tokens: np.ndarray, sched: Schedule,
                 out_path: str | None = None, log=print):
        if sched.batch % sched.micro:
            raise ValueError("batch must be a multiple of micro")
        self.model, self.s, self.out, self.log = model, sched, out_path, log
        t = model.cfg.block_size
        self.t = t
        self.train = DeviceCorpus(model.ctx, train_tokens, sched.micro, t)
        self.val = DeviceCorpus(model.ctx, val_tokens, sched.micro, t)
        self.step = 0          # optimizer steps done
        self.adam_step = 0     # bias-correction count (tstep)
        self.best_val = math.inf
        self.rng = Mulberry32(42)

    def resume(self, path: str) -> dict:
        """Loads a TURTCKPT file (and its .adam sidecar when present) and continues from its step."""
        meta = ckpt.load_checkpoint(path, self.model)
        self.step = int(meta["step"])
        self.best_val = float(meta["bestValLoss"])
        self.adam_step = self.step
        side = path + ".adam"
        if os.path.exists(side):
            self.adam_step = ckpt.load_optimizer_state(side, self.model)
        self.rng = Mulberry32(42 + self.step)
        return meta

    def eval_loss(self) -> float:
        total = 0.0
        for i in range(self.s.eval_batches):
            d_ids, d_tgt = self.val.sample(self.s.micro, Mulberry32(90000 + i))
            total += self.model.forward_device(d_ids, d_tgt, self.s.micro, self.t)
        return total / self.s.eval_batches

    def train_step(self, want_loss: bool = False):
        s, m = self.s, self.model
        m.zero_grad()
        for _ in range(s.batch // s.micro):
            d_ids, d_tgt = self.train.sample(s.micro, self.rng)
            m.forward_backward_device(d_ids, d_tgt, s.micro, self.t, loss_scale=1.0)
        loss = m.read_loss() if want_loss else None
        self.adam_step += 1
        b1, b2 = s.betas
        lr = lr_at(self.step, s.warmup, s.steps, s.peak_lr, s.min_lr_frac)
        m.adamw_step(lr, b1, b2, s.eps, s.weight_decay, 1 - b1 ** self.adam_step, 1 - b2 ** self.adam_step)
        self.step += 1
        return loss

    def save(self, path: str) -> None:
        ckpt.save_checkpoint(path, self.model, self.step, self.best_val)
        ckpt.save_optimizer_state(path + ".adam", self.model, self.adam_step)

    def run(self, until: int | None = None, print_every: int = 20) -> float:
        """Trains to step `until` (default: the schedule's end); returns the best val loss."""
        end = self.s.steps if until is None else min(until, self.s.steps)
        t0, first = time.perf_counter(), self.step
        while self.step < end:
            printing = (self.step + 1) % print_every == 0
            loss = self.train_step(want_loss=printing)
            if printing:
                secs = time.perf_counter() - t0
                tps = (self.step - first) * self.s.batch * self.t / max(secs, 1e-9)
                self.log(f"step {self.step:6d}/{self.s.steps}  loss {loss:.4f}  "
                         f"lr {lr_at(self.step - 1, self.s.warmup, self.s.steps, self.s.peak_lr):.2e}  {tps:.0f} tok/s")
            if self.step % self.s.eval_every == 0 or self.step == self.s.steps:
                vl = self.eval_loss()
                self.best_val = min(self.best_val, vl)
                if self.out:
                    self.save(self.out)
                self.log(f"  eval @ {self.step}: val loss {vl:.4f} (best {self.best_val:.4f})")
        return self.best_val


def main(argv=None) -> float:
    """Command line of scripts/gpu-pretrain.ts: --data DIR (meta.json, train.bin, val.bin),
    --out / --resume (TURTCKPT paths; a resume adopts the checkpoint's config), --arch, --block,
    --layers, --heads, --embd, --batch, --micro, --steps, --lr, --warmup, --eval, --seed."""
    import argparse
    import json

    from .runtime import Context, Model, make_config
    ap = argparse.ArgumentParser(prog="python -m turt_b200.pretrain")
    ap.add_argument("--data", default="data")
    ap.add_argument("--out", default="gpt-big.bin")
    ap.add_argument("--resume", default="")
    ap.add_argument("--arch", default="modern", choices=["modern", "gpt2"])
    ap.add_argument("--block", type=int, default=256)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--embd", type=int, default=512)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--micro", type=int, default=0, help="micro-batch (default: logits chunks near 64 MB)")
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--lr", type=float, default=6e-4)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--eval", type=int, default=500)
    ap.add_argument("--seed", type=int, default=1337)
    a = ap.parse_args(argv)
    with open(os.path.join(a.data, "meta.json")) as f:
        vocab = int(json.load(f)["vocabSize"])
    cfg = dict(vocab=vocab, block=a.block, layers=a.layers, heads=a.heads, embd=a.embd, arch=a.arch)
    if a.resume:
        c = ckpt.read_checkpoint_meta(a.resume)["config"]
        cfg = dict(vocab=c["vocabSize"], block=c["blockSize"], layers=c["nLayer"], heads=c["nHead"],
                   embd=c["nEmbd"], arch=c.get("arch", "gpt2"))
    micro = a.micro or min(a.batch, max(1, (64 * 1024 * 1024 // 4 // cfg["vocab"]) // cfg["block"]))
    while a.batch % micro:
        micro -= 1
    ctx = Context(0)
    model = Model(ctx, make_config(cfg["vocab"], cfg["block"], cfg["layers"], cfg["heads"], cfg["embd"],
                                   cfg["arch"]))
    try:
        sched = Schedule(steps=a.steps, batch=a.batch, micro=micro, warmup=a.warmup, peak_lr=a.lr,
                         eval_every=a.eval)
        train = load_tokens(os.path.join(a.data, "train.bin"))
        val = load_tokens(os.path.join(a.data, "val.bin"))
        trainer = Pretrainer(model, train, val, sched, out_path=a.out)
        if a.resume:
            trainer.resume(a.resume)
            print(f"Resumed from {a.resume} at step {trainer.step} (best val {trainer.best_val:.4f})")
        else:
            model.init_reference(a.seed)
        print(f"GPU pretraining a {model.num_params() / 1e6:.2f}M-param GPT ({cfg['arch']}): "
              f"{cfg['layers']}L {cfg['heads']}H {cfg['embd']}E block {cfg['block']} vocab {cfg['vocab']}, "
              f"batch {a.batch} (micro {micro}), {a.steps} steps, peak lr {a.lr}")
        best = trainer.run()
        print(f"Done. Best val loss {best:.4f}. Saved to {a.out}")
        return best
    finally:
        model.close()
        ctx.close()


if __name__ == "__main__":
    main()
