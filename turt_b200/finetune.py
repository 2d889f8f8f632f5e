"""Fine-tuning a pretrained checkpoint on the GPU: scripts/finetune-chat.ts on the fused step.

The reference loads a TURTCKPT base model (its config, arch included, comes from the file),
copies it into the GPU model and trains on a second token corpus with the same GpuGPT step
(finetune-chat.ts:75-158).  Its schedule differs from pretraining and is kept here:

* one batch of 16 windows of blockSize per step, drawn by sampleBatch from one mulberry32(7)
  stream (:43-54, :97); no micro-batches and no gradient clip;
* AdamW beta 0.9 / 0.999, eps 1e-8, weight decay 0.05, bias corrections from a step count
  starting at 1 (:127-132); LR warmup of 100 steps then cosine to 10 % (:103-107);
* every 500 steps and at the end: eval loss over 8 validation batches drawn with
  mulberry32(1000 + i) (:109-118), then a TURTCKPT checkpoint whose bestValLoss slot holds that
  eval loss (:143-145), then a 24-token sample (temperature 0.7, top-k 40) drawn with the
  training rng (:146-148).  The sample therefore consumes 24 draws of the batch stream; when no
  prompt is given the same 24 draws are still taken, so the batches after a checkpoint are the
  reference's.  The reference encodes the prompt "User: Hello!\\nTurt:" with its BPE tokenizer,
  which is not on this path: pass the encoded ids.
"""
from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass
from typing import List, Optional

import numpy as np

from . import checkpoint as ckpt
from .generate import generate
from .pretrain import DeviceCorpus, Mulberry32, load_tokens, lr_at


@dataclass
class FinetuneSchedule:
    steps: int = 3000
    batch: int = 16
    warmup: int = 100
    peak_lr: float = 2e-4
    min_lr_frac: float = 0.1
    betas: tuple = (0.9, 0.999)
    eps: float = 1e-8
    weight_decay: float = 0.05
    eval_every: int = 500
    eval_batches: int = 8
    log_every: int = 100
    sample_tokens: int = 24
    sample_temperature: float = 0.7
    sample_top_k: int = 40


class Finetuner:
    """finetune-chat.ts's loop on a turt_b200 Model already holding the base weights."""

    def __init__(self, model, train_tokens: np.ndarray, val_tokens: np.ndarray, sched: FinetuneSchedule,
                 out_path: Optional[str] = None, sample_prompt: Optional[List[int]] = None, log=print):
        self.model, self.s, self.out, self.log = model, sched, out_path, log
        self.t = model.cfg.block_size
        self.train = DeviceCorpus(model.ctx, train_tokens, sched.batch, self.t)
        self.val = DeviceCorpus(model.ctx, val_tokens, sched.batch, self.t)
        self.rng = Mulberry32(7)
        self.step = 0
        self.tstep = 0
        self.sample_prompt = list(sample_prompt) if sample_prompt else None
        self.samples: List[List[int]] = []

    def eval_loss(self) -> float:
        total = 0.0
        for i in range(self.s.eval_batches):
            d_ids, d_tgt = self.val.sample(self.s.batch, Mulberry32(1000 + i))
            total += self.model.forward_device(d_ids, d_tgt, self.s.batch, self.t)
        return total / self.s.eval_batches

    def train_step(self, want_loss: bool = False):
        s, m = self.s, self.model
        m.zero_grad()
        d_ids, d_tgt = self.train.sample(s.batch, self.rng)
        m.forward_backward_device(d_ids, d_tgt, s.batch, self.t, loss_scale=1.0)
        self.tstep += 1
        lr = lr_at(self.step, s.warmup, s.steps, s.peak_lr, s.min_lr_frac)
        b1, b2 = s.betas
        m.adamw_step(lr, b1, b2, s.eps, s.weight_decay, 1 - b1 ** self.tstep, 1 - b2 ** self.tstep)
        self.step += 1
        return m.read_loss() if want_loss else None

    def sample(self) -> Optional[List[int]]:
        """The periodic sample continuation; takes sample_tokens draws of the training rng."""
        s = self.s
        if self.sample_prompt is None:
            for _ in range(s.sample_tokens):
                self.rng()
            return None
        out = generate(self.model, self.sample_prompt, s.sample_tokens, temperature=s.sample_temperature,
                       top_k=s.sample_top_k, rng=self.rng)
        self.samples.append(out)
        return out

    def run(self) -> float:
        """Runs the whole schedule; returns the last eval loss."""
        s = self.s
        t0 = time.perf_counter()
        vl = math.nan
        while self.step < s.steps:
            printing = (self.step + 1) % s.log_every == 0
            loss = self.train_step(want_loss=printing)
            if printing:
                tps = self.step * s.batch * self.t / max(time.perf_counter() - t0, 1e-9)
                lr = lr_at(self.step - 1, s.warmup, s.steps, s.peak_lr, s.min_lr_frac)
                self.log(f"step {self.step}/{s.steps}  loss {loss:.4f}  lr {lr:.2e}  {tps:.0f} tok/s")
            if self.step % s.eval_every == 0 or self.step == s.steps:
                vl = self.eval_loss()
                if self.out:
                    ckpt.save_checkpoint(self.out, self.model, self.step, vl)
                gen = self.sample()
                self.log(f"  eval val loss {vl:.4f}" + (f" — saved {self.out}" if self.out else ""))
                if gen is not None:
                    self.log(f"  sample ids: {gen[len(self.sample_prompt):]}")
        return vl


def main(argv=None) -> float:
    """Command line of scripts/finetune-chat.ts: --steps, --lr, --base, --out (names under
    --ckpt-dir), the chat corpus chat-train.bin / chat-val.bin under --data, and --sample-ids
    (comma-separated prompt ids for the periodic sample)."""
    import argparse

    from .runtime import Context, Model, make_config
    ap = argparse.ArgumentParser(prog="python -m turt_b200.finetune")
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--lr", type=float, default=2e-4)
    ap.add_argument("--base", default="gpt.bin")
    ap.add_argument("--out", default="chat.bin")
    ap.add_argument("--data", default="data")
    ap.add_argument("--ckpt-dir", default="checkpoints")
    ap.add_argument("--sample-ids", default="")
    a = ap.parse_args(argv)
    base = os.path.join(a.ckpt_dir, a.base)
    out = os.path.join(a.ckpt_dir, a.out)
    c = ckpt.read_checkpoint_meta(base)["config"]
    ctx = Context(0)
    model = Model(ctx, make_config(c["vocabSize"], c["blockSize"], c["nLayer"], c["nHead"], c["nEmbd"],
                                   c.get("arch", "gpt2"), c.get("mlpHidden", 0)))
    try:
        ckpt.load_checkpoint(base, model)
        train = load_tokens(os.path.join(a.data, "chat-train.bin"))
        val = load_tokens(os.path.join(a.data, "chat-val.bin"))
        prompt = [int(x) for x in a.sample_ids.split(",") if x.strip()] or None
        sched = FinetuneSchedule(steps=a.steps, peak_lr=a.lr)
        print(f"Fine-tuning {model.num_params() / 1e6:.2f}M-param GPT into a chatbot")
        print(f"  {a.steps} steps, batch {sched.batch}x{model.cfg.block_size}, lr {a.lr}, "
              f"chat data {len(train) / 1e6:.2f}M tokens\n")
        t0 = time.perf_counter()
        vl = Finetuner(model, train, val, sched, out_path=out, sample_prompt=prompt).run()
        print(f"Done in {(time.perf_counter() - t0) / 60:.1f} min. Chatbot saved to {out}")
        return vl
    finally:
        model.close()
        ctx.close()


if __name__ == "__main__":
    main()
