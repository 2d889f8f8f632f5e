"""Fine-tuning on the GPU (scripts/finetune-chat.ts on the fused step).

* A few fine-tune steps from a base model equal the oracle running the reference's recipe on
  the same batches: sampleBatch windows from one mulberry32(7) stream, AdamW with weight decay
  0.05, no clip, warmup + cosine LR, bias corrections from step 1 (finetune-chat.ts:97-132).
* The periodic eval / checkpoint / sample takes 24 draws of the batch stream, with or without a
  prompt, and the checkpoint's bestValLoss slot holds that eval loss (:143-148).
* The command line fine-tunes a TURTCKPT base model (config and arch taken from the file) on a
  chat corpus and writes the tuned checkpoint.
"""
import json
import math

import numpy as np
import pytest

from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from turt_b200.runtime import Context
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def _corpus(n, period=61):
    return (np.arange(n) % period).astype(np.uint16)


@pytest.mark.parametrize("arch", ["modern", "gpt2"])
def test_steps_match_oracle_recipe(ctx, orc, arch):
    from turt_b200.finetune import Finetuner, FinetuneSchedule
    from turt_b200.pretrain import Mulberry32, lr_at, sample_batch
    from turt_b200.runtime import Model, make_config
    V, T, L, H, E = 64, 32, 2, 2, 64
    c = orc.cfg(V, T, L, H, E, arch)
    base = orc.init(c, 3)
    rs = np.random.default_rng(5)
    train = rs.integers(0, V, 5000).astype(np.uint16)
    val = rs.integers(0, V, 3000).astype(np.uint16)
    sched = FinetuneSchedule(steps=4, batch=4, warmup=2, peak_lr=1e-3, eval_every=1000)
    m = Model(ctx, make_config(V, T, L, H, E, arch))
    try:
        m.load_flat(base)
        ft = Finetuner(m, train, val, sched, log=lambda *_: None)
        vl = ft.run()
        got = m.params_flat()
    finally:
        m.close()
    p = base.copy()
    mm, vv = np.zeros_like(p), np.zeros_like(p)
    rng = Mulberry32(7)
    for step in range(sched.steps):
        ids, tgt = sample_batch(train, sched.batch, T, rng)
        _, g = orc.loss_grad(c, p, ids.astype(np.int32), tgt.astype(np.int32), sched.batch, T)
        lr = lr_at(step, sched.warmup, sched.steps, sched.peak_lr)
        orc.adamw_bc(p, g, mm, vv, lr, 0.9, 0.999, 1e-8, 0.05, 1 - 0.9 ** (step + 1), 1 - 0.999 ** (step + 1))
    diff = np.abs(got - p)
    # Adam moves each weight by about lr per step whatever the gradient's size, so a gradient
    # that is ~0 in the oracle and a rounding-noise value of either sign on the GPU may differ
    # by up to 2 lr per step; every other weight must agree closely.
    assert diff.max() <= 2 * sched.peak_lr * sched.steps + 1e-6
    assert np.mean(diff <= 2e-6) > 0.99
    # eval at the end (step == steps), then 24 sample draws of the batch stream
    want = Mulberry32(7)
    for _ in range(sched.steps * sched.batch + sched.sample_tokens):
        want()
    assert ft.rng.state == want.state
    assert math.isfinite(vl)


def test_checkpoint_and_sample(ctx, tmp_path):
    from turt_b200 import checkpoint as ck
    from turt_b200.finetune import Finetuner, FinetuneSchedule
    from turt_b200.pretrain import Mulberry32
    from turt_b200.runtime import Model, make_config
    m = Model(ctx, make_config(64, 32, 2, 2, 64, "modern"))
    try:
        m.init_reference(9)
        out = str(tmp_path / "chat.bin")
        sched = FinetuneSchedule(steps=6, batch=4, warmup=2, peak_lr=3e-3, eval_every=3, log_every=2)
        ft = Finetuner(m, _corpus(4000), _corpus(2000), sched, out_path=out, sample_prompt=[1, 2, 3],
                       log=lambda *_: None)
        vl = ft.run()
        meta = ck.read_checkpoint_meta(out)
        assert meta["step"] == 6 and abs(meta["bestValLoss"] - vl) < 1e-6
        assert len(ft.samples) == 2 and all(len(s) == 3 + 24 and s[:3] == [1, 2, 3] for s in ft.samples)
        want = Mulberry32(7)
        for _ in range(6 * 4 + 2 * 24):
            want()
        assert ft.rng.state == want.state
    finally:
        m.close()


def test_command_line(ctx, tmp_path):
    from turt_b200 import checkpoint as ck
    from turt_b200.finetune import main
    from turt_b200.runtime import Model, make_config
    cdir, ddir = tmp_path / "checkpoints", tmp_path / "data"
    cdir.mkdir()
    ddir.mkdir()
    m = Model(ctx, make_config(64, 32, 2, 2, 64, "gpt2"))
    try:
        m.init_reference(4)
        ck.save_checkpoint(str(cdir / "gpt.bin"), m, 100, 3.5)
    finally:
        m.close()
    _corpus(20_000).astype("<u2").tofile(ddir / "chat-train.bin")
    _corpus(4_000).astype("<u2").tofile(ddir / "chat-val.bin")
    vl = main(["--steps", "150", "--lr", "3e-3", "--data", str(ddir), "--ckpt-dir", str(cdir),
               "--sample-ids", "5,6,7"])
    meta = ck.read_checkpoint_meta(str(cdir / "chat.bin"))
    assert meta["step"] == 150 and meta["config"]["arch"] == "gpt2" and meta["config"]["nEmbd"] == 64
    assert abs(meta["bestValLoss"] - vl) < 1e-6 and vl < math.log(64) - 0.5
    json.dumps(meta)
