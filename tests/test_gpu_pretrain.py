"""Pretraining path on the GPU: reference init, device data feed, checkpoints and resume.

* turt_model_init reproduces the reference CPU constructor GPT(config, mulberry32(seed))
  bit for bit (checked against the oracle's restatement of src/models/gpt.ts init).
* turt_sample_windows gathers exactly the windows of sampleBatch (gpu-pretrain.ts:57-68).
* A checkpoint written from device parameters reloads bit for bit into a differently
  initialised model (checkpoint.test.ts:20-38 on the GPU model) and gives the same loss.
* Resuming from a checkpoint with its AdamW sidecar continues the optimizer trajectory: the
  parameters after the resumed steps match an uninterrupted run (same batches) to rounding
  noise, while dropping the moments (what the reference's resume does) changes them.
* The Pretrainer loop learns a predictable corpus (train and eval loss fall).
"""
import numpy as np
import pytest

from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import torch

    from turt_b200.runtime import Context
    c = Context(0)
    c.set_stream(torch.cuda.current_stream().cuda_stream)
    yield c
    c.close()


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def _model(ctx, V=64, T=32, L=2, H=2, E=64, arch="modern"):
    from turt_b200.runtime import Model, make_config
    return Model(ctx, make_config(V, T, L, H, E, arch))


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
def test_reference_init(ctx, orc, arch):
    m = _model(ctx, 48, 16, 2, 2, 32, arch)
    try:
        m.init_reference(1337)
        ref = orc.init(orc.cfg(48, 16, 2, 2, 32, arch), 1337)
        got = m.params_flat()
        assert np.array_equal(got.view(np.uint32), ref.astype(np.float32).view(np.uint32))
    finally:
        m.close()


def test_device_windows_match_sample_batch(ctx):
    from turt_b200.pretrain import DeviceCorpus, Mulberry32, sample_batch
    rng_tokens = np.random.default_rng(3)
    tokens = rng_tokens.integers(0, 65535, 100_000).astype(np.uint16)
    b, t = 7, 129
    dc = DeviceCorpus(ctx, tokens, b, t)
    d_ids, d_tgt = dc.sample(b, Mulberry32(1234))
    ctx.synchronize()
    ids = dc.ids.cpu().numpy().view(np.uint32)
    tgt = dc.tgt.cpu().numpy().view(np.uint32)
    ref_ids, ref_tgt = sample_batch(tokens, b, t, Mulberry32(1234))
    np.testing.assert_array_equal(ids, ref_ids)
    np.testing.assert_array_equal(tgt, ref_tgt)


def test_checkpoint_round_trip(ctx, tmp_path):
    from turt_b200 import checkpoint as ck
    a, b = _model(ctx), _model(ctx)
    try:
        a.init_reference(1)
        b.init_reference(999)
        rng = np.random.default_rng(0)
        ids = rng.integers(0, 64, 4 * 32).astype(np.uint32)
        tgt = rng.integers(0, 64, 4 * 32).astype(np.uint32)
        la = a.forward(ids, tgt, 4, 32)
        assert b.forward(ids, tgt, 4, 32) != la
        path = str(tmp_path / "m.bin")
        ck.save_checkpoint(path, a, 42, 1.234)
        meta = ck.load_checkpoint(path, b)
        assert meta["step"] == 42 and meta["config"]["arch"] == "modern" and meta["config"]["nEmbd"] == 64
        pa, pb = a.params_flat(), b.params_flat()
        assert np.array_equal(pa.view(np.uint32), pb.view(np.uint32))
        assert b.forward(ids, tgt, 4, 32) == la
        wider = _model(ctx, E=128)
        try:
            with pytest.raises(ValueError, match="mismatch"):
                ck.load_checkpoint(path, wider)
        finally:
            wider.close()
    finally:
        a.close()
        b.close()


def _corpus(n=20_000, period=61):
    return (np.arange(n) % period).astype(np.uint16)


def test_resume_with_optimizer_state(ctx, tmp_path):
    from turt_b200.pretrain import Mulberry32, Pretrainer, Schedule
    sched = Schedule(steps=8, batch=8, micro=4, warmup=2, peak_lr=3e-3, eval_every=1000, eval_batches=2)
    path = str(tmp_path / "run.bin")
    tokens = _corpus()
    a = _model(ctx)
    b = _model(ctx)
    c = _model(ctx)
    try:
        a.init_reference(5)
        pa = Pretrainer(a, tokens, tokens, sched, log=lambda *_: None)
        pa.run(until=4)
        pa.save(path)
        pa.rng = Mulberry32(42 + pa.step)  # a resumed run reseeds the batch stream this way
        pa.run(until=8)
        final_a = a.params_flat()

        pb = Pretrainer(b, tokens, tokens, sched, log=lambda *_: None)
        meta = pb.resume(path)
        assert meta["step"] == 4 and pb.adam_step == 4
        pb.run(until=8)
        final_b = b.params_flat()
        np.testing.assert_allclose(final_b, final_a, rtol=1e-5, atol=1e-6)

        import os
        os.rename(path + ".adam", path + ".adam.off")  # resume without the moments
        pc = Pretrainer(c, tokens, tokens, sched, log=lambda *_: None)
        pc.resume(path)
        pc.run(until=8)
        assert np.max(np.abs(c.params_flat() - final_a)) > 100 * np.max(np.abs(final_b - final_a))
    finally:
        for m in (a, b, c):
            m.close()


def test_pretrainer_learns(ctx, tmp_path):
    from turt_b200 import checkpoint as ck
    from turt_b200.pretrain import Pretrainer, Schedule
    sched = Schedule(steps=60, batch=8, micro=8, warmup=5, peak_lr=3e-3, eval_every=30, eval_batches=4)
    m = _model(ctx)
    try:
        m.init_reference(1337)
        tokens = _corpus()
        path = str(tmp_path / "learn.bin")
        p = Pretrainer(m, tokens, tokens, sched, out_path=path, log=lambda *_: None)
        first = p.eval_loss()
        best = p.run()
        assert best < 0.5 * first
        meta = ck.read_checkpoint_meta(path)
        assert meta["step"] == 60 and abs(meta["bestValLoss"] - best) < 1e-6
    finally:
        m.close()


def test_command_line(tmp_path):
    """python -m turt_b200.pretrain on a data directory laid out like prepare-data's output."""
    import json

    from turt_b200 import checkpoint as ck
    from turt_b200.pretrain import main
    d = tmp_path / "data"
    d.mkdir()
    (d / "meta.json").write_text(json.dumps({"vocabSize": 64}))
    _corpus(30_000).astype("<u2").tofile(d / "train.bin")
    _corpus(5_000).astype("<u2").tofile(d / "val.bin")
    out = str(tmp_path / "cli.bin")
    args = ["--data", str(d), "--out", out, "--block", "32", "--layers", "2", "--heads", "2", "--embd", "64",
            "--batch", "8", "--steps", "20", "--warmup", "4", "--lr", "3e-3", "--eval", "10"]
    best = main(args)
    meta = ck.read_checkpoint_meta(out)
    assert meta["step"] == 20 and meta["config"]["vocabSize"] == 64 and best < 4.0
    best2 = main(args[:4] + ["--resume", out, "--steps", "30", "--eval", "10", "--batch", "8", "--lr", "3e-3"])
    assert ck.read_checkpoint_meta(out)["step"] == 30 and best2 <= best
