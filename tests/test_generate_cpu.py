"""Host side of GPU generation, on the CPU.

* sample_from_logits against a scalar restatement of sampleFromLogits (src/models/gpt.ts:324-341).
* Temperature and top-k as GPT.generate applies them (gpt.ts:306-314), ties at the threshold kept.
* generate() driven by a stand-in model whose prefill / step logits come from the oracle's
  forward reproduces the oracle's GPT.generate token for token, across the point where the
  context outgrows the block, and issues one prefill, then decode steps until the block is full,
  then one prefill per token (the window slides).
"""
import math
from types import SimpleNamespace

import numpy as np
import pytest

from oracle.oracle import Oracle
from turt_b200.generate import Generator, apply_temperature_top_k, generate, sample_from_logits
from turt_b200.pretrain import Mulberry32


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def _scalar_sample(logits, rng):
    mx = -math.inf
    for v in logits:
        if v > mx:
            mx = float(v)
    probs, total = [], 0.0
    for v in logits:
        e = math.exp(float(v) - mx)
        probs.append(float(np.float32(e)))
        total += e
    r = rng() * total
    for j, p in enumerate(probs):
        r -= p
        if r <= 0:
            return j
    return len(probs) - 1


def test_sample_from_logits_matches_scalar_loop():
    rs = np.random.default_rng(0)
    for trial in range(200):
        V = int(rs.integers(2, 300))
        logits = (rs.standard_normal(V) * rs.uniform(0.1, 8)).astype(np.float32)
        if trial % 3 == 0:
            logits[rs.random(V) < 0.5] = -np.inf
            logits[rs.integers(0, V)] = 1.0
        a, b = Mulberry32(trial), Mulberry32(trial)
        for _ in range(5):
            assert sample_from_logits(logits, a) == _scalar_sample(logits, b)


def test_temperature_and_top_k():
    logits = np.array([1.0, 3.0, 3.0, -2.0, 0.5, 2.0], dtype=np.float32)
    out = apply_temperature_top_k(logits, 0.7, 2)
    # the 2nd largest is 3/0.7 (a tie): both copies stay, everything below goes
    assert np.isinf(out[[0, 3, 4, 5]]).all() and (out[[0, 3, 4, 5]] < 0).all()
    assert out[1] == out[2] == np.float32(np.float64(np.float32(3.0)) / 0.7)
    assert np.array_equal(apply_temperature_top_k(logits, 1.0, None), logits)
    assert np.array_equal(apply_temperature_top_k(logits, 1.0, 6), logits)  # top_k >= V: off
    assert np.array_equal(apply_temperature_top_k(logits, 1.0, 0), logits)  # falsy: off


class OracleModel:
    """Stand-in for runtime.Model: prefill / step logits from the oracle's forward."""

    def __init__(self, orc, cfg, params, block, vocab):
        self.orc, self.c, self.p = orc, cfg, params
        self.cfg = SimpleNamespace(block_size=block, vocab_size=vocab)
        self.ctx_ids, self.calls = [], []

    def _last(self):
        t = len(self.ctx_ids)
        return self.orc.logits(self.c, self.p, self.ctx_ids, 1, t)[t - 1]

    def generate_prefill(self, ids):
        assert 0 < len(ids) <= self.cfg.block_size
        self.ctx_ids = list(ids)
        self.calls.append(("prefill", len(ids)))
        return self._last()

    def generate_step(self, token, pos):
        assert pos == len(self.ctx_ids) < self.cfg.block_size
        self.ctx_ids.append(token)
        self.calls.append(("step", pos))
        return self._last()


@pytest.mark.parametrize("arch,temperature,top_k", [("modern", 1.0, None), ("gpt2", 0.8, 5), ("modern", 1.3, 3)])
def test_generate_matches_oracle(orc, arch, temperature, top_k):
    V, T = 40, 12
    c = orc.cfg(V, T, 2, 2, 16, arch)
    p = orc.init(c, 7)
    prompt = [3, 1, 4, 1, 5]
    want = orc.generate(c, p, prompt, 14, temperature=temperature, topk=top_k or 0, rng_state=orc.rng(99))
    fake = OracleModel(orc, c, p, T, V)
    got = generate(fake, prompt, 14, temperature=temperature, top_k=top_k, rng=Mulberry32(99))
    assert got == want
    # one prefill of the prompt, steps at positions 5..11, then a prefill per token of the
    # sliding window (13 tokens and more do not fit the block of 12)
    assert fake.calls[0] == ("prefill", 5)
    assert fake.calls[1:8] == [("step", q) for q in range(5, 12)]
    assert fake.calls[8:] == [("prefill", 12)] * 6


def test_generate_stops_on_callback(orc):
    c = orc.cfg(20, 8, 1, 2, 16, "modern")
    p = orc.init(c, 1)
    seen = []
    out = generate(OracleModel(orc, c, p, 8, 20), [1, 2], 10, rng=Mulberry32(5),
                   on_token=lambda i: seen.append(i) if len(seen) < 3 else False)
    assert len(out) == 2 + 4 and seen == out[2:5]


def test_empty_prompt_rejected(orc):
    c = orc.cfg(20, 8, 1, 2, 16, "modern")
    with pytest.raises(ValueError):
        Generator(OracleModel(orc, c, orc.init(c, 1), 8, 20)).next_logits([])
