"""GPU generation with a KV cache vs the oracle's GPT.generate (src/models/gpt.ts:291-341).

* turt_generate_prefill logits = the oracle's forward logits at the last position.
* Every turt_generate_step (one token appended to the cached keys / values) gives the logits
  of a full forward over the grown context, up to a full block; both architectures, both
  attention paths of the prefill (the cache is filled from either), ragged head dims.
* Sampling through the cache (temperature, top-k, the reference's mulberry32 stream) draws the
  oracle's tokens, including past the block size where the window slides.
* The reference's overfit-then-generate test (tests/models/gpt.test.ts:45-70) on the GPU:
  AdamW + clip on one sequence, then near-greedy generation reproduces it.
* Bad positions / ids / lengths are rejected with an error, not run.
Logit tolerance: maxRelErr <= 1e-3 (floor 1e-3), the training-gradient bound's order.
"""
import numpy as np
import pytest

from oracle.oracle import Oracle, max_rel_err

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


@pytest.fixture(scope="module")
def ctx():
    from turt_b200.runtime import Context
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def _setup(ctx, orc, V, T, L, H, E, arch, seed=7, attn=0):
    from turt_b200.runtime import Model, make_config
    c = orc.cfg(V, T, L, H, E, arch)
    p = orc.init(c, seed)
    m = Model(ctx, make_config(V, T, L, H, E, arch))
    m.set_attention(attn)
    m.load_flat(p)
    return c, p, m


@pytest.mark.parametrize("arch,attn,E,H", [("modern", 1, 64, 2), ("modern", 2, 64, 2), ("gpt2", 1, 64, 4),
                                           ("gpt2", 2, 64, 4), ("modern", 1, 96, 2), ("gpt2", 0, 96, 6)])
def test_prefill_and_steps_match_full_forward(ctx, orc, arch, attn, E, H):
    V, T = 100, 24
    c, p, m = _setup(ctx, orc, V, T, 2, H, E, arch, attn=attn)
    try:
        rs = np.random.default_rng(1)
        ids = [int(x) for x in rs.integers(0, V, T)]
        n0 = 5
        got = m.generate_prefill(ids[:n0])
        want = orc.logits(c, p, ids[:n0], 1, n0)[n0 - 1]
        assert max_rel_err(got, want) <= LOGIT_TOL
        for pos in range(n0, T):
            got = m.generate_step(ids[pos], pos)
            want = orc.logits(c, p, ids[:pos + 1], 1, pos + 1)[pos]
            assert max_rel_err(got, want) <= LOGIT_TOL, pos
        # a second prefill replaces the cache (a shorter context, then steps again)
        got = m.generate_prefill(ids[3:10])
        assert max_rel_err(got, orc.logits(c, p, ids[3:10], 1, 7)[6]) <= LOGIT_TOL
        got = m.generate_step(ids[10], 7)
        assert max_rel_err(got, orc.logits(c, p, ids[3:11], 1, 8)[7]) <= LOGIT_TOL
    finally:
        m.close()


@pytest.mark.parametrize("arch,temperature,top_k", [("modern", 1.0, None), ("gpt2", 0.9, 8), ("modern", 0.7, 4)])
def test_sampling_matches_oracle(ctx, orc, arch, temperature, top_k):
    from turt_b200.generate import generate
    from turt_b200.pretrain import Mulberry32
    V, T = 64, 16
    c, p, m = _setup(ctx, orc, V, T, 2, 2, 32, arch, seed=11)
    try:
        prompt = [5, 9, 2]
        want = orc.generate(c, p, prompt, 20, temperature=temperature, topk=top_k or 0, rng_state=orc.rng(123))
        got = generate(m, prompt, 20, temperature=temperature, top_k=top_k, rng=Mulberry32(123))
        assert got == want
    finally:
        m.close()


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
def test_overfit_then_generate(ctx, orc, arch):
    """gpt.test.ts:45-70 at nEmbd 32, two heads of 16 (the CUDA path's smallest sizes): AdamW
    (lr 0.01, wd 0.01) + clip 1.0 for 120 steps on one sequence, then generation at
    temperature 0.01 from its first token reproduces it, the rng shared with the init."""
    from turt_b200.generate import generate
    from turt_b200.pretrain import Mulberry32
    from turt_b200.runtime import Model, make_config
    V, T, L, H, E = 16, 8, 2, 2, 32
    c = orc.cfg(V, T, L, H, E, arch)
    st = orc.rng(7)
    p = orc.init_state(c, st)
    seq = [1, 2, 3, 4, 5, 6, 7, 8]
    ids, tgt = seq[:7], seq[1:]
    m = Model(ctx, make_config(V, T, L, H, E, arch))
    try:
        m.load_flat(p)
        b1, b2 = 0.9, 0.999
        for step in range(1, 121):
            m.zero_grad()
            m.forward_backward(ids, tgt, 1, 7, want_loss=False)
            m.adamw_step(0.01, b1, b2, 1e-8, 0.01, 1 - b1 ** step, 1 - b2 ** step, clip=1.0)
        assert m.forward(ids, tgt, 1, 7) < 0.05
        assert generate(m, [1], 7, temperature=0.01, rng=Mulberry32(int(st[0]))) == seq
    finally:
        m.close()


def test_rejects_bad_calls(ctx, orc):
    from turt_b200._lib import TurtError
    c, p, m = _setup(ctx, orc, 32, 8, 1, 2, 32, "modern")
    try:
        with pytest.raises(TurtError):
            m.generate_step(1, 0)  # nothing cached yet
        m.generate_prefill([1, 2, 3])
        with pytest.raises(TurtError):
            m.generate_step(1, 2)  # not the next position
        with pytest.raises(TurtError):
            m.generate_step(32, 3)  # id out of range
        with pytest.raises(TurtError):
            m.generate_prefill(list(range(9)))  # longer than the block
        m.generate_prefill(list(range(8)))
        with pytest.raises(TurtError):
            m.generate_step(1, 8)  # the block is full
        # the model still generates after the rejected calls
        m.generate_prefill([4, 5])
        m.generate_step(6, 2)
    finally:
        m.close()
