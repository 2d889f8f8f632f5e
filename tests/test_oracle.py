"""Pins the CPU oracle against the reference's own known-answer tests (CPU only).

Each test restates one assertion of the turt reference's vitest suite (cited per case in
tests/golden/reference_known_answers.json) against the C oracle, plus central-difference
gradient checks of every op and of the whole model (double build of the same source).
"""
import json
import math
import os

import numpy as np
import pytest

from oracle.oracle import Oracle, max_rel_err

HERE = os.path.dirname(os.path.abspath(__file__))
KA = json.load(open(os.path.join(HERE, "golden", "reference_known_answers.json")))


@pytest.fixture(scope="module")
def o():
    return Oracle()


@pytest.fixture(scope="module")
def o64():
    return Oracle(f64=True)


def close(a, b, digits):
    """vitest toBeCloseTo(b, digits): |a - b| < 10^-digits / 2."""
    return abs(a - b) < 10 ** (-digits) / 2


def numeric_grad(f, vals, eps=1e-3):
    out = []
    for i in range(len(vals)):
        p = list(vals)
        m = list(vals)
        p[i] += eps
        m[i] -= eps
        out.append((f(p) - f(m)) / (2 * eps))
    return np.array(out)


def rand_vals(o, n, seed=5):
    st = o.rng(seed)
    return [o.rng_next(st) * 2 - 1 for _ in range(n)]


# ------------------------------------------------------------------ RNG
def test_mulberry32_first_values(o):
    # Values of the restated mulberry32(42) (src/math/random.ts:8-17), pinned in golden/rng.json.
    gold = json.load(open(os.path.join(HERE, "golden", "rng.json")))
    st = o.rng(gold["seed"])
    got = [o.rng_next(st) for _ in range(len(gold["values"]))]
    np.testing.assert_array_equal(got, gold["values"])
    assert all(0 <= v < 1 for v in got)


# ------------------------------------------------------------- gpt-ops tests
def test_permute(o):
    k = KA["permute"]
    y = o.permute(np.array(k["input"], dtype=np.float32).reshape(k["shape"]), k["perm"])
    assert list(y.shape) == k["expected_shape"]
    assert y.ravel().tolist() == k["expected"]


def test_permute_self_inverse(o):
    x = np.array(rand_vals(o, 24), dtype=np.float32).reshape(2, 3, 4)
    np.testing.assert_array_equal(o.permute(o.permute(x, [2, 1, 0]), [2, 1, 0]), x)


def test_bmm(o):
    k = KA["bmm"]
    y = o.bmm(np.array(k["a"], np.float32).reshape(k["shape"]), np.array(k["b"], np.float32).reshape(k["shape"]))
    assert y.ravel().tolist() == k["expected"]


def test_bmm_numeric_grads(o64):
    a = np.array(rand_vals(o64, 12, 11)).reshape(2, 2, 3)
    b = np.array(rand_vals(o64, 12, 12)).reshape(2, 3, 2)
    y = o64.bmm(a, b)
    g = 1 - np.tanh(y) ** 2  # d sum(tanh(y)) / dy
    da, db = o64.bmm_bwd(a, b, g)
    na = numeric_grad(lambda v: np.tanh(o64.bmm(np.array(v).reshape(2, 2, 3), b)).sum(), a.ravel().tolist())
    nb = numeric_grad(lambda v: np.tanh(o64.bmm(a, np.array(v).reshape(2, 3, 2))).sum(), b.ravel().tolist())
    np.testing.assert_allclose(da.ravel(), na, atol=5e-3)
    np.testing.assert_allclose(db.ravel(), nb, atol=5e-3)


def test_gather(o):
    k = KA["gather"]
    t = np.array(k["table"], np.float32).reshape(k["shape"])
    assert o.gather(t, k["idx"]).ravel().tolist() == k["expected"]


def test_gather_scatter_repeated(o):
    k = KA["gather_scatter"]
    g = np.ones((len(k["idx"]), k["table_shape"][1]), np.float32)
    assert o.gather_bwd(k["idx"], g, k["table_shape"][0]).ravel().tolist() == k["expected_grad"]


def test_gather_rejects_out_of_range(o):
    with pytest.raises(IndexError):
        o.gather(np.zeros((2, 2), np.float32), [5])


def test_softmax_rows(o):
    k = KA["softmax_uniform"]
    y = o.softmax(np.array(k["input"], np.float32).reshape(k["shape"]))
    for row in y:
        assert close(row.sum(), 1, 5) and np.all(row > 0)
    for v, e in zip(y[1], k["expected_row1"]):
        assert close(v, e, k["digits"])


def test_softmax_large_logits(o):
    k = KA["softmax_large"]
    y = o.softmax(np.array(k["input"], np.float32).reshape(k["shape"]))
    assert np.all(np.isfinite(y)) and close(y.sum(), 1, 5)


def test_softmax_numeric_grads(o64):
    x = rand_vals(o64, 6, 13)
    w = np.arange(1, 7, dtype=np.float64).reshape(2, 3)
    y = o64.softmax(np.array(x).reshape(2, 3))
    gx = o64.softmax_bwd(y, w)
    num = numeric_grad(lambda v: (o64.softmax(np.array(v).reshape(2, 3)) * w).sum(), x)
    np.testing.assert_allclose(gx.ravel(), num, atol=5e-3)


def test_mask_then_softmax(o):
    k = KA["mask_softmax"]
    a = o.softmax(o.mask(np.array(k["input"], np.float32).reshape(k["shape"]))).ravel()
    for i in k["zeros"]:
        assert close(a[i], 0, 6)
    assert close(a[0], 1, 6)
    assert close(a[3] + a[4], 1, 5)


def test_mask_grad(o):
    k = KA["mask_grad"]
    assert o.mask_bwd(np.ones(k["shape"], np.float32)).ravel().tolist() == k["expected_grad"]


def test_gelu_known(o):
    k = KA["gelu"]
    y = o.gelu(np.array(k["input"], np.float32))
    for v, e, d in zip(y, k["expected"], k["digits"]):
        assert close(v, e, d)


def test_gelu_numeric_grad(o64):
    x = np.array(rand_vals(o64, 6, 14))
    g = o64.gelu_bwd(x, np.ones_like(x))
    num = numeric_grad(lambda v: o64.gelu(np.array(v)).sum(), x.tolist())
    np.testing.assert_allclose(g, num, atol=5e-3)


def test_cross_entropy_known(o):
    k = KA["ce_uniform"]
    loss, _ = o.cross_entropy(np.zeros(k["shape"], np.float32), k["targets"])
    assert close(loss, math.log(4), k["digits"])
    k = KA["ce_confident"]
    loss, _ = o.cross_entropy(np.array(k["logits"], np.float32).reshape(k["shape"]), k["targets"])
    assert loss < k["less_than"]
    k = KA["ce_large"]
    loss, _ = o.cross_entropy(np.array(k["logits"], np.float32).reshape(k["shape"]), k["targets"])
    assert math.isfinite(loss)


def test_cross_entropy_grad_numeric(o):
    k = KA["ce_grad"]
    x = np.array(k["logits"], np.float32).reshape(k["shape"])
    _, g = o.cross_entropy(x, k["targets"])
    num = numeric_grad(lambda v: o.cross_entropy(np.array(v, np.float32).reshape(k["shape"]), k["targets"])[0],
                       k["logits"])
    for a, b in zip(g.ravel(), num):
        assert close(a, b, k["digits"])


def test_cross_entropy_rejects_bad_target(o):
    with pytest.raises(IndexError):
        o.cross_entropy(np.zeros((1, 4), np.float32), [4])


def test_silu(o, o64):
    k = KA["silu"]
    xs = np.array(k["input"], np.float32)
    y = o.silu(xs)
    for v, x in zip(y, k["input"]):
        assert close(v, x / (1 + math.exp(-x)), k["digits"])
    big = o.silu(np.array(k["large"], np.float32))
    assert big[0] == 0 and close(big[1], 20, 4)
    x = np.array(rand_vals(o64, 6, 15))
    num = numeric_grad(lambda v: o64.silu(np.array(v)).sum(), x.tolist())
    np.testing.assert_allclose(o64.silu_bwd(x, np.ones_like(x)), num, atol=5e-4)


def test_rope_properties(o, o64):
    # identity at position 0 (gpt-ops.test.ts:198-203)
    v = np.array(rand_vals(o, 4, 16), np.float32).reshape(1, 1, 4)
    np.testing.assert_allclose(o.rope(v), v, atol=1e-5)
    # norm preserving (:205-213)
    x = np.array(rand_vals(o, 40, 17), np.float32).reshape(2, 5, 4)
    y = o.rope(x)
    np.testing.assert_allclose(np.linalg.norm(y, axis=-1), np.linalg.norm(x, axis=-1), atol=1e-4)
    # relative-distance dot products (:215-235)
    vec = rand_vals(o, 4, 18)
    r = o.rope(np.array([vec] * 6, np.float32).reshape(1, 6, 4))[0]
    for gap in range(4):
        ref = float(r[0] @ r[gap])
        for i in range(6 - gap):
            assert abs(float(r[i] @ r[i + gap]) - ref) < 5e-5
    # numeric gradient of sum(rope(t) * rope(t)) (:237-239)
    t = np.array(rand_vals(o64, 12, 19)).reshape(1, 3, 4)
    yy = o64.rope(t)
    g = o64.rope_bwd(2 * yy)
    num = numeric_grad(lambda v: (o64.rope(np.array(v).reshape(1, 3, 4)) ** 2).sum(), t.ravel().tolist())
    np.testing.assert_allclose(g.ravel(), num, atol=5e-4)
    # odd head dim rejected (:241-243)
    with pytest.raises(ValueError, match="even headDim"):
        o.rope(np.zeros((1, 1, 3), np.float32))


def test_norm_composites_numeric(o64):
    rows, d = 3, 8
    x = np.array(rand_vals(o64, rows * d, 20)).reshape(rows, d)
    g = 1 + 0.5 * np.array(rand_vals(o64, d, 21))
    bt = 0.5 * np.array(rand_vals(o64, d, 22))
    R = np.array(rand_vals(o64, rows * d, 23)).reshape(rows, d)
    _, dx, dg = o64.rmsnorm(x, g, R)
    num = numeric_grad(lambda v: (o64.rmsnorm(np.array(v).reshape(rows, d), g) * R).sum(), x.ravel().tolist(), 1e-5)
    np.testing.assert_allclose(dx.ravel(), num, atol=1e-6)
    numg = numeric_grad(lambda v: (o64.rmsnorm(x, np.array(v)) * R).sum(), g.tolist(), 1e-5)
    np.testing.assert_allclose(dg, numg, atol=1e-6)
    _, dx, dg, db = o64.layernorm(x, g, bt, R)
    num = numeric_grad(lambda v: (o64.layernorm(np.array(v).reshape(rows, d), g, bt) * R).sum(), x.ravel().tolist(),
                       1e-5)
    np.testing.assert_allclose(dx.ravel(), num, atol=1e-6)
    np.testing.assert_allclose(db, R.sum(0), atol=1e-12)


def test_layernorm_and_rmsnorm_stats(o):
    """tests/nn/nn.test.ts:72-85 and :98-107: unit variance rows / unit RMS rows."""
    st = o.rng(3)
    x = np.empty(32, np.float32)
    o.lib.oc_randn(x.ctypes.data, 32, st.ctypes.data, 1.0)
    x = x.reshape(4, 8)
    y = o.layernorm(x, np.ones(8, np.float32), np.zeros(8, np.float32))
    for row in y:
        assert close(row.mean(), 0, 4) and close(((row - row.mean()) ** 2).mean(), 1, 2)
    y = o.rmsnorm(x, np.ones(8, np.float32))
    for row in y:
        assert close(math.sqrt((row.astype(np.float64) ** 2).mean()), 1, 3)
    z = np.array([[1, 2, 3, 4]], np.float32)
    assert o.rmsnorm(z, np.ones(4, np.float32)).mean() > 0.5
    assert close(o.layernorm(z, np.ones(4, np.float32), np.zeros(4, np.float32)).mean(), 0, 5)


def test_clip_to_max_norm(o):
    """tests/nn/nn.test.ts:71-80: mse(10p, 0) grads clipped to norm 1."""
    p = np.array([3.0, 4.0])
    g = (2 * (10 * p) * 10 / 2).astype(np.float32)  # d mean((10p)^2)/dp
    before = o.clip(g, 1.0)
    assert before > 1 and close(float(np.hypot(*g.astype(np.float64))), 1, 4)


# ------------------------------------------------------------------ model tests
def _cfg(o, arch):
    k = KA["gpt_config"]
    return o.cfg(k["vocabSize"], k["blockSize"], k["nLayer"], k["nHead"], k["nEmbd"], arch)


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
def test_param_count_formula(o, arch):
    c = _cfg(o, arch)
    V, T, L, E = 16, 8, 2, 16
    h = o.hidden(c)
    if arch == "gpt2":
        expect = V * E + T * E + L * (12 * E * E + 13 * E) + 2 * E
    else:
        expect = V * E + L * (4 * E * E + 3 * E * h + 2 * E) + E
    assert o.num_params(c) == expect


def test_swiglu_width_matches_gelu(o):
    m = o.cfg(16, 8, 2, 2, 384, "modern")
    g = o.cfg(16, 8, 2, 2, 384, "gpt2")
    assert close(3 * 384 * o.hidden(m) / (2 * 384 * o.hidden(g)), 1, 1)
    assert o.hidden(o.cfg(8192, 128, 4, 4, 128, "modern")) == 320
    assert o.hidden(o.cfg(8192, 256, 6, 6, 384, "modern")) == 1024


def test_init_loss_near_uniform(o):
    k = KA["gpt_init_loss"]
    for arch in ("gpt2", "modern"):
        c = _cfg(o, arch)
        p = o.init(c, k["seed"])
        loss = o.loss_grad(c, p, k["idx"], k["targets"], 1, 8, grads=False)
        assert abs(loss - math.log(16)) < k["tolerance"]


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
def test_causality(o, arch):
    k = KA["gpt_causal"]
    c = _cfg(o, arch)
    p = o.init(c, k["seed"])
    a = o.logits(c, p, k["a"], 1, 4)
    b = o.logits(c, p, k["b"], 1, 4)
    np.testing.assert_allclose(a[:3], b[:3], atol=10 ** -k["digits"] / 2)
    assert not np.array_equal(a[3], b[3])


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
def test_every_param_gets_grad(o, arch):
    k = KA["gpt_every_param_grad"]
    c = _cfg(o, arch)
    p = o.init(c, k["seed"])
    _, g = o.loss_grad(c, p, k["idx"], k["targets"], 1, 4)
    for t in o.split(c, g):
        assert np.any(t != 0)


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
def test_model_numeric_gradient(o64, arch):
    """Every parameter of a tiny model: analytic vs central difference (double build)."""
    c = o64.cfg(11, 8, 2, 2, 8, arch)
    p = o64.init(c, 3)
    ids, tg = [1, 2, 3, 4, 5, 6], [2, 3, 4, 5, 6, 7]
    _, g = o64.loss_grad(c, p, ids, tg, 2, 3)
    h = 1e-5
    for i in range(p.size):
        pp = p.copy()
        pp[i] += h
        pm = p.copy()
        pm[i] -= h
        num = (o64.loss_grad(c, pp, ids, tg, 2, 3, grads=False) - o64.loss_grad(c, pm, ids, tg, 2, 3, grads=False)) / (2 * h)
        assert abs(num - g[i]) < 1e-7 + 1e-5 * abs(num)


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
def test_overfit_fixed_sequence(o, arch):
    """gpt.test.ts:45-70 / :154-171: AdamW(lr .01, wd .01) + clip 1.0, 120 steps -> loss < 0.05,
    then near-greedy generation reproduces the sequence."""
    k = KA["gpt_overfit"]
    c = _cfg(o, arch)
    st = o.rng(k["seed"])
    p = o.init_state(c, st)  # one rng shared by init and generate, as in the reference test
    seq = k["sequence"]
    ids, tgt = seq[:7], seq[1:]
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    for step in range(1, k["steps"] + 1):
        loss, g = o.loss_grad(c, p, ids, tgt, 1, 7)
        o.clip(g, k["clip"])
        o.adamw(p, g, m, v, k["lr"], 0.9, 0.999, 1e-8, k["weight_decay"], step)
    final = o.loss_grad(c, p, ids, tgt, 1, 7, grads=False)
    assert final < k["final_below"]
    gen = o.generate(c, p, [1], 7, temperature=k["temperature"], rng_state=st)
    assert gen == seq


def test_dp_sharded_mean_equals_full_batch(o):
    """checkpoint.test.ts:83-107: mean of per-shard grads (weight rows/batch) == full-batch grads."""
    k = KA["dp_sharded_mean"]
    cc = k["config"]
    c = o.cfg(cc["vocabSize"], cc["blockSize"], cc["nLayer"], cc["nHead"], cc["nEmbd"], "gpt2")
    p = o.init(c, k["seed"])
    _, full = o.loss_grad(c, p, k["inputs"], k["targets"], 2, 4)
    _, sharded = o.dp_grads(c, p, k["inputs"], k["targets"], 2, 4, workers=2)
    np.testing.assert_allclose(sharded, full, atol=10 ** -k["digits"] / 2)


def test_dp_worker_counts_agree(o):
    """1, 2, 3 and 4 workers (ragged shards included) give the same step (docs: loss matches across workers)."""
    c = o.cfg(64, 16, 2, 2, 32, "modern")
    p = o.init(c, 7)
    ids = o.uniform_ints(6 * 16, 99, 64)
    tgt = o.uniform_ints(6 * 16, 100, 64)
    base_loss, base = o.dp_grads(c, p, ids, tgt, 6, 16, 1)
    for w in (2, 3, 4):
        loss, g = o.dp_grads(c, p, ids, tgt, 6, 16, w)
        assert abs(loss - base_loss) < 1e-5
        assert max_rel_err(g, base) < 1e-4
