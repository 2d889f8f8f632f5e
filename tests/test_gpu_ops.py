"""Op-level parity through the GpuEngine / GpuTensor mirror (the op-by-op C ABI entry points).

Restates the reference's GPU validators against the CPU oracle:
* scripts/gpu-ops-validate.ts -- each op with loss = sum(op(x) * R), input / parameter
  gradients compared with maxRelErr <= 3e-3 (same seeds and sizes);
* scripts/gpu-train.ts -- a 2-layer MLP, one step and 100 SGD steps, tolerance 2e-3;
* scripts/gpu-gpt-validate.ts -- the whole GPT built op by op on the tape, tolerance 5e-3,
  and the fused model agreeing with the tape;
* scripts/gpu-bench.ts -- host-array matmul cases.
"""
import numpy as np
import pytest

from oracle.oracle import Oracle, max_rel_err

pytestmark = pytest.mark.gpu
TOL = 3e-3


@pytest.fixture(scope="module")
def eng():
    from turt_b200.engine import GpuEngine
    e = GpuEngine.create(0)
    yield e
    e.ctx.close()


@pytest.fixture(scope="module")
def o():
    return Oracle()


def _loss_with(eng, out, R):
    return out.mul(eng.tensor(R, out.shape)).sum()


def test_gather_rows(eng, o):
    V, D, N = 20, 12, 16
    table = o.randn(V * D, 1, 0.3)
    idx = [(i * 7 + 3) % V for i in range(N)]
    R = o.randn(N * D, 2)
    t = eng.tensor(table, [V, D], True)
    _loss_with(eng, t.gatherRows(idx), R).backward()
    ref = o.gather_bwd(idx, R.reshape(N, D), V)
    assert max_rel_err(eng.read(t.grad, t.size), ref) <= TOL


def test_bmm(eng, o):
    G, M, K, N = 4, 8, 6, 10
    a, b, R = o.randn(G * M * K, 3), o.randn(G * K * N, 4), o.randn(G * M * N, 5)
    ga, gb = eng.tensor(a, [G, M, K], True), eng.tensor(b, [G, K, N], True)
    _loss_with(eng, ga.bmm(gb), R).backward()
    da, db = o.bmm_bwd(a.reshape(G, M, K), b.reshape(G, K, N), R.reshape(G, M, N))
    assert max_rel_err(eng.read(ga.grad, ga.size), da) <= TOL
    assert max_rel_err(eng.read(gb.grad, gb.size), db) <= TOL


def test_softmax(eng, o):
    rows, d = 12, 9
    x, R = o.randn(rows * d, 6), o.randn(rows * d, 7)
    gx = eng.tensor(x, [rows, d], True)
    _loss_with(eng, gx.softmax(), R).backward()
    y = o.softmax(x.reshape(rows, d))
    assert max_rel_err(eng.read(gx.grad, gx.size), o.softmax_bwd(y, R.reshape(rows, d))) <= TOL


def test_masked_fill_causal(eng, o):
    G, T = 2, 5
    x, R = o.randn(G * T * T, 8), o.randn(G * T * T, 9)
    gx = eng.tensor(x, [G, T, T], True)
    _loss_with(eng, gx.maskedFillCausal().softmax(), R).backward()
    P = o.softmax(o.mask(x.reshape(G, T, T)))
    ref = o.mask_bwd(o.softmax_bwd(P, R.reshape(G, T, T)))
    assert max_rel_err(eng.read(gx.grad, gx.size), ref) <= TOL


def test_gelu(eng, o):
    n = 40
    x, R = o.randn(n, 10), o.randn(n, 11)
    gx = eng.tensor(x, [n], True)
    _loss_with(eng, gx.gelu(), R).backward()
    assert max_rel_err(eng.read(gx.grad, n), o.gelu_bwd(x, R)) <= TOL


def test_permute(eng, o):
    s = [2, 3, 4, 5]
    n = 120
    x, R = o.randn(n, 12), o.randn(n, 13)
    gx = eng.tensor(x, s, True)
    _loss_with(eng, gx.permute([0, 2, 1, 3]), R).backward()
    ref = o.permute_bwd(R.reshape(2, 4, 3, 5), s, [0, 2, 1, 3])
    assert max_rel_err(eng.read(gx.grad, n), ref) <= TOL
    np.testing.assert_array_equal(gx.permute([0, 2, 1, 3]).read(), o.permute(x.reshape(s), [0, 2, 1, 3]))


def test_matmul_bt(eng, o):
    N, D, V = 8, 6, 11
    x, w, R = o.randn(N * D, 14), o.randn(V * D, 15, 0.2), o.randn(N * V, 16)
    gx, gw = eng.tensor(x, [N, D], True), eng.tensor(w, [V, D], True)
    _loss_with(eng, gx.matmulBT(gw), R).backward()
    X, W, Rm = x.reshape(N, D).astype(np.float64), w.reshape(V, D).astype(np.float64), R.reshape(N, V)
    assert max_rel_err(eng.read(gx.grad, gx.size), Rm @ W) <= TOL
    assert max_rel_err(eng.read(gw.grad, gw.size), Rm.T @ X) <= TOL


def test_layer_norm(eng, o):
    rows, d = 10, 8
    x, R = o.randn(rows * d, 17), o.randn(rows * d, 18)
    gamma = o.randn(d, 19, 0.5) + 1
    beta = o.randn(d, 20, 0.5)
    gx = eng.tensor(x, [rows, d], True)
    gg, gb = eng.tensor(gamma, [d], True), eng.tensor(beta, [d], True)
    _loss_with(eng, gx.layerNorm(gg, gb), R).backward()
    _, dx, dg, db = o.layernorm(x.reshape(rows, d), gamma, beta, R.reshape(rows, d))
    assert max_rel_err(eng.read(gx.grad, gx.size), dx) <= TOL
    assert max_rel_err(eng.read(gg.grad, d), dg) <= TOL
    assert max_rel_err(eng.read(gb.grad, d), db) <= TOL


def test_rms_norm(eng, o):
    rows, d = 10, 64
    x, R = o.randn(rows * d, 21), o.randn(rows * d, 22)
    gamma = o.randn(d, 23, 0.5) + 1
    gx, gg = eng.tensor(x, [rows, d], True), eng.tensor(gamma, [d], True)
    out = gx.rmsNorm(gg)
    y, dx, dg = o.rmsnorm(x.reshape(rows, d), gamma, R.reshape(rows, d))
    assert max_rel_err(out.read(), y) <= TOL
    _loss_with(eng, out, R).backward()
    assert max_rel_err(eng.read(gx.grad, gx.size), dx) <= TOL
    assert max_rel_err(eng.read(gg.grad, d), dg) <= TOL


def test_cross_entropy(eng, o):
    N, V = 14, 17
    x = o.randn(N * V, 21, 0.5)
    tgt = [(i * 5 + 2) % V for i in range(N)]
    gx = eng.tensor(x, [N, V], True)
    loss = gx.crossEntropyLogits(tgt)
    loss.backward()
    ref_loss, ref_g = o.cross_entropy(x.reshape(N, V), tgt)
    assert max_rel_err(loss.read(), [ref_loss]) <= TOL
    assert max_rel_err(eng.read(gx.grad, gx.size), ref_g) <= TOL


def test_silu_rope_and_mul(eng, o):
    G, T, hd = 3, 7, 8
    n = G * T * hd
    x, R = o.randn(n, 24), o.randn(n, 25)
    gx = eng.tensor(x, [G, T, hd], True)
    _loss_with(eng, gx.rope(), R).backward()
    assert max_rel_err(eng.read(gx.grad, n), o.rope_bwd(R.reshape(G, T, hd))) <= TOL
    np.testing.assert_allclose(gx.rope().read(), o.rope(x.reshape(G, T, hd)), atol=1e-5)
    gs = eng.tensor(x, [n], True)
    _loss_with(eng, gs.silu(), R).backward()
    assert max_rel_err(eng.read(gs.grad, n), o.silu_bwd(x, R)) <= TOL
    with pytest.raises(ValueError, match="even headDim"):
        eng.tensor(np.zeros(3), [1, 1, 3]).rope()


def test_broadcast_bias_add_and_scale(eng):
    rows, d = 6, 5
    rng = np.random.default_rng(0)
    x = rng.standard_normal(rows * d).astype(np.float32)
    b = rng.standard_normal(d).astype(np.float32)
    R = rng.standard_normal(rows * d).astype(np.float32)
    gx, gb = eng.tensor(x, [rows, d], True), eng.tensor(b, [d], True)
    _loss_with(eng, gx.add(gb).scale(0.5).sub(gb), R).backward()
    Rm = R.reshape(rows, d).astype(np.float64)
    np.testing.assert_allclose(eng.read(gx.grad, gx.size).reshape(rows, d), 0.5 * Rm, atol=1e-6)
    np.testing.assert_allclose(eng.read(gb.grad, d), 0.5 * Rm.sum(0) - Rm.sum(0), atol=1e-5)


def test_adamw_kernel_matches_oracle(eng, o):
    n = 1000
    p, g = o.randn(n, 30), o.randn(n, 31)
    m, v = np.abs(o.randn(n, 32)) * 0.1, np.abs(o.randn(n, 33)) * 0.01
    dp, dg, dm, dv = (eng.tensor(a, [n]).buffer for a in (p, g, m, v))
    eng.adamw(dg, dp, dm, dv, n, 3e-4, 0.9, 0.999, 1e-8, 0.1, 0.19, 0.002)
    pr, mr, vr = p.copy(), m.copy(), v.copy()
    o.adamw_bc(pr, g, mr, vr, 3e-4, 0.9, 0.999, 1e-8, 0.1, 0.19, 0.002)
    # f32 device arithmetic vs the oracle's double intermediates: a few f32 ulps
    np.testing.assert_allclose(eng.read(dp, n), pr, rtol=5e-6, atol=1e-7)
    np.testing.assert_allclose(eng.read(dm, n), mr, rtol=5e-5, atol=1e-8)
    np.testing.assert_allclose(eng.read(dv, n), vr, rtol=5e-5, atol=1e-10)


def test_mlp_sgd_training(eng, o):
    """scripts/gpu-train.ts: y = relu(x W1 + b1) W2 + b2, loss = mean((y - t)^2), SGD lr 0.05."""
    B, din, hid, dout = 32, 24, 40, 12
    x, tgt = o.randn(B * din, 1), o.randn(B * dout, 2)
    W1, W2 = o.randn(din * hid, 3, 0.2), o.randn(hid * dout, 4, 0.2)
    b1, b2 = np.zeros(hid, np.float32), np.zeros(dout, np.float32)

    def cpu_grads(W1, b1, W2, b2):
        X = x.reshape(B, din).astype(np.float64)
        pre = X @ W1.reshape(din, hid) + b1
        h = np.maximum(pre, 0)
        y = h @ W2.reshape(hid, dout) + b2
        d = y - tgt.reshape(B, dout)
        loss = (d * d).mean()
        gy = 2 * d / d.size
        gW2 = h.T @ gy
        gh = gy @ W2.reshape(hid, dout).T * (pre > 0)
        return loss, (X.T @ gh).ravel(), gh.sum(0), gW2.ravel(), gy.sum(0)

    gX, gT = eng.tensor(x, [B, din]), eng.tensor(tgt, [B, dout])
    ps = [eng.tensor(W1, [din, hid], True), eng.tensor(b1, [hid], True), eng.tensor(W2, [hid, dout], True),
          eng.tensor(b2, [dout], True)]

    def forward():
        h = gX.matmul(ps[0]).add(ps[1]).relu()
        y = h.matmul(ps[2]).add(ps[3])
        d = y.sub(gT)
        return d.mul(d).mean()
    loss = forward()
    loss.backward()
    ref = cpu_grads(W1, b1, W2, b2)
    assert max_rel_err(loss.read(), [ref[0]]) <= 2e-3
    for p, r in zip(ps, ref[1:]):
        assert max_rel_err(eng.read(p.grad, p.size), r) <= 2e-3
    # 100 SGD steps on both engines
    cw = [W1.astype(np.float64), b1.astype(np.float64), W2.astype(np.float64), b2.astype(np.float64)]
    for p, a in zip(ps, (W1, b1, W2, b2)):
        eng.write(p.buffer, a)
    for step in range(100):
        for p in ps:
            p.zeroGrad()
        lg = forward()
        lg.backward()
        for p in ps:
            eng.sgd(p.grad, p.buffer, p.size, 0.05)
        gpu_loss = float(lg.read()[0])
        lg.freeGraph()
        c = cpu_grads(*cw)
        cw = [w - 0.05 * g for w, g in zip(cw, c[1:])]
        cpu_loss = c[0]
    eng.reclaim()
    assert max_rel_err([gpu_loss], [cpu_loss]) <= 2e-3


@pytest.mark.parametrize("arch", ["gpt2", "modern"])
def test_gpt_tape_and_fused_match_oracle(eng, o, arch):
    """scripts/gpu-gpt-validate.ts:52-91 through the op-by-op tape, then the fused model."""
    from turt_b200.engine import GpuGPT
    cfg = dict(vocabSize=48, blockSize=16, nLayer=2, nHead=2, nEmbd=32, arch=arch)
    ocfg = o.cfg(48, 16, 2, 2, 32, arch)
    params = o.init(ocfg, 7)
    st = o.rng(99)
    b, t = 2, 8
    ids = np.array([int(o.rng_next(st) * 48) for _ in range(b * t)], np.uint32)
    tgt = np.array([int(o.rng_next(st) * 48) for _ in range(b * t)], np.uint32)
    ref_loss, ref_g = o.loss_grad(ocfg, params, ids, tgt, b, t)

    tape = GpuGPT(eng, cfg, skipInit=True)
    assert tape.numParams() == params.size
    tape.loadFlat(params)
    loss = tape.loss(ids, tgt, b, t)
    loss.backward()
    assert max_rel_err(loss.read(), [ref_loss]) <= 1e-4
    assert max_rel_err(tape.gradsFlat(), ref_g) <= 5e-3
    loss.freeGraph()
    eng.reclaim()

    fused = GpuGPT(eng, cfg, skipInit=True, fused=True)
    fused.loadFlat(params)
    fl = fused.loss(ids, tgt, b, t)
    assert max_rel_err([fl], [ref_loss]) <= 1e-4
    assert max_rel_err(fused.gradsFlat(), ref_g) <= 2e-3


def _rand_array(o, n, seed):
    """randArray of scripts/gpu-bench.ts:34-46: mulberry32 uniforms mapped to [-1, 1)."""
    st = o.rng(seed)
    return np.array([o.rng_next(st) * 2 - 1 for _ in range(n)], np.float32)


def _max_rel_error(a, b):
    """maxRelError of scripts/gpu-bench.ts:49-56 (denominator floor 1e-4)."""
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(np.max(np.abs(a - b) / np.maximum(1e-4, np.maximum(np.abs(a), np.abs(b)))))


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (16, 16, 16), (17, 33, 9), (64, 128, 384), (256, 160, 1024)])
def test_backend_matmul(o, m, k, n):
    """scripts/gpu-bench.ts:64-116: the GPU matmul against the reference's f32 CPU matmul
    (i-k-j order, restated in the oracle) on the script's own inputs, tolerance 5e-3."""
    from turt_b200.engine import CudaBackend
    be = CudaBackend(0)
    a = _rand_array(o, m * k, m * 7 + k).reshape(m, k)
    b = _rand_array(o, k * n, n * 13 + k).reshape(k, n)
    assert _max_rel_error(be.matmul(a, b), o.matmul(a, b)) <= 5e-3
    if (m, k, n) == (1, 1, 1):
        # batched, attention-shaped (gpu-bench.ts:85-107)
        g, bm, bk, bn = 8, 128, 40, 128
        A = _rand_array(o, g * bm * bk, 3)
        B = _rand_array(o, g * bk * bn, 5)
        out = be.compute.bmm(A, g, bm, bk, B, bn).reshape(g, bm, bn)
        want = o.bmm(A.reshape(g, bm, bk), B.reshape(g, bk, bn))
        assert _max_rel_error(out, want) <= 5e-3
