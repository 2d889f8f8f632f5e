"""Checkpoint format and pretraining data feed, on the CPU.

The reference's checkpoint tests (tests/scripts/checkpoint.test.ts:20-55) restated for the
TURTCKPT writer / reader: exact round trip with step and bestValLoss, a shape mismatch and a
foreign file rejected.  The header bytes are compared with what JSON.stringify writes for the
same meta object (compact, key order kept, Infinity as null), and the file is also parsed with
an independent restatement of the reference loader (checkpoint.ts:53-60,99-123).  The data feed's
mulberry32 stream is compared with the oracle's, its window sampler with sampleBatch
(scripts/gpu-pretrain.ts:57-68), and the LR schedule with lrAt (:182-186).
"""
import json
import math
import struct

import numpy as np
import pytest

from oracle.oracle import Oracle
from turt_b200 import checkpoint as ck
from turt_b200.pretrain import Mulberry32, lr_at, sample_batch, sample_starts

CONFIG = {"vocabSize": 32, "blockSize": 8, "nLayer": 2, "nHead": 2, "nEmbd": 16}


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def _params(orc, seed):
    cfg = orc.cfg(32, 8, 2, 2, 16, "gpt2")  # the reference test's config has no arch: gpt2
    return [np.array(p, dtype=np.float32) for p in orc.split(cfg, orc.init(cfg, seed))]


def _reference_load(path):
    """checkpoint.ts parseHeader + loadCheckpoint, restated independently of the writer."""
    buf = open(path, "rb").read()
    if buf[0:8].decode("ascii").rstrip("\0") != "TURTCKPT":
        raise ValueError("not a Turt checkpoint")
    n = int.from_bytes(buf[8:12], "little")
    meta = json.loads(buf[12:12 + n].decode("utf-8"))
    off, out = 12 + n, []
    for shp in meta["shapes"]:
        k = int(np.prod(shp))
        out.append(np.array(struct.unpack_from(f"<{k}f", buf, off), dtype=np.float32).reshape(shp))
        off += 4 * k
    return meta, out


def test_round_trip_exact(orc, tmp_path):
    params = _params(orc, 1)
    path = str(tmp_path / "gpt.bin")
    ck.write_checkpoint(path, CONFIG, 42, 1.234, params)
    meta, got = ck.read_checkpoint(path)
    assert meta["step"] == 42 and abs(meta["bestValLoss"] - 1.234) < 1e-6 and meta["config"] == CONFIG
    assert len(got) == len(params)
    for a, b in zip(got, params):
        assert a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))
    meta2, got2 = _reference_load(path)
    assert meta2 == meta
    for a, b in zip(got2, params):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_header_bytes_match_json_stringify(orc, tmp_path):
    params = _params(orc, 2)
    path = str(tmp_path / "h.bin")
    ck.write_checkpoint(path, CONFIG, 7, math.inf, params)
    buf = open(path, "rb").read()
    shapes = ",".join("[" + ",".join(str(d) for d in p.shape) + "]" for p in params)
    expected = ('{"config":{"vocabSize":32,"blockSize":8,"nLayer":2,"nHead":2,"nEmbd":16},"step":7,'
                '"bestValLoss":null,"shapes":[' + shapes + ']}').encode()
    assert buf[:8] == b"TURTCKPT"
    assert int.from_bytes(buf[8:12], "little") == len(expected)
    assert buf[12:12 + len(expected)] == expected
    assert len(buf) == 12 + len(expected) + 4 * sum(p.size for p in params)
    assert ck.read_checkpoint_meta(path)["bestValLoss"] == math.inf


def test_shape_mismatch_rejected(orc, tmp_path):
    path = str(tmp_path / "mismatch.bin")
    ck.write_checkpoint(path, CONFIG, 1, 0.0, _params(orc, 2))
    _, arrays = ck.read_checkpoint(path)
    cfg_wide = orc.cfg(32, 8, 2, 2, 32, "gpt2")
    wider = [tuple(s) for s in orc.param_shapes(cfg_wide)]
    with pytest.raises(ValueError, match="mismatch|params"):
        ck.check_shapes(wider, [a.shape for a in arrays])
    with pytest.raises(ValueError, match="params"):
        ck.check_shapes(wider[:-1], [a.shape for a in arrays])


def test_foreign_file_rejected(tmp_path):
    path = str(tmp_path / "garbage.bin")
    open(path, "wb").write(bytes([7]) * 256)
    with pytest.raises(ValueError, match="not a Turt"):
        ck.read_checkpoint(path)


def test_mulberry32_matches_oracle(orc):
    for seed in (0, 1, 42, 1337, 90000, 2 ** 32 - 1):
        st = orc.rng(seed)
        r = Mulberry32(seed)
        for _ in range(2000):
            assert r() == orc.rng_next(st)


def test_sample_batch(orc):
    tokens = (np.arange(5000) * 7919 % 8192).astype(np.uint16)
    b, t = 5, 33
    ids, tgt = sample_batch(tokens, b, t, Mulberry32(42))
    st = orc.rng(42)
    for i in range(b):
        s = math.floor(orc.rng_next(st) * (len(tokens) - t - 1))
        np.testing.assert_array_equal(ids[i * t:(i + 1) * t], tokens[s:s + t])
        np.testing.assert_array_equal(tgt[i * t:(i + 1) * t], tokens[s + 1:s + t + 1])
    with pytest.raises(ValueError):
        sample_starts(t + 1, 1, t, Mulberry32(1))


def test_lr_schedule():
    peak, warm, steps = 6e-4, 200, 20000
    assert lr_at(0, warm, steps, peak) == pytest.approx(peak / warm)
    assert lr_at(warm - 1, warm, steps, peak) == pytest.approx(peak)
    assert lr_at(warm, warm, steps, peak) == pytest.approx(peak)
    mid = warm + (steps - warm) // 2
    assert lr_at(mid, warm, steps, peak) == pytest.approx(peak * (0.1 + 0.9 * 0.5), rel=1e-3)
    assert lr_at(steps, warm, steps, peak) == pytest.approx(0.1 * peak)
    assert lr_at(10 * steps, warm, steps, peak) == pytest.approx(0.1 * peak)
