"""Checkpoints in the reference's portable format, and AdamW state beside them.

TURTCKPT (scripts/checkpoint.ts:21-60,99-123): the 8 ASCII bytes "TURTCKPT", a little-endian
uint32 header length, a UTF-8 JSON header {config, step, bestValLoss, shapes} and then every
parameter as raw little-endian float32 in parameters() order.  Files written here load with the
reference's `loadCheckpoint` (generate.ts, chat, resume of gpu-pretrain.ts) and the reference's
files load here; shapes are checked on load so that a mismatch fails loudly.

The reference format has no optimizer state, so gpu-pretrain.ts restarts AdamW's moments at
zero on --resume (scripts/gpu-pretrain.ts:171-173).  `save_optimizer_state` writes them to a
sidecar file (<checkpoint>.adam: "TURTADAM", uint32 header length, JSON {adamStep, shapes},
then all first moments and all second moments in parameters() order), leaving the checkpoint
itself readable by the reference.
"""
from __future__ import annotations

import json
import math
import struct

import numpy as np

MAGIC = b"TURTCKPT"
ADAM_MAGIC = b"TURTADAM"


def config_dict(cfg) -> dict:
    """GPTConfig (src/models/gpt.ts:40-51) of a turt_config: vocabSize, blockSize, nLayer, nHead,
    nEmbd, arch.  A hidden-width override has no GPTConfig field; it is recorded as mlpHidden,
    which the reference ignores (its model then fails the shape check, as it should)."""
    d = {"vocabSize": cfg.vocab_size, "blockSize": cfg.block_size, "nLayer": cfg.n_layer, "nHead": cfg.n_head,
         "nEmbd": cfg.n_embd, "arch": "modern" if cfg.arch == 1 else "gpt2"}
    if cfg.hidden:
        d["mlpHidden"] = cfg.hidden
    return d


def _js_number(x):
    # JSON.stringify writes non-finite numbers as null (bestValLoss starts at Infinity)
    return x if isinstance(x, (int,)) or math.isfinite(x) else None


def _pack(magic: bytes, header: dict, blocks) -> bytes:
    head = json.dumps(header, separators=(",", ":")).encode("utf-8")
    out = [magic.ljust(8, b"\0"), struct.pack("<I", len(head)), head]
    out += [np.ascontiguousarray(b, dtype="<f4").tobytes() for b in blocks]
    return b"".join(out)


def _unpack(buf: bytes, magic: bytes, path: str):
    if buf[:8].rstrip(b"\0") != magic.rstrip(b"\0"):
        what = "Turt checkpoint" if magic == MAGIC else "Turt optimizer state"
        raise ValueError(f"{path} is not a {what}")
    (n,) = struct.unpack_from("<I", buf, 8)
    return json.loads(buf[12:12 + n].decode("utf-8")), 12 + n


def write_checkpoint(path: str, config: dict, step: int, best_val_loss: float, params) -> None:
    """Writes `params` (arrays in parameters() order) as a TURTCKPT file."""
    params = [np.asarray(p, dtype=np.float32) for p in params]
    meta = {"config": config, "step": int(step), "bestValLoss": _js_number(float(best_val_loss)),
            "shapes": [list(p.shape) for p in params]}
    with open(path, "wb") as f:
        f.write(_pack(MAGIC, meta, params))


def read_checkpoint_meta(path: str) -> dict:
    """The JSON header only (checkpoint.ts readCheckpointMeta); bestValLoss null -> inf."""
    with open(path, "rb") as f:
        buf = f.read()
    meta, _ = _unpack(buf, MAGIC, path)
    if meta.get("bestValLoss") is None:
        meta["bestValLoss"] = math.inf
    return meta


def read_checkpoint(path: str):
    """(meta, [arrays of the recorded shapes]) from a TURTCKPT file."""
    with open(path, "rb") as f:
        buf = f.read()
    meta, off = _unpack(buf, MAGIC, path)
    if meta.get("bestValLoss") is None:
        meta["bestValLoss"] = math.inf
    arrays = []
    for shp in meta["shapes"]:
        n = int(np.prod(shp)) if shp else 1
        if off + 4 * n > len(buf):
            raise ValueError(f"{path} is truncated")
        arrays.append(np.frombuffer(buf, dtype="<f4", count=n, offset=off).astype(np.float32).reshape(shp))
        off += 4 * n
    return meta, arrays


def check_shapes(expected, got) -> None:
    """loadCheckpoint's count and per-parameter shape checks (checkpoint.ts:103-115)."""
    if len(expected) != len(got):
        raise ValueError(f"Checkpoint has {len(got)} params, model has {len(expected)}")
    for i, (e, g) in enumerate(zip(expected, got)):
        if tuple(e) != tuple(g):
            raise ValueError(f"Param {i} shape mismatch: checkpoint [{','.join(map(str, g))}], "
                             f"model [{','.join(map(str, e))}]")


def save_checkpoint(path: str, model, step: int, best_val_loss: float) -> None:
    """Downloads the device parameters of a turt_b200 Model into a TURTCKPT file."""
    write_checkpoint(path, config_dict(model.cfg), step, best_val_loss, model.param_list())


def load_checkpoint(path: str, model) -> dict:
    """Uploads a TURTCKPT file into a Model of the same shapes; returns the header."""
    meta, arrays = read_checkpoint(path)
    check_shapes([tuple(s) for s in model.shapes], [tuple(a.shape) for a in arrays])
    model.load_param_list(arrays)
    return meta


def save_optimizer_state(path: str, model, adam_step: int) -> None:
    """AdamW moments and the bias-correction step count into a TURTADAM sidecar file."""
    ms, vs = model.adam_state()
    header = {"adamStep": int(adam_step), "shapes": [list(m.shape) for m in ms]}
    with open(path, "wb") as f:
        f.write(_pack(ADAM_MAGIC, header, ms + vs))


def load_optimizer_state(path: str, model) -> int:
    """Restores AdamW moments from a TURTADAM file; returns the step count they belong to."""
    with open(path, "rb") as f:
        buf = f.read()
    header, off = _unpack(buf, ADAM_MAGIC, path)
    shapes = [tuple(s) for s in header["shapes"]]
    check_shapes([tuple(s) for s in model.shapes], shapes)
    arrays = []
    for shp in shapes + shapes:
        n = int(np.prod(shp))
        arrays.append(np.frombuffer(buf, dtype="<f4", count=n, offset=off).reshape(shp))
        off += 4 * n
    k = len(shapes)
    model.load_adam_state(arrays[:k], arrays[k:])
    return int(header["adamStep"])
