"""Sampling continuations from a GPU model: GPT.generate with a KV cache.

GPT.generate (src/models/gpt.ts:291-321) re-runs the whole forward over the last blockSize
tokens for every new token and samples from the last position's logits.  Here the forward of
a context that still fits the block is split into one prefill (turt_generate_prefill, which
fills the per-layer key / value cache) and one decode step per new token
(turt_generate_step); once the context outgrows the block the window slides, every position
shifts, and each token re-prefills the cropped window, as the reference does.  The logits come
back to the host, where temperature, top-k and sampleFromLogits (gpt.ts:324-341) run with the
reference's arithmetic: f32 logits divided by the temperature into a Float32Array, the top-k
threshold taken from a descending sort, exp in double stored as f32 probabilities whose double
sum scales rng(), and a sequential subtraction scan.
"""
from __future__ import annotations

from typing import Callable, Iterable, List, Optional

import numpy as np

from .pretrain import Mulberry32

# The reference's module-level defaultRng (src/math/random.ts:27): one mulberry32(42) stream
# shared by every call that passes no rng.
default_rng = Mulberry32(42)


def apply_temperature_top_k(logits: np.ndarray, temperature: float = 1.0, top_k: Optional[int] = None) -> np.ndarray:
    """last[j] = logits[j] / temperature (stored as f32); with 0 < top_k < V, entries below the
    top_k-th largest become -inf (gpt.ts:306-314)."""
    last = (np.asarray(logits, dtype=np.float32).astype(np.float64) / float(temperature)).astype(np.float32)
    V = last.shape[0]
    if top_k and top_k < V:
        threshold = np.sort(last)[::-1][top_k - 1]
        last[last < threshold] = -np.inf
    return last


def sample_from_logits(logits: np.ndarray, rng: Callable[[], float]) -> int:
    """sampleFromLogits (gpt.ts:324-341): one index drawn from softmax(logits)."""
    last = np.asarray(logits, dtype=np.float32)
    mx = float(np.max(last)) if last.size else -np.inf
    e = np.exp(last.astype(np.float64) - mx)
    probs = e.astype(np.float32)
    total = float(np.cumsum(e)[-1])  # a sequential double sum, as the reference's loop
    r = rng() * total
    # r -= probs[j] one after another; the first j where r <= 0 is drawn
    scan = np.subtract.accumulate(np.concatenate(([r], probs.astype(np.float64))))[1:]
    hit = np.flatnonzero(scan <= 0)
    return int(hit[0]) if hit.size else last.shape[0] - 1


class Generator:
    """KV-cached decoding state of one model: which window of ids the cache holds."""

    def __init__(self, model):
        self.model = model
        self.block = model.cfg.block_size
        self.win_start = 0
        self.cached = 0

    def next_logits(self, ids: List[int]) -> np.ndarray:
        """Logits of the last position of ids[-block_size:]: one decode step when the cache
        already holds every earlier position of that window, else a prefill of the window."""
        if not ids:
            raise ValueError("generate: the prompt must hold at least one token")
        start = max(0, len(ids) - self.block)
        if self.cached > 0 and start == self.win_start and self.win_start + self.cached == len(ids) - 1:
            out = self.model.generate_step(ids[-1], self.cached)
            self.cached += 1
            return out
        out = self.model.generate_prefill(ids[start:])
        self.win_start, self.cached = start, len(ids) - start
        return out


def generate(model, prompt: Iterable[int], max_new_tokens: int, temperature: float = 1.0,
             top_k: Optional[int] = None, rng: Optional[Callable[[], float]] = None,
             on_token: Optional[Callable[[int], Optional[bool]]] = None) -> List[int]:
    """GPT.generate on the GPU model: returns prompt + sampled ids; on_token returning False
    stops early (gpt.ts:291-321)."""
    rng = default_rng if rng is None else rng
    ids = [int(i) for i in prompt]
    gen = Generator(model)
    for _ in range(max_new_tokens):
        last = apply_temperature_top_k(gen.next_logits(ids), temperature, top_k)
        nxt = sample_from_logits(last, rng)
        ids.append(nxt)
        if on_token is not None and on_token(nxt) is False:
            break
    return ids
