"""Synthetic token data (restates src/ferrite/model/data.py:23-34, 45-56).

``synthetic`` is the reference's offline Markov byte corpus (the TinyShakespeare
download is out of scope: no network); ``get_batch`` draws random windows;
``uniform_batch`` draws token ids uniform in [0, vocab) -- the generator the
32000-vocabulary GPT config needs (the reference's data path is byte-level).
"""

from __future__ import annotations

import numpy as np


def synthetic(n: int = 1_000_000, seed: int = 0) -> np.ndarray:
    """A learnable corpus: an order-2 Markov chain over 64 symbols, each step
    picking one of 3 successors from a random table, with 5% uniform noise
    (data.py:23-34).  uint8 bytes."""
    rng = np.random.default_rng(seed)
    table = rng.integers(0, 64, size=(64, 64, 3))
    out = np.empty(n, dtype=np.uint8)
    out[:2] = rng.integers(0, 64, size=2)
    pick = rng.integers(0, 3, size=n)
    noisy = rng.random(n) < 0.05
    uniform = rng.integers(0, 64, size=n)
    prev2, prev1 = int(out[0]), int(out[1])
    for i in range(2, n):
        nxt = int(uniform[i]) if noisy[i] else int(table[prev2, prev1, pick[i]])
        out[i] = nxt
        prev2, prev1 = prev1, nxt
    return out


def split(corpus: np.ndarray, frac: float = 0.9):
    k = int(len(corpus) * frac)
    return corpus[:k], corpus[k:]


def get_batch(rng: np.random.Generator, corpus: np.ndarray, batch: int, seq: int):
    """Random contiguous windows -> (inputs, targets) int64 [batch, seq] (data.py:51-56)."""
    starts = rng.integers(0, len(corpus) - seq - 1, size=batch)
    window = corpus[starts[:, None] + np.arange(seq + 1)[None, :]].astype(np.int64)
    return window[:, :-1].copy(), window[:, 1:].copy()


def uniform_batch(rng: np.random.Generator, batch: int, seq: int, vocab: int):
    """Token ids uniform in [0, vocab); targets are the next ids of the same stream."""
    ids = rng.integers(0, vocab, size=(batch, seq + 1), dtype=np.int64)
    return ids[:, :-1].copy(), ids[:, 1:].copy()
