"""Softmax cross-entropy oracle (numpy) -- test infrastructure only; see ``oracle/__init__.py``.

Restates the training loss of anxnd2211/ferrite-tpu, src/ferrite/model/gpt.py:147-152
(``loss_fn``): ``logp = jax.nn.log_softmax(logits)`` over the vocabulary in f32,
``nll = -logp[target]``, loss = mean(nll); and its gradient with respect to the
logits, ``(softmax(logits) - onehot(target)) / rows`` (the VJP of that
expression, scaled by the upstream gradient).  ``acc=np.float64`` gives the
float64 twin for triage.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def lse(logits: np.ndarray, acc=F32) -> np.ndarray:
    """log(sum(exp(x))) per row with the max subtracted first (log_softmax's form)."""
    x = logits.astype(acc)
    m = np.max(x, axis=-1, keepdims=True)
    return (m[..., 0] + np.log(np.sum(np.exp(x - m), axis=-1, dtype=acc))).astype(acc)


def xent_fwd(logits: np.ndarray, targets: np.ndarray, acc=F32):
    """(lse, nll) per row; nll = lse - x[target] (= -log_softmax(x)[target])."""
    l = lse(logits, acc)
    picked = np.take_along_axis(logits.astype(acc), targets.reshape(-1, 1).astype(np.int64), axis=-1)[:, 0]
    return l, (l - picked).astype(acc)


def loss(logits: np.ndarray, targets: np.ndarray, acc=F32) -> float:
    """Mean next-token cross-entropy (gpt.py:147-152)."""
    return float(np.mean(xent_fwd(logits, targets, acc)[1], dtype=acc))


def xent_bwd(logits: np.ndarray, targets: np.ndarray, g: float = 1.0, acc=F32) -> np.ndarray:
    """d loss / d logits for loss = mean(nll): g * (softmax - onehot) / rows, in f32."""
    rows = logits.shape[0]
    x = logits.astype(acc)
    p = np.exp(x - lse(logits, acc)[:, None])
    p[np.arange(rows), targets.reshape(-1).astype(np.int64)] -= acc(1.0)
    return (p * acc(g / rows)).astype(acc)
