"""Matmul oracle (numpy) -- test infrastructure only; see ``oracle/__init__.py``.

Restates src/ferrite/kernels/matmul.py of anxnd2211/ferrite-tpu:
  * ``matmul_reference``  matmul.py:129-131: f32 accumulation, cast to out dtype
                          (bf16 products are exact in f32; ``acc=np.float64``
                          gives the float64 twin used for the f32 HIGHEST case),
  * ``matmul_vjp``        matmul.py:99-104: dX = G Y^T (in x.dtype),
                          dY = X^T G (in y.dtype), G cast to the operand dtype
                          first.  Zero padding (:58-63) contributes nothing, so
                          ragged shapes need no special case here.
"""

from __future__ import annotations

import numpy as np


def matmul_reference(x: np.ndarray, y: np.ndarray, out_dtype=None, acc=np.float32) -> np.ndarray:
    return np.matmul(x.astype(acc), y.astype(acc)).astype(out_dtype or x.dtype)


def matmul_vjp(x: np.ndarray, y: np.ndarray, g: np.ndarray, acc=np.float32):
    gx = g.astype(x.dtype)
    gy = g.astype(y.dtype)
    dx = np.matmul(gx.astype(acc), y.astype(acc).T).astype(x.dtype)
    dy = np.matmul(x.astype(acc).T, gy.astype(acc)).astype(y.dtype)
    return dx, dy


def matmul_flops(m: int, n: int, k: int) -> int:
    """matmul.py:134-135."""
    return 2 * m * n * k
