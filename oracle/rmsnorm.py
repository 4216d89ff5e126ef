"""RMSNorm oracle (numpy) -- test infrastructure only; see ``oracle/__init__.py``.

Restates src/ferrite/kernels/rmsnorm.py of anxnd2211/ferrite-tpu:
  * ``rmsnorm_reference``  rmsnorm.py:193-199 (the plain-JAX reference),
  * ``add_rmsnorm_fwd``    _add_rmsnorm_kernel rmsnorm.py:52-56 with _inv_rms :39-43
                           (y from the unrounded f32 h; h and y rounded to x.dtype),
  * ``rmsnorm_fwd``        _rmsnorm_kernel rmsnorm.py:46-49,
  * ``rmsnorm_bwd``        _rmsnorm_bwd_math rmsnorm.py:159-166 plus
                           _add_norm_bwd :148-153 (dh + dh_direct, returned twice)
                           and _norm_bwd :128-131.
All statistics are float32 (``acc=np.float64`` gives the float64 twin used to
triage rounding differences).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def _inv_rms(h: np.ndarray, eps: float, acc=F32) -> np.ndarray:
    """1/sqrt(mean(h^2) + eps) per row (rmsnorm.py:39-43)."""
    dim = h.shape[-1]
    ss = np.sum(h * h, axis=-1, keepdims=True, dtype=acc)
    return (1.0 / np.sqrt(ss * acc(1.0 / dim) + acc(eps))).astype(acc)


def rmsnorm_fwd(x: np.ndarray, w: np.ndarray, eps: float = 1e-6, acc=F32) -> np.ndarray:
    """y = x * inv_rms(x) * w in f32, rounded to x.dtype (rmsnorm.py:46-49)."""
    h = x.astype(acc)
    y = h * _inv_rms(h, eps, acc) * w.astype(acc)
    return y.astype(x.dtype)


def add_rmsnorm_fwd(x: np.ndarray, r: np.ndarray, w: np.ndarray, eps: float = 1e-6, acc=F32):
    """(h, y): h = x + r in f32; y from the UNROUNDED h (rmsnorm.py:52-56)."""
    h = x.astype(acc) + r.astype(acc)
    y = h * _inv_rms(h, eps, acc) * w.astype(acc)
    return h.astype(x.dtype), y.astype(x.dtype)


def rmsnorm_reference(x, w, residual=None, eps: float = 1e-6, acc=F32):
    """The reference's plain reference (rmsnorm.py:193-199)."""
    if residual is None:
        return rmsnorm_fwd(x, w, eps, acc)
    return add_rmsnorm_fwd(x, residual, w, eps, acc)


def rmsnorm_bwd(h: np.ndarray, w: np.ndarray, dy: np.ndarray, dh_direct: np.ndarray | None = None, eps: float = 1e-6, acc=F32):
    """(dh, dw) from the saved rounded h (rmsnorm.py:159-166, :148-153).

    dh is rounded to h.dtype, dw to w.dtype.  With ``dh_direct`` the reference
    returns ``(dh, dh, dw)`` (dx = dr = dh); callers take dh twice.
    """
    hf, wf, dyf = h.astype(acc), w.astype(acc), dy.astype(acc)
    dim = h.shape[-1]
    inv = 1.0 / np.sqrt(np.mean(hf * hf, axis=-1, keepdims=True, dtype=acc) + acc(eps))
    xhat = hf * inv
    dw = np.sum(dyf * xhat, axis=0, dtype=acc)
    dxhat = dyf * wf
    dh = inv * (dxhat - xhat * np.mean(dxhat * xhat, axis=-1, keepdims=True, dtype=acc))
    if dh_direct is not None:
        dh = dh + dh_direct.astype(acc)
    del dim
    return dh.astype(h.dtype), dw.astype(w.dtype)
