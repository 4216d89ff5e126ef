"""Flash-attention oracle (numpy) -- test infrastructure only; see ``oracle/__init__.py``.

Restates src/ferrite/kernels/flash_attention.py of anxnd2211/ferrite-tpu:
  * ``reference_fwd``   flash_attention_reference :370-380 (materialised f32
                        scores, finite MASK_VALUE :44, softmax, cast back),
  * ``reference_bwd``   the analytic VJP of that reference (what ``jax.grad`` of
                        it computes in the reference tests :242-263), in f32 or
                        f64, with the gradients cast to the input dtype,
  * ``flash_fwd``       the blockwise forward _fwd_kernel :91-127 (online
                        softmax, causal block skip :65-67/:117-118, P rounded to
                        v.dtype before P@V :114, normalise once at the end
                        :122-127, lse = m + log l),
  * ``flash_bwd``       delta (:326-330), _recompute_p_ds :184-194,
                        _bwd_dkv_kernel :197-221 and _bwd_dq_kernel :224-243
                        (P and dS rounded to the operand dtype before each
                        product, scale applied to dK/dQ at the end).
and, from src/ferrite/serving/engine.py,
  * ``decode_reference`` the decode step's cache write and cache attention
                        (:89-104).
Arrays are ``[b, h, s, d]``; bfloat16 is ``ml_dtypes.bfloat16``.  The (b, h)
slices are independent, so callers may pass a subset of heads.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32
MASK_VALUE = -0.7 * float(np.finfo(np.float32).max)


def _scale(d: int, scale):
    return 1.0 / math.sqrt(d) if scale is None else float(scale)


def _mask(sq: int, sk: int) -> np.ndarray:
    """jnp.tril(ones((sq, sk)), k=sk-sq) (flash_attention.py:377)."""
    return np.tril(np.ones((sq, sk), dtype=bool), k=sk - sq)


def reference_fwd(q, k, v, causal=True, scale=None, acc=F32):
    """Materialised reference (flash_attention.py:370-380); returns q.dtype."""
    scale = _scale(q.shape[-1], scale)
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(acc), k.astype(acc)) * acc(scale)
    if causal:
        s = np.where(_mask(q.shape[2], k.shape[2]), s, acc(MASK_VALUE))
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v.astype(acc)).astype(q.dtype)


def reference_bwd(q, k, v, do, causal=True, scale=None, acc=F32):
    """Gradients (dq, dk, dv) of sum(reference_fwd(q,k,v) * do), in q.dtype."""
    scale = _scale(q.shape[-1], scale)
    qf, kf, vf, dof = (a.astype(acc) for a in (q, k, v, do))
    s = np.einsum("bhqd,bhkd->bhqk", qf, kf) * acc(scale)
    if causal:
        s = np.where(_mask(q.shape[2], k.shape[2]), s, acc(MASK_VALUE))
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(-1, keepdims=True)
    dv = np.einsum("bhqk,bhqd->bhkd", p, dof)
    dp = np.einsum("bhqd,bhkd->bhqk", dof, vf)
    ds = p * (dp - np.sum(dp * p, -1, keepdims=True))
    dq = np.einsum("bhqk,bhkd->bhqd", ds, kf) * acc(scale)
    dk = np.einsum("bhqk,bhqd->bhkd", ds, qf) * acc(scale)
    return dq.astype(q.dtype), dk.astype(k.dtype), dv.astype(v.dtype)


def _on_or_below_diag(qi, bq, ki, bk) -> bool:
    """flash_attention.py:65-67."""
    return (qi + 1) * bq - 1 >= ki * bk


def _causal_mask_block(s, qi, ki, bq, bk):
    """flash_attention.py:80-83 (iota compare, MASK_VALUE)."""
    rows = qi * bq + np.arange(bq)[:, None]
    cols = ki * bk + np.arange(bk)[None, :]
    return np.where(cols <= rows, s, F32(MASK_VALUE))


def _round(x: np.ndarray, dtype) -> np.ndarray:
    """Round an f32 array to ``dtype`` and back (the ``.astype(x.dtype)`` points)."""
    return x.astype(dtype).astype(F32)


def flash_fwd(q, k, v, causal=True, scale=None, bq=128, bk=128):
    """Blockwise forward (flash_attention.py:91-175); returns (out [q.dtype], lse f32 [b,h,s])."""
    b, h, sq, d = q.shape
    sk = k.shape[2]
    scale = _scale(d, scale)
    nq, nk = sq // bq, sk // bk
    out = np.empty(q.shape, q.dtype)
    lse = np.empty((b, h, sq), F32)
    qf, kf, vf = q.astype(F32), k.astype(F32), v.astype(F32)
    for qi in range(nq):
        qb = qf[:, :, qi * bq:(qi + 1) * bq]
        m = np.full((b, h, bq), -np.inf, F32)
        l = np.zeros((b, h, bq), F32)
        accum = np.zeros((b, h, bq, d), F32)
        for ki in range(nk):
            if causal and not _on_or_below_diag(qi, bq, ki, bk):
                continue
            kb, vb = kf[:, :, ki * bk:(ki + 1) * bk], vf[:, :, ki * bk:(ki + 1) * bk]
            s = np.matmul(qb, kb.transpose(0, 1, 3, 2))
            if scale != 1.0:
                s = s * F32(scale)
            if causal:
                s = _causal_mask_block(s, qi, ki, bq, bk)
            m_next = np.maximum(m, s.max(-1))
            p = np.exp(s - m_next[..., None])
            alpha = np.exp(m - m_next)
            l = alpha * l + p.sum(-1, dtype=F32)
            m = m_next
            pv = np.matmul(_round(p, v.dtype), vb)
            accum = accum * alpha[..., None] + pv
        out[:, :, qi * bq:(qi + 1) * bq] = (accum * (F32(1.0) / l)[..., None]).astype(q.dtype)
        lse[:, :, qi * bq:(qi + 1) * bq] = m + np.log(l)
    return out, lse


def delta(do, out):
    """rowsum(dO * O) in f32 (flash_attention.py:328)."""
    return np.sum(do.astype(F32) * out.astype(F32), axis=-1, dtype=F32)


def _recompute_p_ds(qb, kb, vb, dob, lseb, deltab, scale, causal, qi, ki, bq, bk):
    """flash_attention.py:184-194 on f32 blocks [b,h,bq,d] / [b,h,bk,d]."""
    s = np.matmul(qb, kb.transpose(0, 1, 3, 2))
    if scale != 1.0:
        s = s * F32(scale)
    if causal:
        s = _causal_mask_block(s, qi, ki, bq, bk)
    p = np.exp(s - lseb[..., None])
    dp = np.matmul(dob, vb.transpose(0, 1, 3, 2))
    ds = p * (dp - deltab[..., None])
    return p, ds


def flash_bwd(q, k, v, out, lse, do, causal=True, scale=None, bq=128, bk=128):
    """Blockwise backward (flash_attention.py:197-307): returns (dq, dk, dv)."""
    b, h, sq, d = q.shape
    sk = k.shape[2]
    scale = _scale(d, scale)
    nq, nk = sq // bq, sk // bk
    dlt = delta(do, out)
    qf, kf, vf, dof = (a.astype(F32) for a in (q, k, v, do))
    dq = np.empty(q.shape, q.dtype)
    dk = np.empty(k.shape, k.dtype)
    dv = np.empty(v.shape, v.dtype)
    # dK, dV: kv block outer, q block inner (:197-221)
    for ki in range(nk):
        kb, vb = kf[:, :, ki * bk:(ki + 1) * bk], vf[:, :, ki * bk:(ki + 1) * bk]
        dk_acc = np.zeros((b, h, bk, d), F32)
        dv_acc = np.zeros((b, h, bk, d), F32)
        for qi in range(nq):
            if causal and not _on_or_below_diag(qi, bq, ki, bk):
                continue
            sl = slice(qi * bq, (qi + 1) * bq)
            p, ds = _recompute_p_ds(qf[:, :, sl], kb, vb, dof[:, :, sl], lse[:, :, sl], dlt[:, :, sl], scale, causal, qi, ki, bq, bk)
            dv_acc += np.matmul(_round(p, do.dtype).transpose(0, 1, 3, 2), dof[:, :, sl])
            dk_acc += np.matmul(_round(ds, q.dtype).transpose(0, 1, 3, 2), qf[:, :, sl])
        dk[:, :, ki * bk:(ki + 1) * bk] = (dk_acc * F32(scale)).astype(k.dtype)
        dv[:, :, ki * bk:(ki + 1) * bk] = dv_acc.astype(v.dtype)
    # dQ: q block outer, kv block inner (:224-243)
    for qi in range(nq):
        sl = slice(qi * bq, (qi + 1) * bq)
        dq_acc = np.zeros((b, h, bq, d), F32)
        for ki in range(nk):
            if causal and not _on_or_below_diag(qi, bq, ki, bk):
                continue
            kb, vb = kf[:, :, ki * bk:(ki + 1) * bk], vf[:, :, ki * bk:(ki + 1) * bk]
            _, ds = _recompute_p_ds(qf[:, :, sl], kb, vb, dof[:, :, sl], lse[:, :, sl], dlt[:, :, sl], scale, causal, qi, ki, bq, bk)
            dq_acc += np.matmul(_round(ds, k.dtype), kb)
        dq[:, :, sl] = (dq_acc * F32(scale)).astype(q.dtype)
    return dq, dk, dv


def attention_flops(b, h, sq, sk, d, causal=True, backward=False) -> int:
    """flash_attention.py:383-390."""
    frac = 0.5 if causal else 1.0
    fwd = 4 * b * h * sq * sk * d * frac
    return int(fwd if not backward else fwd * 2.5)


def decode_reference(q, k_cache, v_cache, pos, scale, k_new=None, v_new=None):
    """One decode step against a static KV cache, src/ferrite/serving/engine.py of the
    reference: ``_write_cache`` :98-104 (the new row stored at ``pos[b]``, cast to the
    cache dtype) then ``_cache_attention`` :89-95 (f32 scores over every cache
    position, positions after ``pos[b]`` set to -1e30, softmax, P V in f32, cast to
    q's dtype).

    q [b, h, d]; k_cache, v_cache [b, h, max_len, d]; pos [b] ints in [0, max_len);
    k_new / v_new [b, h, d] or None.  Returns (o [b, h, d], k_cache, v_cache), the
    caches as new arrays.
    """
    kc, vc = k_cache.copy(), v_cache.copy()
    pos = np.asarray(pos, dtype=np.int64)
    assert np.all((pos >= 0) & (pos < kc.shape[2])), "pos outside the cache"
    if k_new is not None:
        for bi, p in enumerate(pos):
            kc[bi, :, p] = k_new[bi].astype(kc.dtype)
            vc[bi, :, p] = v_new[bi].astype(vc.dtype)
    s = np.einsum("bhd,bhkd->bhk", q.astype(F32), kc.astype(F32)) * F32(scale)
    idx = np.arange(kc.shape[2])[None, :]
    s = np.where((idx <= pos[:, None])[:, None, :], s, F32(-1e30))
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(-1, keepdims=True)
    return np.einsum("bhk,bhkd->bhd", p, vc.astype(F32)).astype(q.dtype), kc, vc
