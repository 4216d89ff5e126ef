"""Decode attention against a static KV cache, with the cache write fused in.

The reference runs its decode step in XLA (src/ferrite/serving/engine.py:12-15):
``_write_cache`` (:98-104) stores the new token's K/V row at ``pos[b]``, then
``_cache_attention`` (:89-95) computes f32 scores of the one query row against
every cache position, masks the positions after ``pos[b]`` to -1e30, and takes
the softmax-weighted sum of V.  :func:`decode_attention` does both in one kernel
(``ferrite_attn_decode``): it reads only the rows ``<= pos[b]`` (a masked row's
weight is exactly 0 in f32), splits them over a thread-block cluster per
(batch, head) and merges the partial softmax states in distributed shared memory.
"""

from __future__ import annotations

import math

import torch

from ferrite import _native as nat

_HEAD_DIMS = {torch.bfloat16: (32, 64, 128, 256), torch.float16: (32, 64, 128, 256), torch.float32: (32, 64, 128)}


@nat.on_tensor_device
def decode_attention(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    pos: torch.Tensor,
    *,
    scale: float | None = None,
    k_new: torch.Tensor | None = None,
    v_new: torch.Tensor | None = None,
) -> torch.Tensor:
    """softmax(scale * q K^T) V over the cache positions ``<= pos[b]``; returns ``[b, h, d]``.

    q, k_new, v_new: ``[b, h, d]`` with unit-stride d and head stride d; they share
    one batch stride (the slots of a ``[b, 3, h, d]`` projection are read in place).
    k_cache, v_cache: ``[b, h, max_len, d]``, contiguous (one layer of the
    ``[L, b, h, max_len, d]`` cache).  pos: ``[b]`` integer positions, each in
    ``[0, max_len)``.  With k_new / v_new given, they are written into the caches at
    ``pos`` (in place) and attended to, as the reference's decode step does.
    """
    nat.require_cuda(q, k_cache, v_cache, pos, k_new, v_new)
    if q.dim() != 3 or k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError(f"expected q [b, h, d] and caches [b, h, max_len, d]; got {tuple(q.shape)}, {tuple(k_cache.shape)}, {tuple(v_cache.shape)}")
    b, h, d = q.shape
    if k_cache.shape[0] != b or k_cache.shape[1] != h or k_cache.shape[3] != d:
        raise ValueError(f"cache {tuple(k_cache.shape)} does not match q {tuple(q.shape)}")
    if (k_new is None) != (v_new is None):
        raise ValueError("k_new and v_new must be given together")
    dtypes = {q.dtype, k_cache.dtype, v_cache.dtype} | ({k_new.dtype, v_new.dtype} if k_new is not None else set())
    if len(dtypes) != 1:
        raise ValueError(f"q, caches and new rows must share one dtype; got {sorted(map(str, dtypes))}")
    if q.dtype not in _HEAD_DIMS or d not in _HEAD_DIMS[q.dtype]:
        raise ValueError(f"head_dim {d} with {q.dtype} is not supported (head dims {_HEAD_DIMS.get(q.dtype, ())})")
    if pos.shape != (b,):
        raise ValueError(f"pos must have shape ({b},); got {tuple(pos.shape)}")
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    k_cache, v_cache = _dense(k_cache, "k_cache"), _dense(v_cache, "v_cache")
    rows = [q] + ([k_new, v_new] if k_new is not None else [])
    ld = q.stride(0)
    if any(t.stride(2) != 1 or t.stride(1) != d or t.stride(0) != ld or t.data_ptr() % 16 for t in rows) or ld % (16 // q.element_size()):
        rows = [t.contiguous() for t in rows]
        ld = h * d
    pos = pos.to(torch.int64).contiguous()
    out = torch.empty(b, h, d, dtype=q.dtype, device=q.device)
    kn = rows[1] if k_new is not None else None
    vn = rows[2] if k_new is not None else None
    nat.check(
        nat.lib().ferrite_attn_decode(
            nat.stream_ptr(q.device), rows[0].data_ptr(), nat.ptr(kn), nat.ptr(vn), k_cache.data_ptr(), v_cache.data_ptr(),
            pos.data_ptr(), out.data_ptr(), b, h, k_cache.shape[2], d, ld, scale, nat.dtype_code(q.dtype),
        )
    )
    return out


def _dense(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous (the cache is updated in place)")
    return t


def decode_attention_reference(q, k_cache, v_cache, pos, scale=None):
    """The reference's ``_cache_attention`` (serving/engine.py:89-95) in torch f32: every
    cache position scored, positions after ``pos[b]`` masked to -1e30."""
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    s = torch.einsum("bhd,bhkd->bhk", q.float(), k_cache.float()) * scale
    idx = torch.arange(k_cache.shape[2], device=q.device)[None, :]
    s = torch.where((idx <= pos[:, None])[:, None, :], s, -1e30)
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhk,bhkd->bhd", p, v_cache.float()).to(q.dtype)
