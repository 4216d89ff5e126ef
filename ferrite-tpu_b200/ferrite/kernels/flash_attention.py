"""Causal flash attention (forward, dK/dV, dQ) on B200, with a custom backward.

Drop-in for the reference's ``ferrite.kernels.flash_attention``
(src/ferrite/kernels/flash_attention.py): same public names (``BlockSizes``
:49-62, ``flash_attention`` :356-367, ``flash_attention_reference`` :370-380,
``attention_flops`` :383-390, ``MASK_VALUE`` :44), same validation
(``_validate`` :336-353, raising ``ValueError``), same numerics contract:

* scores ``s = scale * q k^T`` in f32, causal mask with the finite
  ``MASK_VALUE``, online softmax with f32 row statistics, output normalised once
  after the last key block, ``lse = m + log(l)`` kept for the backward;
* ``P`` is rounded to the input dtype before ``P @ V`` (:114), ``P`` and ``dS``
  before the backward products (:210-211, :234), and the scale is applied to
  dK / dQ at the end (:220, :243);
* backward = FlashAttention-2 recompute from ``lse`` and
  ``delta = rowsum(dO * O)`` (:326-330) without atomics: dK/dV with one CTA per
  key tile sweeping query tiles, which also writes the bf16 ``dS`` it forms to a
  scratch buffer, then dQ = scale * dS K as one tensor-core GEMM per (batch,
  head) slice -- the reference's dQ kernel recomputes S, P, dP and dS instead
  (:224-243); both give the same rounded ``dS`` operand.  Without scratch (or on
  the CUDA-core path) the recompute dQ kernel runs.

The reference's ``jax.custom_vjp`` (:315-333) becomes a ``torch.autograd.Function``
whose residuals are ``(q, k, v, out, lse)``; ``lse`` and ``delta`` are compact f32
``[b, h, s]`` tensors instead of the reference's lane-replicated ``[b, h, s, 128]``
(that layout is internal to the residuals, so callers see no difference).
Block sizes are validated exactly as in the reference; the kernels tile
internally (128 x 128 on the tensor cores).
"""

from __future__ import annotations

import ctypes
import dataclasses
import math
import os

import numpy as np
import torch

from ferrite import _native as nat
from ferrite import platform

NUM_LANES = platform.LANES
# Large negative finite value instead of -inf so masked rows never produce inf - inf.
MASK_VALUE = -0.7 * float(np.finfo(np.float32).max)


@dataclasses.dataclass(frozen=True)
class BlockSizes:
    """Tile sizes. ``block_q`` is a multiple of 8, ``block_k`` a multiple of 128."""

    block_q: int = 128
    block_k: int = 128
    block_q_bwd: int = 128
    block_k_bwd: int = 128

    @classmethod
    def for_device(cls) -> "BlockSizes":
        t = platform.default_tile()
        return cls(t, t, t, t)


def _on_or_below_diag(qi: int, bq: int, ki: int, bk: int) -> bool:
    """True when block (qi, ki) has at least one unmasked (col <= row) entry (:65-67)."""
    return (qi + 1) * bq - 1 >= ki * bk


def _validate(q, k, v, causal, bs: BlockSizes):
    if not (q.ndim == 4 and k.shape == v.shape and q.shape[:2] == k.shape[:2] and q.shape[3] == k.shape[3]):
        raise ValueError(f"expected q,k,v as [b,h,s,d] with matching b,h,d; got {tuple(q.shape)} {tuple(k.shape)} {tuple(v.shape)}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, v must share a dtype")
    d = q.shape[3]
    if d % NUM_LANES and d > NUM_LANES:
        raise ValueError(f"head_dim must be <= {NUM_LANES} or a multiple of it; got {d}")
    if causal and q.shape[2] != k.shape[2]:
        raise ValueError("causal attention needs equal q and k sequence lengths")
    for name, blk, dim, mult in [
        ("block_q", bs.block_q, q.shape[2], platform.SUBLANES),
        ("block_k", bs.block_k, k.shape[2], NUM_LANES),
        ("block_q_bwd", bs.block_q_bwd, q.shape[2], platform.SUBLANES),
        ("block_k_bwd", bs.block_k_bwd, k.shape[2], NUM_LANES),
    ]:
        if blk % mult or dim % blk:
            raise ValueError(f"{name}={blk} must be a multiple of {mult} and divide the sequence length {dim}")


def _unit_d(t):
    """The kernels read any [b, h, s, d] view whose head_dim is unit-stride."""
    return t if t.stride(3) == 1 else t.contiguous()


@nat.on_tensor_device
def _forward(q, k, v, causal: bool, scale: float, bs: BlockSizes, out=None):
    """``(out, lse)``; ``out`` may be a caller-provided strided [b, h, s, d] view."""
    nat.require_cuda(q, k, v)
    b, h, sq, d = q.shape
    sk = k.shape[2]
    q, k, v = _unit_d(q), _unit_d(k), _unit_d(v)
    if out is None:
        out = torch.empty((b, h, sq, d), dtype=q.dtype, device=q.device)
    lse = torch.empty((b, h, sq), dtype=torch.float32, device=q.device)
    st = nat.attn_strides(q=q, k=k, v=v, o=out)
    nat.check(
        nat.lib().ferrite_attn_fwd_strided(
            nat.stream_ptr(q.device), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(),
            ctypes.byref(st), b, h, sq, sk, d, scale, int(causal), bs.block_q, bs.block_k, nat.dtype_code(q.dtype),
        )
    )
    return out, lse


@nat.on_tensor_device
def _backward(q, k, v, out, lse, do, causal: bool, scale: float, bs: BlockSizes, dq=None, dk=None, dv=None):
    """``(dq, dk, dv)``; the gradients may be caller-provided strided views."""
    nat.require_cuda(q, k, v, out, lse, do)
    b, h, sq, d = q.shape
    sk = k.shape[2]
    q, k, v, out = _unit_d(q), _unit_d(k), _unit_d(v), _unit_d(out)
    do = _unit_d(do.to(q.dtype))
    lib = nat.lib()
    s = nat.stream_ptr(q.device)
    code = nat.dtype_code(q.dtype)
    dq = torch.empty((b, h, sq, d), dtype=q.dtype, device=q.device) if dq is None else dq
    dk = torch.empty((b, h, sk, d), dtype=k.dtype, device=q.device) if dk is None else dk
    dv = torch.empty((b, h, sk, d), dtype=v.dtype, device=q.device) if dv is None else dv
    st = ctypes.byref(nat.attn_strides(q=q, k=k, v=v, o=out, dout=do, dq=dq, dk=dk, dv=dv))
    delta = torch.empty((b, h, sq), dtype=torch.float32, device=q.device)
    nat.check(lib.ferrite_attn_bwd_prep_strided(s, do.data_ptr(), out.data_ptr(), delta.data_ptr(), st, b, h, sq, d, code))
    ws = _ds_workspace(lib, b, h, sq, sk, d, code, q.device)
    nat.check(
        lib.ferrite_attn_bwd_ds(
            s, q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(), delta.data_ptr(),
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), st, None if ws is None else ws.data_ptr(),
            0 if ws is None else ws.numel(), b, h, sq, sk, d, scale, int(causal), bs.block_q_bwd, bs.block_k_bwd, code,
        )
    )
    return dq, dk, dv


# Upper bound on the dS scratch of one backward call; slices beyond it are
# processed in chunks (the kernels loop over them).
DS_WORKSPACE_BUDGET = int(os.environ.get("FERRITE_ATTN_DS_BUDGET_MB", "4096")) << 20


def _ds_workspace(lib, b, h, sq, sk, d, code, device):
    """Scratch for the materialised-dS backward (None: the recompute path runs)."""
    full = lib.ferrite_attn_bwd_ds_workspace_size(b, h, sq, sk, d, code)
    if not full:
        return None
    per_slice = full // (b * h)
    size = max(per_slice, min(full, DS_WORKSPACE_BUDGET // per_slice * per_slice))
    return torch.empty(size, dtype=torch.uint8, device=device)


class _Flash(torch.autograd.Function):
    """custom_vjp of ``_flash`` (flash_attention.py:315-333)."""

    @staticmethod
    def forward(ctx, q, k, v, causal, scale, bs):
        out, lse = _forward(q, k, v, causal, scale, bs)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal, ctx.scale, ctx.bs = causal, scale, bs
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = _backward(q, k, v, out, lse, do, ctx.causal, ctx.scale, ctx.bs)
        return dq, dk, dv, None, None, None


def flash_attention(q, k, v, *, causal: bool = True, scale: float | None = None, block_sizes: BlockSizes | None = None):
    """Memory-efficient attention ``softmax(q k^T * scale) v`` with exact numerics.

    Differentiable through autograd (custom backward kernels).  Shapes
    ``[batch, heads, seq, head_dim]``; sequence lengths must be multiples of the
    block sizes (pad upstream if needed).
    """
    bs = block_sizes or BlockSizes()
    _validate(q, k, v, causal, bs)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    return _Flash.apply(q, k, v, bool(causal), float(scale), bs)


def _split_packed(qkv):
    """[b, s, 3, h, d] -> q, k, v as [b, h, s, d] views (no copies)."""
    return tuple(qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))


class _FlashPacked(torch.autograd.Function):
    """Attention over a packed [b, s, 3, h, d] projection, output [b, s, h, d].

    The kernels read q, k and v in place through strided tensor maps and write
    the output, and in the backward dq/dk/dv, straight into the layouts the
    transformer block's linears use, so the head split and the transposes
    around the reference's attention call (gpt.py:136-138) cost no copies."""

    @staticmethod
    def forward(ctx, qkv, causal, scale, bs):
        b, s, _, h, d = qkv.shape
        q, k, v = _split_packed(qkv)
        out = torch.empty((b, s, h, d), dtype=qkv.dtype, device=qkv.device)
        _, lse = _forward(q, k, v, causal, scale, bs, out=out.permute(0, 2, 1, 3))
        ctx.save_for_backward(qkv, out, lse)
        ctx.causal, ctx.scale, ctx.bs = causal, scale, bs
        return out

    @staticmethod
    def backward(ctx, do):
        qkv, out, lse = ctx.saved_tensors
        q, k, v = _split_packed(qkv)
        dqkv = torch.empty_like(qkv)
        dq, dk, dv = _split_packed(dqkv)
        do = do if do.stride(3) == 1 else do.contiguous()
        _backward(q, k, v, out.permute(0, 2, 1, 3), lse, do.permute(0, 2, 1, 3), ctx.causal, ctx.scale, ctx.bs, dq=dq, dk=dk, dv=dv)
        return dqkv, None, None, None


def flash_attention_packed(qkv, *, causal: bool = True, scale: float | None = None, block_sizes: BlockSizes | None = None):
    """``flash_attention`` on a packed ``[b, s, 3, h, d]`` q/k/v projection.

    Returns ``[b, s, h, d]`` -- the same values as
    ``flash_attention(q, k, v).transpose(1, 2)`` with ``q, k, v = qkv.unbind(2)``
    transposed to ``[b, h, s, d]`` -- without materialising any transpose, in the
    forward or the backward.
    """
    if qkv.ndim != 5 or qkv.shape[2] != 3:
        raise ValueError(f"expected qkv as [b, s, 3, h, d]; got {tuple(qkv.shape)}")
    qkv = qkv if qkv.is_contiguous() else qkv.contiguous()
    bs = block_sizes or BlockSizes()
    q, k, v = _split_packed(qkv)
    _validate(q, k, v, causal, bs)
    if scale is None:
        scale = 1.0 / math.sqrt(qkv.shape[-1])
    return _FlashPacked.apply(qkv, bool(causal), float(scale), bs)


def flash_forward_with_lse(q, k, v, *, causal: bool = True, scale: float | None = None, block_sizes: BlockSizes | None = None):
    """Forward only, returning ``(out, lse)`` (lse f32 ``[b, h, s]``); no autograd."""
    bs = block_sizes or BlockSizes()
    _validate(q, k, v, causal, bs)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    return _forward(q, k, v, bool(causal), float(scale), bs)


def flash_backward(q, k, v, out, lse, do, *, causal: bool = True, scale: float | None = None, block_sizes: BlockSizes | None = None):
    """Backward only: ``(dq, dk, dv)`` from the forward residuals and ``dO``."""
    bs = block_sizes or BlockSizes()
    _validate(q, k, v, causal, bs)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    return _backward(q, k, v, out, lse, do, bool(causal), float(scale), bs)


def flash_attention_reference(q, k, v, *, causal: bool = True, scale: float | None = None):
    """Materialised-scores reference in f32, same contract as :func:`flash_attention` (:370-380)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), k.float()) * scale
    if causal:
        sq, sk = q.shape[2], k.shape[2]
        mask = torch.tril(torch.ones((sq, sk), dtype=torch.bool, device=q.device), diagonal=sk - sq)
        s = torch.where(mask, s, MASK_VALUE)  # a Python scalar: no host-to-device copy (graph-capture safe)
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhqk,bhkd->bhqd", p, v.float()).to(q.dtype)


def attention_flops(b: int, h: int, sq: int, sk: int, d: int, *, causal: bool, backward: bool = False) -> int:
    """Tensor-core FLOPs for one forward (and optionally backward) pass, counting skipped blocks as free (:383-390)."""
    frac = 0.5 if causal else 1.0
    fwd = 4 * b * h * sq * sk * d * frac  # QK^T and PV, 2 flops per MAC
    if not backward:
        return int(fwd)
    # backward recomputes S (1 matmul) and does dP, dV, dK, dQ (4 matmuls) = 5 matmuls vs 2 in forward
    return int(fwd * 2.5)
