"""Fused residual-add + RMSNorm on B200, with a custom backward.

Drop-in for the reference's ``ferrite.kernels.rmsnorm`` (src/ferrite/kernels/rmsnorm.py):
same public functions (``rmsnorm`` :174-190, ``rmsnorm_reference`` :193-199),
same argument meaning and errors (``ValueError`` for a weight of the wrong shape
:181-182, a residual that does not match :187-188, or ``block_rows`` that is not
a multiple of 8 :72-73), same numerics (f32 statistics; y from the unrounded f32
``h = x + residual``; backward from the saved rounded ``h``; ``dx = dr = dh``).

The reference's ``jax.custom_vjp`` pairs (``_norm`` :118-134, ``_add_norm``
:137-156) become ``torch.autograd.Function``s whose forward and backward both
call the native library (the reference leaves its backward to XLA; here it is
one CUDA kernel plus a deterministic dw reduction).  ``block_rows`` is accepted
and validated but the kernel picks its own row tiling.
"""

from __future__ import annotations

import torch

from ferrite import _native as nat
from ferrite import platform


def _check_block_rows(block_rows):
    if block_rows is not None and block_rows % platform.SUBLANES:
        raise ValueError(f"block_rows must be a multiple of {platform.SUBLANES}")


@nat.on_tensor_device
def _fwd(x2d: torch.Tensor, w: torch.Tensor, r2d: torch.Tensor | None, eps: float):
    nat.require_cuda(x2d, w, r2d)
    rows, dim = x2d.shape
    y = torch.empty_like(x2d)
    lib = nat.lib()
    s = nat.stream_ptr(x2d.device)
    if r2d is None:
        nat.check(lib.ferrite_rmsnorm_fwd(s, x2d.data_ptr(), w.data_ptr(), y.data_ptr(), rows, dim, eps, nat.dtype_code(x2d.dtype), nat.dtype_code(w.dtype)))
        return None, y
    h = torch.empty_like(x2d)
    nat.check(
        lib.ferrite_add_rmsnorm_fwd(
            s, x2d.data_ptr(), r2d.data_ptr(), w.data_ptr(), h.data_ptr(), y.data_ptr(), rows, dim, eps, nat.dtype_code(x2d.dtype), nat.dtype_code(w.dtype)
        )
    )
    return h, y


@nat.on_tensor_device
def rmsnorm_backward(h: torch.Tensor, w: torch.Tensor, dy: torch.Tensor, dh_direct: torch.Tensor | None, eps: float):
    """Native backward: returns (dh, dw) with dh in h.dtype and dw in w.dtype."""
    nat.require_cuda(h, w, dy, dh_direct)
    rows, dim = h.shape
    dy = dy.to(h.dtype).contiguous()
    if dh_direct is not None:
        dh_direct = dh_direct.to(h.dtype).contiguous()
    dh = torch.empty_like(h)
    dw = torch.empty_like(w)
    lib = nat.lib()
    ws_bytes = int(lib.ferrite_rmsnorm_bwd_workspace_size(rows, dim))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=h.device)
    nat.check(
        lib.ferrite_rmsnorm_bwd(
            nat.stream_ptr(h.device),
            h.data_ptr(),
            w.data_ptr(),
            dy.data_ptr(),
            nat.ptr(dh_direct),
            dh.data_ptr(),
            dw.data_ptr(),
            ws.data_ptr(),
            ws.numel(),
            rows,
            dim,
            eps,
            nat.dtype_code(h.dtype),
            nat.dtype_code(w.dtype),
        )
    )
    return dh, dw


class _Norm(torch.autograd.Function):
    """custom_vjp of ``_norm`` (rmsnorm.py:118-134)."""

    @staticmethod
    def forward(ctx, x2d, w, eps):
        _, y = _fwd(x2d, w, None, eps)
        ctx.save_for_backward(x2d, w)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, dy):
        x2d, w = ctx.saved_tensors
        dx, dw = rmsnorm_backward(x2d, w, dy, None, ctx.eps)
        return dx, dw, None


class _AddNorm(torch.autograd.Function):
    """custom_vjp of ``_add_norm`` (rmsnorm.py:137-156): residuals are (h, w)."""

    @staticmethod
    def forward(ctx, x2d, r2d, w, eps):
        h, y = _fwd(x2d, w, r2d, eps)
        ctx.save_for_backward(h, w)
        ctx.eps = eps
        return h, y

    @staticmethod
    def backward(ctx, dh_direct, dy):
        h, w = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(h)
        dh, dw = rmsnorm_backward(h, w, dy, dh_direct, ctx.eps)
        return dh, dh, dw, None


def rmsnorm(x, weight, *, residual=None, eps: float = 1e-6, block_rows: int | None = None):
    """RMSNorm over the last axis of ``x``.

    With ``residual`` given, returns ``(h, y)`` where ``h = x + residual`` is the
    new residual stream and ``y = rmsnorm(h) * weight``; otherwise returns ``y``.
    """
    dim = x.shape[-1]
    if tuple(weight.shape) != (dim,):
        raise ValueError(f"weight must have shape ({dim},), got {tuple(weight.shape)}")
    _check_block_rows(block_rows)
    lead = x.shape[:-1]
    x2d = x.reshape(-1, dim).contiguous()
    w = weight.contiguous()
    if residual is None:
        return _Norm.apply(x2d, w, float(eps)).reshape(*lead, dim)
    if residual.shape != x.shape:
        raise ValueError("residual must match x")
    r2d = residual.reshape(-1, dim).contiguous()
    if r2d.dtype != x2d.dtype:
        r2d = r2d.to(x2d.dtype)
    h, y = _AddNorm.apply(x2d, r2d, w, float(eps))
    return h.reshape(*lead, dim), y.reshape(*lead, dim)


def rmsnorm_reference(x, weight, *, residual=None, eps: float = 1e-6):
    """Plain-torch reference with identical f32 numerics (rmsnorm.py:193-199)."""
    h = x.float() + (0 if residual is None else residual.float())
    y = h * torch.rsqrt(torch.mean(h * h, dim=-1, keepdim=True) + eps) * weight.float()
    if residual is None:
        return y.to(x.dtype)
    return h.to(x.dtype), y.to(x.dtype)
