"""Matmul with an f32 accumulator on B200, with a custom backward.

Drop-in for the reference's ``ferrite.kernels.matmul`` (src/ferrite/kernels/matmul.py):
``matmul`` (:110-126), ``matmul_reference`` (:129-131), ``matmul_flops``
(:134-135).  Same contract: any ``[M, K] @ [K, N]`` shape, f32 accumulation,
``out_dtype`` defaulting to ``x.dtype``, ``ValueError`` for non-2-D operands or
mismatched K (:53-54) and for block sizes that are not multiples of (8, 128, 128)
(:46-47).  The VJP (:99-104) computes ``dX = G Y^T`` and ``dY = X^T G`` through
the same native GEMM, but as transposed-operand calls (no materialised
transposes; the reference transposes in XLA first).

Ragged shapes need no padding copies (the reference pads to the block grid,
:58-63): the TMA loads zero-fill out-of-range tiles and the epilogue masks the
stores.  bf16/f16 operands run on tcgen05 tensor cores; f32 operands run the
exact-f32 path, matching ``dot_precision`` (_compat.py:17-26).
"""

from __future__ import annotations

import torch

from ferrite import _native as nat
from ferrite import platform


def _pick_blocks(m: int, n: int, k: int, bm, bn, bk):
    """Validate caller block sizes like the reference (:41-49); the kernel tiles internally."""
    for name, b, mult in (("bm", bm, platform.SUBLANES), ("bn", bn, platform.LANES), ("bk", bk, platform.LANES)):
        if b is not None and b % mult:
            raise ValueError(f"blocks must be multiples of ({platform.SUBLANES}, {platform.LANES}); got bm={bm} bn={bn} bk={bk}")
    return bm, bn, bk


@nat.on_tensor_device
def gemm(a: torch.Tensor, b: torch.Tensor, *, trans_a: bool = False, trans_b: bool = False, out_dtype=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``op(a) @ op(b)`` through ``ferrite_gemm``; ``op`` transposes the stored 2-D tensor.

    ``a`` is stored ``[M, K]`` (or ``[K, M]`` with ``trans_a``), ``b`` is stored
    ``[K, N]`` (or ``[N, K]`` with ``trans_b``).  Row strides other than the
    packed ones are honoured (``a.stride(0)``), the inner stride must be 1.
    """
    nat.require_cuda(a, b)
    if a.dtype != b.dtype:
        raise ValueError(f"operands must share a dtype, got {a.dtype} and {b.dtype}")
    if a.stride(1) != 1:
        a = a.contiguous()
    if b.stride(1) != 1:
        b = b.contiguous()
    m, ka = (a.shape[1], a.shape[0]) if trans_a else (a.shape[0], a.shape[1])
    kb, n = (b.shape[1], b.shape[0]) if trans_b else (b.shape[0], b.shape[1])
    if ka != kb:
        raise ValueError(f"inner dimensions differ: {ka} vs {kb}")
    out_dtype = out_dtype or a.dtype
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    lib = nat.lib()
    code = nat.dtype_code(a.dtype)
    # split-K scratch for few-tile outputs (weight gradients); 0 bytes otherwise
    ws_bytes = lib.ferrite_gemm_workspace_size(m, n, ka, a.stride(0), b.stride(0), int(trans_a), int(trans_b), code) if m and n and ka else 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=a.device) if ws_bytes else None
    nat.check(
        lib.ferrite_gemm_ws(
            nat.stream_ptr(a.device), a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, ka,
            a.stride(0), b.stride(0), out.stride(0), int(trans_a), int(trans_b),
            code, nat.dtype_code(out.dtype), None if ws is None else ws.data_ptr(), ws_bytes,
        )
    )
    return out


@nat.on_tensor_device
def rmsnorm_matmul(x: torch.Tensor, w_norm: torch.Tensor, b: torch.Tensor, *, residual: torch.Tensor | None = None, eps: float = 1e-6,
                   trans_b: bool = False, gelu: bool = False, out_dtype=None):
    """Residual-add + RMSNorm folded in front of a product with at most 16 rows -- the
    decode step's norm feeding its next linear -- in one launch (``ferrite_gemm_rmsnorm``).

    ``h = x + residual`` (``x`` alone without one), ``y = rmsnorm(h) * w_norm`` (statistics
    from the unrounded f32 sum, as ``rmsnorm`` with a residual), ``c = y @ op(b)`` with an f32
    accumulator, ``op`` transposing ``b`` when ``trans_b``.  Returns ``(h, c)``, or with
    ``gelu`` (the MLP up-projection) ``(h, u, gelu_tanh(u))``; ``h`` is ``x`` itself when no
    residual is given.  Inference only (no autograd).  Shapes the fused kernel does not take
    (more rows, misaligned or ragged operands) run the norm and the product as two launches.
    """
    from ferrite.kernels.rmsnorm import rmsnorm

    m, k = x.shape
    kb, n = (b.shape[1], b.shape[0]) if trans_b else (b.shape[0], b.shape[1])
    if kb != k:
        raise ValueError(f"inner dimensions differ: {k} vs {kb}")
    if residual is not None and (residual.shape != x.shape or residual.dtype != x.dtype):
        raise ValueError("residual must match x in shape and dtype")
    out_dtype = out_dtype or x.dtype
    w32 = w_norm.float().contiguous()
    fits = (x.dtype in (torch.bfloat16, torch.float16) and b.dtype == x.dtype and 1 <= m <= 16 and k % 8 == 0
            and out_dtype in (x.dtype, torch.float32) and (not gelu or (x.dtype == torch.bfloat16 and not trans_b and out_dtype == x.dtype)))
    if fits:
        x = x.contiguous()
        residual = residual.contiguous() if residual is not None else None
        bb = b if b.stride(1) == 1 else b.contiguous()
        fits = all(t.data_ptr() % 16 == 0 for t in (x, bb, w32) + ((residual,) if residual is not None else ())) and bb.stride(0) % 8 == 0
        fits = fits and (trans_b or n % 8 == 0)
    if not fits:
        if residual is None:
            h, y = x, rmsnorm(x, w_norm, eps=eps)
        else:
            h, y = rmsnorm(x, w_norm, residual=residual, eps=eps)
        if gelu:
            u = gemm(y, b, trans_b=trans_b, out_dtype=out_dtype)
            return h, u, torch.nn.functional.gelu(u.float(), approximate="tanh").to(u.dtype)
        return h, gemm(y, b, trans_b=trans_b, out_dtype=out_dtype)
    h = torch.empty_like(x) if residual is not None else x
    c = torch.empty((m, n), dtype=out_dtype, device=x.device)
    act = torch.empty_like(c) if gelu else None
    nat.check(
        nat.lib().ferrite_gemm_rmsnorm(
            nat.stream_ptr(x.device), x.data_ptr(), nat.ptr(residual), w32.data_ptr(), float(eps),
            h.data_ptr() if residual is not None else None, bb.data_ptr(), c.data_ptr(), m, n, k, x.stride(0), bb.stride(0),
            c.stride(0), int(trans_b), 1 if gelu else 0, nat.ptr(act), act.stride(0) if gelu else 0,
            nat.dtype_code(x.dtype), nat.dtype_code(out_dtype),
        )
    )
    return (h, c, act) if gelu else (h, c)


class _Matmul(torch.autograd.Function):
    """custom_vjp of ``_matmul_vjp`` (matmul.py:89-107)."""

    @staticmethod
    def forward(ctx, x, y, out_dtype):
        ctx.save_for_backward(x, y)
        return gemm(x, y, out_dtype=out_dtype)

    @staticmethod
    def backward(ctx, g):
        x, y = ctx.saved_tensors
        dx = dy = None
        if ctx.needs_input_grad[0]:
            dx = gemm(g.to(x.dtype), y, trans_b=True, out_dtype=x.dtype)  # G @ Y^T
        if ctx.needs_input_grad[1]:
            dy = gemm(x, g.to(y.dtype), trans_a=True, out_dtype=y.dtype)  # X^T @ G
        return dx, dy, None


def matmul(x: torch.Tensor, y: torch.Tensor, *, block_m: int | None = None, block_n: int | None = None, block_k: int | None = None, out_dtype=None) -> torch.Tensor:
    """``x @ y`` for 2-D ``x: [M, K]`` and ``y: [K, N]`` on the B200 GEMM kernels.

    Any shape is accepted (ragged edges are handled in-kernel); differentiable:
    the backward runs the transposed products through the same kernel.
    """
    if x.ndim != 2 or y.ndim != 2 or x.shape[1] != y.shape[0]:
        raise ValueError(f"expected [M,K] @ [K,N], got {tuple(x.shape)} @ {tuple(y.shape)}")
    _pick_blocks(x.shape[0], y.shape[1], x.shape[1], block_m, block_n, block_k)
    if x.dtype != y.dtype:
        ct = torch.promote_types(x.dtype, y.dtype)
        x, y = x.to(ct), y.to(ct)
    return _Matmul.apply(x, y, out_dtype or x.dtype)


def matmul_reference(x: torch.Tensor, y: torch.Tensor, *, out_dtype=None) -> torch.Tensor:
    """Plain-torch baseline with the same numerics contract (f32 accumulation, :129-131)."""
    return torch.matmul(x.float(), y.float()).to(out_dtype or x.dtype)


def matmul_flops(m: int, n: int, k: int) -> int:
    return 2 * m * n * k
