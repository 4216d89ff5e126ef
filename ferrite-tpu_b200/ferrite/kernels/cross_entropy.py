"""Softmax cross-entropy on B200, and the tied LM head fused with it.

The reference computes its training loss in XLA (src/ferrite/model/gpt.py:147-152:
``log_softmax`` over the vocabulary, the target's log-probability gathered, the
mean taken) on f32 logits.  Here the same loss is two HBM-bound row kernels of
the native library (``ferrite_xent_fwd`` / ``ferrite_xent_bwd``): the forward
reads each logit row once (online max / sum) and keeps only ``lse`` per row;
the backward writes ``softmax - onehot`` scaled by the upstream gradient
directly in the dtype of the LM-head GEMMs, so no f32 gradient of the logits is
ever materialised.

:func:`tied_head_cross_entropy` chains the tied LM head (``y @ E^T`` with f32
output, the reference's gpt.py:143) with the loss in one autograd node; its
backward feeds the bf16 ``dlogits`` straight into the two GEMMs
``dY = dL E`` and ``dE = dL^T Y``.
"""

from __future__ import annotations

import torch

from ferrite import _native as nat
from ferrite.kernels.matmul import gemm


def _target_code(t: torch.Tensor) -> int:
    if t.dtype == torch.int64:
        return 1
    if t.dtype == torch.int32:
        return 0
    raise TypeError(f"targets must be int32 or int64, got {t.dtype}")


@nat.on_tensor_device
def xent_forward(logits: torch.Tensor, targets: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``(lse, nll)`` per row of f32 ``logits [rows, vocab]``."""
    nat.require_cuda(logits, targets)
    if logits.dtype != torch.float32 or logits.ndim != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a 2-D f32 tensor with unit column stride")
    rows, vocab = logits.shape
    targets = targets.reshape(-1).contiguous()
    if targets.numel() != rows:
        raise ValueError(f"{targets.numel()} targets for {rows} rows")
    lse = torch.empty(rows, dtype=torch.float32, device=logits.device)
    nll = torch.empty(rows, dtype=torch.float32, device=logits.device)
    nat.check(
        nat.lib().ferrite_xent_fwd(
            nat.stream_ptr(logits.device), logits.data_ptr(), targets.data_ptr(), lse.data_ptr(), nll.data_ptr(),
            rows, vocab, logits.stride(0), _target_code(targets),
        )
    )
    return lse, nll


@nat.on_tensor_device
def xent_backward(logits, targets, lse, dloss: torch.Tensor | None, scale: float, out_dtype=torch.float32) -> torch.Tensor:
    """``dlogits = dloss * scale * (softmax(logits) - onehot(targets))`` as ``out_dtype``."""
    nat.require_cuda(logits, targets, lse)
    rows, vocab = logits.shape
    targets = targets.reshape(-1).contiguous()
    out = torch.empty((rows, vocab), dtype=out_dtype, device=logits.device)
    if dloss is not None:
        dloss = dloss.reshape(()).to(torch.float32).contiguous()
    nat.check(
        nat.lib().ferrite_xent_bwd(
            nat.stream_ptr(logits.device), logits.data_ptr(), targets.data_ptr(), lse.data_ptr(),
            None if dloss is None else dloss.data_ptr(), float(scale), out.data_ptr(), rows, vocab,
            logits.stride(0), out.stride(0), _target_code(targets), nat.dtype_code(out_dtype),
        )
    )
    return out


class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets):
        lse, nll = xent_forward(logits, targets)
        ctx.save_for_backward(logits, targets, lse)
        return nll.mean()

    @staticmethod
    def backward(ctx, g):
        logits, targets, lse = ctx.saved_tensors
        return xent_backward(logits, targets, lse, g, 1.0 / logits.shape[0], torch.float32), None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean next-token cross-entropy of f32 ``logits [rows, vocab]`` (gpt.py:147-152)."""
    return _CrossEntropy.apply(logits, targets)


class _TiedHeadXent(torch.autograd.Function):
    """loss = mean_r(lse_r - (y E^T)_{r, t_r}); logits f32 are a forward-only residual."""

    @staticmethod
    def forward(ctx, y, e, targets):
        logits = gemm(y, e, trans_b=True, out_dtype=torch.float32)  # [T, V]
        lse, nll = xent_forward(logits, targets)
        ctx.save_for_backward(y, e, targets, logits, lse)
        return nll.mean()

    @staticmethod
    def backward(ctx, g):
        y, e, targets, logits, lse = ctx.saved_tensors
        dl = xent_backward(logits, targets, lse, g, 1.0 / logits.shape[0], y.dtype)  # [T, V] bf16
        dy = gemm(dl, e, out_dtype=y.dtype) if ctx.needs_input_grad[0] else None  # [T, V] @ [V, d]
        de = gemm(dl, y, trans_a=True, out_dtype=e.dtype) if ctx.needs_input_grad[1] else None  # [V, T] @ [T, d]
        return dy, de, None


def tied_head_cross_entropy(y: torch.Tensor, e: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean cross-entropy of the tied LM head ``y [T, d] @ e[V, d]^T`` (f32 logits)."""
    if y.dtype != e.dtype:
        raise ValueError("y and the embedding must share a dtype")
    return _TiedHeadXent.apply(y, e, targets)
