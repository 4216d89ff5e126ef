"""A small pre-norm, decoder-only transformer whose attention, norms and linears run
on the B200 kernels (the reference's ``pallas`` slot) or on plain torch (``xla``).

Restates the reference's model (src/ferrite/model/gpt.py): ``GPTConfig`` (:29-63),
``init_params`` (:66-88, GPT-2 residual-projection scaling), ``param_count``
(:91-92), the routing helpers ``_linear`` / ``_norm`` / ``_attention`` (:95-121),
``forward`` (:124-144, the add that closes one sub-layer fused into the norm that
opens the next), ``loss_fn`` (:147-152) and ``flops_per_token`` (:155-163).
Parameters live in f32; activations and matmuls use ``cfg.dtype`` (bf16 by
default); softmax, RMS and loss statistics are f32.

Differences from the reference, all on the ``pallas`` slot: the tied LM head also
runs on the B200 GEMM when ``cfg.linear == "pallas"`` (the reference always leaves
it to XLA), with the embedding passed as the transposed operand (no copy); attention reads
q/k/v in place from the packed ``[B, S, 3, H, hd]`` projection and writes
``[B, S, H, hd]`` (``flash_attention_packed``), so the head split and the
transposes of gpt.py:136-138 are folded into the kernels' tensor maps; the
loss (gpt.py:147-152) runs on the native cross-entropy kernels, fused with the
tied head into one autograd node (no f32 logit gradient is materialised); the
MLP's GELU runs in the epilogues of its GEMMs (forward and backward); the
``xla`` slot is plain torch (cuBLAS matmuls, materialised attention).
"""

from __future__ import annotations

import dataclasses
import math
from typing import Any

import torch
import torch.nn.functional as F

from ferrite import platform
from ferrite.kernels.flash_attention import BlockSizes, flash_attention, flash_attention_packed, flash_attention_reference
from ferrite.kernels.cross_entropy import tied_head_cross_entropy
from ferrite.kernels.matmul import gemm, matmul
from ferrite.kernels.rmsnorm import rmsnorm, rmsnorm_reference


@dataclasses.dataclass(frozen=True)
class GPTConfig:
    vocab_size: int = 256
    seq_len: int = 256
    d_model: int = 512
    n_head: int = 4
    n_layer: int = 4
    d_ff: int = 2048
    attention: str = "pallas"  # "pallas" | "xla"
    norm: str = "pallas"  # "pallas" | "xla"
    linear: str = "xla"  # "xla" | "pallas"
    dtype: Any = torch.bfloat16
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        assert self.d_model % self.n_head == 0
        return self.d_model // self.n_head

    def replace(self, **kw) -> "GPTConfig":
        return dataclasses.replace(self, **kw)

    def attention_blocks(self, seq_len: int | None = None) -> BlockSizes | None:
        """Tile sizes for ``seq_len``, or None when the kernel cannot tile it (gpt.py:51-63)."""
        s = seq_len or self.seq_len
        if s % 128:
            return None
        t = min(platform.default_tile(), s)
        while s % t:
            t -= 128
        return BlockSizes(t, t, t, t)


def init_params(seed: int, cfg: GPTConfig, device="cuda") -> dict:
    """normal(0, 0.02) weights, GPT-2 scaling 0.02/sqrt(2L) on wo and w2 (gpt.py:66-88)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    std = 0.02
    out_std = std / math.sqrt(2 * cfg.n_layer)
    d, f = cfg.d_model, cfg.d_ff

    def rn(*shape, s=std):
        return s * torch.randn(*shape, generator=g, device=device, dtype=torch.float32)

    layers = []
    for _ in range(cfg.n_layer):
        layers.append(
            {
                "ln1": torch.ones(d, device=device),
                "wqkv": rn(d, 3 * d),
                "wo": rn(d, d, s=out_std),
                "ln2": torch.ones(d, device=device),
                "w1": rn(d, f),
                "w2": rn(f, d, s=out_std),
            }
        )
    return {"tok_emb": rn(cfg.vocab_size, d), "pos_emb": rn(cfg.seq_len, d), "layers": layers, "ln_f": torch.ones(d, device=device)}


def param_leaves(params) -> list[torch.Tensor]:
    out = [params["tok_emb"], params["pos_emb"]]
    for layer in params["layers"]:
        out += [layer[k] for k in ("ln1", "wqkv", "wo", "ln2", "w1", "w2")]
    out.append(params["ln_f"])
    return out


def param_count(params) -> int:
    return sum(int(x.numel()) for x in param_leaves(params))


def _linear(x, w, cfg: GPTConfig):
    """[..., in] @ [in, out] in cfg.dtype with f32 accumulation (gpt.py:95-104)."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1]).to(cfg.dtype)
    w = w.to(cfg.dtype)
    if cfg.linear == "pallas":
        y = matmul(x2, w)
    else:
        y = torch.matmul(x2, w)
    return y.reshape(*lead, w.shape[1])


def _norm(x, w, residual, cfg: GPTConfig):
    if cfg.norm == "pallas":
        return rmsnorm(x, w, residual=residual, eps=cfg.eps)
    return rmsnorm_reference(x, w, residual=residual, eps=cfg.eps)


def _attention(q, k, v, cfg: GPTConfig):
    """q, k, v: [B, H, S, hd] -> [B, H, S, hd], causal (gpt.py:113-121)."""
    blocks = cfg.attention_blocks(q.shape[2]) if cfg.attention == "pallas" else None
    if blocks is not None:
        return flash_attention(q, k, v, causal=True, block_sizes=blocks)
    return flash_attention_reference(q, k, v, causal=True)


def _lm_head(y2d, tok_emb, cfg: GPTConfig):
    """Tied LM head: y @ tok_emb^T -> f32 logits."""
    w = tok_emb.to(cfg.dtype)
    if cfg.linear == "pallas":
        return _TiedHead.apply(y2d, w)
    return torch.matmul(y2d.float(), w.float().t())


class _TiedHead(torch.autograd.Function):
    """logits = y @ E^T (f32 out) on the B200 GEMM with E as the transposed operand;
    backward dY = dL E, dE = dL^T Y, both without materialised transposes."""

    @staticmethod
    def forward(ctx, y, e):
        ctx.save_for_backward(y, e)
        return gemm(y, e, trans_b=True, out_dtype=torch.float32)

    @staticmethod
    def backward(ctx, g):
        y, e = ctx.saved_tensors
        g16 = g.to(y.dtype)
        dy = gemm(g16, e, out_dtype=y.dtype)  # [T, V] @ [V, d]
        de = gemm(g16, y, trans_a=True, out_dtype=e.dtype)  # [V, T] @ [T, d]
        return dy, de


class _FusedMlp(torch.autograd.Function):
    """``gelu_tanh(y W1) W2`` (gpt.py:141) with the activation in GEMM epilogues
    (``ferrite_gemm_epilogue``): the forward's up-projection writes the
    pre-activation u (kept for the backward) and a = gelu(u) in one pass; the
    backward's dA = dP W2^T product writes dU = dA * gelu'(u) directly.  Same
    rounding points as the unfused chain (u, a, dA and dU rounded to bf16)."""

    @staticmethod
    def forward(ctx, y, w1, w2):
        from ferrite import _native as nat

        t, d = y.shape
        f = w1.shape[1]
        u = torch.empty((t, f), dtype=y.dtype, device=y.device)
        a = torch.empty_like(u)
        with torch.cuda.device(y.device):
            nat.check(nat.lib().ferrite_gemm_epilogue(nat.stream_ptr(y.device), y.data_ptr(), w1.data_ptr(), u.data_ptr(),
                                                      t, f, d, y.stride(0), w1.stride(0), u.stride(0), 0, 0, 1, a.data_ptr(), a.stride(0)))
        ctx.save_for_backward(y, w1, w2, u, a)
        return gemm(a, w2)

    @staticmethod
    def backward(ctx, dp):
        from ferrite import _native as nat

        y, w1, w2, u, a = ctx.saved_tensors
        dp = dp.to(y.dtype).contiguous()
        t, f = u.shape
        du = torch.empty_like(u)
        with torch.cuda.device(y.device):
            nat.check(nat.lib().ferrite_gemm_epilogue(nat.stream_ptr(y.device), dp.data_ptr(), w2.data_ptr(), du.data_ptr(),
                                                      t, f, dp.shape[1], dp.stride(0), w2.stride(0), du.stride(0), 0, 1, 2, u.data_ptr(), u.stride(0)))
        dw2 = gemm(a, dp, trans_a=True, out_dtype=w2.dtype)  # A^T dP
        dy = gemm(du, w1, trans_b=True, out_dtype=y.dtype)  # dU W1^T
        dw1 = gemm(y, du, trans_a=True, out_dtype=w1.dtype)  # Y^T dU
        return dy, dw1, dw2


def _mlp(y2, w1, w2, cfg: GPTConfig):
    """The block's MLP, gelu(approximate=True) between the two linears (gpt.py:141)."""
    b, s, d = y2.shape
    if cfg.linear == "pallas" and cfg.dtype == torch.bfloat16 and d % 8 == 0 and w1.shape[1] % 8 == 0:
        return _FusedMlp.apply(y2.reshape(-1, d).to(cfg.dtype), w1.to(cfg.dtype), w2.to(cfg.dtype)).reshape(b, s, -1)
    return _linear(F.gelu(_linear(y2, w1, cfg), approximate="tanh"), w2, cfg)


def block(layer, h, pending, cfg: GPTConfig):
    """One transformer block; returns (h, pending, k, v) (gpt.py:131-141, engine.py:53-66)."""
    b, s, _ = h.shape
    if pending is None:
        y = _norm(h, layer["ln1"], None, cfg)
    else:
        h, y = _norm(pending, layer["ln1"], h, cfg)
    qkv = _linear(y, layer["wqkv"], cfg).reshape(b, s, 3, cfg.n_head, cfg.head_dim)
    q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))  # [B, H, S, hd] views
    blocks = cfg.attention_blocks(s) if cfg.attention == "pallas" else None
    if blocks is not None:
        # q/k/v read in place and the output written as [B, S, H, hd]: no transposes
        a = flash_attention_packed(qkv, causal=True, block_sizes=blocks).reshape(b, s, cfg.d_model)
    else:
        a = _attention(q, k, v, cfg).transpose(1, 2).reshape(b, s, cfg.d_model)
    a = _linear(a, layer["wo"], cfg)
    h, y2 = _norm(a, layer["ln2"], h, cfg)
    pending = _mlp(y2, layer["w1"], layer["w2"], cfg)
    return h, pending, k, v


def hidden(params, tokens, cfg: GPTConfig):
    """tokens [B, S] int -> final-norm output [B*S, d_model] (gpt.py:124-142)."""
    b, s = tokens.shape
    if s > cfg.seq_len:
        raise ValueError(f"sequence {s} longer than cfg.seq_len={cfg.seq_len}")
    h = (params["tok_emb"][tokens] + params["pos_emb"][:s]).to(cfg.dtype)  # residual stream
    pending = None  # sub-layer output whose residual add is fused into the next norm
    for layer in params["layers"]:
        h, pending, _, _ = block(layer, h, pending, cfg)
    _, y = _norm(pending, params["ln_f"], h, cfg)
    return y.reshape(-1, cfg.d_model)


def forward(params, tokens, cfg: GPTConfig):
    """tokens [B, S] int -> logits [B, S, vocab] f32 (gpt.py:124-144)."""
    b, s = tokens.shape
    logits = _lm_head(hidden(params, tokens, cfg), params["tok_emb"], cfg)
    return logits.reshape(b, s, cfg.vocab_size)


def loss_fn(params, tokens, targets, cfg: GPTConfig):
    """Mean next-token cross-entropy in f32 (gpt.py:147-152).

    On the ``pallas`` linear slot the tied LM head and the loss run as one
    autograd node on the native kernels (f32 logits, ``log_softmax`` / gather
    in two row passes, bf16 ``dlogits`` straight into the head's GEMMs)."""
    y = hidden(params, tokens, cfg)
    if cfg.linear == "pallas":
        return tied_head_cross_entropy(y, params["tok_emb"].to(cfg.dtype), targets.reshape(-1))
    logits = _lm_head(y, params["tok_emb"], cfg)
    return F.cross_entropy(logits, targets.reshape(-1))


def flops_per_token(cfg: GPTConfig, n_params_nonembed: int) -> dict:
    """Analytic FLOPs per token (forward; training = 3x), gpt.py:155-163."""
    dense = 2 * (n_params_nonembed + cfg.vocab_size * cfg.d_model)
    attn = 4 * cfg.seq_len * cfg.d_model * cfg.n_layer * 0.5
    return {"dense": dense, "attention": attn, "total": dense + attn}
