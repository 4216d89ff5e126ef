"""GPT training-step restatement on the CPU (torch, f32) -- test infrastructure /
CPU baseline only; see ``oracle/__init__.py``.

Follows src/ferrite/model/gpt.py of anxnd2211/ferrite-tpu with every slot on
its plain (``xla``) path: embedding + positional table (:129), per layer
add+RMSNorm fused into the next norm (:131-141), causal softmax attention over
materialised scores (:113-121, :370-380 of flash_attention.py), tanh-GELU MLP,
tied LM head (:143) and mean next-token NLL (:147-152).  Used to time the
reference's CPU path for the GPT config on a bounded sample (one sequence).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def init(cfg: dict, seed: int = 0) -> dict:
    g = torch.Generator().manual_seed(seed)
    d, f, L = cfg["d_model"], cfg["d_ff"], cfg["n_layer"]
    std, out_std = 0.02, 0.02 / math.sqrt(2 * L)

    def rn(*s, sd=std):
        return (sd * torch.randn(*s, generator=g)).requires_grad_(True)

    layers = [
        {"ln1": torch.ones(d, requires_grad=True), "wqkv": rn(d, 3 * d), "wo": rn(d, d, sd=out_std),
         "ln2": torch.ones(d, requires_grad=True), "w1": rn(d, f), "w2": rn(f, d, sd=out_std)}
        for _ in range(L)
    ]
    return {"tok_emb": rn(cfg["vocab_size"], d), "pos_emb": rn(cfg["seq_len"], d), "layers": layers, "ln_f": torch.ones(d, requires_grad=True)}


def _norm(x, w, r, eps):
    h = x if r is None else x + r
    y = h * torch.rsqrt(torch.mean(h * h, -1, keepdim=True) + eps) * w
    return h, y


def loss(params: dict, tokens: torch.Tensor, targets: torch.Tensor, cfg: dict) -> torch.Tensor:
    b, s = tokens.shape
    H, d = cfg["n_head"], cfg["d_model"]
    hd = d // H
    h = params["tok_emb"][tokens] + params["pos_emb"][:s]
    pending = None
    mask = torch.tril(torch.ones(s, s, dtype=torch.bool))
    for layer in params["layers"]:
        if pending is None:
            _, y = _norm(h, layer["ln1"], None, 1e-6)
        else:
            h, y = _norm(pending, layer["ln1"], h, 1e-6)
        qkv = (y @ layer["wqkv"]).reshape(b, s, 3, H, hd)
        q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
        sc = (q @ k.transpose(-1, -2)) / math.sqrt(hd)
        sc = sc.masked_fill(~mask, -0.7 * torch.finfo(torch.float32).max)
        a = (torch.softmax(sc, -1) @ v).transpose(1, 2).reshape(b, s, d)
        h, y2 = _norm(a @ layer["wo"], layer["ln2"], h, 1e-6)
        pending = F.gelu(y2 @ layer["w1"], approximate="tanh") @ layer["w2"]
    _, y = _norm(pending, params["ln_f"], h, 1e-6)
    logits = y.reshape(-1, d) @ params["tok_emb"].t()
    return F.cross_entropy(logits, targets.reshape(-1))
