"""Bucketed prefill on the B200 kernels into a static KV cache, plus greedy decode.

Restates src/ferrite/serving/engine.py: ``ServeConfig`` (:35-40), ``bucket_for``
(:43-47), ``prefill`` (:69-86: right-padded prompts, per-layer block on the
kernels, K/V padded to ``max_len`` and stacked into ``[L, B, H, max_len, hd]``),
``decode_step`` (:107-131), ``Engine`` (:137-209) and ``reference_greedy``
(:231-242).

B200 mapping of the reference's ahead-of-time compilation: each bucket's prefill
is captured once into a CUDA graph over static input/output buffers at engine
construction (the counterpart of ``jit(...).lower(...).compile()``), so serving
a prompt replays a graph -- no Python-level launch overhead and no shape seen at
serving time triggers new work.  The decode step is captured the same way, once: its
positions live on the device, so one graph serves every step.

Decode is one query row against the cache.  The reference keeps the whole decode
step in XLA (engine.py:12-15); here, with ``ServeConfig.decode_kernels="pallas"`` (the
default), its attention and cache write run as one kernel (``decode_attention``), its
residual-add + RMSNorms on the fused norm kernel, and for 16-bit models its linears
(one row per sequence) and the tied LM head on the skinny GEMM kernels (B stored
[K][N] for the layer matrices, the MLP's GELU fused into the up-projection; [N][K]
for the embedding), each norm folded into the product it feeds; f32 models keep the
plain linears.  ``"xla"`` gives the reference's plain path throughout.  ``jax.export`` of
the decode step has no counterpart here.
"""

from __future__ import annotations

import dataclasses
import time
from typing import Any

import numpy as np
import torch
import torch.nn.functional as F

from ferrite.kernels.decode_attention import decode_attention
from ferrite.kernels.matmul import rmsnorm_matmul
from ferrite.model.gpt import GPTConfig, _linear, _lm_head, _mlp, _norm, block


@dataclasses.dataclass(frozen=True)
class ServeConfig:
    batch: int = 1
    max_len: int = 512
    buckets: tuple[int, ...] = (128, 256, 512)
    prefill_kernels: str = "pallas"  # "pallas" | "xla" for attention + norms in prefill
    decode_kernels: str = "pallas"  # "pallas": decode attention + norms on the B200 kernels; "xla": plain
    use_graphs: bool = True


def bucket_for(length: int, buckets: tuple[int, ...]) -> int:
    for b in buckets:
        if length <= b:
            return b
    raise ValueError(f"prompt length {length} exceeds largest bucket {buckets[-1]}")


_MATRICES = ("wqkv", "wo", "w1", "w2")


def cast_weights(params, dtype):
    """The parameters with every layer matrix in the compute dtype, plus the tied embedding
    in the compute dtype under ``lm_head`` for the output projection.  The model casts
    these at every use (``w.to(cfg.dtype)``, gpt.py:95-104 and :143 of the reference);
    casting once gives the same values, and inside a captured graph it saves re-reading
    and re-writing every weight on each replay.  Norm weights and the f32 embedding
    tables (the lookup adds them in f32 before casting) are shared, not copied."""
    out = dict(params)
    out["layers"] = [{k: (v.to(dtype) if k in _MATRICES else v) for k, v in layer.items()} for layer in params["layers"]]
    out["lm_head"] = params["tok_emb"].to(dtype)
    return out


@torch.no_grad()
def prefill(params, tokens, lengths, cfg: GPTConfig, max_len: int):
    """tokens [B, L] (right-padded), lengths [B] -> (next-token logits [B, V] f32, k_cache, v_cache).

    Caches are [layers, B, H, max_len, hd]; positions >= length hold padding garbage
    that decode never attends to and overwrites in order.
    """
    b, s = tokens.shape
    h = (params["tok_emb"][tokens] + params["pos_emb"][:s]).to(cfg.dtype)
    pending = None
    kc = torch.zeros(cfg.n_layer, b, cfg.n_head, max_len, cfg.head_dim, dtype=cfg.dtype, device=tokens.device)
    vc = torch.zeros_like(kc)
    for i, layer in enumerate(params["layers"]):
        h, pending, k, v = block(layer, h, pending, cfg)
        kc[i, :, :, :s] = k
        vc[i, :, :, :s] = v
    _, y = _norm(pending, params["ln_f"], h, cfg)
    last = y[torch.arange(b, device=y.device), (lengths - 1).long()]  # [B, D]
    logits = _lm_head(last, params.get("lm_head", params["tok_emb"]), cfg)
    return logits, kc, vc


def _cache_attention(q, k_cache, v_cache, pos, scale):
    """q [B, H, hd]; caches [B, H, max_len, hd]; pos [B] = index of the current token (engine.py:89-95)."""
    s = torch.einsum("bhd,bhkd->bhk", q.float(), k_cache.float()) * scale
    idx = torch.arange(k_cache.shape[2], device=q.device)[None, :]
    s = torch.where((idx <= pos[:, None])[:, None, :], s, -1e30)
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhk,bhkd->bhd", p, v_cache.float()).to(q.dtype)


@torch.no_grad()
def decode_step(params, token, pos, k_cache, v_cache, cfg: GPTConfig):
    """One greedy decode step (engine.py:107-131); updates the caches in place.

    ``cfg.attention == "pallas"`` runs the cache write and the cache attention as one
    kernel (:func:`ferrite.kernels.decode_attention.decode_attention`); otherwise
    they run as the reference writes them (``_write_cache`` + ``_cache_attention``).
    With the norms and linears both on the kernels (16-bit, at most 16 sequences) each
    residual-add + RMSNorm is folded into the product it feeds
    (:func:`ferrite.kernels.matmul.rmsnorm_matmul`): ln1 into the QKV projection, ln2
    into the MLP up-projection (with its GELU), ln_f into the tied head -- five launches
    a layer instead of seven, same rounding points.
    """
    b = token.shape[0]
    h = (params["tok_emb"][token] + params["pos_emb"][pos]).to(cfg.dtype)  # [B, D]
    scale = 1.0 / np.sqrt(cfg.head_dim)
    pending = None
    ar = torch.arange(b, device=token.device)
    fused = cfg.norm == "pallas" and cfg.linear == "pallas" and cfg.dtype in (torch.bfloat16, torch.float16) and b <= 16
    for i, layer in enumerate(params["layers"]):
        if fused:
            w = layer["wqkv"].to(cfg.dtype)
            if pending is None:
                _, qkv = rmsnorm_matmul(h, layer["ln1"], w, eps=cfg.eps)
            else:
                h, qkv = rmsnorm_matmul(pending, layer["ln1"], w, residual=h, eps=cfg.eps)
        else:
            if pending is None:
                y = _norm(h, layer["ln1"], None, cfg)
            else:
                h, y = _norm(pending, layer["ln1"], h, cfg)
            qkv = _linear(y, layer["wqkv"], cfg)
        qkv = qkv.reshape(b, 3, cfg.n_head, cfg.head_dim)
        q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
        if cfg.attention == "pallas":
            a = decode_attention(q, k_cache[i], v_cache[i], pos, scale=scale, k_new=k.to(k_cache.dtype), v_new=v.to(v_cache.dtype))
        else:
            k_cache[i, ar, :, pos] = k.to(k_cache.dtype)
            v_cache[i, ar, :, pos] = v.to(v_cache.dtype)
            a = _cache_attention(q, k_cache[i], v_cache[i], pos, scale)
        a = a.reshape(b, cfg.d_model)
        a = _linear(a, layer["wo"], cfg)
        if fused:
            h, _, act = rmsnorm_matmul(a, layer["ln2"], layer["w1"].to(cfg.dtype), residual=h, eps=cfg.eps, gelu=True)
            pending = _linear(act, layer["w2"], cfg)
        else:
            h, y2 = _norm(a, layer["ln2"], h, cfg)
            pending = _mlp(y2[:, None], layer["w1"], layer["w2"], cfg)[:, 0]
    # tied head in cfg.dtype with f32 accumulation (engine.py:130): exact 16-bit products
    # summed in f32 on either path, f32 logits
    head = params.get("lm_head", params["tok_emb"])
    if fused:
        _, logits = rmsnorm_matmul(pending, params["ln_f"], head.to(cfg.dtype), residual=h, eps=cfg.eps, trans_b=True,
                                   out_dtype=torch.float32)
        return logits
    _, y = _norm(pending, params["ln_f"], h, cfg)
    return _lm_head(y, head, cfg)


class Engine:
    """Captures prefill per bucket and the decode step (CUDA graphs) and generates greedily
    (engine.py:137-209)."""

    def __init__(self, params, model_cfg: GPTConfig, serve_cfg: ServeConfig):
        if max(serve_cfg.buckets) > model_cfg.seq_len or serve_cfg.max_len > model_cfg.seq_len:
            raise ValueError("buckets and max_len must fit within the model's trained seq_len (positional table)")
        # the weights as of construction, matrices cast once to the compute dtype
        params = cast_weights(params, model_cfg.dtype)
        self.params = params
        self.cfg = model_cfg
        self.serve = serve_cfg
        self.prefill_cfg = model_cfg if serve_cfg.prefill_kernels == "pallas" else model_cfg.replace(attention="xla", norm="xla", linear="xla")
        if serve_cfg.decode_kernels not in ("pallas", "xla"):
            raise ValueError(f"decode_kernels must be 'pallas' or 'xla', got {serve_cfg.decode_kernels!r}")
        dk = serve_cfg.decode_kernels
        # the skinny GEMM kernels take 16-bit operands: f32 models keep the plain linears
        dl = dk if model_cfg.dtype in (torch.bfloat16, torch.float16) else "xla"
        self.decode_cfg = model_cfg.replace(attention=dk, norm=dk, linear=dl)
        self.device = params["tok_emb"].device
        self.compile_seconds: dict[str, float] = {}
        self._graphs: dict[int, Any] = {}
        b = serve_cfg.batch
        for bucket in serve_cfg.buckets:
            t0 = time.perf_counter()
            tok = torch.zeros(b, bucket, dtype=torch.long, device=self.device)
            lens = torch.ones(b, dtype=torch.long, device=self.device)
            if serve_cfg.use_graphs:
                s = torch.cuda.Stream(self.device)
                s.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(s):
                    for _ in range(2):  # warm-up: module loading, allocator pools
                        prefill(params, tok, lens, self.prefill_cfg, serve_cfg.max_len)
                torch.cuda.current_stream(self.device).wait_stream(s)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    out = prefill(params, tok, lens, self.prefill_cfg, serve_cfg.max_len)
                self._graphs[bucket] = (g, tok, lens, out)
            else:
                self._graphs[bucket] = (None, tok, lens, None)
            torch.cuda.synchronize(self.device)
            self.compile_seconds[f"prefill_{bucket}"] = time.perf_counter() - t0
        self._decode_graph = None
        if serve_cfg.use_graphs:
            self._capture_decode()
        # every bucket's prefill + the decode step (a captured graph, or one eager function)
        self.n_compiles = len(self.compile_seconds) + (0 if self._decode_graph is not None else 1)

    def _capture_decode(self):
        """Captures one decode step into a CUDA graph over static buffers: the token and
        position inputs, both caches and the next-token output (the counterpart of the
        reference compiling its decode step once, engine.py:9-10).  Positions are read on
        the device, so one graph serves every position."""
        t0 = time.perf_counter()
        cfg, b = self.cfg, self.serve.batch
        shape = (cfg.n_layer, b, cfg.n_head, self.serve.max_len, cfg.head_dim)
        self._dkc = torch.zeros(shape, dtype=cfg.dtype, device=self.device)
        self._dvc = torch.zeros_like(self._dkc)
        self._dtok = torch.zeros(b, dtype=torch.long, device=self.device)
        self._dpos = torch.zeros(b, dtype=torch.long, device=self.device)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up: module loading, per-device kernel set-up, allocator pools
                decode_step(self.params, self._dtok, self._dpos, self._dkc, self._dvc, self.decode_cfg)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            logits = decode_step(self.params, self._dtok, self._dpos, self._dkc, self._dvc, self.decode_cfg)
            self._dnext = torch.argmax(logits, dim=-1)
        self._decode_graph = g
        self._dkc.zero_()  # the warm-up steps wrote rows at position 0
        self._dvc.zero_()
        torch.cuda.synchronize(self.device)
        self.compile_seconds["decode"] = time.perf_counter() - t0

    def prefill(self, prompts: list[list[int]]):
        """Returns (first token [B], pos [B], caches). Prompts are right-padded to a bucket."""
        token, pos, kc, vc, graph_owned = self._run_prefill(prompts)
        if graph_owned:  # the graph's buffers are reused by the next replay
            kc, vc = kc.clone(), vc.clone()
        return token, pos, kc, vc

    def _run_prefill(self, prompts: list[list[int]]):
        """prefill() without copying the caches out of a captured graph's buffers:
        (token, pos, kc, vc, graph_owned), valid until the bucket's next replay."""
        b = self.serve.batch
        if len(prompts) != b:
            raise ValueError(f"engine built for batch {b}, got {len(prompts)} prompts")
        lengths = np.array([len(p) for p in prompts], np.int64)
        bucket = bucket_for(int(lengths.max()), self.serve.buckets)
        tokens = np.zeros((b, bucket), np.int64)
        for i, p in enumerate(prompts):
            tokens[i, : len(p)] = p
        g, tok, lens, out = self._graphs[bucket]
        tok.copy_(torch.from_numpy(tokens), non_blocking=True)
        lens.copy_(torch.from_numpy(lengths), non_blocking=True)
        if g is not None:
            g.replay()
            logits, kc, vc = out
        else:
            logits, kc, vc = prefill(self.params, tok, lens, self.prefill_cfg, self.serve.max_len)
        return torch.argmax(logits, dim=-1), torch.from_numpy(lengths).to(self.device), kc, vc, g is not None

    def decode(self, token, pos, kc, vc):
        """One greedy step; updates kc / vc in place.  Caches that are the engine's own decode
        buffers (as ``generate`` passes them) replay the captured graph; others run eagerly."""
        if self._decode_graph is not None and kc.data_ptr() == self._dkc.data_ptr() and vc.data_ptr() == self._dvc.data_ptr():
            self._dtok.copy_(token)
            self._dpos.copy_(pos)
            self._decode_graph.replay()
            return self._dnext.clone(), kc, vc
        logits = decode_step(self.params, token, pos, kc, vc, self.decode_cfg)
        return torch.argmax(logits, dim=-1), kc, vc

    def generate(self, prompts: list[list[int]], max_new_tokens: int) -> tuple[np.ndarray, dict]:
        if max(len(p) for p in prompts) + max_new_tokens > self.serve.max_len:
            raise ValueError("prompt + new tokens exceed max_len")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        token, pos, kc, vc, graph_owned = self._run_prefill(prompts)
        if self._decode_graph is not None:
            # continue in the captured decode graph's own caches, copied straight from the
            # prefill output (one copy of each cache, no intermediate clone)
            self._dkc.copy_(kc)
            self._dvc.copy_(vc)
            kc, vc = self._dkc, self._dvc
        elif graph_owned:
            kc, vc = kc.clone(), vc.clone()
        e1.record()
        out = [token.cpu().numpy()]
        ttft = e0.elapsed_time(e1)
        step_times = []
        for _ in range(max_new_tokens - 1):
            t = time.perf_counter()
            token, kc, vc = self.decode(token, pos, kc, vc)
            out.append(token.cpu().numpy())
            step_times.append(time.perf_counter() - t)
            pos = pos + 1
        total = time.perf_counter() - t0
        stats = {
            "ttft_ms": ttft,
            "itl_ms_median": float(np.median(step_times)) * 1e3 if step_times else float("nan"),
            "tokens_per_second": len(prompts) * max_new_tokens / total,
            "total_s": total,
            "n_compiles": self.n_compiles,
        }
        return np.stack(out, axis=1), stats


@torch.no_grad()
def reference_greedy(params, cfg: GPTConfig, prompt: list[int], max_new_tokens: int) -> np.ndarray:
    """Slow but obviously-correct greedy decoding by re-running the full model each step."""
    from ferrite.model.gpt import forward

    toks = list(prompt)
    out = []
    dev = params["tok_emb"].device
    for _ in range(max_new_tokens):
        logits = forward(params, torch.tensor([toks], device=dev), cfg)
        nxt = int(torch.argmax(logits[0, -1]))
        out.append(nxt)
        toks.append(nxt)
    return np.array(out)
