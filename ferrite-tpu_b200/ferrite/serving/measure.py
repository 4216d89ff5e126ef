"""Greedy-generation latency of the serving engine, per decode mode.

    PYTHONPATH=ferrite-tpu_b200 python -m ferrite.serving.measure [--prompts 8] [--prompt-len 400] [--new 64]

Builds the GPT config of the benchmarks (d_model 1024, 24 layers, 16 heads, vocab
32000, bf16, random init) and one :class:`Engine` per decode mode -- the B200
kernels or the plain path, each with and without CUDA graphs -- then generates from
the same seeded prompts (prefill bucket 512) and prints one JSON line: per mode the
median inter-token latency, tokens/s and time to first token; whether the graph and
eager engines produced identical tokens; and how far the kernel and plain paths'
greedy tokens agree (they round differently in bf16).

``--breakdown`` instead times, per call, the kernels one decode step of that model runs
(graph-replayed back to back over 24 distinct weights or inputs, as the 24 layers
do): the four layer linears and the tied LM head on the skinny GEMM against
``torch.matmul`` (cuBLAS) on the same bf16 operands, the fused residual-add + RMSNorm,
and the cache attention at the engine's shape (512-slot cache, position 400).
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from ferrite.model.gpt import GPTConfig, init_params
from ferrite.serving.engine import Engine, ServeConfig


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--prompts", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=400)
    ap.add_argument("--new", type=int, default=64, help="tokens generated per prompt in the timed run")
    ap.add_argument("--breakdown", action="store_true", help="per-call kernel times of one decode step instead")
    a = ap.parse_args(argv)
    if a.breakdown:
        print(json.dumps(breakdown(a.prompts)), flush=True)
        return
    if a.prompt_len + a.new > 512:
        raise SystemExit("prompt-len + new must fit the 512-token cache")
    cfg = GPTConfig(vocab_size=32000, seq_len=1024, d_model=1024, n_head=16, n_layer=24, d_ff=4096,
                    attention="pallas", norm="pallas", linear="pallas", dtype=torch.bfloat16)
    params = init_params(0, cfg, device=torch.device("cuda"))
    rng = np.random.default_rng(0)
    prompts = [list(rng.integers(0, cfg.vocab_size, size=a.prompt_len)) for _ in range(a.prompts)]
    out, tokens = {"config": {"model": "GPT d1024 L24 H16 V32000 bf16", "prompts": a.prompts, "prompt_len": a.prompt_len,
                              "new_tokens": a.new, "max_len": 512}}, []
    for kernels in ("pallas", "xla"):
        for graphs in (True, False):
            eng = Engine(params, cfg, ServeConfig(batch=a.prompts, max_len=512, buckets=(512,), use_graphs=graphs, decode_kernels=kernels))
            eng.generate(prompts, max_new_tokens=8)  # warm-up
            gen, st = eng.generate(prompts, max_new_tokens=a.new)
            out[f"decode_{kernels}_{'graph' if graphs else 'eager'}"] = {
                "itl_ms_median": round(st["itl_ms_median"], 3), "tokens_per_second": round(st["tokens_per_second"], 1),
                "ttft_ms": round(st["ttft_ms"], 3)}
            tokens.append(gen)
            del eng
            torch.cuda.empty_cache()
    # graph replay runs the same kernels as the eager step: bit-identical tokens expected
    out["graph_equals_eager"] = {"pallas": bool(np.array_equal(tokens[0], tokens[1])), "xla": bool(np.array_equal(tokens[2], tokens[3]))}
    # the kernel and plain paths round differently in bf16 (fused norm from the unrounded f32
    # sum, another summation order in attention); a random-init model has near-tied logits,
    # so greedy tokens drift apart after a while: report the agreement, position by position
    out["token_agreement_pallas_vs_xla"] = round(float(np.mean(tokens[0] == tokens[2])), 4)
    out["first_divergence_pallas_vs_xla"] = [int(np.argmax(r)) if r.any() else None for r in (tokens[0] != tokens[2])]
    print(json.dumps(out), flush=True)


def _graph_us(fn, reps: int = 30) -> float:
    """Microseconds per replay of ``fn`` captured as one CUDA graph (CUDA events, after warm-up)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1000.0


@torch.no_grad()
def breakdown(batch: int = 8) -> dict:
    """Per-call times (us) of the kernels of one decode step of GPT d1024 L24 with ``batch``
    sequences; each call class replayed 24 times back to back with distinct operands."""
    from ferrite.kernels.decode_attention import decode_attention
    from ferrite.kernels.matmul import gemm
    from ferrite.kernels.rmsnorm import rmsnorm

    dev, bf = torch.device("cuda"), torch.bfloat16
    out = {"config": {"model": "GPT d1024 L24 H16 V32000 bf16", "batch": batch, "cache": [24, batch, 16, 512, 64], "pos": 400,
                      "timing": "CUDA graph of 24 calls, us per call"}}
    x = torch.randn(batch, 4096, device=dev).to(bf)
    for name, (k, n) in {"qkv": (1024, 3072), "out": (1024, 1024), "up": (1024, 4096), "down": (4096, 1024)}.items():
        ws = [torch.randn(k, n, device=dev).to(bf) for _ in range(24)]
        xk = x[:, :k]
        ours = _graph_us(lambda: [gemm(xk, w) for w in ws]) / 24
        ref = _graph_us(lambda: [torch.matmul(xk, w) for w in ws]) / 24
        out[f"linear_{name}_{k}x{n}"] = {"skinny_us": round(ours, 2), "cublas_us": round(ref, 2),
                                         "skinny_GBps": round(k * n * 2 / ours / 1e3, 1)}
        del ws
    e = torch.randn(32000, 1024, device=dev).to(bf)
    y = x[:, :1024]
    ours = _graph_us(lambda: gemm(y, e, trans_b=True, out_dtype=torch.float32))
    ref = _graph_us(lambda: torch.matmul(y.float(), e.float().t()))
    out["lm_head_32000x1024_f32_logits"] = {"skinny_us": round(ours, 2), "torch_f32_us": round(ref, 2)}
    del e
    hs = [torch.randn(batch, 1024, device=dev).to(bf) for _ in range(24)]
    rs = [torch.randn(batch, 1024, device=dev).to(bf) for _ in range(24)]
    wn = torch.ones(1024, device=dev)
    out["add_rmsnorm_us"] = round(_graph_us(lambda: [rmsnorm(hs[i], wn, residual=rs[i], eps=1e-5) for i in range(24)]) / 24, 2)
    kc = torch.randn(24, batch, 16, 512, 64, device=dev).to(bf)
    vc = torch.randn_like(kc)
    q = torch.randn(batch, 3, 16, 64, device=dev).to(bf)
    pos = torch.full((batch,), 400, dtype=torch.long, device=dev)
    out["cache_attention_us"] = round(_graph_us(
        lambda: [decode_attention(q[:, 0], kc[i], vc[i], pos, scale=0.125, k_new=q[:, 1], v_new=q[:, 2]) for i in range(24)]) / 24, 2)
    return out


if __name__ == "__main__":
    main()
