"""Greedy-generation latency of the serving engine, per decode mode.

    PYTHONPATH=ferrite-tpu_b200 python -m ferrite.serving.measure [--prompts 8] [--prompt-len 400] [--new 64]

Builds the GPT config of the benchmarks (d_model 1024, 24 layers, 16 heads, vocab
32000, bf16, random init) and one :class:`Engine` per decode mode -- the B200
kernels or the plain path, each with and without CUDA graphs -- then generates from
the same seeded prompts (prefill bucket 512) and prints one JSON line: per mode the
median inter-token latency, tokens/s and time to first token; whether the graph and
eager engines produced identical tokens; and how far the kernel and plain paths'
greedy tokens agree (they round differently in bf16).
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
    a = ap.parse_args(argv)
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


if __name__ == "__main__":
    main()
