"""GPU tests of the bucketed-prefill engine (tests/test_serving.py of
anxnd2211/ferrite-tpu re-pointed at the B200 kernels): greedy generation through
the CUDA-graph prefill equals full-recompute greedy, and the prefill KV cache
matches the plain path."""

import numpy as np
import pytest
import torch

from ferrite.model.gpt import GPTConfig, init_params
from ferrite.serving.engine import Engine, ServeConfig, prefill, reference_greedy

pytestmark = pytest.mark.gpu
torch.backends.cuda.matmul.allow_tf32 = False
CFG = GPTConfig(vocab_size=256, seq_len=256, d_model=128, n_head=1, n_layer=2, d_ff=256, dtype=torch.float32)


def test_engine_matches_reference_greedy():
    params = init_params(0, CFG)
    eng = Engine(params, CFG, ServeConfig(batch=2, max_len=256, buckets=(128,)))
    assert eng.n_compiles == 2  # one prefill bucket + decode
    prompts = [[1, 2, 3, 4, 5, 6, 7, 8, 9, 10], [42, 7, 99]]
    gen, stats = eng.generate(prompts, max_new_tokens=6)
    assert gen.shape == (2, 6) and stats["ttft_ms"] > 0
    for i, p in enumerate(prompts):
        ref = reference_greedy(params, CFG.replace(attention="xla", norm="xla"), p, 6)
        np.testing.assert_array_equal(gen[i], ref)


def test_graph_replay_matches_eager_prefill_bf16():
    cfg = GPTConfig(vocab_size=512, seq_len=512, d_model=256, n_head=4, n_layer=2, d_ff=1024, linear="pallas")
    params = init_params(0, cfg)
    eng = Engine(params, cfg, ServeConfig(batch=4, max_len=512, buckets=(128, 256)))
    rng = np.random.default_rng(0)
    prompts = [list(rng.integers(0, 512, size=n)) for n in (200, 17, 256, 130)]
    tok, pos, kc, vc = eng.prefill(prompts)
    tokens = torch.zeros(4, 256, dtype=torch.long, device="cuda")
    for i, p in enumerate(prompts):
        tokens[i, : len(p)] = torch.tensor(p)
    logits, kc2, vc2 = prefill(params, tokens, pos, cfg, 512)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(tok, torch.argmax(logits, -1))
    # plain (xla) prefill agrees within bf16 tolerance
    _, kc3, vc3 = prefill(params, tokens, pos, cfg.replace(attention="xla", norm="xla", linear="xla"), 512)
    assert (kc.float() - kc3.float()).abs().max().item() < 5e-2
    assert (vc.float() - vc3.float()).abs().max().item() < 5e-2


def test_bucket_errors():
    params = init_params(0, CFG)
    with pytest.raises(ValueError):
        Engine(params, CFG, ServeConfig(batch=1, max_len=512, buckets=(128,)))
