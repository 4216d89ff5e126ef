"""CPU tests of the caller-side host logic: parameter/FLOP accounting, data
generators, the LR schedule and AdamW arithmetic (restated from the reference's
formulas), bucket selection."""

import math

import numpy as np
import pytest
import torch

from ferrite.model import data as data_lib
from ferrite.model.gpt import GPTConfig, flops_per_token, init_params, param_count
from ferrite.model.train import AdamW, TrainConfig, lr_at
from ferrite.serving.engine import bucket_for


def test_gpt_config_flops_match_baseline():
    cfg = GPTConfig(vocab_size=32000, seq_len=1024, d_model=1024, n_head=16, n_layer=24, d_ff=4096)
    params = init_params(0, cfg.replace(n_layer=1), device="cpu")
    one = param_count(params)
    n_total = one + 23 * (2 * 1024 + 4 * 1024 * 1024 + 2 * 1024 * 4096)
    n_nonembed = n_total - 32000 * 1024 - 1024 * 1024
    assert n_total == 335_856_640 and n_nonembed == 302_040_064
    fpt = flops_per_token(cfg, n_nonembed)["total"]
    assert 3 * fpt * 64 * 1024 == pytest.approx(1.4155e14, rel=1e-4)


def test_attention_blocks_rule():
    cfg = GPTConfig()
    assert cfg.attention_blocks(1024).block_q == 128
    assert cfg.attention_blocks(100) is None


def test_synthetic_data_batches():
    corpus = data_lib.synthetic(20_000, seed=1)
    assert corpus.dtype == np.uint8 and corpus.max() < 64
    x, y = data_lib.get_batch(np.random.default_rng(0), corpus, 4, 16)
    assert x.shape == (4, 16) and y.shape == (4, 16)
    np.testing.assert_array_equal(x[:, 1:], y[:, :-1])
    np.testing.assert_array_equal(data_lib.synthetic(20_000, seed=1), corpus)
    xu, yu = data_lib.uniform_batch(np.random.default_rng(0), 3, 8, 32000)
    assert xu.max() < 32000 and np.array_equal(xu[:, 1:], yu[:, :-1])


def test_lr_schedule():
    cfg = TrainConfig(steps=100, lr=1.0, warmup=10)
    assert lr_at(0, cfg) == pytest.approx(0.1)
    assert lr_at(10, cfg) == pytest.approx(1.0)
    assert lr_at(100, cfg) == pytest.approx(0.1)
    assert lr_at(55, cfg) == pytest.approx(0.1 + 0.9 * 0.5 * (1 + math.cos(math.pi * 0.5)))


def test_adamw_matches_reference_formula():
    rng = np.random.default_rng(0)
    cfg = TrainConfig(steps=10, lr=0.01, warmup=2, weight_decay=0.1, clip=1.0)
    p2 = rng.standard_normal((4, 3)).astype(np.float32)
    p1 = rng.standard_normal(3).astype(np.float32)
    params = [torch.tensor(p2), torch.tensor(p1)]
    opt = AdamW(params, cfg)
    m = [np.zeros_like(p2), np.zeros_like(p1)]
    v = [np.zeros_like(p2), np.zeros_like(p1)]
    ref = [p2.astype(np.float64), p1.astype(np.float64)]
    for step in range(1, 4):
        g = [rng.standard_normal(p.shape).astype(np.float32) * 3 for p in (p2, p1)]
        opt.update([torch.tensor(x) for x in g])
        lr = lr_at(step, cfg)
        gn = math.sqrt(sum(float(np.sum(x.astype(np.float64) ** 2)) for x in g))
        sc = min(1.0, cfg.clip / (gn + 1e-6))
        for i, (gi, dec) in enumerate(zip(g, (0.1, 0.0))):
            gi = gi * sc
            m[i] = 0.9 * m[i] + 0.1 * gi
            v[i] = 0.95 * v[i] + 0.05 * gi * gi
            upd = (m[i] / (1 - 0.9**step)) / (np.sqrt(v[i] / (1 - 0.95**step)) + 1e-8) + dec * ref[i]
            ref[i] = ref[i] - lr * upd
    for p, r in zip(params, ref):
        np.testing.assert_allclose(p.numpy(), r, atol=1e-5, rtol=1e-5)


def test_bucket_selection():
    assert bucket_for(1, (64, 128)) == 64 and bucket_for(64, (64, 128)) == 64 and bucket_for(65, (64, 128)) == 128
    with pytest.raises(ValueError):
        bucket_for(129, (64, 128))
