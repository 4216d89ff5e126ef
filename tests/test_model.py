"""GPU tests of the callers on the kernels: the GPT forward/gradients through the
``pallas`` slot agree with the plain (``xla``) slot, training reduces the loss,
and the data-parallel step runs (tests/test_model.py of anxnd2211/ferrite-tpu
re-pointed at the B200 kernels)."""

import numpy as np
import pytest
import torch

from ferrite.model import data as data_lib
from ferrite.model.gpt import GPTConfig, forward, init_params, loss_fn, param_count, param_leaves
from ferrite.model.train import TrainConfig, train

pytestmark = pytest.mark.gpu
torch.backends.cuda.matmul.allow_tf32 = False
TINY = GPTConfig(vocab_size=256, seq_len=128, d_model=256, n_head=2, n_layer=2, d_ff=512, dtype=torch.float32)


def _tokens(b=2, s=128, v=256, seed=1):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randint(0, v, (b, s), device="cuda", generator=g)


def test_pallas_and_xla_paths_agree():
    params = init_params(0, TINY)
    tokens = _tokens()
    out_pallas = forward(params, tokens, TINY)
    out_xla = forward(params, tokens, TINY.replace(attention="xla", norm="xla"))
    assert out_pallas.shape == (2, 128, 256)
    torch.testing.assert_close(out_pallas, out_xla, atol=2e-4, rtol=2e-4)


def test_pallas_linear_path_agrees():
    params = init_params(0, TINY)
    tokens = _tokens()
    a = forward(params, tokens, TINY.replace(linear="pallas"))
    b = forward(params, tokens, TINY.replace(attention="xla", norm="xla", linear="xla"))
    torch.testing.assert_close(a, b, atol=5e-4, rtol=5e-4)


def test_gradients_agree_between_paths():
    x = _tokens()
    y = torch.roll(x, -1, dims=1)

    def grads(cfg):
        params = init_params(0, TINY)
        leaves = param_leaves(params)
        for p in leaves:
            p.requires_grad_(True)
        loss_fn(params, x, y, cfg).backward()
        return [p.grad for p in leaves]

    g1 = grads(TINY.replace(linear="pallas"))
    g2 = grads(TINY.replace(attention="xla", norm="xla"))
    for a, b in zip(g1, g2):
        torch.testing.assert_close(a, b, atol=2e-4, rtol=2e-3)


def test_bf16_all_kernels_forward_close_to_xla():
    cfg = GPTConfig(vocab_size=512, seq_len=256, d_model=256, n_head=4, n_layer=2, d_ff=1024, linear="pallas")
    params = init_params(0, cfg)
    tokens = _tokens(2, 256, 512)
    a = forward(params, tokens, cfg)
    b = forward(params, tokens, cfg.replace(attention="xla", norm="xla", linear="xla"))
    assert torch.isfinite(a).all()
    assert (a - b).abs().max().item() < 5e-2


def test_param_count_matches_formula():
    params = init_params(0, TINY)
    d, f, L, V, S = TINY.d_model, TINY.d_ff, TINY.n_layer, TINY.vocab_size, TINY.seq_len
    assert param_count(params) == V * d + S * d + d + L * (2 * d + 3 * d * d + d * d + d * f + f * d)


def test_short_training_run_reduces_loss(tmp_path):
    cfg = TINY.replace(seq_len=128, d_model=128, n_head=1, n_layer=1, d_ff=256)
    tcfg = TrainConfig(steps=12, batch=8, lr=3e-3, warmup=2, log_every=100, data="synthetic", out=str(tmp_path / "r.json"), save_params=str(tmp_path / "p.npz"))
    res = train(cfg, tcfg, verbose=False)
    assert res["loss_last"] < res["loss_first"]
    assert (tmp_path / "r.json").exists() and (tmp_path / "p.npz").exists()
    assert res["tokens_per_second"] > 0


def test_bf16_training_on_all_kernels_reduces_loss():
    cfg = GPTConfig(vocab_size=256, seq_len=256, d_model=256, n_head=2, n_layer=2, d_ff=1024, linear="pallas")
    tcfg = TrainConfig(steps=30, batch=16, lr=3e-3, warmup=3, log_every=100, data="synthetic")
    res = train(cfg, tcfg, verbose=False)
    assert np.isfinite(res["loss_last"]) and res["loss_last"] < res["loss_first"] - 0.5
