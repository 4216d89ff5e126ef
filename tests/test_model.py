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


def test_fused_adamw_matches_reference_adamw():
    """ferrite_adamw_step over flat buffers vs the per-tensor restatement of
    adamw_update (train.py:59-74): clipping active (large grads) and inactive,
    decay on ndim >= 2 only, a summed-gradient pre-scale."""
    from ferrite.model.train import AdamW, FusedAdamW, TrainConfig

    tcfg = TrainConfig(steps=10, lr=1e-2, warmup=2, weight_decay=0.1, clip=1.0)

    def make():
        p = init_params(0, TINY)
        leaves = param_leaves(p)
        for t in leaves:
            t.requires_grad_(True)
        return leaves

    ref_leaves, fused_leaves = make(), make()
    ref = AdamW(ref_leaves, tcfg)
    fused = FusedAdamW(fused_leaves, tcfg)
    g = torch.Generator(device="cuda").manual_seed(3)
    for step, mag in enumerate((5.0, 0.01, 3.0)):
        grads = [mag * torch.randn(t.shape, device="cuda", generator=g) for t in ref_leaves]
        slot = {id(t): i for i, t in enumerate(fused.order)}  # identity, not tensor ==
        for t, gr in zip(fused_leaves, grads):
            fused.grads.views[slot[id(t)]].copy_(2.0 * gr)  # summed over 2 "ranks"
        gn_ref = ref.update(grads)
        gn = fused.update(grad_scale=0.5)
        torch.testing.assert_close(gn, gn_ref.float(), rtol=1e-5, atol=1e-6)
        for a, b in zip(fused_leaves, ref_leaves):
            torch.testing.assert_close(a.detach(), b.detach(), rtol=2e-5, atol=2e-6)
        torch.testing.assert_close(fused.m.sum(), torch.stack([m.sum() for m in ref.m]).sum(), rtol=1e-4, atol=1e-4)


def test_train_step_with_fused_optimizer_reduces_loss():
    from ferrite.model.train import TrainConfig, build_train_step, make_optimizer

    cfg = TINY.replace(dtype=torch.bfloat16, linear="pallas")
    params = init_params(0, cfg)
    leaves = param_leaves(params)
    for p in leaves:
        p.requires_grad_(True)
    tcfg = TrainConfig(steps=20, lr=3e-3, warmup=2)
    opt, flat = make_optimizer(leaves, tcfg, late=(params["tok_emb"], params["pos_emb"]))
    step = build_train_step(cfg, tcfg, leaves, opt, flat, params)
    x = _tokens(4, 128, 256)
    y = torch.roll(x, -1, dims=1)
    losses = [float(step(x, y)[0]) for _ in range(8)]
    assert losses[-1] < losses[0] and all(np.isfinite(losses))


def test_fused_mlp_matches_unfused_chain():
    """GELU in the GEMM epilogues (forward u/a, backward dU) against the unfused
    matmul -> torch gelu(tanh) -> matmul chain with the same rounding points."""
    import torch.nn.functional as F

    from ferrite.kernels.matmul import matmul
    from ferrite.model.gpt import _FusedMlp

    g = torch.Generator(device="cuda").manual_seed(0)
    T, d, f = 512, 256, 1024
    y = torch.randn(T, d, device="cuda", generator=g).to(torch.bfloat16).requires_grad_(True)
    w1 = (0.05 * torch.randn(d, f, device="cuda", generator=g)).to(torch.bfloat16).requires_grad_(True)
    w2 = (0.05 * torch.randn(f, d, device="cuda", generator=g)).to(torch.bfloat16).requires_grad_(True)
    dp = torch.randn(T, d, device="cuda", generator=g).to(torch.bfloat16)
    out = _FusedMlp.apply(y, w1, w2)
    out.backward(dp)
    y2, w1b, w2b = (t.detach().clone().requires_grad_(True) for t in (y, w1, w2))
    ref = matmul(F.gelu(matmul(y2, w1b), approximate="tanh"), w2b)
    ref.backward(dp)
    torch.testing.assert_close(out, ref, rtol=1e-2, atol=1e-2)
    assert (out != ref).float().mean().item() < 0.01  # all but rare last-bit differences
    for got, want in ((y.grad, y2.grad), (w1.grad, w1b.grad), (w2.grad, w2b.grad)):
        scale = want.float().abs().max().item()
        assert (got.float() - want.float()).abs().max().item() <= 1e-2 * scale
