"""CPU checks of the oracle: pinned against its float64 twin, the restated
materialised references (within the reference tests' own tolerances), analytic
identities and the committed golden fixtures."""

import os

import numpy as np
import pytest
import torch

from helpers import BF16, load_arrays, max_abs, normal, rel_l2
from oracle import attention as oa
from oracle import matmul as om
from oracle import rmsnorm as on

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# ---------------------------------------------------------------- rmsnorm


@pytest.mark.parametrize("shape", [(4, 64, 256), (300, 384), (2, 8, 128)])
def test_rmsnorm_f32_matches_f64_twin(rng, shape):
    x = normal(rng, shape)
    w = (1 + 0.1 * rng.standard_normal(shape[-1])).astype(np.float32)
    y32 = on.rmsnorm_fwd(x, w)
    y64 = on.rmsnorm_fwd(x, w, acc=np.float64)
    np.testing.assert_allclose(y32, y64, atol=1e-5, rtol=1e-5)  # test_rmsnorm.py:14 tolerance


def test_add_rmsnorm_y_uses_unrounded_h(rng):
    x, r = normal(rng, (8, 256), BF16), normal(rng, (8, 256), BF16)
    w = np.ones(256, np.float32)
    h, y = on.add_rmsnorm_fwd(x, r, w)
    hf = x.astype(np.float32) + r.astype(np.float32)
    y_unrounded = (hf / np.sqrt(np.mean(hf * hf, -1, keepdims=True) + 1e-6)).astype(BF16)
    assert np.array_equal(y.view(np.uint16), y_unrounded.view(np.uint16))
    assert h.dtype == BF16


def test_rmsnorm_bwd_matches_numeric_gradient(rng):
    """_rmsnorm_bwd_math (rmsnorm.py:159-166) is the exact VJP: check with float64 finite differences."""
    n, d = 6, 32
    h = rng.standard_normal((n, d))
    w = 1 + 0.1 * rng.standard_normal(d)
    dy = rng.standard_normal((n, d))
    dhd = rng.standard_normal((n, d))
    eps = 1e-6

    def loss(hh, ww):
        y = hh / np.sqrt(np.mean(hh * hh, -1, keepdims=True) + eps) * ww
        return float(np.sum(y * dy) + np.sum(hh * dhd))

    dh, dw = on.rmsnorm_bwd(h, w, dy, dhd, eps, acc=np.float64)
    step = 1e-6
    num_dh = np.zeros_like(h)
    for i in range(n):
        for j in range(d):
            e = np.zeros_like(h)
            e[i, j] = step
            num_dh[i, j] = (loss(h + e, w) - loss(h - e, w)) / (2 * step)
    num_dw = np.array([(loss(h, w + step * np.eye(d)[j]) - loss(h, w - step * np.eye(d)[j])) / (2 * step) for j in range(d)])
    np.testing.assert_allclose(dh, num_dh, atol=1e-6, rtol=1e-6)
    np.testing.assert_allclose(dw, num_dw, atol=1e-6, rtol=1e-6)


def test_rmsnorm_golden_fixtures_reproduce():
    g = load_arrays(os.path.join(GOLDEN, "add_rmsnorm_bf16_16x4096.npz"))
    h, y = on.add_rmsnorm_fwd(g["x"], g["r"], g["w"], 1e-6)
    dh, dw = on.rmsnorm_bwd(h, g["w"], g["dy"], g["dh_direct"], 1e-6)
    for a, b in ((h, g["h"]), (y, g["y"]), (dh, g["dh"]), (dw, g["dw"])):
        assert np.array_equal(np.asarray(a).view(np.uint8), np.asarray(b).view(np.uint8))
    g = load_arrays(os.path.join(GOLDEN, "rmsnorm_f32_40x384.npz"))
    y = on.rmsnorm_fwd(g["x"], g["w"], 1e-6)
    dx, dw = on.rmsnorm_bwd(g["x"], g["w"], g["dy"], None, 1e-6)
    np.testing.assert_array_equal(y, g["y"])
    np.testing.assert_array_equal(dx, g["dx"])
    np.testing.assert_array_equal(dw, g["dw"])


# ---------------------------------------------------------------- attention


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("s,d,bq,bk", [(256, 128, 128, 128), (512, 64, 128, 256), (256, 256, 64, 128)])
def test_flash_fwd_f32_matches_reference(rng, causal, s, d, bq, bk):
    """test_flash_attention.py:18-24 restated on the oracle (atol=rtol=2e-5)."""
    q, k, v = (normal(rng, (1, 2, s, d)) for _ in range(3))
    out, lse = oa.flash_fwd(q, k, v, causal=causal, bq=bq, bk=bk)
    ref = oa.reference_fwd(q, k, v, causal=causal)
    np.testing.assert_allclose(out, ref, atol=2e-5, rtol=2e-5)
    # lse = log sum exp of the scaled, masked scores
    sc = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), k.astype(np.float64)) / np.sqrt(d)
    if causal:
        sc = np.where(np.tril(np.ones((s, s), bool)), sc, -np.inf)
    mx = sc.max(-1, keepdims=True)
    lse64 = (mx + np.log(np.exp(sc - mx).sum(-1, keepdims=True)))[..., 0]
    np.testing.assert_allclose(lse, lse64, atol=1e-4, rtol=1e-5)


def test_flash_fwd_bf16_matches_reference(rng):
    q, k, v = (normal(rng, (2, 2, 256, 128), BF16) for _ in range(3))
    out, _ = oa.flash_fwd(q, k, v, causal=True)
    ref = oa.reference_fwd(q, k, v, causal=True)
    assert out.dtype == BF16
    assert max_abs(out, ref) < 2e-2


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("s,d,bq,bk", [(256, 128, 128, 128), (384, 64, 64, 128)])
def test_flash_bwd_f32_matches_reference(rng, causal, s, d, bq, bk):
    """test_flash_attention.py:35-47 restated (5e-4)."""
    q, k, v, do = (normal(rng, (1, 2, s, d)) for _ in range(4))
    out, lse = oa.flash_fwd(q, k, v, causal=causal)
    g = oa.flash_bwd(q, k, v, out, lse, do, causal=causal, bq=bq, bk=bk)
    g_ref = oa.reference_bwd(q, k, v, do, causal=causal, acc=np.float64)
    for a, b in zip(g, g_ref):
        np.testing.assert_allclose(a, b, atol=5e-4, rtol=5e-4)


def test_flash_bwd_bf16_is_close(rng):
    q, k, v = (normal(rng, (1, 2, 256, 128), BF16) for _ in range(3))
    out, lse = oa.flash_fwd(q, k, v, causal=True)
    do = (2 * out.astype(np.float32)).astype(BF16)  # d/dout sum(out^2)
    g = oa.flash_bwd(q, k, v, out, lse, do, causal=True)
    ref_out = oa.reference_fwd(q, k, v, causal=True).astype(np.float32)
    g_ref = oa.reference_bwd(q, k, v, (2 * ref_out), causal=True)
    for a, b in zip(g, g_ref):
        assert rel_l2(a, b) < 5e-2


def test_flash_prefix_invariance(rng):
    q, k, v = (normal(rng, (1, 1, 512, 128)) for _ in range(3))
    full, _ = oa.flash_fwd(q, k, v, causal=True)
    short, _ = oa.flash_fwd(q[:, :, :256], k[:, :, :256], v[:, :, :256], causal=True)
    np.testing.assert_allclose(full[:, :, :256], short, atol=2e-5, rtol=2e-5)


def test_attention_golden_fixture_reproduces():
    g = load_arrays(os.path.join(GOLDEN, "attn_causal_bf16_1x2x256x64.npz"))
    out, lse = oa.flash_fwd(g["q"], g["k"], g["v"], causal=True, scale=1 / 8)
    dq, dk, dv = oa.flash_bwd(g["q"], g["k"], g["v"], out, lse, g["do"], causal=True, scale=1 / 8)
    for a, name in ((out, "out"), (lse, "lse"), (dq, "dq"), (dk, "dk"), (dv, "dv")):
        assert np.array_equal(np.asarray(a).view(np.uint8), np.asarray(g[name]).view(np.uint8)), name


def test_attention_flops_formula():
    assert oa.attention_flops(2, 4, 512, 512, 64, causal=True) == 268435456
    assert oa.attention_flops(8, 32, 8192, 8192, 128, causal=True, backward=True) + oa.attention_flops(8, 32, 8192, 8192, 128, causal=True) == 15393162788864


# ---------------------------------------------------------------- matmul


def test_matmul_oracle_and_vjp(rng):
    x, y = normal(rng, (77, 130)), normal(rng, (130, 203))
    g = normal(rng, (77, 203))
    out = om.matmul_reference(x, y)
    np.testing.assert_allclose(out, x.astype(np.float64) @ y.astype(np.float64), atol=1e-4, rtol=1e-5)
    dx, dy = om.matmul_vjp(x, y, g)
    np.testing.assert_allclose(dx, g.astype(np.float64) @ y.T.astype(np.float64), atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(dy, x.T.astype(np.float64) @ g.astype(np.float64), atol=1e-4, rtol=1e-5)


def test_matmul_golden_fixture_reproduces():
    g = load_arrays(os.path.join(GOLDEN, "matmul_ragged_bf16_77x130x203.npz"))
    assert np.array_equal(om.matmul_reference(g["x"], g["y"]).view(np.uint16), g["out"].view(np.uint16))
    np.testing.assert_array_equal(om.matmul_reference(g["x"], g["y"], out_dtype=np.float32), g["out_f32"])


# ---------------------------------------------------------------- cross-entropy oracle


def test_xent_oracle_against_torch_log_softmax():
    """The loss restatement (gpt.py:147-152) against torch's f32 log_softmax/NLL on CPU."""
    from oracle import xent as ox

    rng = np.random.default_rng(0)
    x = (3.0 * rng.standard_normal((64, 1000))).astype(np.float32)
    t = rng.integers(0, 1000, 64)
    xt = torch.from_numpy(x).requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(xt, torch.from_numpy(t))
    ref.backward()
    assert abs(ox.loss(x, t) - ref.item()) < 1e-5
    np.testing.assert_allclose(ox.xent_bwd(x, t), xt.grad.numpy(), atol=1e-7, rtol=1e-4)
    l, nll = ox.xent_fwd(x, t)
    np.testing.assert_allclose(l, torch.logsumexp(torch.from_numpy(x), -1).numpy(), rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(nll, ox.xent_fwd(x, t, acc=np.float64)[1], rtol=1e-5, atol=1e-5)
