"""GPU parity of the flash-attention kernels (forward, delta prep, dK/dV, dQ)
against the oracle (blockwise restatement of the reference kernels and the
materialised reference), the golden fixture, and the reference's own test
cases (tests/test_flash_attention.py of anxnd2211/ferrite-tpu, re-pointed at
the CUDA path).

Tolerances: the reference's (f32 forward 2e-5, f32 gradients 5e-4, bf16 forward
2e-2, bf16 gradients relative L2 < 5e-2) and the north star's max-abs 2e-2 on
bf16 outputs and gradients.
"""

import os

import numpy as np
import pytest
import torch

from ferrite import _native as nat
from ferrite.kernels.flash_attention import (
    BlockSizes,
    flash_attention,
    flash_attention_reference,
    flash_backward,
    flash_forward_with_lse,
)
from helpers import BF16, load_arrays, max_abs, normal, rel_l2, to_numpy, to_torch
from oracle import attention as oa

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _qkv(rng, b, h, s, d, dtype, n=3):
    return tuple(normal(rng, (b, h, s, d), dtype) for _ in range(n))


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("s,d,bs", [(256, 128, BlockSizes(128, 128)), (512, 64, BlockSizes(128, 256)), (256, 256, BlockSizes(64, 128))])
def test_forward_f32(rng, causal, s, d, bs):
    """test_flash_attention.py:18-24 (f32, 2e-5)."""
    q, k, v = _qkv(rng, 1, 2, s, d, np.float32)
    out = flash_attention(to_torch(q), to_torch(k), to_torch(v), causal=causal, block_sizes=bs)
    np.testing.assert_allclose(to_numpy(out), oa.reference_fwd(q, k, v, causal=causal), atol=2e-5, rtol=2e-5)


def test_forward_bf16(rng):
    """test_flash_attention.py:27-32 (bf16, 2e-2)."""
    q, k, v = _qkv(rng, 2, 2, 256, 128, BF16)
    out = flash_attention(to_torch(q), to_torch(k), to_torch(v), causal=True)
    assert out.dtype == torch.bfloat16
    ref = oa.reference_fwd(q, k, v, causal=True)
    np.testing.assert_allclose(to_numpy(out).astype(np.float32), ref.astype(np.float32), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("s,d,bs", [(256, 128, BlockSizes()), (384, 64, BlockSizes(128, 128, 64, 128))])
def test_backward_matches_reference(rng, causal, s, d, bs):
    """test_flash_attention.py:35-47 (f32 grads, 5e-4)."""
    q, k, v = _qkv(rng, 1, 2, s, d, np.float32)
    cot = normal(rng, q.shape)
    qt, kt, vt = (to_torch(a).requires_grad_(True) for a in (q, k, v))
    (flash_attention(qt, kt, vt, causal=causal, block_sizes=bs) * to_torch(cot)).sum().backward()
    g_ref = oa.reference_bwd(q, k, v, cot, causal=causal, acc=np.float64)
    for name, a, b in zip("qkv", (qt.grad, kt.grad, vt.grad), g_ref):
        np.testing.assert_allclose(to_numpy(a), b, atol=5e-4, rtol=5e-4, err_msg=f"d{name}")


def test_backward_bf16_is_close(rng):
    """test_flash_attention.py:50-58 (bf16, relative L2 < 5e-2)."""
    q, k, v = _qkv(rng, 1, 2, 256, 128, BF16)
    qt, kt, vt = (to_torch(a).requires_grad_(True) for a in (q, k, v))
    (flash_attention(qt, kt, vt, causal=True).float() ** 2).sum().backward()
    qr, kr, vr = (to_torch(a).float().requires_grad_(True) for a in (q, k, v))
    (flash_attention_reference(qr, kr, vr, causal=True).float() ** 2).sum().backward()
    for a, b in zip((qt.grad, kt.grad, vt.grad), (qr.grad, kr.grad, vr.grad)):
        assert rel_l2(a, b) < 5e-2


def test_causal_output_is_prefix_invariant(rng):
    """test_flash_attention.py:61-66 (f32), and the bf16 tensor-core path bitwise."""
    q, k, v = _qkv(rng, 1, 1, 512, 128, np.float32)
    qt, kt, vt = to_torch(q), to_torch(k), to_torch(v)
    full = flash_attention(qt, kt, vt, causal=True)
    short = flash_attention(qt[:, :, :256], kt[:, :, :256], vt[:, :, :256], causal=True)
    torch.testing.assert_close(full[:, :, :256], short, atol=2e-5, rtol=2e-5)
    qb, kb, vb = (t.to(torch.bfloat16) for t in (qt, kt, vt))
    full = flash_attention(qb, kb, vb, causal=True)
    short = flash_attention(qb[:, :, :256].contiguous(), kb[:, :, :256].contiguous(), vb[:, :, :256].contiguous(), causal=True)
    assert torch.equal(full[:, :, :256], short)


def test_golden_fixture():
    g = load_arrays(os.path.join(GOLDEN, "attn_causal_bf16_1x2x256x64.npz"))
    q, k, v, do = (to_torch(g[n]) for n in ("q", "k", "v", "do"))
    out, lse = flash_forward_with_lse(q, k, v, causal=True, scale=1 / 8)
    assert max_abs(out, g["out"]) <= 2e-2
    np.testing.assert_allclose(to_numpy(lse), g["lse"], atol=1e-4, rtol=1e-5)
    dq, dk, dv = flash_backward(q, k, v, out, lse, do, causal=True, scale=1 / 8)
    for got, name in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        assert max_abs(got, g[name]) <= 2e-2, name


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("d", [64, 128])
def test_small_config_vs_blockwise_oracle(causal, d):
    """Small benchmark config: b2 h4 s512 (d64; also d128), bf16 N(0,1) seed 0, block 128."""
    rng = np.random.default_rng(0)
    q, k, v, do = _qkv(rng, 2, 4, 512, d, BF16, n=4)
    scale = 1 / np.sqrt(d)
    out, lse = flash_forward_with_lse(to_torch(q), to_torch(k), to_torch(v), causal=causal)
    o_ref, lse_ref = oa.flash_fwd(q, k, v, causal=causal, scale=scale)
    assert max_abs(out, o_ref) <= 2e-2
    np.testing.assert_allclose(to_numpy(lse), lse_ref, atol=2e-4, rtol=1e-5)
    dq, dk, dv = flash_backward(to_torch(q), to_torch(k), to_torch(v), out, lse, to_torch(do), causal=causal)
    g_ref = oa.flash_bwd(q, k, v, o_ref, lse_ref, do, causal=causal, scale=scale)
    for got, ref, name in zip((dq, dk, dv), g_ref, ("dq", "dk", "dv")):
        assert max_abs(got, ref) <= 2e-2, name
        assert rel_l2(got, ref) < 1e-2, name


def test_noncausal_unequal_lengths_and_short_query():
    rng = np.random.default_rng(4)
    q = normal(rng, (1, 2, 200, 64), BF16)
    k, v = normal(rng, (1, 2, 384, 64), BF16), normal(rng, (1, 2, 384, 64), BF16)
    out = flash_attention(to_torch(q), to_torch(k), to_torch(v), causal=False, block_sizes=BlockSizes(8, 128, 8, 128))
    assert max_abs(out, oa.reference_fwd(q, k, v, causal=False)) <= 2e-2


@pytest.mark.parametrize("d", [64, 128])
def test_backward_ragged_query_length(d):
    """sq = 200 against sk = 384 (non-causal): the last 128-query tile of the dK/dV
    kernel and the last dS block of the dQ kernel are partly past sq."""
    rng = np.random.default_rng(40 + d)
    q, do = normal(rng, (1, 2, 200, d), BF16), normal(rng, (1, 2, 200, d), BF16)
    k, v = normal(rng, (1, 2, 384, d), BF16), normal(rng, (1, 2, 384, d), BF16)
    bs = BlockSizes(8, 128, 8, 128)
    out, lse = flash_forward_with_lse(to_torch(q), to_torch(k), to_torch(v), causal=False, block_sizes=bs)
    dq, dk, dv = flash_backward(to_torch(q), to_torch(k), to_torch(v), out, lse, to_torch(do), causal=False, block_sizes=bs)
    o_ref, lse_ref = oa.flash_fwd(q, k, v, causal=False, bq=8, bk=128)
    g_ref = oa.flash_bwd(q, k, v, o_ref, lse_ref, do, causal=False, bq=8, bk=128)
    for got, ref, name in zip((dq, dk, dv), g_ref, ("dq", "dk", "dv")):
        assert max_abs(got, ref) <= 2e-2, name
        assert rel_l2(got, ref) < 1e-2, name


@pytest.mark.slow
def test_long_config_forward_sampled_heads():
    """Long-context benchmark config: b8 h32 s8192 d128 bf16; full-size run on the GPU,
    oracle on two (b, h) slices (heads are independent)."""
    b, h, s, d = 8, 32, 8192, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(b, h, s, d, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    out, lse = flash_forward_with_lse(q, k, v, causal=True)
    for bi, hi in ((0, 0), (7, 31)):
        qs, ks, vs = (to_numpy(t[bi : bi + 1, hi : hi + 1]) for t in (q, k, v))
        o_ref, lse_ref = oa.flash_fwd(qs, ks, vs, causal=True)
        assert max_abs(out[bi : bi + 1, hi : hi + 1], o_ref) <= 2e-2
        np.testing.assert_allclose(to_numpy(lse[bi, hi]), lse_ref[0, 0], atol=2e-4, rtol=1e-5)


@pytest.mark.parametrize("s,d,dtype", [(256, 64, BF16), (300, 128, BF16), (129, 256, BF16), (256, 64, np.float32), (77, 96, np.float16), (200, 8, BF16)])
def test_delta_prep(s, d, dtype):
    """Vectorised kernel (16-byte rows of up to 32 vectors) and the generic one (d = 96)."""
    rng = np.random.default_rng(2)
    do, o = normal(rng, (2, 3, s, d), dtype), normal(rng, (2, 3, s, d), dtype)
    delta = torch.empty(2, 3, s, device="cuda")
    dot, ot = to_torch(do), to_torch(o)
    nat.check(nat.lib().ferrite_attn_bwd_prep(nat.stream_ptr(), dot.data_ptr(), ot.data_ptr(), delta.data_ptr(), 2, 3, s, d, nat.dtype_code(dot.dtype)))
    np.testing.assert_allclose(to_numpy(delta), oa.delta(do, o), atol=1e-4, rtol=1e-5)


def test_delta_prep_unaligned_takes_the_generic_kernel():
    rng = np.random.default_rng(6)
    do, o = normal(rng, (1, 2, 128, 64), BF16), normal(rng, (1, 2, 128, 64), BF16)
    store = torch.empty(do.size + 1, dtype=torch.bfloat16, device="cuda")
    dot = store[1:].view(1, 2, 128, 64)
    dot.copy_(to_torch(do))
    ot = to_torch(o)
    delta = torch.empty(1, 2, 128, device="cuda")
    nat.check(nat.lib().ferrite_attn_bwd_prep(nat.stream_ptr(), dot.data_ptr(), ot.data_ptr(), delta.data_ptr(), 1, 2, 128, 64, nat.BF16))
    np.testing.assert_allclose(to_numpy(delta), oa.delta(do, o), atol=1e-4, rtol=1e-5)


def test_deterministic_forward_and_backward():
    g = torch.Generator(device="cuda").manual_seed(1)
    q, k, v, do = (torch.randn(2, 4, 512, 64, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
    o1, l1 = flash_forward_with_lse(q, k, v)
    o2, l2 = flash_forward_with_lse(q, k, v)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    g1 = flash_backward(q, k, v, o1, l1, do)
    g2 = flash_backward(q, k, v, o1, l1, do)
    assert all(torch.equal(a, b) for a, b in zip(g1, g2))


def test_c_abi_rejects_bad_blocks_on_device():
    q = torch.zeros(1, 1, 256, 64, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(1, 1, 256, device="cuda")
    rc = nat.lib().ferrite_attn_fwd(nat.stream_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), lse.data_ptr(), 1, 1, 256, 256, 64, 0.125, 1, 128, 100, nat.BF16)
    assert rc == nat.BAD_SHAPE


def test_device_status_clean_after_attention():
    nat.device_status(clear=True)
