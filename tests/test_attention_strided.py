"""GPU parity of the strided attention entry points.

The kernels read q/k/v and write o, dq/dk/dv through per-operand (batch, head,
sequence) strides.  The packed ``[b, s, 3, h, d]`` projection of the GPT block
(``flash_attention_packed``) must give bitwise the same outputs and gradients as
the contiguous path on copied-out q/k/v -- the same kernels run the same
arithmetic, only the addresses differ -- and layouts the tensor-core path cannot
read (unaligned bases) must still be correct on the CUDA-core path.
"""

import numpy as np
import pytest
import torch

from ferrite.kernels.flash_attention import BlockSizes, flash_attention, flash_attention_packed
from helpers import BF16, assert_bf16_close, max_abs, normal, rel_l2, to_numpy, to_torch
from oracle import attention as oa

pytestmark = pytest.mark.gpu


def _packed(rng, b, s, h, d, dtype):
    return to_torch(normal(rng, (b, s, 3, h, d), dtype))


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", [BF16, np.float16])
def test_packed_equals_contiguous_bitwise(d, dtype):
    rng = np.random.default_rng(d)
    b, s, h = 2, 512, 4
    qkv = _packed(rng, b, s, h, d, dtype).requires_grad_(True)
    do = to_torch(normal(rng, (b, s, h, d), dtype))
    out = flash_attention_packed(qkv, causal=True)
    out.backward(do)
    q, k, v = (qkv.detach()[:, :, i].transpose(1, 2).contiguous().requires_grad_(True) for i in range(3))
    ref = flash_attention(q, k, v, causal=True)
    ref.backward(do.transpose(1, 2).contiguous())
    assert out.shape == (b, s, h, d) and out.is_contiguous()
    assert torch.equal(out, ref.transpose(1, 2))
    for i, t in enumerate((q, k, v)):
        assert torch.equal(qkv.grad[:, :, i], t.grad.transpose(1, 2)), "qkv"[i]


def test_packed_vs_oracle_bf16():
    rng = np.random.default_rng(11)
    b, s, h, d = 1, 256, 2, 64
    qkv_np = normal(rng, (b, s, 3, h, d), BF16)
    do_np = normal(rng, (b, s, h, d), BF16)
    qkv = to_torch(qkv_np).requires_grad_(True)
    out = flash_attention_packed(qkv, causal=True)
    out.backward(to_torch(do_np))
    q, k, v = (np.ascontiguousarray(qkv_np[:, :, i].transpose(0, 2, 1, 3)) for i in range(3))
    do_bhsd = np.ascontiguousarray(do_np.transpose(0, 2, 1, 3))
    o_ref, lse = oa.flash_fwd(q, k, v, causal=True)
    dq, dk, dv = oa.flash_bwd(q, k, v, o_ref, lse, do_bhsd, causal=True)
    assert_bf16_close(out.transpose(1, 2), o_ref)
    for i, ref in enumerate((dq, dk, dv)):
        g = qkv.grad[:, :, i].transpose(1, 2)
        assert max_abs(g, ref) <= 2e-2 and rel_l2(g, ref) < 1e-2, "qkv"[i]


def test_packed_f32_runs_the_cuda_core_path_exactly():
    """f32 (Precision.HIGHEST contract) through the strided CUDA-core kernels."""
    rng = np.random.default_rng(3)
    b, s, h, d = 1, 256, 2, 64
    qkv_np = normal(rng, (b, s, 3, h, d))
    do_np = normal(rng, (b, s, h, d))
    qkv = to_torch(qkv_np).requires_grad_(True)
    out = flash_attention_packed(qkv, causal=True)
    out.backward(to_torch(do_np))
    q, k, v = (np.ascontiguousarray(qkv_np[:, :, i].transpose(0, 2, 1, 3)) for i in range(3))
    np.testing.assert_allclose(to_numpy(out.transpose(1, 2)), oa.reference_fwd(q, k, v, causal=True), atol=2e-5, rtol=2e-5)
    dq, dk, dv = oa.reference_bwd(q, k, v, np.ascontiguousarray(do_np.transpose(0, 2, 1, 3)), causal=True)
    for i, ref in enumerate((dq, dk, dv)):
        np.testing.assert_allclose(to_numpy(qkv.grad[:, :, i].transpose(1, 2)), ref, atol=5e-4, rtol=5e-4)


def test_transposed_views_and_noncausal():
    """q, k, v as separate [b, s, h, d] buffers viewed as [b, h, s, d]; non-causal."""
    rng = np.random.default_rng(5)
    b, s, h, d = 2, 256, 3, 128
    bshd = [to_torch(normal(rng, (b, s, h, d), BF16)) for _ in range(3)]
    views = [t.transpose(1, 2) for t in bshd]
    out = flash_attention(*views, causal=False, block_sizes=BlockSizes(128, 128))
    ref = flash_attention(*(t.contiguous() for t in views), causal=False, block_sizes=BlockSizes(128, 128))
    assert torch.equal(out, ref)


def test_unaligned_base_falls_back_to_cuda_cores():
    """A q whose base is 8 bytes off a 16-byte boundary cannot feed TMA; the call
    still succeeds (CUDA-core path) and matches the oracle."""
    rng = np.random.default_rng(9)
    b, h, s, d = 1, 2, 256, 64
    qn, kn, vn = (normal(rng, (b, h, s, d), BF16) for _ in range(3))
    store = torch.empty(b * h * s * d + 4, dtype=torch.bfloat16, device="cuda")
    q = store[4:].view(b, h, s, d)
    q.copy_(to_torch(qn))
    assert q.data_ptr() % 16 == 8
    out = flash_attention(q, to_torch(kn), to_torch(vn), causal=True)
    ref = oa.reference_fwd(qn, kn, vn, causal=True)
    assert max_abs(out, ref) <= 2e-2


# ---------------------------------------------------------------- materialised-dS backward


def _bwd(q, k, v, do, causal):
    from ferrite.kernels.flash_attention import flash_backward, flash_forward_with_lse

    out, lse = flash_forward_with_lse(q, k, v, causal=causal)
    return flash_backward(q, k, v, out, lse, do, causal=causal), out, lse


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("budget_slices", [1, 4, None])
def test_ds_backward_matches_recompute_and_oracle(monkeypatch, d, causal, budget_slices):
    """dQ from the stored dS (a workspace of the whole batch, or of 1 / 4 of the 6
    slices: the fused backward then recycles its dS slots) against the recompute
    path and the blockwise oracle.  The fused backward accumulates dK/dV over the
    query tiles last-first, the recompute kernel first-last: equal up to f32
    summation order, so compared at the dQ bound."""
    import importlib

    from ferrite import _native as nat

    fa = importlib.import_module("ferrite.kernels.flash_attention")  # the module, not the re-exported function

    rng = np.random.default_rng(d + causal)
    b, h, s = 2, 3, 512
    qn, kn, vn, don = (normal(rng, (b, h, s, d), BF16) for _ in range(4))
    q, k, v, do = (to_torch(a) for a in (qn, kn, vn, don))
    per_slice = nat.lib().ferrite_attn_bwd_ds_workspace_size(1, 1, s, s, d, nat.BF16)
    assert per_slice >= s * s * 2  # one dS slice (+ the fused backward's scheduler state)
    if budget_slices is not None:
        monkeypatch.setattr(fa, "DS_WORKSPACE_BUDGET", budget_slices * per_slice)
    (dq, dk, dv), out, lse = _bwd(q, k, v, do, causal)
    monkeypatch.setenv("FERRITE_ATTN_BWD_DS", "0")
    (dq0, dk0, dv0), _, _ = _bwd(q, k, v, do, causal)
    for a, b_ in ((dq, dq0), (dk, dk0), (dv, dv0)):
        assert_bf16_close(a, b_, atol=4e-3)
    o_ref, lse_ref = oa.flash_fwd(qn, kn, vn, causal=causal)
    g_ref = oa.flash_bwd(qn, kn, vn, o_ref, lse_ref, don, causal=causal)
    for got, ref, name in zip((dq, dk, dv), g_ref, ("dq", "dk", "dv")):
        assert max_abs(got, ref) <= 2e-2, name
        assert rel_l2(got, ref) < 1e-2, name


def test_ds_backward_ragged_noncausal_query_length():
    """sq = 200 (not a multiple of the 64-query tile; dS rows padded to 256) with
    sk = 384, non-causal."""
    rng = np.random.default_rng(21)
    qn = normal(rng, (1, 2, 200, 64), BF16)
    kn, vn = normal(rng, (1, 2, 384, 64), BF16), normal(rng, (1, 2, 384, 64), BF16)
    don = normal(rng, (1, 2, 200, 64), BF16)
    from ferrite.kernels.flash_attention import flash_backward, flash_forward_with_lse

    bs = BlockSizes(8, 128, 8, 128)
    q, k, v, do = (to_torch(a) for a in (qn, kn, vn, don))
    out, lse = flash_forward_with_lse(q, k, v, causal=False, block_sizes=bs)
    dq, dk, dv = flash_backward(q, k, v, out, lse, do, causal=False, block_sizes=bs)
    dq_r, dk_r, dv_r = oa.reference_bwd(qn, kn, vn, don, causal=False)
    for got, ref, name in zip((dq, dk, dv), (dq_r, dk_r, dv_r), ("dq", "dk", "dv")):
        assert max_abs(got, ref) <= 2e-2, name


def test_ds_backward_is_deterministic():
    g = torch.Generator(device="cuda").manual_seed(4)
    q, k, v, do = (torch.randn(2, 4, 1024, 128, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
    a, _, _ = _bwd(q, k, v, do, True)
    b_, _, _ = _bwd(q, k, v, do, True)
    for x, y in zip(a, b_):
        assert torch.equal(x, y)


def test_split_dkv_ds_and_dq_ds_entry_points_over_slice_ranges():
    """The two halves called separately on slice ranges [0, 2) and [2, 6) give
    the same gradients as the one-call (fused) backward: dQ bitwise (same dS, same
    product order), dK/dV up to the order of their f32 sums over query tiles."""
    import ctypes

    from ferrite import _native as nat
    from ferrite.kernels.flash_attention import flash_backward, flash_forward_with_lse

    g = torch.Generator(device="cuda").manual_seed(8)
    b, h, s, d = 2, 3, 256, 128
    q, k, v, do = (torch.randn(b, h, s, d, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
    out, lse = flash_forward_with_lse(q, k, v, causal=True)
    dq_ref, dk_ref, dv_ref = flash_backward(q, k, v, out, lse, do, causal=True)
    lib = nat.lib()
    sp = nat.stream_ptr()
    delta = torch.empty(b, h, s, device="cuda")
    nat.check(lib.ferrite_attn_bwd_prep(sp, do.data_ptr(), out.data_ptr(), delta.data_ptr(), b, h, s, d, nat.BF16))
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    st = nat.attn_strides(q=q, k=k, v=v, o=out, dout=do, dq=dq, dk=dk, dv=dv)
    ds = torch.empty(4 * s * s * 2, dtype=torch.uint8, device="cuda")  # room for 4 slices
    for begin, count in ((0, 2), (2, 4)):
        nat.check(lib.ferrite_attn_bwd_dkv_ds(sp, q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(), delta.data_ptr(),
                                              dk.data_ptr(), dv.data_ptr(), ds.data_ptr(), ctypes.byref(st), begin, count, b, h, s, s, d,
                                              d**-0.5, 1, 128, 128, nat.BF16))
        nat.check(lib.ferrite_attn_bwd_dq_ds(sp, ds.data_ptr(), k.data_ptr(), dq.data_ptr(), ctypes.byref(st), begin, count, b, h, s, s, d,
                                             d**-0.5, 1, 128, 128, nat.BF16))
    assert torch.equal(dq, dq_ref)
    assert_bf16_close(dk, dk_ref, atol=4e-3)
    assert_bf16_close(dv, dv_ref, atol=4e-3)


# ---------------------------------------------------------------- kernel variants


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal,sq,sk", [(True, 512, 512), (True, 384, 384), (False, 256, 384), (False, 640, 256)])
def test_dkv_128_and_64_query_tiles_agree(monkeypatch, d, causal, sq, sk):
    """The 128-query-tile dK/dV kernel (default) and the 64-query template
    (FERRITE_ATTN_DKV_WIDE=0) form the same rounded P and dS; only the order of
    the f32 accumulation differs.  Both meet the oracle; their dS-based dQ too."""
    rng = np.random.default_rng(d * 7 + sq + sk + causal)
    b, h = 1, 3
    qn, don = normal(rng, (b, h, sq, d), BF16), normal(rng, (b, h, sq, d), BF16)
    kn, vn = normal(rng, (b, h, sk, d), BF16), normal(rng, (b, h, sk, d), BF16)
    q, k, v, do = (to_torch(a) for a in (qn, kn, vn, don))
    (dq, dk, dv), out, lse = _bwd(q, k, v, do, causal)
    monkeypatch.setenv("FERRITE_ATTN_DKV_WIDE", "0")
    (dq0, dk0, dv0), _, _ = _bwd(q, k, v, do, causal)
    for a, b_, name in ((dq, dq0, "dq"), (dk, dk0, "dk"), (dv, dv0, "dv")):
        assert_bf16_close(a, b_, atol=4e-3)
    o_ref, lse_ref = oa.flash_fwd(qn, kn, vn, causal=causal)
    g_ref = oa.flash_bwd(qn, kn, vn, o_ref, lse_ref, don, causal=causal)
    for got, ref, name in zip((dq, dk, dv), g_ref, ("dq", "dk", "dv")):
        assert max_abs(got, ref) <= 2e-2, name
        assert rel_l2(got, ref) < 1e-2, name


@pytest.mark.parametrize("causal", [True, False])
def test_forward_one_and_two_query_tiles_per_cta_agree(monkeypatch, causal):
    """d = 64 forward: one 128-row query tile per CTA (default, two CTAs per SM)
    and two per CTA (FERRITE_ATTN_FWD_NG=2) run the same per-tile arithmetic."""
    from ferrite.kernels.flash_attention import flash_forward_with_lse

    rng = np.random.default_rng(11 + causal)
    qn, kn, vn = (normal(rng, (2, 3, 640, 64), BF16) for _ in range(3))
    q, k, v = (to_torch(a) for a in (qn, kn, vn))
    out1, lse1 = flash_forward_with_lse(q, k, v, causal=causal)
    monkeypatch.setenv("FERRITE_ATTN_FWD_NG", "2")
    out2, lse2 = flash_forward_with_lse(q, k, v, causal=causal)
    assert torch.equal(out1, out2)
    assert torch.equal(lse1, lse2)
    o_ref, lse_ref = oa.flash_fwd(qn, kn, vn, causal=causal)
    assert max_abs(out1, o_ref) <= 2e-2
    np.testing.assert_allclose(to_numpy(lse1), lse_ref, atol=2e-4, rtol=1e-5)
