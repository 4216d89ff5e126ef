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
