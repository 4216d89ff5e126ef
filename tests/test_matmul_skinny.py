"""The skinny 16-bit GEMM path (at most 16 rows of A, B stored [N][K]): the serving
prefill's LM head over the last position of each sequence, y = h W^T with W the tied
embedding (gpt.py:143 of anxnd2211/ferrite-tpu).  Checked against a torch fp32 reference
and the oracle (f32 accumulation of exact 16-bit products: differences are summation
order only), at the edges of the path (1 and 16 rows, N not a multiple of 4, K = 8) and
just past them (17 rows, K not a multiple of 8), which take the other kernels.
"""

import numpy as np
import pytest
import torch

from ferrite import _native as nat
from helpers import BF16, normal, to_numpy, to_torch
from oracle import matmul as om

pytestmark = pytest.mark.gpu


def _gemm_tb(a, b, out_dtype):
    """a [m, k], b [n, k] -> a b^T through ferrite_gemm (trans_b)."""
    m, k = a.shape
    n = b.shape[0]
    c = torch.empty(m, n, dtype=out_dtype, device="cuda")
    nat.check(nat.lib().ferrite_gemm(nat.stream_ptr(), a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, a.stride(0), b.stride(0),
                                     c.stride(0), 0, 1, nat.dtype_code(a.dtype), nat.dtype_code(c.dtype)))
    torch.cuda.synchronize()
    return c


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(1, 5, 8), (3, 1000, 1024), (8, 32000, 1024), (9, 777, 2048), (16, 4099, 3072), (17, 300, 512), (8, 64, 1001)])
def test_skinny_matches_fp32_reference(dtype, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m * 1000 + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).to(dtype)
    b = (torch.randn(n, k, device="cuda", generator=g) / np.sqrt(k)).to(dtype)
    ref = a.float() @ b.float().t()
    got = _gemm_tb(a, b, torch.float32)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-4)
    got16 = _gemm_tb(a, b, dtype)
    torch.testing.assert_close(got16.float(), ref, rtol=2**-7, atol=1e-3)


def test_lm_head_shape_against_the_oracle():
    """bf16 h [8, 1024] against a [32000, 1024] tied embedding, f32 logits."""
    rng = np.random.default_rng(5)
    h = normal(rng, (8, 1024), BF16)
    w = normal(rng, (32000, 1024), BF16, std=0.02)
    got = to_numpy(_gemm_tb(to_torch(h), to_torch(w), torch.float32))
    ref = om.matmul_reference(h, np.ascontiguousarray(w.T), out_dtype=np.float32)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)


def test_strided_rows_and_deterministic():
    """A and B as row slices of larger buffers (lda, ldb > k); repeated calls agree bitwise."""
    g = torch.Generator(device="cuda").manual_seed(3)
    abuf = torch.randn(8, 1536, device="cuda", generator=g).to(torch.bfloat16)
    bbuf = torch.randn(2048, 1536, device="cuda", generator=g).to(torch.bfloat16)
    a, b = abuf[:, :1024], bbuf[:2000, :1024]
    ref = a.float() @ b.float().t()
    got = _gemm_tb(a, b, torch.float32)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-4)
    assert torch.equal(got, _gemm_tb(a, b, torch.float32))
