"""The skinny 16-bit GEMM paths (at most 16 rows of A).  B stored [N][K]: the serving
LM head over the last position of each sequence, y = h W^T with W the tied embedding
(gpt.py:143 of anxnd2211/ferrite-tpu).  B stored [K][N]: the decode step's linears,
y = x W (gpt.py:95-104, engine.py:107-131), K split over a thread-block cluster.
Checked against a torch fp32 reference and the oracle (f32 accumulation of exact 16-bit
products: differences are summation order only), at the edges of each path (1, 8, 9 and
16 rows, N not a multiple of 4 or of the 64-column tile, K = 8, K past one load batch
per CTA) and just past them (17 rows, K or N not a multiple of 8), which take the
other kernels.
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
@pytest.mark.parametrize("m,n,k", [(1, 5, 8), (3, 1000, 1024), (8, 32000, 1024), (9, 777, 2048), (16, 4099, 3072), (8, 100, 520),
                                   (16, 300, 8192), (17, 300, 512), (8, 64, 1001)])
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


def _gemm_kn(a, b, out_dtype):
    """a [m, k], b [k, n] -> a b through ferrite_gemm (no transposes)."""
    m, k = a.shape
    n = b.shape[1]
    c = torch.empty(m, n, dtype=out_dtype, device="cuda")
    nat.check(nat.lib().ferrite_gemm(nat.stream_ptr(), a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, a.stride(0), b.stride(0),
                                     c.stride(0), 0, 0, nat.dtype_code(a.dtype), nat.dtype_code(c.dtype)))
    torch.cuda.synchronize()
    return c


# decode linears of GPT d1024 (qkv, out, up, down), edges of the tile and of the cluster
# split, K past one batch of loads per CTA (8192, 20000), more 64-column tiles than
# clusters fit at once (32768, 20000: each cluster loops over several), and shapes that
# leave the path
KN_SHAPES = [(8, 3072, 1024), (8, 1024, 1024), (8, 4096, 1024), (8, 1024, 4096), (1, 8, 8), (3, 1000, 1000),
             (9, 200, 777), (16, 4096, 8192), (8, 136, 20000), (8, 32768, 1024), (4, 20000, 256), (17, 256, 512),
             (8, 1002, 64)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", KN_SHAPES)
def test_skinny_kn_matches_fp32_reference(dtype, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n * 3 + k)
    a = torch.randn(m, k, device="cuda", generator=g).to(dtype)
    b = (torch.randn(k, n, device="cuda", generator=g) / np.sqrt(k)).to(dtype)
    ref = a.float() @ b.float()
    got = _gemm_kn(a, b, torch.float32)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-4)
    got16 = _gemm_kn(a, b, dtype)
    torch.testing.assert_close(got16.float(), ref, rtol=2**-7, atol=1e-3)


def test_skinny_kn_decode_shape_against_the_oracle():
    """bf16 x [8, 1024] against the fused QKV weight [1024, 3072], bf16 out (the decode step)."""
    rng = np.random.default_rng(11)
    x = normal(rng, (8, 1024), BF16)
    w = normal(rng, (1024, 3072), BF16, std=0.02)
    got = to_numpy(_gemm_kn(to_torch(x), to_torch(w), torch.bfloat16)).astype(np.float32)
    ref = om.matmul_reference(x, w, out_dtype=np.float32)
    np.testing.assert_allclose(got, ref, rtol=2**-7, atol=1e-3)


def test_skinny_kn_strided_and_deterministic():
    """A and B as slices of larger buffers (lda > k, ldb > n); repeated calls agree bitwise."""
    g = torch.Generator(device="cuda").manual_seed(4)
    abuf = torch.randn(16, 5000, device="cuda", generator=g).to(torch.bfloat16)
    bbuf = (torch.randn(4100, 1536, device="cuda", generator=g) / 64).to(torch.bfloat16)
    a, b = abuf[:12, :4096], bbuf[:4096, 256:1280]
    ref = a.float() @ b.float()
    got = _gemm_kn(a, b, torch.float32)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-4)
    for _ in range(3):
        assert torch.equal(got, _gemm_kn(a, b, torch.float32))


def test_matmul_api_routes_decode_rows():
    """The reference-facing ``matmul`` on a decode-sized product: forward on the [K][N]
    skinny path, backward products through their own paths, all against fp32."""
    from ferrite.kernels.matmul import matmul

    g = torch.Generator(device="cuda").manual_seed(8)
    x = torch.randn(8, 1024, device="cuda", generator=g).to(torch.bfloat16).requires_grad_()
    w = (torch.randn(1024, 4096, device="cuda", generator=g) / 32).to(torch.bfloat16).requires_grad_()
    y = matmul(x, w)
    ref = x.detach().float() @ w.detach().float()
    torch.testing.assert_close(y.float(), ref, rtol=2**-7, atol=1e-3)
    gy = torch.randn(8, 4096, device="cuda", generator=g).to(torch.bfloat16)
    y.backward(gy)
    torch.testing.assert_close(x.grad.float(), gy.float() @ w.detach().float().t(), rtol=2**-7, atol=2e-2)
    torch.testing.assert_close(w.grad.float(), x.detach().float().t() @ gy.float(), rtol=2**-7, atol=2e-2)


@pytest.mark.parametrize("m", [1, 8, 16])
def test_skinny_kn_gelu_epilogue(m):
    """ferrite_gemm_epilogue's GELU form on a decode-sized up-projection: u = x W1 rounded
    to bf16 and a = gelu_tanh(u) rounded, the MLP's rounding points (gpt.py:141)."""
    g = torch.Generator(device="cuda").manual_seed(20 + m)
    d, f = 1024, 4096
    x = torch.randn(m, d, device="cuda", generator=g).to(torch.bfloat16)
    w1 = (torch.randn(d, f, device="cuda", generator=g) / 32).to(torch.bfloat16)
    u = torch.empty(m, f, dtype=torch.bfloat16, device="cuda")
    a = torch.empty_like(u)
    nat.check(nat.lib().ferrite_gemm_epilogue(nat.stream_ptr(), x.data_ptr(), w1.data_ptr(), u.data_ptr(), m, f, d, d, f, f, 0, 0, 1,
                                              a.data_ptr(), f))
    torch.cuda.synchronize()
    ref = x.float() @ w1.float()
    torch.testing.assert_close(u.float(), ref, rtol=2**-7, atol=1e-3)
    ga = torch.nn.functional.gelu(u.float(), approximate="tanh")
    torch.testing.assert_close(a.float(), ga, rtol=2**-7, atol=1e-3)
    assert torch.equal(u, _gemm_kn(x, w1, torch.bfloat16))  # same kernel, same sums as the plain product


# ---------------------------------------------------------------------------
# residual-add + RMSNorm folded in front of the skinny product (the decode step's norms)
# ---------------------------------------------------------------------------

def _norm_case(m, k, seed, residual=True):
    rng = np.random.default_rng(seed)
    x = normal(rng, (m, k), BF16)
    r = normal(rng, (m, k), BF16) if residual else None
    w = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    return x, r, w


@pytest.mark.parametrize("m,k,n", [(8, 1024, 3072), (1, 256, 768), (16, 1024, 1024), (5, 512, 200)])
def test_gemm_rmsnorm_against_the_oracle(m, k, n):
    """h = round(x + r) bitwise equal to the oracle's add_rmsnorm (rmsnorm.py:52-56 of the
    reference); c = rmsnorm(h) w @ W within the bf16 tolerance (y may differ from the norm
    kernel's by one rounding: another order of the same f32 statistics)."""
    from ferrite.kernels.matmul import rmsnorm_matmul
    from oracle import rmsnorm as orn

    x, r, w = _norm_case(m, k, 30 + m)
    wm = normal(np.random.default_rng(31), (k, n), BF16, std=k ** -0.5)
    h, c = rmsnorm_matmul(to_torch(x), to_torch(w), to_torch(wm), residual=to_torch(r), eps=1e-6)
    h_ref, y_ref = orn.add_rmsnorm_fwd(x, r, w, eps=1e-6)
    np.testing.assert_array_equal(to_numpy(h), h_ref)
    ref = om.matmul_reference(y_ref, wm, out_dtype=np.float32)
    np.testing.assert_allclose(to_numpy(c).astype(np.float32), ref, rtol=2**-6, atol=2e-2)


def test_gemm_rmsnorm_gelu_head_and_no_residual():
    """The three decode forms: ln2 into the up-projection with its GELU (u and gelu(u)),
    ln_f into the tied head (B stored [N][K], f32 logits), and the first layer's ln1
    without a residual (h is x itself)."""
    from ferrite.kernels.matmul import rmsnorm_matmul
    from oracle import rmsnorm as orn

    x, r, w = _norm_case(8, 1024, 40)
    w1 = normal(np.random.default_rng(41), (1024, 4096), BF16, std=1 / 32)
    h, u, a = rmsnorm_matmul(to_torch(x), to_torch(w), to_torch(w1), residual=to_torch(r), eps=1e-6, gelu=True)
    _, y_ref = orn.add_rmsnorm_fwd(x, r, w, eps=1e-6)
    u_ref = om.matmul_reference(y_ref, w1, out_dtype=np.float32)
    np.testing.assert_allclose(to_numpy(u).astype(np.float32), u_ref, rtol=2**-6, atol=2e-2)
    g = torch.nn.functional.gelu(u.float(), approximate="tanh")
    torch.testing.assert_close(a.float(), g, rtol=2**-7, atol=1e-3)

    e = normal(np.random.default_rng(42), (5000, 1024), BF16, std=0.02)
    _, logits = rmsnorm_matmul(to_torch(x), to_torch(w), to_torch(e), residual=to_torch(r), eps=1e-6, trans_b=True,
                               out_dtype=torch.float32)
    assert logits.dtype == torch.float32
    np.testing.assert_allclose(to_numpy(logits), om.matmul_reference(y_ref, np.ascontiguousarray(e.T), out_dtype=np.float32),
                               rtol=2**-6, atol=5e-3)

    xt = to_torch(x)
    h0, c0 = rmsnorm_matmul(xt, to_torch(w), to_torch(w1), eps=1e-6)
    assert h0 is xt
    y0 = orn.rmsnorm_fwd(x, w, eps=1e-6)
    np.testing.assert_allclose(to_numpy(c0).astype(np.float32), om.matmul_reference(y0, w1, out_dtype=np.float32), rtol=2**-6, atol=2e-2)


def test_gemm_rmsnorm_fallback_and_errors():
    """More than 16 rows take the norm kernel and the product as two launches (same
    results within tolerance); the C entry rejects h_out overlapping its inputs."""
    from ferrite.kernels.matmul import rmsnorm_matmul

    x, r, w = _norm_case(20, 512, 50)
    wm = to_torch(normal(np.random.default_rng(51), (512, 256), BF16, std=512 ** -0.5))
    h, c = rmsnorm_matmul(to_torch(x), to_torch(w), wm, residual=to_torch(r), eps=1e-6)
    h8, c8 = rmsnorm_matmul(to_torch(x[:8]), to_torch(w), wm, residual=to_torch(r[:8]), eps=1e-6)
    assert torch.equal(h[:8], h8)
    torch.testing.assert_close(c[:8].float(), c8.float(), rtol=2**-6, atol=2e-2)

    xt, rt, wt = to_torch(x[:8]), to_torch(r[:8]), to_torch(w)
    out = torch.empty(8, 256, dtype=torch.bfloat16, device="cuda")
    rc = nat.lib().ferrite_gemm_rmsnorm(nat.stream_ptr(), xt.data_ptr(), rt.data_ptr(), wt.data_ptr(), 1e-6, rt.data_ptr(),
                                        wm.data_ptr(), out.data_ptr(), 8, 256, 512, 512, 256, 256, 0, 0, None, 0, nat.BF16, nat.BF16)
    assert rc == nat.BAD_SHAPE
