"""GPU parity of the matmul kernels (tcgen05 bf16/f16 path and the exact-f32
CUDA-core path) against the oracle / a torch fp32 reference, the golden
fixture, and the reference's own test cases (tests/test_matmul.py of
anxnd2211/ferrite-tpu re-pointed at the CUDA path).

Tolerances: the reference's (f32 atol 1e-3, bf16 atol 0.5 / rtol 1e-2 for
N(0,1) inputs), the north star's rtol = atol = 1e-5 for the f32 2048^3
Precision.HIGHEST case, and for bf16 outputs "within one bf16 rounding of the
f32-accumulated product" (|err| <= 2^-7 |ref| + 1e-3 * scale) plus max-abs
2e-2 on N(0,1)/sqrt(K) inputs.
"""

import os

import numpy as np
import pytest
import torch

from ferrite.kernels.matmul import gemm, matmul, matmul_reference
from helpers import BF16, load_arrays, max_abs, normal, to_numpy, to_torch
from oracle import matmul as om

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
torch.backends.cuda.matmul.allow_tf32 = False


def _ref32(a: torch.Tensor, b: torch.Tensor, ta=False, tb=False) -> torch.Tensor:
    a = a.float().t() if ta else a.float()
    b = b.float().t() if tb else b.float()
    return a @ b


def _assert_bf16_close(got: torch.Tensor, ref32: torch.Tensor, scale: float = 1.0):
    g = got.float()
    err = (g - ref32).abs()
    bound = ref32.abs() * 2.0**-7 + 1e-3 * scale
    bad = (err > bound).sum().item()
    assert bad == 0, f"{bad} elements outside one bf16 rounding; max err {err.max().item()}"


@pytest.mark.parametrize("dtype,atol", [(torch.float32, 1e-3), (torch.bfloat16, 0.5)])
def test_matches_reference_aligned(rng, dtype, atol):
    """test_matmul.py:13-20."""
    x = to_torch(normal(rng, (256, 384))).to(dtype)
    y = to_torch(normal(rng, (384, 512))).to(dtype)
    out = matmul(x, y, block_m=128, block_n=256, block_k=128)
    ref = matmul_reference(x, y)
    assert out.shape == (256, 512) and out.dtype == dtype
    torch.testing.assert_close(out.float(), ref.float(), atol=atol, rtol=1e-2)


def test_ragged_shapes_are_exact(rng):
    """test_matmul.py:23-27 (f32 77x130x203, no padding copies)."""
    x, y = normal(rng, (77, 130)), normal(rng, (130, 203))
    out = matmul(to_torch(x), to_torch(y), block_m=64, block_n=128, block_k=128)
    np.testing.assert_allclose(to_numpy(out), om.matmul_reference(x, y), atol=1e-3, rtol=1e-3)


def test_f32_output_from_bf16_inputs(rng):
    """test_matmul.py:30-35."""
    x, y = normal(rng, (128, 256), BF16), normal(rng, (256, 128), BF16)
    out = matmul(to_torch(x), to_torch(y), out_dtype=torch.float32)
    assert out.dtype == torch.float32
    np.testing.assert_allclose(to_numpy(out), om.matmul_reference(x, y, out_dtype=np.float32), atol=1e-2, rtol=1e-2)


def test_golden_fixture():
    g = load_arrays(os.path.join(GOLDEN, "matmul_ragged_bf16_77x130x203.npz"))
    x, y, gg = to_torch(g["x"]), to_torch(g["y"]), to_torch(g["g"])
    out = matmul(x, y)
    assert max_abs(out, g["out"]) <= 2e-2
    out32 = matmul(x, y, out_dtype=torch.float32)
    np.testing.assert_allclose(to_numpy(out32), g["out_f32"], atol=1e-4, rtol=1e-5)
    xr, yr = x.clone().requires_grad_(True), y.clone().requires_grad_(True)
    matmul(xr, yr).backward(gg)
    assert max_abs(xr.grad, g["dx"]) <= 2e-2 and max_abs(yr.grad, g["dy"]) <= 2e-2


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("m,n,k", [(256, 512, 384), (1000, 696, 328), (128, 128, 64), (384, 256, 4096)])
def test_tensor_core_transpose_variants(ta, tb, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn((k, m) if ta else (m, k), device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn((n, k) if tb else (k, n), device="cuda", generator=g).to(torch.bfloat16)
    ref = _ref32(a, b, ta, tb)
    out = gemm(a, b, trans_a=ta, trans_b=tb)
    _assert_bf16_close(out, ref, scale=float(np.sqrt(k)))
    out32 = gemm(a, b, trans_a=ta, trans_b=tb, out_dtype=torch.float32)
    torch.testing.assert_close(out32, ref, atol=1e-3 * np.sqrt(k), rtol=1e-4)


def test_f16_operands():
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(512, 256, device="cuda", generator=g).half()
    b = torch.randn(256, 384, device="cuda", generator=g).half()
    out = gemm(a, b, out_dtype=torch.float32)
    torch.testing.assert_close(out, _ref32(a, b), atol=2e-3, rtol=1e-4)


def test_bf16_8192_cubed_vs_oracle_rows():
    """Benchmark config: bf16 8192^3, A, B ~ N(0,1)/sqrt(K), checked against the
    oracle on a sample of rows and against torch fp32 everywhere."""
    m = n = k = 8192
    rng = np.random.default_rng(0)
    a = normal(rng, (m, k), BF16, std=1 / np.sqrt(k))
    b = normal(rng, (k, n), BF16, std=1 / np.sqrt(k))
    at, bt = to_torch(a), to_torch(b)
    out = matmul(at, bt)
    ref = _ref32(at, bt)
    _assert_bf16_close(out, ref, scale=1 / np.sqrt(k))
    assert (out.float() - ref).abs().max().item() <= 2e-2
    rows = rng.choice(m, 48, replace=False)
    o_rows = om.matmul_reference(a[rows], b)
    assert max_abs(to_numpy(out)[rows], o_rows) <= 2e-2
    assert np.array_equal(to_numpy(out)[rows].view(np.uint16), o_rows.view(np.uint16)) or max_abs(to_numpy(out)[rows], o_rows) < 1e-3


def test_bf16_ragged_4000x3000x5000_fwd_and_vjp():
    m, n, k = 4000, 3000, 5000
    g = torch.Generator(device="cuda").manual_seed(1)
    x = (torch.randn(m, k, device="cuda", generator=g) / np.sqrt(k)).to(torch.bfloat16).requires_grad_(True)
    y = (torch.randn(k, n, device="cuda", generator=g) / np.sqrt(k)).to(torch.bfloat16).requires_grad_(True)
    gout = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
    out = matmul(x, y)
    _assert_bf16_close(out, _ref32(x.detach(), y.detach()), scale=1 / np.sqrt(k))
    out.backward(gout)
    _assert_bf16_close(x.grad, gout.float() @ y.detach().float().t(), scale=1.0)
    _assert_bf16_close(y.grad, x.detach().float().t() @ gout.float(), scale=1.0)


def test_f32_2048_cubed_highest_precision():
    """North star: f32 2048^3 at Precision.HIGHEST within rtol = atol = 1e-5 (float64 oracle)."""
    rng = np.random.default_rng(0)
    k = 2048
    a = normal(rng, (k, k), std=1 / np.sqrt(k))
    b = normal(rng, (k, k), std=1 / np.sqrt(k))
    out = to_numpy(matmul(to_torch(a), to_torch(b)))
    ref = om.matmul_reference(a, b, out_dtype=np.float64, acc=np.float64)
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5)


def test_f32_vjp(rng):
    x, y, g = normal(rng, (96, 200)), normal(rng, (200, 136)), normal(rng, (96, 136))
    xt, yt = to_torch(x).requires_grad_(True), to_torch(y).requires_grad_(True)
    matmul(xt, yt).backward(to_torch(g))
    dx, dy = om.matmul_vjp(x, y, g, acc=np.float64)
    np.testing.assert_allclose(to_numpy(xt.grad), dx, atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(to_numpy(yt.grad), dy, atol=1e-4, rtol=1e-5)


def test_degenerate_sizes():
    a = torch.zeros(0, 64, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(64, 32, device="cuda", dtype=torch.bfloat16)
    assert matmul(a, b).shape == (0, 32)
    a = torch.ones(16, 1, device="cuda")
    b = torch.ones(1, 16, device="cuda")
    assert torch.equal(matmul(a, b), torch.ones(16, 16, device="cuda"))


def test_deterministic():
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(1024, 2048, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(2048, 1536, device="cuda", generator=g).to(torch.bfloat16)
    assert torch.equal(matmul(a, b), matmul(a, b))


def test_device_status_clean_after_gemm():
    from ferrite import _native as nat

    nat.device_status(clear=True)


# ---------------------------------------------------------------- split-K


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("m,n,k", [(256, 256, 8192), (296, 520, 4000), (1024, 1024, 65536), (128, 384, 2048)])
def test_split_k_matches_fp32_reference(ta, m, n, k):
    """Few-tile outputs with long K (weight-gradient shapes) take the split-K
    launch; the sum of the f32 slices is rounded once, like the unsplit kernel."""
    from ferrite import _native as nat

    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = (torch.randn((k, m) if ta else (m, k), device="cuda", generator=g) / k**0.5).to(torch.bfloat16)
    b = torch.randn(k, n, device="cuda", generator=g).to(torch.bfloat16)
    ws = nat.lib().ferrite_gemm_workspace_size(m, n, k, a.stride(0), b.stride(0), int(ta), 0, nat.BF16)
    assert ws > 0, "shape expected to split"
    ref = _ref32(a, b, ta=ta)
    for out_dtype in (torch.bfloat16, torch.float32):
        c = gemm(a, b, trans_a=ta, out_dtype=out_dtype)
        if out_dtype == torch.float32:
            torch.testing.assert_close(c, ref, rtol=1e-4, atol=1e-4)
        else:
            _assert_bf16_close(c, ref)
        assert torch.equal(c, gemm(a, b, trans_a=ta, out_dtype=out_dtype))  # deterministic


@pytest.mark.parametrize("splits", [2, 3, 7])
def test_forced_split_counts_agree_with_unsplit(monkeypatch, splits):
    """Uneven slices (k blocks not divisible by the split count) and the no-split
    path agree to f32 summation order."""
    g = torch.Generator(device="cuda").manual_seed(splits)
    m, n, k = 512, 768, 64 * 29
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(k, n, device="cuda", generator=g).to(torch.bfloat16)
    monkeypatch.setenv("FERRITE_GEMM_SPLITS", str(splits))
    c_split = gemm(a, b, out_dtype=torch.float32)
    monkeypatch.setenv("FERRITE_GEMM_SPLITS", "1")
    c_one = gemm(a, b, out_dtype=torch.float32)
    # N(0,1) operands, K = 1856: |c| ~ 43, f32 summation-order noise ~ 1e-4
    torch.testing.assert_close(c_split, c_one, rtol=1e-5, atol=1e-3)
    torch.testing.assert_close(c_split, _ref32(a, b), rtol=1e-4, atol=2e-3)


def test_no_workspace_entry_point_never_splits():
    """ferrite_gemm (no scratch) on a split-eligible shape runs the unsplit kernel."""
    from ferrite import _native as nat

    g = torch.Generator(device="cuda").manual_seed(7)
    m, n, k = 256, 256, 8192
    a = (torch.randn(m, k, device="cuda", generator=g) / k**0.5).to(torch.bfloat16)
    b = torch.randn(k, n, device="cuda", generator=g).to(torch.bfloat16)
    c = torch.empty(m, n, device="cuda", dtype=torch.float32)
    nat.check(nat.lib().ferrite_gemm(nat.stream_ptr(), a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, k, n, n, 0, 0, nat.BF16, nat.F32))
    torch.testing.assert_close(c, _ref32(a, b), rtol=1e-4, atol=1e-4)
    # too-small scratch: same as no scratch
    ws = torch.empty(64, dtype=torch.uint8, device="cuda")
    c2 = torch.empty_like(c)
    nat.check(nat.lib().ferrite_gemm_ws(nat.stream_ptr(), a.data_ptr(), b.data_ptr(), c2.data_ptr(), m, n, k, k, n, n, 0, 0, nat.BF16, nat.F32, ws.data_ptr(), 64))
    assert torch.equal(c, c2)
