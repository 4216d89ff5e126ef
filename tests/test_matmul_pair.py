"""The CTA-pair tensor-core GEMM (two CTAs of a cluster computing one 256 x 256
tile with tcgen05.mma.cta_group::2) against the one-CTA kernel, a torch fp32
reference and the oracle.

Both kernels accumulate each output element over the same K order (64-wide
K blocks, four K=16 MMAs each, f32 in TMEM), so the pair path is compared with
the one-CTA path bitwise and with the fp32 reference at one bf16 rounding.
Cases: every transpose combination, ragged M (the last pair tile's second CTA
entirely past M) and N, more pair tiles than resident clusters (several units
per cluster), f32 and f16 outputs, the GPT MLP's fused GELU epilogues, and the
reference's matmul sizes (src/ferrite/kernels/matmul.py:52-86 of
anxnd2211/ferrite-tpu).  The unsplit cases go through ``ferrite_gemm`` (no
split-K scratch) and the split-K case through ``gemm`` with a forced split
count; 256-wide tiles are forced (FERRITE_GEMM_BN=256) and FERRITE_GEMM_PAIR
selects the pair (1) or the one-CTA (0) kernel.
"""

import numpy as np
import pytest
import torch

from ferrite import _native as nat
from helpers import BF16, max_abs, normal, to_numpy, to_torch
from oracle import matmul as om

pytestmark = pytest.mark.gpu
torch.backends.cuda.matmul.allow_tf32 = False


def _ref32(a, b, ta=False, tb=False):
    a = a.float().t() if ta else a.float()
    b = b.float().t() if tb else b.float()
    return a @ b


def _gemm(a, b, ta=False, tb=False, out_dtype=None):
    """ferrite_gemm (no split-K scratch: every shape runs unsplit)."""
    m, k = (a.shape[1], a.shape[0]) if ta else a.shape
    n = b.shape[0] if tb else b.shape[1]
    c = torch.empty(m, n, dtype=out_dtype or a.dtype, device="cuda")
    nat.check(nat.lib().ferrite_gemm(nat.stream_ptr(), a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, a.stride(0), b.stride(0),
                                     c.stride(0), int(ta), int(tb), nat.dtype_code(a.dtype), nat.dtype_code(c.dtype)))
    return c


def _both(monkeypatch, fn):
    """fn() on the pair path, then on the one-CTA path (256-wide tiles on both)."""
    monkeypatch.setenv("FERRITE_GEMM_BN", "256")
    monkeypatch.setenv("FERRITE_GEMM_PAIR", "1")
    got = fn()
    monkeypatch.setenv("FERRITE_GEMM_PAIR", "0")
    one = fn()
    monkeypatch.delenv("FERRITE_GEMM_PAIR")
    monkeypatch.delenv("FERRITE_GEMM_BN")
    torch.cuda.synchronize()
    nat.device_status(clear=True)  # no bounded wait expired
    return got, one


def _bf16_close(got, ref32, scale):
    err = (got.float() - ref32).abs()
    bad = (err > ref32.abs() * 2.0**-7 + 1e-3 * scale).sum().item()
    assert bad == 0, f"{bad} elements outside one bf16 rounding; max err {err.max().item()}"


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("m,n,k", [(512, 768, 1024), (300, 520, 4000), (1000, 696, 328), (4096, 3072, 768)])
def test_pair_matches_one_cta_and_reference(monkeypatch, ta, tb, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    a = torch.randn((k, m) if ta else (m, k), device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn((n, k) if tb else (k, n), device="cuda", generator=g).to(torch.bfloat16)
    ref = _ref32(a, b, ta, tb)
    for out_dtype in (torch.bfloat16, torch.float32):
        got, one = _both(monkeypatch, lambda: _gemm(a, b, ta, tb, out_dtype))
        assert torch.equal(got, one), (out_dtype, (got.float() - one.float()).abs().max().item())
        if out_dtype == torch.float32:
            torch.testing.assert_close(got, ref, atol=1e-3 * np.sqrt(k), rtol=1e-4)
        else:
            _bf16_close(got, ref, float(np.sqrt(k)))


def test_many_units_per_cluster_f16(monkeypatch):
    """8192 x 8192: 1024 pair tiles over the resident clusters."""
    g = torch.Generator(device="cuda").manual_seed(5)
    m = n = 8192
    k = 512
    a = torch.randn(m, k, device="cuda", generator=g).half()
    b = torch.randn(k, n, device="cuda", generator=g).half()
    got, one = _both(monkeypatch, lambda: _gemm(a, b))
    assert torch.equal(got, one)
    rows = torch.arange(0, m, 97, device="cuda")
    _bf16_close(got[rows], _ref32(a[rows], b), float(np.sqrt(k)))


def test_oracle_rows_8192_cubed(monkeypatch):
    """The benchmark's bf16 8192^3 on the pair path, rows checked against the oracle."""
    rng = np.random.default_rng(0)
    m = n = k = 8192
    a = normal(rng, (m, k), BF16, std=1 / np.sqrt(k))
    b = normal(rng, (k, n), BF16, std=1 / np.sqrt(k))
    at, bt = to_torch(a), to_torch(b)
    monkeypatch.setenv("FERRITE_GEMM_PAIR", "1")
    out = _gemm(at, bt)
    torch.cuda.synchronize()
    nat.device_status(clear=True)
    rows = rng.choice(m, 32, replace=False)
    o_rows = om.matmul_reference(a[rows], b)
    assert max_abs(to_numpy(out)[rows], o_rows) <= 2e-2


@pytest.mark.parametrize("t", [512, 1000])
def test_gelu_epilogues(monkeypatch, t):
    """The MLP's fused epilogues (up-projection writing u and gelu(u); dU = dA *
    gelu'(u)) on the pair path equal the one-CTA path."""
    g = torch.Generator(device="cuda").manual_seed(t)
    d, f = 768, 3072
    y = torch.randn(t, d, device="cuda", generator=g).to(torch.bfloat16)
    w1 = (0.05 * torch.randn(d, f, device="cuda", generator=g)).to(torch.bfloat16)
    w2 = (0.05 * torch.randn(f, d, device="cuda", generator=g)).to(torch.bfloat16)
    dp = torch.randn(t, d, device="cuda", generator=g).to(torch.bfloat16)
    lib = nat.lib()

    def fwd():
        u = torch.empty(t, f, dtype=torch.bfloat16, device="cuda")
        a = torch.empty_like(u)
        nat.check(lib.ferrite_gemm_epilogue(nat.stream_ptr(), y.data_ptr(), w1.data_ptr(), u.data_ptr(), t, f, d, d, f, f, 0, 0, 1,
                                            a.data_ptr(), f))
        return torch.cat([u, a])

    def bwd(u):
        du = torch.empty(t, f, dtype=torch.bfloat16, device="cuda")
        nat.check(lib.ferrite_gemm_epilogue(nat.stream_ptr(), dp.data_ptr(), w2.data_ptr(), du.data_ptr(), t, f, d, d, d, f, 0, 1, 2,
                                            u.data_ptr(), f))
        return du

    ua, ua1 = _both(monkeypatch, fwd)
    assert torch.equal(ua, ua1)
    u = ua[:t]
    torch.testing.assert_close(u.float(), _ref32(y, w1), atol=2e-2, rtol=1e-2)
    du, du1 = _both(monkeypatch, lambda: bwd(u))
    assert torch.equal(du, du1)


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("splits", [2, 3])
def test_pair_split_k_matches_one_cta(monkeypatch, ta, splits):
    """Split-K on pairs (the weight gradients X^T G: few output tiles, long K): the
    f32 partial slices and their ordered sum equal the one-CTA kernel's."""
    from ferrite.kernels.matmul import gemm

    g = torch.Generator(device="cuda").manual_seed(splits)
    m, n, k = 768, 1024, 64 * 61
    a = torch.randn((k, m) if ta else (m, k), device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(k, n, device="cuda", generator=g).to(torch.bfloat16)
    monkeypatch.setenv("FERRITE_GEMM_SPLITS", str(splits))
    for out_dtype in (torch.float32, torch.bfloat16):
        got, one = _both(monkeypatch, lambda: gemm(a, b, trans_a=ta, out_dtype=out_dtype))
        assert torch.equal(got, one)
        ref = _ref32(a, b, ta)
        if out_dtype == torch.float32:
            torch.testing.assert_close(got, ref, atol=1e-3 * np.sqrt(k), rtol=1e-4)
        else:
            _bf16_close(got, ref, float(np.sqrt(k)))
