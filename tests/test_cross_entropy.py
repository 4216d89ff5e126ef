"""GPU parity of the softmax cross-entropy kernels and the fused tied-head loss
against the oracle (oracle/xent.py, the reference's loss_fn at
src/ferrite/model/gpt.py:147-152) and torch's f32 log_softmax / NLL.

Tolerances: f32 loss and lse 1e-5 relative; f32 dlogits 1e-4 relative (the
kernels use the fast exponential); bf16 dlogits within one bf16 rounding of the
f32 gradient; the fused head's gradients within the bf16 GEMM tolerance.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from ferrite.kernels.cross_entropy import cross_entropy, tied_head_cross_entropy, xent_backward, xent_forward
from ferrite.kernels.matmul import gemm
from helpers import to_numpy, to_torch
from oracle import xent as ox

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,vocab", [(300, 32000), (64, 1001), (7, 4), (1, 50257)])
@pytest.mark.parametrize("tdtype", [torch.int64, torch.int32])
def test_forward_and_backward_vs_oracle(rows, vocab, tdtype):
    rng = np.random.default_rng(rows + vocab)
    x = (4.0 * rng.standard_normal((rows, vocab))).astype(np.float32)
    t = rng.integers(0, vocab, rows)
    xt, tt = to_torch(x), torch.from_numpy(t).to("cuda", tdtype)
    lse, nll = xent_forward(xt, tt)
    l_ref, nll_ref = ox.xent_fwd(x, t)
    np.testing.assert_allclose(to_numpy(lse), l_ref, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(to_numpy(nll), nll_ref, rtol=1e-5, atol=2e-5)
    g_ref = ox.xent_bwd(x, t, g=1.0)
    d32 = xent_backward(xt, tt, lse, None, 1.0 / rows, torch.float32)
    np.testing.assert_allclose(to_numpy(d32), g_ref, rtol=1e-4, atol=1e-9)
    d16 = xent_backward(xt, tt, lse, None, 1.0 / rows, torch.bfloat16).float()
    err = (d16 - d32).abs()
    assert bool((err <= d32.abs() * 2.0**-8 + 1e-12).all())  # round-to-nearest of the f32 value


def test_autograd_loss_matches_torch():
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (3 * torch.randn(512, 32000, device="cuda", generator=g)).requires_grad_(True)
    t = torch.randint(0, 32000, (512,), device="cuda", generator=g)
    loss = cross_entropy(x, t)
    (2.0 * loss).backward()
    xr = x.detach().clone().requires_grad_(True)
    ref = F.cross_entropy(xr, t)
    (2.0 * ref).backward()
    torch.testing.assert_close(loss, ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(x.grad, xr.grad, rtol=1e-4, atol=1e-10)


def test_tied_head_cross_entropy_matches_unfused():
    g = torch.Generator(device="cuda").manual_seed(1)
    T, d, V = 1024, 256, 4096
    y = (torch.randn(T, d, device="cuda", generator=g)).to(torch.bfloat16).requires_grad_(True)
    e = (0.02 * torch.randn(V, d, device="cuda", generator=g)).to(torch.bfloat16).requires_grad_(True)
    t = torch.randint(0, V, (T,), device="cuda", generator=g)
    loss = tied_head_cross_entropy(y, e, t)
    loss.backward()
    y2, e2 = y.detach().clone().requires_grad_(True), e.detach().clone().requires_grad_(True)
    logits = y2.float() @ e2.float().t()
    ref = F.cross_entropy(logits, t)
    ref.backward()
    torch.testing.assert_close(loss, ref, rtol=1e-4, atol=1e-4)
    for got, want in ((y.grad, y2.grad), (e.grad, e2.grad)):
        scale = want.float().abs().max().item()
        assert (got.float() - want.float()).abs().max().item() <= 2e-2 * scale


def test_out_of_range_target_gives_nan_not_a_read():
    x = torch.zeros(3, 128, device="cuda")
    t = torch.tensor([0, 128, -1], device="cuda")
    _, nll = xent_forward(x, t)
    assert torch.isfinite(nll[0]) and torch.isnan(nll[1]) and torch.isnan(nll[2])


def test_deterministic():
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(256, 32000, device="cuda", generator=g)
    t = torch.randint(0, 32000, (256,), device="cuda", generator=g)
    a, b = xent_forward(x, t), xent_forward(x, t)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
