"""Backward parity at the full benchmark sizes, through the product path.

* Long-context config: b8 h32 s8192 d128 bf16, causal.  ``flash_attention`` +
  autograd runs the whole problem on the GPU: the forward, the delta prep, the
  dK/dV kernel that stores dS, and the dQ-from-dS GEMM, with the dS scratch cut into
  chunks of slices by the Python API's budget (4 GiB: 32 slices of 8192 x 8192 bf16
  per chunk).  The oracle (blockwise restatement of the reference's kernels,
  src/ferrite/kernels/flash_attention.py:91-127 and :184-243) recomputes sampled
  (b, h) slices -- heads are independent -- including the first and last slice and
  the slices on both sides of the first chunk boundary.
* GPT attention shape: b64 h16 s1024 d64 (per-layer attention of the GPT training
  step at global batch 64), through ``flash_attention`` and through the packed
  ``[b, s, 3, h, d]`` form the GPT block uses.

Tolerances: the north star's max-abs 2e-2 on bf16 outputs and gradients, and
relative L2 < 1e-2.
"""

import numpy as np
import pytest
import torch

from ferrite.kernels.flash_attention import DS_WORKSPACE_BUDGET, flash_attention, flash_attention_packed
from helpers import max_abs, rel_l2, to_numpy
from oracle import attention as oa

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _inputs(shape, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return tuple(torch.randn(*shape, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))


def _check_slices(q, k, v, do, out, grads, slices, scale):
    """Compare out / dq / dk / dv of the given (b, h) slices with the oracle."""
    for bi, hi in slices:
        qs, ks, vs, dos = (to_numpy(t[bi : bi + 1, hi : hi + 1]) for t in (q, k, v, do))
        o_ref, lse_ref = oa.flash_fwd(qs, ks, vs, causal=True, scale=scale)
        assert max_abs(out[bi : bi + 1, hi : hi + 1], o_ref) <= 2e-2, ("out", bi, hi)
        g_ref = oa.flash_bwd(qs, ks, vs, o_ref, lse_ref, dos, causal=True, scale=scale)
        for got, ref, name in zip(grads, g_ref, ("dq", "dk", "dv")):
            sl = got[bi : bi + 1, hi : hi + 1]
            assert max_abs(sl, ref) <= 2e-2, (name, bi, hi, max_abs(sl, ref))
            assert rel_l2(sl, ref) < 1e-2, (name, bi, hi, rel_l2(sl, ref))


def test_long_config_backward_sampled_slices():
    b, h, s, d = 8, 32, 8192, 128
    q, k, v, do = _inputs((b, h, s, d), seed=0)
    per_slice = s * s * 2
    chunk = DS_WORKSPACE_BUDGET // per_slice  # slices per dS chunk
    assert 0 < chunk < b * h, "the test must cross at least one chunk boundary"
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    out = flash_attention(qg, kg, vg, causal=True)
    out.backward(do)
    torch.cuda.synchronize()
    flat = sorted({0, chunk - 1, chunk, 2 * chunk + 5, b * h - 1})
    slices = [(i // h, i % h) for i in flat]
    _check_slices(q, k, v, do, out.detach(), (qg.grad, kg.grad, vg.grad), slices, 1 / np.sqrt(d))


@pytest.mark.parametrize("packed", [False, True])
def test_gpt_shape_backward_sampled_slices(packed):
    b, h, s, d = 64, 16, 1024, 64
    q, k, v, do = _inputs((b, h, s, d), seed=3)
    if packed:
        qkv = torch.stack([t.transpose(1, 2) for t in (q, k, v)], dim=2).contiguous().requires_grad_(True)  # [b, s, 3, h, d]
        out = flash_attention_packed(qkv, causal=True)  # [b, s, h, d]
        out.backward(do.transpose(1, 2))
        torch.cuda.synchronize()
        out = out.detach().transpose(1, 2)
        grads = tuple(qkv.grad[:, :, i].transpose(1, 2) for i in range(3))
    else:
        qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
        out = flash_attention(qg, kg, vg, causal=True)
        out.backward(do)
        torch.cuda.synchronize()
        out, grads = out.detach(), (qg.grad, kg.grad, vg.grad)
    slices = [(0, 0), (17, 9), (31, 15), (32, 0), (63, 15)]
    _check_slices(q, k, v, do, out, grads, slices, 1 / np.sqrt(d))
