"""GPU test of ``ferrite_rmsnorm_bwd_noalloc``, the allocation-free RMSNorm backward.

That entry point is for callers that cannot allocate device memory (a framework
that owns all device memory and gives kernels no scratch allocator, or a runtime
whose device arena is fixed at start-up): it keeps the dw partial sums in a
library-owned device array instead of a caller workspace.  This test calls it
through the C ABI twice in a row and compares each result with the workspace
entry point ``ferrite_rmsnorm_bwd`` on the same inputs, with the tolerances of
the other RMSNorm tests (dh: max-abs 2e-2 for bf16, 1e-5 for f32; dw: rtol 2e-4).
It lives in its own file, collected last, and holds no state between tests.
"""

import numpy as np
import pytest
import torch

from ferrite import _native as nat

pytestmark = pytest.mark.gpu


def _inputs(rows, dim, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    h = torch.randn(rows, dim, device="cuda", generator=g).to(dtype)
    dy = torch.randn(rows, dim, device="cuda", generator=g).to(dtype)
    dhd = torch.randn(rows, dim, device="cuda", generator=g).to(dtype)
    w = (1.0 + 0.1 * torch.randn(dim, device="cuda", generator=g)).float()
    return h, w, dy, dhd


def _with_workspace(h, w, dy, dhd, eps=1e-6):
    rows, dim = h.shape
    lib = nat.lib()
    dh, dw = torch.empty_like(h), torch.empty_like(w)
    ws = torch.empty(int(lib.ferrite_rmsnorm_bwd_workspace_size(rows, dim)), dtype=torch.uint8, device="cuda")
    nat.check(lib.ferrite_rmsnorm_bwd(nat.stream_ptr(), h.data_ptr(), w.data_ptr(), dy.data_ptr(), nat.ptr(dhd), dh.data_ptr(), dw.data_ptr(),
                                      ws.data_ptr(), ws.numel(), rows, dim, eps, nat.dtype_code(h.dtype), nat.F32))
    return dh, dw


def _no_alloc(h, w, dy, dhd, eps=1e-6):
    rows, dim = h.shape
    dh, dw = torch.empty_like(h), torch.empty_like(w)
    nat.check(nat.lib().ferrite_rmsnorm_bwd_noalloc(nat.stream_ptr(), h.data_ptr(), w.data_ptr(), dy.data_ptr(), nat.ptr(dhd), dh.data_ptr(),
                                                    dw.data_ptr(), rows, dim, eps, nat.dtype_code(h.dtype), nat.F32))
    return dh, dw


@pytest.mark.parametrize(
    "rows,dim,dtype,with_dh",
    [(8192, 4096, torch.bfloat16, True), (300, 384, torch.float32, False), (1000, 8192, torch.bfloat16, True), (33, 1000, torch.bfloat16, False)],
)
def test_no_alloc_backward_matches_workspace_backward_twice(rows, dim, dtype, with_dh):
    atol_dh = 2e-2 if dtype == torch.bfloat16 else 1e-5
    for call in range(2):  # two calls in a row share (and must fully rewrite) the library buffer
        h, w, dy, dhd = _inputs(rows, dim, dtype, seed=10 * call + rows)
        dhd = dhd if with_dh else None
        ref_dh, ref_dw = _with_workspace(h, w, dy, dhd)
        dh, dw = _no_alloc(h, w, dy, dhd)
        torch.cuda.synchronize()
        assert (dh.float() - ref_dh.float()).abs().max().item() <= atol_dh
        np.testing.assert_allclose(dw.cpu().numpy(), ref_dw.cpu().numpy(), rtol=2e-4, atol=2e-3 * np.sqrt(rows / 64 + 1))
    nat.device_status(clear=True)


def test_no_alloc_rejects_rows_longer_than_its_buffer():
    rc = nat.lib().ferrite_rmsnorm_bwd_noalloc(nat.stream_ptr(), 1, 1, 1, None, 1, 1, 4, 131072 + 8, 1e-6, nat.BF16, nat.F32)
    assert rc == nat.BAD_SHAPE
    assert "allocation-free maximum" in nat.last_error()
