"""The fused persistent backward (dK/dV and dQ-from-dS units in one launch, dS kept
in L2 between them) against the oracle and against the two-kernel path.  The product
picks the fused kernel from 4096 queries on; these tests force it at small sizes
(FERRITE_ATTN_BWD_FUSED=2).

Both paths form the same rounded dS operand (flash_attention.py:184-194 of the
reference) and compute dQ = scale * dS K with the same product order, so dQ is
bitwise equal between them; dK and dV accumulate their query tiles in the other
order (last tile first) and are compared with the oracle at the north star's
max-abs 2e-2.  Workspaces of one and two dS slots make the scheduler recycle slots
(a slice starts only after the dQ units of the slice that held its slot)."""

import ctypes
import os

import numpy as np
import pytest
import torch

from ferrite import _native as nat
from helpers import BF16, max_abs, normal, rel_l2, to_torch
from oracle import attention as oa

pytestmark = pytest.mark.gpu


def _bwd(q, k, v, o, lse, do, causal, ws_bytes=None, fused=True):
    """ferrite_attn_bwd_ds with an explicit workspace; returns (dq, dk, dv)."""
    b, h, sq, d = q.shape
    sk = k.shape[2]
    lib = nat.lib()
    code = nat.dtype_code(q.dtype)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty(b, h, sq, device="cuda")
    st = nat.attn_strides(q=q, k=k, v=v, o=o, dout=do, dq=dq, dk=dk, dv=dv)
    nat.check(lib.ferrite_attn_bwd_prep_strided(nat.stream_ptr(), do.data_ptr(), o.data_ptr(), delta.data_ptr(), ctypes.byref(st), b, h, sq, d, code))
    full = lib.ferrite_attn_bwd_ds_workspace_size(b, h, sq, sk, d, code)
    ws = torch.empty(full if ws_bytes is None else ws_bytes, dtype=torch.uint8, device="cuda")
    old = os.environ.get("FERRITE_ATTN_BWD_FUSED")
    os.environ["FERRITE_ATTN_BWD_FUSED"] = "2" if fused else "0"  # 2: the fused kernel at any eligible size
    try:
        nat.check(lib.ferrite_attn_bwd_ds(nat.stream_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                          delta.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ctypes.byref(st), ws.data_ptr(),
                                          ws.numel(), b, h, sq, sk, d, 1 / np.sqrt(d), int(causal), 128, 128, code))
    finally:
        if old is None:
            os.environ.pop("FERRITE_ATTN_BWD_FUSED", None)
        else:
            os.environ["FERRITE_ATTN_BWD_FUSED"] = old
    torch.cuda.synchronize()
    nat.device_status(clear=True)  # no bounded wait expired
    return dq, dk, dv


def _case(seed, b, h, sq, sk, d):
    rng = np.random.default_rng(seed)
    q, do = normal(rng, (b, h, sq, d), BF16), normal(rng, (b, h, sq, d), BF16)
    k, v = normal(rng, (b, h, sk, d), BF16), normal(rng, (b, h, sk, d), BF16)
    return q, k, v, do


def _fwd(q, k, v, causal):
    b, h, sq, d = q.shape
    o = torch.empty_like(q)
    lse = torch.empty(b, h, sq, device="cuda")
    nat.check(nat.lib().ferrite_attn_fwd(nat.stream_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                         b, h, sq, k.shape[2], d, 1 / np.sqrt(d), int(causal), 128, 128, nat.dtype_code(q.dtype)))
    return o, lse


def _slice_bytes(sq, sk):
    return (sq + 63) // 64 * 64 * sk * 2


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal,sq,sk", [(True, 512, 512), (False, 256, 384), (True, 1024, 1024)])
def test_fused_matches_oracle_and_two_kernel_path(d, causal, sq, sk):
    q, k, v, do = _case(7 + d + sq, 2, 3, sq, sk, d)
    qt, kt, vt, dot = (to_torch(a) for a in (q, k, v, do))
    o, lse = _fwd(qt, kt, vt, causal)
    dq, dk, dv = _bwd(qt, kt, vt, o, lse, dot, causal)
    dq0, dk0, dv0 = _bwd(qt, kt, vt, o, lse, dot, causal, fused=False)
    assert torch.equal(dq, dq0), "dQ differs from the two-kernel path"
    o_ref, lse_ref = oa.flash_fwd(q, k, v, causal=causal)
    g_ref = oa.flash_bwd(q, k, v, o_ref, lse_ref, do, causal=causal)
    for got, ref, name in zip((dq, dk, dv), g_ref, ("dq", "dk", "dv")):
        assert max_abs(got, ref) <= 2e-2, name
        assert rel_l2(got, ref) < 1e-2, name
    for a, b_ in ((dk, dk0), (dv, dv0)):
        assert max_abs(a, b_) <= 2e-2


@pytest.mark.parametrize("slots", [1, 2, 5])
def test_fused_slot_recycling(slots):
    """A workspace of `slots` dS slices (+ the scheduler state) for 2 x 4 slices."""
    b, h, s, d = 2, 4, 512, 128
    q, k, v, do = _case(3, b, h, s, s, d)
    qt, kt, vt, dot = (to_torch(a) for a in (q, k, v, do))
    o, lse = _fwd(qt, kt, vt, True)
    ref = _bwd(qt, kt, vt, o, lse, dot, True)  # every slice its own slot
    full = nat.lib().ferrite_attn_bwd_ds_workspace_size(b, h, s, s, d, nat.BF16)
    sched = full - b * h * _slice_bytes(s, s)
    got = _bwd(qt, kt, vt, o, lse, dot, True, ws_bytes=slots * _slice_bytes(s, s) + sched)
    for a, b_ in zip(got, ref):
        assert torch.equal(a, b_)


def test_fused_is_deterministic():
    q, k, v, do = _case(11, 2, 8, 1024, 1024, 64)
    qt, kt, vt, dot = (to_torch(a) for a in (q, k, v, do))
    o, lse = _fwd(qt, kt, vt, True)
    g1 = _bwd(qt, kt, vt, o, lse, dot, True)
    g2 = _bwd(qt, kt, vt, o, lse, dot, True)
    assert all(torch.equal(a, b) for a, b in zip(g1, g2))


def test_workspace_size_covers_the_scheduler_state():
    b, h, s, d = 2, 4, 512, 128
    full = nat.lib().ferrite_attn_bwd_ds_workspace_size(b, h, s, s, d, nat.BF16)
    assert full > b * h * _slice_bytes(s, s)
