"""CPU checks of the C-ABI library and the host-side API logic (no GPU compute).

* the shared library loads and exports every entry point ``include/*.h`` declares,
  with the signatures the ctypes binding uses;
* host-side validation returns the documented status codes before touching a
  device (bad shapes / dtypes, host fault injection);
* the Python API raises the reference's ``ValueError``s and refuses CPU tensors
  (no fallback path).
"""

import ctypes
import glob
import os
import re

import pytest
import torch

from ferrite import _native as nat
from ferrite.kernels.flash_attention import BlockSizes, attention_flops, flash_attention
from ferrite.kernels.matmul import matmul, matmul_flops
from ferrite.kernels.rmsnorm import rmsnorm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols() -> set[str]:
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        names |= set(re.findall(r"FERRITE_API\s+[\w\s\*]+?\b(ferrite_\w+)\s*\(", txt))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    lib = nat.lib()
    declared = _declared_symbols()
    assert len(declared) >= 12, declared
    for name in declared:
        assert hasattr(lib, name), name
    assert declared <= set(nat.SIGNATURES), declared - set(nat.SIGNATURES)
    assert "sm_100a" in nat.version()


def test_library_is_built_for_sm100a_only():
    out = os.popen(f"cuobjdump --list-elf {nat.LIB_PATH} 2>/dev/null").read()
    if not out:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out
    assert "sm_90" not in out and "sm_80" not in out


def test_status_codes_without_a_gpu():
    lib = nat.lib()
    # negative rows -> BAD_SHAPE, before any CUDA call
    rc = lib.ferrite_rmsnorm_fwd(None, 1, 1, 1, -1, 4096, 1e-6, nat.BF16, nat.F32)
    assert rc == nat.BAD_SHAPE and "bad shape" in nat.last_error()
    rc = lib.ferrite_add_rmsnorm_fwd(None, 1, 1, 1, 1, 1, 8, 4096, 1e-6, 7, nat.F32)
    assert rc == nat.UNSUPPORTED_DTYPE
    rc = lib.ferrite_rmsnorm_bwd(None, 1, 1, 1, None, 1, 1, 1, 16, 8, 0, 1e-6, nat.BF16, nat.F32)
    assert rc == nat.BAD_SHAPE
    with pytest.raises(nat.FerriteError) as e:
        nat.check(nat.UNSUPPORTED_DTYPE)
    assert e.value.status == nat.UNSUPPORTED_DTYPE


def test_strided_attention_validation_without_a_gpu():
    """The strided entry points check their stride block on the host, after the
    shape checks and before any CUDA call."""
    lib = nat.lib()
    args = (1, 2, 256, 256, 64, 0.125, 1, 128, 128, nat.BF16)
    rc = lib.ferrite_attn_fwd_strided(None, 1, 1, 1, 1, 1, None, *args)
    assert rc == nat.BAD_SHAPE and "null strides" in nat.last_error()
    st = nat.AttnStrides()
    st.k[:] = (0, -64, 64)
    rc = lib.ferrite_attn_fwd_strided(None, 1, 1, 1, 1, 1, ctypes.byref(st), *args)
    assert rc == nat.BAD_SHAPE and "negative stride" in nat.last_error()
    rc = lib.ferrite_attn_bwd_dq_strided(None, 1, 1, 1, 1, 1, 1, 1, ctypes.byref(st), *args)
    assert rc == nat.BAD_SHAPE
    rc = lib.ferrite_attn_bwd_dkv_strided(None, 1, 1, 1, 1, 1, 1, 1, 1, None, *args)
    assert rc == nat.BAD_SHAPE
    rc = lib.ferrite_attn_bwd_prep_strided(None, 1, 1, 1, None, 1, 2, 256, 64, nat.BF16)
    assert rc == nat.BAD_SHAPE
    # shape errors come first, as in the contiguous entry points
    rc = lib.ferrite_attn_fwd_strided(None, 1, 1, 1, 1, 1, ctypes.byref(st), 1, 2, 256, 256, 64, 0.125, 1, 100, 128, nat.BF16)
    assert rc == nat.BAD_SHAPE and "block_q" in nat.last_error()


def test_ds_backward_host_checks_without_a_gpu():
    lib = nat.lib()
    def sched(slices, sq):  # the fused backward's scheduler state after the dS slots, 256-byte aligned
        return -(-(8 + 2 * slices * -(-sq // 128) + slices) * 4 // 256) * 256

    assert lib.ferrite_attn_bwd_ds_workspace_size(2, 3, 512, 512, 64, nat.BF16) == 6 * 512 * 512 * 2 + sched(6, 512)
    assert lib.ferrite_attn_bwd_ds_workspace_size(1, 1, 200, 384, 64, nat.BF16) == 256 * 384 * 2 + sched(1, 200)  # rows padded to 64
    assert lib.ferrite_attn_bwd_ds_workspace_size(1, 1, 512, 512, 64, nat.F32) == 0  # CUDA-core path: no dS
    assert lib.ferrite_attn_bwd_ds_workspace_size(1, 1, 512, 512, 96, nat.BF16) == 0
    st = nat.AttnStrides()
    args = (1, 2, 256, 256, 64, 0.125, 1, 128, 128, nat.BF16)
    rc = lib.ferrite_attn_bwd_dkv_ds(None, 1, 1, 1, 1, 1, 1, 1, 1, 1, ctypes.byref(st), 1, 2, *args)
    assert rc == nat.BAD_SHAPE and "slice range" in nat.last_error()
    rc = lib.ferrite_attn_bwd_dq_ds(None, 1, 1, 1, ctypes.byref(st), -1, 1, *args)
    assert rc == nat.BAD_SHAPE


def test_attn_strides_struct_matches_views():
    qkv = torch.zeros(2, 256, 3, 4, 64)
    q = qkv[:, :, 0].permute(0, 2, 1, 3)
    st = nat.attn_strides(q=q)
    assert tuple(st.q) == (256 * 3 * 4 * 64, 64, 3 * 4 * 64) and tuple(st.k) == (0, 0, 0)
    assert ctypes.sizeof(nat.AttnStrides) == 8 * 3 * 8
    with pytest.raises(ValueError):
        nat.attn_strides(q=q.transpose(2, 3))


def test_host_fault_injection(monkeypatch):
    lib = nat.lib()
    monkeypatch.setenv("FERRITE_FAULT_INJECT", "rmsnorm_fwd,add_rmsnorm_fwd")
    rc = lib.ferrite_rmsnorm_fwd(None, 1, 1, 1, 8, 4096, 1e-6, nat.BF16, nat.F32)
    assert rc == nat.INJECTED_FAULT and "injected" in nat.last_error()
    monkeypatch.setenv("FERRITE_FAULT_INJECT", "all")
    assert lib.ferrite_rmsnorm_bwd(None, 1, 1, 1, None, 1, 1, 1, 16, 8, 8, 1e-6, nat.BF16, nat.F32) == nat.INJECTED_FAULT
    monkeypatch.delenv("FERRITE_FAULT_INJECT")


def test_last_error_is_thread_local():
    import threading

    lib = nat.lib()
    lib.ferrite_rmsnorm_fwd(None, 1, 1, 1, -1, 8, 1e-6, nat.BF16, nat.F32)
    seen = []

    def other():
        seen.append(nat.last_error())

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen == [""]
    assert "bad shape" in nat.last_error()


def test_workspace_query_is_bounded():
    lib = nat.lib()
    # f32 operands never split (exact CUDA-core path); answered without a device
    assert lib.ferrite_gemm_workspace_size(1024, 1024, 65536, 1024, 1024, 1, 0, nat.F32) == 0
    assert lib.ferrite_gemm_workspace_size(0, 1024, 65536, 1024, 1024, 1, 0, nat.BF16) == 0
    ws = lib.ferrite_rmsnorm_bwd_workspace_size(8192, 4096)
    assert 0 < ws <= 8192 * 4096 * 4
    assert lib.ferrite_rmsnorm_bwd_workspace_size(1, 128) >= 8 * 128 * 4 or lib.ferrite_rmsnorm_bwd_workspace_size(1, 128) >= 128 * 4


# ---------------------------------------------------------------- Python API validation


def test_rmsnorm_validation_errors():
    x = torch.zeros(4, 64)
    with pytest.raises(ValueError):
        rmsnorm(x, torch.ones(63))
    with pytest.raises(ValueError):
        rmsnorm(x, torch.ones(64), residual=torch.zeros(4, 32))
    with pytest.raises(ValueError):
        rmsnorm(x, torch.ones(64), block_rows=12)


def test_cpu_tensors_are_refused_not_computed():
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        rmsnorm(torch.zeros(4, 64), torch.ones(64))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        matmul(torch.zeros(8, 8), torch.zeros(8, 8))
    q = torch.zeros(1, 1, 128, 64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        flash_attention(q, q, q)


def test_flash_attention_validation_errors():
    q = torch.zeros(1, 1, 256, 128)
    with pytest.raises(ValueError):
        flash_attention(q, q, q, block_sizes=BlockSizes(block_k=100))
    with pytest.raises(ValueError):
        flash_attention(q, q[:, :, :128], q[:, :, :128], causal=True)
    with pytest.raises(ValueError):
        flash_attention(q, q, q.to(torch.bfloat16))
    with pytest.raises(ValueError):
        flash_attention(torch.zeros(1, 1, 256, 200), torch.zeros(1, 1, 256, 200), torch.zeros(1, 1, 256, 200))


def test_matmul_validation_errors():
    x = torch.zeros(128, 128)
    with pytest.raises(ValueError):
        matmul(x, x, block_n=100)
    with pytest.raises(ValueError):
        matmul(x, torch.zeros(64, 8))


def test_flop_formulas():
    assert matmul_flops(256, 256, 256) == 2 * 256**3
    assert attention_flops(2, 4, 512, 512, 64, causal=True) * 3.5 == pytest.approx(9.395e8, rel=1e-3)
