"""A bounded device wait that runs out, on the GPU.

Every mbarrier wait of the tensor-core kernels is bounded; on expiry the kernel
records FERRITE_DEVICE_TIMEOUT in a device status word, raises its CTA's abort flag
so the other roles leave their waits, frees TMEM in its ordinary teardown and
returns.  ``ferrite_wait_probe`` runs that path with a 1 ms limit on a barrier that
nothing arrives on (no fault, no trap, no unbounded loop), and these tests check
that the host reads the status, that the CTA tore down (TMEM freed) and that the
context stays usable: a GEMM on every SM afterwards matches the oracle.

The reference's counterpart is its interpret-mode race detector run over the
kernels (tests/test_flash_attention.py:79-85 of anxnd2211/ferrite-tpu).
"""

import numpy as np
import pytest
import torch

from ferrite import _native as nat
from ferrite.kernels.matmul import matmul
from helpers import BF16, normal, to_numpy, to_torch

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000  # 1 ms


def _probe(limit_ns=LIMIT_NS):
    out = torch.zeros(4, dtype=torch.int64, device="cuda")
    nat.check(nat.lib().ferrite_wait_probe(nat.stream_ptr(), limit_ns, out.data_ptr()))
    return out


def test_expired_wait_reports_timeout_frees_tmem_and_context_survives():
    nat.device_status(clear=True)  # start from a clean status word
    out = _probe()
    rc = nat.lib().ferrite_device_status(nat.stream_ptr(), 1)  # synchronises, reads and clears
    assert rc == nat.DEVICE_TIMEOUT, nat.STATUS_NAMES.get(rc, rc)
    waited, timed_out, left, freed = out.tolist()
    assert timed_out == 1
    assert LIMIT_NS <= waited < 1_000_000_000, waited  # expired after its limit, well before the 2 s bound
    assert left == 4  # the issuer and the three waiters released by the abort flag
    assert freed == 1  # the teardown freed TMEM
    # cleared: the next read is clean
    assert nat.lib().ferrite_device_status(nat.stream_ptr(), 0) == nat.OK
    # the context is usable: a persistent tensor-core GEMM (TMEM on every SM) is correct
    rng = np.random.default_rng(11)
    a, b = normal(rng, (2048, 512), BF16), normal(rng, (512, 4096), BF16)  # 256 output tiles
    c = matmul(to_torch(a), to_torch(b), out_dtype=torch.float32)
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_numpy(c), a.astype(np.float32) @ b.astype(np.float32), rtol=1e-3, atol=1e-2)
    assert nat.lib().ferrite_device_status(nat.stream_ptr(), 0) == nat.OK


def test_device_status_raises_through_the_python_helper():
    nat.device_status(clear=True)
    _probe()
    with pytest.raises(nat.FerriteError, match="DEVICE_TIMEOUT"):
        nat.device_status(clear=True)
    nat.device_status(clear=True)  # cleared by the call above


def test_probe_rejects_limits_outside_the_bound():
    out = torch.zeros(4, dtype=torch.int64, device="cuda")
    assert nat.lib().ferrite_wait_probe(nat.stream_ptr(), 0, out.data_ptr()) == nat.BAD_SHAPE
    assert nat.lib().ferrite_wait_probe(nat.stream_ptr(), 3_000_000_000, out.data_ptr()) == nat.BAD_SHAPE
