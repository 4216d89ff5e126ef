"""The roofline bookkeeping and device timing (tests/test_profiling.py of
anxnd2211/ferrite-tpu, re-pointed at B200 peaks): the bound and percent-of-roof
arithmetic of ``ferrite.profiling`` (src/ferrite/profiling/roofline.py:17-94 of the
reference) off device, and ``timeit`` with CUDA events on one."""

import pytest
import torch

from ferrite import platform
from ferrite.kernels.matmul import matmul, matmul_flops
from ferrite.profiling import analyze, format_table, timeit


def test_roofline_math_off_device():
    peaks = platform.peaks()
    assert peaks.source in ("measured", "fallback")
    assert peaks.cores == 148 or torch.cuda.is_available()
    assert peaks.ridge_point > 100  # bf16 FLOP per HBM byte: ~250 on B200
    p = analyze("mm", flops=2 * 1024**3, bytes_=3 * 1024 * 1024 * 2, seconds=20e-6, peaks=peaks)
    assert p.bound == "compute" and 0 < p.percent_of_roof < 1000
    assert p.achieved_tflops == pytest.approx(2 * 1024**3 / 20e-6 / 1e12)
    q = analyze("norm", flops=4 * 1024 * 1024, bytes_=3 * 1024 * 1024 * 2, seconds=20e-6, peaks=peaks)
    assert q.bound == "memory"
    # memory-bound: percent of roof is bytes / peak bandwidth over the time taken
    assert q.percent_of_roof == pytest.approx(100 * (3 * 1024 * 1024 * 2 / peaks.hbm_bytes_per_s) / 20e-6)
    table = format_table([p, q])
    assert "| kernel |" in table and "| mm |" in table and "memory" in table
    assert matmul_flops(256, 256, 256) == 2 * 256**3


@pytest.mark.gpu
def test_timeit_with_cuda_events():
    x = torch.randn(256, 256, device="cuda").to(torch.bfloat16)
    t = timeit(lambda a: matmul(a, a), x, warmup=1, iters=2)
    assert t.median_s > 0 and t.iters == 2 and t.min_s <= t.median_s
