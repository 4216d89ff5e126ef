"""The roofline bookkeeping and device timing (the cases of tests/test_profiling.py of
anxnd2211/ferrite-tpu, re-pointed at the B200 ceilings): bound and fraction of the
ceiling off device, the benchmark line's roofline object, and ``timeit`` with CUDA
events on a GPU."""

import pytest
import torch

from ferrite import platform
from ferrite.kernels.matmul import matmul, matmul_flops
from ferrite.profiling import analyze, format_table, roofline, timeit


def test_roofline_math_off_device():
    peaks = platform.peaks()
    assert peaks.source in ("measured", "fallback")
    assert peaks.cores == 148 or torch.cuda.is_available()
    assert peaks.ridge_point > 100  # bf16 FLOP per HBM byte: ~250 on B200
    # a GEMM-shaped launch: the tensor floor is the longer one
    p = analyze("mm", flops=2 * 1024**3, bytes_=3 * 1024 * 1024 * 2, seconds=20e-6, peaks=peaks)
    assert p.bound == "tensor" and 0 < p.frac < 10
    assert p.achieved_tflops == pytest.approx(2 * 1024**3 / 20e-6 / 1e12)
    assert p.frac == pytest.approx(2 * 1024**3 / peaks.bf16_flops / 20e-6)
    # a norm-shaped launch: bytes at the copy bandwidth over the time taken
    q = analyze("norm", flops=4 * 1024 * 1024, bytes_=3 * 1024 * 1024 * 2, seconds=20e-6, peaks=peaks)
    assert q.bound == "hbm"
    assert q.frac == pytest.approx(3 * 1024 * 1024 * 2 / peaks.hbm_bytes_per_s / 20e-6)
    assert q.percent_of_roof == pytest.approx(100 * q.frac)
    table = format_table([p, q])
    assert "| kernel |" in table and "| mm |" in table and "hbm" in table
    assert matmul_flops(256, 256, 256) == 2 * 256**3


def test_bench_line_object_and_peak_choice():
    """The ``roofline`` object of the benchmark line: burst tensor peak for a
    sub-second region, sustained for a longer one; bytes against the copy bandwidth."""
    peaks = platform.peaks()
    c = roofline.Ceilings.from_platform(peaks)
    assert not c.for_region(0.5) and c.for_region(5.0)
    burst = analyze("attn_bwd_dkv", flops=8.8e12, bytes_=0.0, seconds=9.67e-3, peaks=peaks).line(traffic=22.6e9)
    assert burst["bound"] == "tensor" and burst["unit"] == "TFLOP/s" and burst["traffic"] == 22.6e9
    assert burst["peak"] == pytest.approx(peaks.bf16_flops / 1e12, rel=1e-3)
    assert burst["frac"] == pytest.approx(8.8e12 / 9.67e-3 / peaks.bf16_flops, rel=1e-3)
    assert burst["frac_of_sustained"] >= burst["frac"]
    sus = analyze("train_step", flops=1e14, bytes_=0.0, seconds=0.2, peaks=peaks, sustained=True).line()
    assert sus["peak"] == pytest.approx(peaks.bf16_flops_sustained / 1e12, rel=1e-3) and "frac_of_sustained" not in sus
    hbm = analyze("rmsnorm_bwd", flops=0.0, bytes_=268_468_224, seconds=60e-6, peaks=peaks).line()
    assert hbm["bound"] == "hbm" and hbm["unit"] == "GB/s"
    assert hbm["achieved"] == pytest.approx(268_468_224 / 60e-6 / 1e9, rel=1e-4)
    assert roofline.dominant({"a": 1.0, "b": 3.0, "c": 5.0}, {"a": 1, "b": 1, "c": 0}) == "b"


@pytest.mark.gpu
def test_timeit_with_cuda_events():
    x = torch.randn(256, 256, device="cuda").to(torch.bfloat16)
    t = timeit(lambda a: matmul(a, a), x, warmup=1, iters=2)
    assert t.median_s > 0 and t.iters == 2 and t.min_s <= t.median_s
