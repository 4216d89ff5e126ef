"""Device timing with CUDA events (reference: src/ferrite/profiling/timing.py:25-35,
which times ``block_until_ready`` wall clock; here the events are recorded on the
launching stream, after warm-up, with a synchronize on both sides)."""

from __future__ import annotations

import dataclasses

import numpy as np
import torch


@dataclasses.dataclass(frozen=True)
class Timing:
    median_s: float
    min_s: float
    mean_s: float
    std_s: float
    iters: int

    @property
    def median_ms(self) -> float:
        return self.median_s * 1e3


def timeit(fn, *args, warmup: int = 3, iters: int = 10, **kw) -> Timing:
    """Time ``fn(*args, **kw)`` per call with CUDA events; the first ``warmup`` calls are discarded."""
    for _ in range(warmup):
        fn(*args, **kw)
    torch.cuda.synchronize()
    samples = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn(*args, **kw)
        b.record()
        b.synchronize()
        samples.append(a.elapsed_time(b) / 1e3)
    s = np.asarray(samples)
    return Timing(float(np.median(s)), float(s.min()), float(s.mean()), float(s.std()), iters)
