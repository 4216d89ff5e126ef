"""Roofline of a kernel launch on B200, against the peaks measured on this pool.

A launch that does ``flops`` tensor-core FLOPs and must move ``bytes`` of HBM
traffic cannot finish faster than the slower of two floors: ``bytes`` at the copy
bandwidth, or ``flops`` at the dense bf16 tensor rate.  Whichever floor is longer
names the bound ("hbm" or "tensor"), and ``frac`` = floor / measured time says
how close the launch came to it (a kernel a little above 1.0 against a measured
copy or cuBLAS peak is possible; far above means the timed launch did not do the
counted work).

Two tensor rates exist on a 1 kW part: the burst rate (a kernel timed alone or in
a sub-second region) and the sustained rate under the power cap (a kernel timed
inside a seconds-long loop).  ``Ceilings`` carries both and ``for_region`` picks
one by the length of the timed region.

The reference keeps the same public names (``RooflinePoint``, ``analyze``,
``format_table``: src/ferrite/profiling/roofline.py of anxnd2211/ferrite-tpu,
re-exported by ferrite.profiling) with chip peaks from JAX's table; here the peaks
come from :func:`ferrite.platform.peaks` and the point also produces the
``roofline`` object of the benchmark's JSON line.
"""

from __future__ import annotations

import dataclasses

from ferrite import platform

# A timed region at least this long runs at the power-capped (sustained) clocks.
SUSTAINED_REGION_S = 1.0


@dataclasses.dataclass(frozen=True)
class Ceilings:
    """Per-device ceilings: HBM bytes/s and dense bf16 FLOP/s (burst, sustained)."""

    hbm_bytes_per_s: float
    tensor_burst: float
    tensor_sustained: float
    source: str  # "measured" (MEASURED_PEAKS.json) | "fallback"

    @classmethod
    def from_platform(cls, peaks: platform.Peaks | None = None) -> "Ceilings":
        p = peaks or platform.peaks()
        return cls(p.hbm_bytes_per_s, p.bf16_flops, p.bf16_flops_sustained or p.bf16_flops, p.source)

    def tensor_rate(self, sustained: bool) -> float:
        return self.tensor_sustained if sustained else self.tensor_burst

    def for_region(self, region_seconds: float) -> bool:
        """True when a region of this length is judged against the sustained rate."""
        return region_seconds >= SUSTAINED_REGION_S


@dataclasses.dataclass(frozen=True)
class RooflinePoint:
    """One launch: algorithmic work, measured time, and the ceilings it is held to."""

    name: str
    flops: float
    bytes: float
    seconds: float
    ceilings: Ceilings
    sustained: bool = False
    devices: int = 1

    @property
    def _tensor(self) -> float:
        return self.ceilings.tensor_rate(self.sustained) * self.devices

    @property
    def _hbm(self) -> float:
        return self.ceilings.hbm_bytes_per_s * self.devices

    @property
    def floors(self) -> dict[str, float]:
        """Seconds each ceiling alone allows for this work."""
        return {"tensor": self.flops / self._tensor, "hbm": self.bytes / self._hbm}

    @property
    def bound(self) -> str:
        f = self.floors
        return "tensor" if f["tensor"] >= f["hbm"] else "hbm"

    @property
    def frac(self) -> float:
        return max(self.floors.values()) / self.seconds

    @property
    def achieved_tflops(self) -> float:
        return self.flops / self.seconds / 1e12

    @property
    def achieved_gbps(self) -> float:
        return self.bytes / self.seconds / 1e9

    @property
    def percent_of_roof(self) -> float:
        return 100.0 * self.frac

    def line(self, traffic: float | None = None) -> dict:
        """The benchmark line's ``roofline`` object for this launch."""
        if self.bound == "tensor":
            achieved, peak, unit = self.achieved_tflops, self._tensor / 1e12, "TFLOP/s"
            which = "bf16_tflops_sustained" if self.sustained else "bf16_tflops"
        else:
            achieved, peak, unit = self.achieved_gbps, self._hbm / 1e9, "GB/s"
            which = "hbm_gbs"
        src = f"measured (MEASURED_PEAKS.json {which})" if self.ceilings.source == "measured" else "fallback"
        out = {"bound": self.bound, "kernel": self.name, "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": unit,
               "frac": round(achieved / peak, 4), "peak_source": src, "traffic": traffic}
        if self.bound == "tensor" and not self.sustained:
            out["frac_of_sustained"] = round(self.flops / self.seconds / (self.ceilings.tensor_sustained * self.devices), 4)
        return out


def analyze(name: str, flops: float, bytes_: float, seconds: float, peaks: platform.Peaks | None = None, devices: int = 1,
            sustained: bool = False) -> RooflinePoint:
    """A :class:`RooflinePoint` for ``flops`` / ``bytes_`` done in ``seconds`` on ``devices`` GPUs."""
    return RooflinePoint(name, float(flops), float(bytes_), float(seconds), Ceilings.from_platform(peaks), sustained, devices)


def dominant(kernel_seconds: dict[str, float], counted: dict[str, float]) -> str:
    """The kernel with the longest time among those that do counted work."""
    return max((k for k in kernel_seconds if counted.get(k)), key=lambda k: kernel_seconds[k])


def format_table(points: list[RooflinePoint]) -> str:
    """Markdown table of points: time, rates, bound and fraction of its ceiling."""
    rows = ["| kernel | ms | TFLOP/s | GB/s | bound | of ceiling |", "|---|---:|---:|---:|---|---:|"]
    for p in points:
        rows.append(f"| {p.name} | {p.seconds * 1e3:.3f} | {p.achieved_tflops:.1f} | {p.achieved_gbps:.0f} | {p.bound} | {p.frac:.2f} |")
    return "\n".join(rows)
