"""Hardware description and roofline peaks for B200 (sm_100a).

Mirrors the reference's ``ferrite.platform`` (src/ferrite/platform.py:20-144):
``LANES``/``SUBLANES`` keep their values because the public validation rules
(block sizes must be multiples of 8 / 128, flash_attention.py:346-353) are part
of the API contract, ``default_tile()`` is the tile the model layer uses for
attention blocks, and ``peaks()`` / ``describe()`` feed the roofline tooling.

Peaks come from ``MEASURED_PEAKS.json`` at the repository root when present (a
STREAM-style copy and a cuBLAS bf16 GEMM measured on this pool's B200s), else
from the pool's earlier measurement (6.65 TB/s, 1.59 PFLOP/s), labelled
"fallback".  TPU interpret mode (platform.py:112-125) has no B200 counterpart:
the kernels only run on the GPU.
"""

from __future__ import annotations

import dataclasses
import json
import os

import torch

LANES = 128  # block-size rule kept from the reference API (flash_attention.py:348)
SUBLANES = 8  # block_q / block_rows multiple (flash_attention.py:347, rmsnorm.py:72)

_REPO_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
PEAKS_FILE = os.path.join(_REPO_ROOT, "MEASURED_PEAKS.json")

# Nominal B200 figures (context only) and the pool's earlier measurement (fallback).
NOMINAL = {"bf16_tflops": 2250.0, "hbm_gbs": 7700.0}
FALLBACK = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}


def backend() -> str:
    return "cuda" if torch.cuda.is_available() else "cpu"


def is_gpu() -> bool:
    return torch.cuda.is_available()


def device_kind() -> str:
    return torch.cuda.get_device_name(0) if torch.cuda.is_available() else "cpu"


def num_devices() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def sm_count(device: int = 0) -> int:
    if not torch.cuda.is_available():
        return 148
    return torch.cuda.get_device_properties(device).multi_processor_count


def default_tile() -> int:
    """Default square tile for matmul-shaped work and attention blocks (128)."""
    return 128


@dataclasses.dataclass(frozen=True)
class Peaks:
    """Per-device roofline peaks (same fields as the reference's Peaks)."""

    name: str
    bf16_flops: float  # FLOP/s (burst)
    hbm_bytes_per_s: float
    hbm_bytes: float
    smem_bytes: float
    cores: int  # SMs
    source: str = "measured"  # "measured" | "fallback"
    bf16_flops_sustained: float | None = None

    @property
    def ridge_point(self) -> float:
        return self.bf16_flops / self.hbm_bytes_per_s


def _load_measured() -> dict | None:
    try:
        with open(PEAKS_FILE) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def peaks(chip: str | None = None) -> Peaks:
    """B200 peaks: measured when MEASURED_PEAKS.json exists, else the fallback."""
    m = _load_measured()
    if m and "hbm_gbs" in m and "bf16_tflops" in m:
        src, bf16, hbm = "measured", float(m["bf16_tflops"]), float(m["hbm_gbs"])
        sus = float(m.get("bf16_tflops_sustained", bf16))
    else:
        src, bf16, hbm, sus = "fallback", FALLBACK["bf16_tflops"], FALLBACK["hbm_gbs"], FALLBACK["bf16_tflops_sustained"]
    return Peaks(
        name=chip or "B200",
        bf16_flops=bf16 * 1e12,
        hbm_bytes_per_s=hbm * 1e9,
        hbm_bytes=183_359 * 2**20,
        smem_bytes=227 * 1024,
        cores=sm_count(),
        source=src,
        bf16_flops_sustained=sus * 1e12,
    )


def describe() -> dict:
    p = peaks()
    out = {
        "backend": backend(),
        "device_kind": device_kind(),
        "num_devices": num_devices(),
        "torch_version": torch.__version__,
        "chip": p.name,
        "sms": p.cores,
        "peak_bf16_tflops": p.bf16_flops / 1e12,
        "peak_hbm_gbps": p.hbm_bytes_per_s / 1e9,
        "peaks_source": p.source,
        "ridge_point_flop_per_byte": p.ridge_point,
    }
    return out
