"""Numerics policy shared by the kernels (reference: src/ferrite/kernels/_compat.py).

``dot_precision`` keeps the reference's contract (_compat.py:17-26): f32 operands
get a true-f32 contraction ("highest"), 16-bit operands a single tensor-core
pass with an f32 accumulator ("default").  On B200 "highest" is the exact-f32
CUDA-core GEMM path of the native library; "default" is tcgen05 kind::f16.
``round_up`` is the reference helper (_compat.py:28-29).
"""

from __future__ import annotations

import torch


def dot_precision(dtype: torch.dtype) -> str:
    return "highest" if dtype == torch.float32 else "default"


def round_up(x: int, m: int) -> int:
    return -(-x // m) * m
