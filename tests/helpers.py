"""Test helpers: seeded inputs, numpy <-> torch conversion with exact bf16 bits."""

from __future__ import annotations

import ml_dtypes
import numpy as np
import torch

BF16 = ml_dtypes.bfloat16

NP_TO_TORCH = {np.dtype(np.float32): torch.float32, np.dtype(BF16): torch.bfloat16, np.dtype(np.float16): torch.float16}


def normal(rng: np.random.Generator, shape, dtype=np.float32, std=1.0, mean=0.0) -> np.ndarray:
    """N(mean, std^2) in f32, then rounded to ``dtype`` (round-to-nearest-even)."""
    return (mean + std * rng.standard_normal(shape, dtype=np.float32)).astype(dtype)


def to_torch(a: np.ndarray, device="cuda") -> torch.Tensor:
    """Bit-exact numpy -> torch (bf16 via its uint16 bit pattern)."""
    if a.dtype == BF16:
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.uint16).astype(np.int16)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to(device)


def to_numpy(t: torch.Tensor) -> np.ndarray:
    """Bit-exact torch -> numpy (bf16 comes back as ml_dtypes.bfloat16)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).view(BF16)
    return t.numpy()


def f32(a) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        a = to_numpy(a)
    return np.asarray(a).astype(np.float32)


def max_abs(a, b) -> float:
    return float(np.max(np.abs(f32(a) - f32(b)))) if np.size(a) else 0.0


def bf16_ulp(x) -> np.ndarray:
    """Spacing of bf16 values at |x|: 2^(e - 7) with e = floor(log2 |x|)."""
    a = np.maximum(np.abs(f32(x)), np.float32(2.0**-126))
    return np.ldexp(np.float32(1.0), np.floor(np.log2(a)).astype(np.int32) - 7)


def assert_bf16_close(got, ref, atol: float = 2e-2) -> None:
    """|got - ref| <= max(atol, one bf16 ulp of ref): the max-abs 2e-2 bound on bf16
    results, widened to bf16's own rounding step where |ref| >= 4 (2^-5 there), since
    two correct implementations may round a value near a tie to neighbouring bf16s."""
    g, r = f32(got), f32(ref)
    bound = np.maximum(np.float32(atol), bf16_ulp(r))
    bad = np.abs(g - r) > bound
    assert not bad.any(), f"{int(bad.sum())} elements off; worst {float(np.max(np.abs(g - r) - bound)):.3g} over the bound"


def rel_l2(a, b) -> float:
    a, b = f32(a).astype(np.float64), f32(b).astype(np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def save_arrays(path: str, **arrays) -> None:
    """npz with bf16 arrays stored as uint16 bits plus a dtype tag."""
    out = {}
    for k, v in arrays.items():
        if isinstance(v, np.ndarray) and v.dtype == BF16:
            out[k] = v.view(np.uint16)
            out[k + "__dtype"] = np.array("bfloat16")
        else:
            out[k] = v
    np.savez_compressed(path, **out)


def load_arrays(path: str) -> dict:
    raw = np.load(path)
    out = {}
    for k in raw.files:
        if k.endswith("__dtype"):
            continue
        v = raw[k]
        if k + "__dtype" in raw.files and str(raw[k + "__dtype"]) == "bfloat16":
            v = v.view(BF16)
        out[k] = v
    return out
