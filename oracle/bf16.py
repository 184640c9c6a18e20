"""bfloat16 emulation on float32 numpy arrays (oracle helper, test-only).

bfloat16 keeps the top 16 bits of an IEEE float32.  Torch rounds float32 to
bfloat16 with round-to-nearest-even and preserves NaN; ``round_bf16`` does
the same on the raw bits, so an oracle value is bit-identical to what a torch
``.to(torch.bfloat16)`` of the same float32 would hold.
"""

from __future__ import annotations

import numpy as np


def round_bf16(a) -> np.ndarray:
    """float32 -> nearest bfloat16 value (ties to even), returned as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).reshape(a.shape).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.nan
    return out


def f32_to_bf16_bits(a) -> np.ndarray:
    """float32 -> uint16 bfloat16 bit patterns (rounded to nearest even)."""
    r = round_bf16(a)
    return (r.view(np.uint32) >> 16).astype(np.uint16)


def bf16_bits_to_f32(bits) -> np.ndarray:
    """uint16 bfloat16 bit patterns -> float32 values (exact)."""
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_to(a, dtype: str) -> np.ndarray:
    """Round float32 values to the storage precision named by ``dtype``
    ("f32" or "bf16"), mirroring a torch op that writes that dtype."""
    if dtype == "f32":
        return np.asarray(a, dtype=np.float32)
    if dtype == "bf16":
        return round_bf16(a)
    raise ValueError(f"oracle: unsupported dtype {dtype!r}")


def promote(*dtypes: str) -> str:
    """torch type promotion restricted to {f32, bf16}: any f32 operand wins."""
    return "f32" if "f32" in dtypes else "bf16"
