"""bfloat16 helpers for numpy (test infrastructure).

numpy has no bfloat16 dtype; values are carried as float32 and rounded with
round-to-nearest-even on the upper 16 bits, which is what torch's
``.to(torch.bfloat16)`` does for finite values.  Storage form is uint16.
"""
from __future__ import annotations

import numpy as np


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.nan
    return out


def to_bits(x: np.ndarray) -> np.ndarray:
    """float32 (already bf16-representable or not) -> bf16 bit pattern uint16."""
    r = round_bf16(x)
    return (r.view(np.uint32) >> 16).astype(np.uint16)


def from_bits(b: np.ndarray) -> np.ndarray:
    """bf16 bit pattern uint16 -> float32."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
