"""Rounding helpers for the CPU oracle -- TEST INFRASTRUCTURE, never the product path.

numpy has no bfloat16, so values are rounded to bf16 by round-to-nearest-even on the float32
bit pattern; f16 uses numpy's own float16. Results stay float64 arrays holding exactly the
representable values, which is how the oracle models a kernel that stores an intermediate in
the 16-bit compute type.
"""
import numpy as np


def round_bf16(x):
    """Round to the nearest bfloat16 (ties to even), returned as float64."""
    f = np.ascontiguousarray(np.asarray(x, np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


def round_to(x, dtype):
    """Round to the 16-bit compute type 'f16' or 'bf16' (anything else: float32)."""
    if dtype == 'f16':
        return np.asarray(x, np.float64).astype(np.float16).astype(np.float64)
    if dtype == 'bf16':
        return round_bf16(x)
    return np.asarray(x, np.float32).astype(np.float64)


def rel_max(a, b):
    """The reference tests' metric: max|a-b| / max(max|b|, 1e-3); NaN or inf counts as inf
    (tests/test_attn_bwd.py:104-111)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    if not np.isfinite(a).all():
        return float('inf')
    if a.size == 0:
        return 0.0
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-3))


def rel_l2(a, b):
    """||a-b||_2 / max(||b||_2, 1e-3 sqrt(n)); NaN or inf counts as inf. The floor is the
    rel_max floor per element: an exactly-zero gradient (one key) has no relative scale."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    if not np.isfinite(a).all():
        return float('inf')
    if a.size == 0:
        return 0.0
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-3 * np.sqrt(a.size)))


def max_abs(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    if not np.isfinite(a).all():
        return float('inf')
    return float(np.abs(a - b).max()) if a.size else 0.0
