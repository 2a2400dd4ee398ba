"""Independent requant model, written like the reference tests' own ``ref_requant``.

gemmkit's tests check the fused requant against a scalar model that rounds with the std
``round_ties_even`` instead of the kernel's 2^52 trick (gemmkit/tests/epilogue/requant.rs:18-23,
gemmkit/src/simd.rs:749-753). This is that model in Python: ``float`` is IEEE binary64 with
round-to-nearest-even arithmetic, and ``round()`` on a float rounds half to even exactly.
It shares no code with the C oracle, so it pins the oracle independently.
"""
from __future__ import annotations

import numpy as np

I64_MIN, I64_MAX = -(1 << 63), (1 << 63) - 1


def wrap_i32(x: int) -> int:
    x &= 0xFFFFFFFF
    return x - (1 << 32) if x >= (1 << 31) else x


def f32(x: float) -> float:
    return float(np.float32(x))


def requant(acc: int, bias: int, scale: float, zp: int, lo: int, hi: int,
            relu: bool = False) -> int:
    """clamp(zp + round_ties_even(f64(acc +wrap bias) * f64(scale_f32)), lo, hi)."""
    v = wrap_i32(acc + bias)
    p = float(v) * f32(scale)
    r = round(p)  # exact integer, ties to even
    q = min(max(r, I64_MIN), I64_MAX)  # `as i64` saturates
    q = min(max(q + zp, I64_MIN), I64_MAX)  # saturating_add
    out = min(max(q, lo), hi)
    if relu:
        out = max(out, min(max(zp, lo), hi))
    return out


def requant_array(acc: np.ndarray, bias_b: np.ndarray, scale_b: np.ndarray, zp: int, lo: int,
                  hi: int, relu: bool = False) -> np.ndarray:
    """Element-wise model over broadcast arrays (python ints; small cases only)."""
    acc, bias_b, scale_b = np.broadcast_arrays(np.asarray(acc, dtype=np.int64),
                                               np.asarray(bias_b, dtype=np.int64),
                                               np.asarray(scale_b, dtype=np.float32))
    out = np.empty(acc.shape, dtype=np.int64)
    it = np.nditer([acc, bias_b, scale_b], flags=["multi_index", "refs_ok"])
    for a, b, s in it:
        out[it.multi_index] = requant(int(a), int(b), float(s), zp, lo, hi, relu)
    return out


def acc_exact(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Exact accumulator (int64 matmul, then i32 wrap) of integer matrices a (m x k), b (k x n)."""
    s = a.astype(np.int64) @ b.astype(np.int64)
    return ((s + (1 << 31)) % (1 << 32) - (1 << 31)).astype(np.int32)
