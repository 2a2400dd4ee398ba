"""The reference test suites' deterministic generators, restated in Python.

gemmkit's tests build their inputs from two tiny generators; re-running them here gives the
parity tests the reference tests' own inputs, bit for bit.

- ``Rng``: xorshift* (gemmkit/tests/epilogue/common.rs:16-33), with ``make_i8`` drawing
  ``[-127, 127]`` as ``next_u64() % 255 - 127`` (gemmkit/tests/epilogue/requant.rs:25-30).
- ``rand_i8``: the xorshift64 stream of gemmkit/tests/correctness/common.rs:137-147 and
  gemmkit/tests/i8_packed_common/mod.rs:14-24, ``(s >> 24) % 201 - 100``.
"""
from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1


class Rng:
    def __init__(self, seed: int):
        self.s = (seed | 1) & M64

    def next_u64(self) -> int:
        x = self.s
        x ^= x >> 12
        x ^= (x << 25) & M64
        x ^= x >> 27
        self.s = x
        return (x * 0x2545F4914F6CDD1D) & M64


def make_i8(rng: Rng, n: int) -> np.ndarray:
    return np.array([(rng.next_u64() % 255) - 127 for _ in range(n)], dtype=np.int8)


def rand_i8(n: int, seed: int) -> np.ndarray:
    s = (seed + 0x9E3779B97F4A7C15) & M64
    out = np.empty(n, dtype=np.int8)
    for i in range(n):
        s ^= (s << 13) & M64
        s ^= s >> 7
        s ^= (s << 17) & M64
        out[i] = ((s >> 24) % 201) - 100
    return out


def bias_vec(rng: Rng, m: int) -> np.ndarray:
    """The per-row bias draw of check_requant (gemmkit/tests/epilogue/requant.rs:48-55)."""
    return np.array([(rng.next_u64() % 2001) - 1000 for _ in range(m)], dtype=np.int32)
