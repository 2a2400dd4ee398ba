"""Generate the golden fixtures the parity tests check against.

Run once in the build container (``python tests/golden/make_golden.py``); the outputs are
committed and nothing at test time regenerates them.

- ``kat.json``: known-answer vectors whose expected outputs are hard-coded constants (or a
  closed-form wrapping formula) in the reference's own tests; each entry cites its source.
- ``model_cases.json``: the reference tests' sweeps, re-run on the reference tests' own
  inputs (the xorshift generators of refrng.py) with expected outputs from the independent
  round_ties_even model of model.py (the same model the reference tests assert against).
  Large outputs are stored as sha256 digests of their little-endian bytes.

gemmkit is Rust and cannot be built or imported here, so no expected value below comes from
running it; each comes from a constant in its tests or from its tests' own model.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from model import acc_exact, f32, requant, requant_array, wrap_i32  # noqa: E402
from refrng import Rng, bias_vec, make_i8, rand_i8  # noqa: E402

I8, U8 = (-128, 127), (0, 255)


def digest(arr: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()


def kat_cases() -> list[dict]:
    out = []
    out.append(dict(
        name="requant_ties_even_exact", source="gemmkit/tests/epilogue/requant.rs:253-272",
        kind="requant", m=6, k=1, n=1, a_colmajor=[1, 3, 5, 7, -1, -3], b=[1], scale=0.5, zp=0,
        out_u8=False, expect=[0, 2, 2, 4, 0, -2]))
    out.append(dict(
        name="requant_u8_saturates", source="gemmkit/tests/epilogue/requant.rs:885-910",
        kind="requant", m=8, k=1, n=1, a_colmajor=[127, -128, 100, -100, 1, -1, 64, -64], b=[1],
        scale=1000.0, zp=0, out_u8=True, expect=[255, 0, 255, 0, 255, 0, 255, 0]))
    out.append(dict(
        name="requant_u8_ties_even_exact", source="gemmkit/tests/epilogue/requant.rs:913-938",
        kind="requant", m=6, k=1, n=1, a_colmajor=[1, 5, 9, -1, -5, -9], b=[1], scale=0.5,
        zp=10, out_u8=True, expect=[10, 12, 14, 10, 8, 6]))
    # i8_wraps_on_overflow: expected = beta.wrapping_mul(c).wrapping_add(alpha.wrapping_mul(acc))
    c0 = [1_000_000, -2_000_000, 3_000_000, -4_000_000]
    alpha, beta, acc = 100_000, 1, 127 * 127 + 127 * 127
    want = [wrap_i32(wrap_i32(beta * c) + wrap_i32(alpha * acc)) for c in c0]
    out.append(dict(
        name="i8_wraps_on_overflow", source="gemmkit/tests/correctness/int8.rs:198-238",
        kind="gemm_i8", m=2, k=2, n=2, a_rowmajor=[127] * 4, b_rowmajor=[127] * 4, c0=c0,
        alpha=alpha, beta=beta, expect=want))
    return out


def model_cases() -> dict:
    cases: dict = {}

    # requant_ties_and_saturation (gemmkit/tests/epilogue/requant.rs:275-320) through
    # check_requant (:34-98): a, b col-major draws from one Rng(0x7135), then an optional bias.
    rng = Rng(0x7135)
    sweep = []
    for k in [1, 8, 300, 1000, 5000]:
        for tag, scale, zp, has_bias in [("ties", 0.5, 3, True), ("sat+", 100.0, 120, False),
                                         ("sat-", 100.0, -120, True)]:
            m, n = 20, 18
            a = make_i8(rng, m * k).reshape(k, m).T  # col-major m x k
            b = make_i8(rng, k * n).reshape(n, k).T  # col-major k x n
            bias = bias_vec(rng, m) if has_bias else np.zeros(m, np.int32)
            acc = acc_exact(a, b)
            want = requant_array(acc, bias[:, None], np.float32(scale), zp, *I8)
            sweep.append(dict(tag=tag, m=m, k=k, n=n, scale=scale, zp=zp, has_bias=has_bias,
                              expect=want.astype(np.int8).reshape(-1).tolist()))
    cases["requant_ties_and_saturation"] = dict(
        source="gemmkit/tests/epilogue/requant.rs:275-320", seed=0x7135, cases=sweep)

    # requant_degenerate_k0 (requant.rs:548-577)
    m, n = 12, 10
    bias = [i * 40 - 200 for i in range(m)]
    want = [[requant(0, bias[i], 0.5, 7, *I8) for _ in range(n)] for i in range(m)]
    cases["requant_degenerate_k0"] = dict(
        source="gemmkit/tests/epilogue/requant.rs:548-577", m=m, n=n, bias=bias, scale=0.5, zp=7,
        expect=want)

    # requant_vector_ties (requant.rs:440-480)
    a = [i - 18 for i in range(37)]
    cases["requant_vector_ties"] = dict(
        source="gemmkit/tests/epilogue/requant.rs:440-480", a=a, scale=0.5, zp=3,
        expect=[requant(v, 0, 0.5, 3, *I8) for v in a])

    # requant_vector_extreme_acc (requant.rs:486-545)
    m, k, n = 37, 1, 7
    a = np.array([-128 if i % 2 == 0 else 127 for i in range(m)], np.int8).reshape(m, 1)
    b = np.array([127 if j % 2 == 0 else -128 for j in range(n)], np.int8).reshape(1, n)
    ext = [2**31 - 1, -2**31, 2**31 - 1 - 200, -2**31 + 200]
    bias = np.array([ext[i % 4] for i in range(m)], np.int64)
    acc = acc_exact(a, b)
    runs = []
    for scale in [1.0, 1e-9, 0.5, 1e30]:
        for zp in [0, -128, 127]:
            want = requant_array(acc, bias[:, None], np.float32(scale), zp, *I8)
            runs.append(dict(scale=scale, zp=zp, expect=want.astype(np.int8).reshape(-1).tolist()))
    cases["requant_vector_extreme_acc"] = dict(
        source="gemmkit/tests/epilogue/requant.rs:486-545", m=m, k=k, n=n,
        a=a.reshape(-1).tolist(), b=b.reshape(-1).tolist(), bias=bias.tolist(), runs=runs)

    # requant_store lane sweep (gemmkit/src/simd.rs:743-853): adversarial i32 + 96 LCG values.
    vals = [-2**31, -2**31 + 1, -1, 0, 1, 1 << 30, 2**31 - 2, 2**31 - 1]
    lcg = 0x123456789ABCDEF0
    for _ in range(96):
        lcg = (lcg * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1)
        vals.append(wrap_i32(lcg >> 32))
    grid = []
    for scale in [1.0, 0.1, 1e30, 1e-30, 0.0078125]:
        for zp in [0, -128, 127]:
            for lo, hi in [I8, U8]:
                grid.append(dict(scale=scale, scale_f32=f32(scale), zp=zp, lo=lo, hi=hi,
                                 expect=[requant(v, 0, scale, zp, lo, hi) & 0xFF for v in vals]))
    cases["requant_store_sweep"] = dict(
        source="gemmkit/src/simd.rs:743-853", note="scales rounded to f32 (the C ABI's type)",
        vals=vals, grid=grid)

    # correctness_i8 (gemmkit/tests/correctness/int8.rs:11-66): exact i32 GEMM digests.
    shapes = [(1, 1, 1), (3, 4, 5), (16, 8, 7), (32, 32, 32), (33, 17, 19), (40, 33, 28),
              (64, 80, 48), (65, 64, 64), (128, 96, 112)]
    rows = []
    for (m, k, n) in shapes:
        for alpha, beta in [(1, 0), (1, 1), (3, -2), (0, 3)]:
            a = rand_i8(m * k, 0x100 + (m * 7 + k)).reshape(m, k)
            b = rand_i8(k * n, 0x200 + (n * 3 + k)).reshape(k, n)
            c0 = np.array([(x % 7) - 3 for x in range(m * n)], np.int64).reshape(m, n)
            v = beta * c0 + alpha * (a.astype(np.int64) @ b.astype(np.int64))
            assert np.all(np.abs(v) < 2**31)
            rows.append(dict(m=m, k=k, n=n, alpha=alpha, beta=beta,
                             sha256=digest(v.astype(np.int32))))
    cases["correctness_i8"] = dict(source="gemmkit/tests/correctness/int8.rs:11-66",
                                   layout="row-major A, col-major B, row-major C", cases=rows)

    # i8_packed_common::check (gemmkit/tests/i8_packed_common/mod.rs:29-90).
    shapes = [(200, 130, 175), (65, 64, 64), (64, 65, 100), (33, 17, 19), (256, 257, 129),
              (8, 1024, 96), (2, 1023, 12)]
    rows = []
    for (m, k, n) in shapes:
        a_cm = rand_i8(m * k, 0x51 + (m * 7 + n))  # col-major m x k
        b_rm = rand_i8(k * n, 0x62 + (n * 3 + k))  # row-major k x n
        a = a_cm.reshape(k, m).T
        b = b_rm.reshape(k, n)
        c0 = np.array([(x % 7) - 3 for x in range(m * n)], np.int64).reshape(n, m).T  # col-major
        for alpha, beta in [(1, 0), (2, 3), (0, 5)]:
            v = beta * c0 + alpha * (a.astype(np.int64) @ b.astype(np.int64))
            v = (v + 2**31) % 2**32 - 2**31
            rows.append(dict(m=m, k=k, n=n, alpha=alpha, beta=beta,
                             sha256_rowmajor=digest(v.astype(np.int32))))
    cases["i8_packed_common"] = dict(source="gemmkit/tests/i8_packed_common/mod.rs:29-90",
                                     cases=rows)
    return cases


def main() -> None:
    with open(os.path.join(HERE, "kat.json"), "w") as f:
        json.dump(kat_cases(), f, indent=1)
    with open(os.path.join(HERE, "model_cases.json"), "w") as f:
        json.dump(model_cases(), f, separators=(",", ":"))
    print("wrote kat.json, model_cases.json")


if __name__ == "__main__":
    main()
