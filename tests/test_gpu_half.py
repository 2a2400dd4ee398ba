"""GPU accuracy of the bf16 / f16 -> f32 path through the C ABI: within 1e-2 relative of an
f64 reference dot (the stated tolerance), and the reference tests' own relative Frobenius
gate 8*k*eps (gemmkit/tests/oracle_common/mod.rs:185-219)."""
import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gpu_util import dev, empty, gather, host, knobs

pytestmark = pytest.mark.gpu

# Per element: |got - ref| <= 1e-2 * (|alpha| * sum_p |a_ip||b_pj| + |beta * c_ij|), i.e. relative
# to the magnitude of the terms of the f64 dot rather than to |ref| itself, which would be
# undefined where the terms cancel to (nearly) zero. The reference tests' own relative
# Frobenius gate (8 * k * eps) is checked on top.
REL_TOL = 1e-2
EPS = {False: 2.0 ** -8, True: 2.0 ** -11}  # bf16 / f16 unit roundoff


@pytest.fixture(autouse=True)
def _reset_tile():
    gk.set_tile_n(0)
    yield
    gk.set_tile_n(0)
    assert gk.device_status(0) == 0


def f16_bits(x):
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def widen(bits, is_f16):
    return (bits.view(np.float16).astype(np.float64) if is_f16
            else O.bf16_to_f32(bits).astype(np.float64))


def make(rng, shape, is_f16):
    x = rng.standard_normal(shape).astype(np.float32)
    return f16_bits(x) if is_f16 else O.f32_to_bf16(x)


def check(got, a, b, alpha, beta, c0, is_f16, rows=None):
    rows = np.arange(a.shape[0]) if rows is None else rows
    ref = O.gemm_half_f64(a[rows], b, alpha, beta, None if c0 is None else c0[rows], is_f16)
    mag = abs(alpha) * (np.abs(widen(a[rows], is_f16)) @ np.abs(widen(b, is_f16)))
    if c0 is not None:
        mag += abs(beta) * np.abs(c0[rows].astype(np.float64))
    err = np.abs(got[rows].astype(np.float64) - ref)
    assert np.all(err <= REL_TOL * mag + 1e-30), float((err / (mag + 1e-30)).max())
    k = a.shape[1]
    fro = np.linalg.norm(got[rows] - ref) / max(np.linalg.norm(ref), 1e-30)
    assert fro <= 8 * k * EPS[is_f16], fro


@pytest.mark.parametrize("is_f16", [False, True])
@pytest.mark.parametrize("shape", [(128, 64, 256), (200, 333, 129), (1, 4096, 999), (517, 8, 61),
                                   (64, 1000, 16)])
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (1.0, 0.5), (-2.0, 1.0)])
def test_half_f32_shapes(is_f16, shape, alpha, beta):
    m, k, n = shape
    rng = np.random.default_rng(m * 31 + k * 7 + n)
    a = make(rng, (m, k), is_f16)
    b = make(rng, (k, n), is_f16)
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    da, db = dev(a.view(np.int16)), dev(b.view(np.int16))
    dc = dev(c0)
    gk.gemm_half_f32(alpha, gk.MatRef.from_row_major(da, m, k), gk.MatRef.from_row_major(db, k, n),
                     beta, gk.MatMut.from_row_major(dc, m, n), is_f16=is_f16)
    check(host(dc).reshape(m, n), a, b, alpha, beta, c0 if beta else None, is_f16)


@pytest.mark.parametrize("layout", ["rc", "cr", "cc"])
def test_half_layouts(layout):
    rng = np.random.default_rng(5)
    m, k, n = 150, 270, 190
    a = make(rng, (m, k), False)
    b = make(rng, (k, n), False)
    abuf = a.reshape(-1) if layout[0] == "r" else np.ascontiguousarray(a.T).reshape(-1)
    rsa, csa = (k, 1) if layout[0] == "r" else (1, m)
    bbuf = b.reshape(-1) if layout[1] == "r" else np.ascontiguousarray(b.T).reshape(-1)
    rsb, csb = (n, 1) if layout[1] == "r" else (1, k)
    dc = empty(m * n, np.float32)
    gk.gemm_half_f32(1.0, gk.MatRef.new(dev(abuf.view(np.int16)), m, k, rsa, csa),
                     gk.MatRef.new(dev(bbuf.view(np.int16)), k, n, rsb, csb), 0.0,
                     gk.MatMut.from_col_major(dc, m, n))
    got = gather(host(dc), m, n, 1, m)
    check(got, a, b, 1.0, 0.0, None, False)


def test_c3_config_full_size_sampled():
    """8192^3 bf16 N(0,1), C f32 N(0,1), alpha 1, beta 0.5. 256 rows (the
    first, the last and 254 spread over the matrix) against an f64 reference of the same
    bf16-widened inputs; at this size the reference uses numpy's f64 matrix product, which
    differs from a sequential f64 dot only by f64 rounding (~1e-13 relative), far inside the
    1e-2 tolerance. The whole output is checked for finiteness."""
    rng = np.random.default_rng(3)
    m = n = k = 8192
    a = O.f32_to_bf16(rng.standard_normal((m, k), dtype=np.float32))
    b = O.f32_to_bf16(rng.standard_normal((k, n), dtype=np.float32))
    c0 = rng.standard_normal((m, n), dtype=np.float32)
    da, db, dc = dev(a.view(np.int16)), dev(b.view(np.int16)), dev(c0)
    gk.gemm_half_f32(1.0, gk.MatRef.from_row_major(da, m, k), gk.MatRef.from_row_major(db, k, n),
                     0.5, gk.MatMut.from_row_major(dc, m, n))
    got = host(dc).reshape(m, n)
    assert np.isfinite(got).all()
    rows = np.unique(np.concatenate([[0, m - 1], rng.choice(m, 254, replace=False)]))
    wa, wb = widen(a[rows], False), widen(b, False)
    ref = wa @ wb + 0.5 * c0[rows].astype(np.float64)
    mag = np.abs(wa) @ np.abs(wb) + 0.5 * np.abs(c0[rows].astype(np.float64))
    err = np.abs(got[rows].astype(np.float64) - ref)
    assert np.all(err <= REL_TOL * mag), float((err / mag).max())
    fro = np.linalg.norm(got[rows] - ref) / np.linalg.norm(ref)
    assert fro <= 8 * k * EPS[False], fro
    # and the scalar f64 restatement on two of those rows
    check(got, a, b, 1.0, 0.5, c0, False, rows=rows[:2])


def test_half_batched():
    rng = np.random.default_rng(8)
    batch, m, k, n = 5, 96, 200, 144
    a = make(rng, (batch, m, k), False)
    b = make(rng, (batch, k, n), False)
    da, db = dev(a.view(np.int16)), dev(b.view(np.int16))
    dc = empty(batch * m * n, np.float32)
    gk.gemm_half_f32_batched(False, batch, m, k, n, 1.0, da.data_ptr(), k, 1, m * k, db.data_ptr(),
                             n, 1, k * n, 0.0, dc.data_ptr(), n, 1, m * n)
    got = host(dc).reshape(batch, m, n)
    for e in range(batch):
        check(got[e], a[e], b[e], 1.0, 0.0, None, False)


def test_half_degenerate():
    dc = dev(np.arange(6, dtype=np.float32))
    gk.gemm_bf16_f32_unchecked(2, 0, 3, 1.0, 0, 0, 1, 0, 3, 1, 2.0, dc.data_ptr(), 3, 1)
    assert host(dc).tolist() == [0.0, 2.0, 4.0, 6.0, 8.0, 10.0]


@pytest.mark.parametrize("shape", [(1000, 1000, 1000), (3000, 640, 700)])
def test_half_stream_k_beta(shape):
    """bf16 shapes with a stream-K tail: f32 partials summed in slot order, beta once."""
    m, k, n = shape
    rng = np.random.default_rng(m + n)
    a = make(rng, (m, k), False)
    b = make(rng, (k, n), False)
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    da, db = dev(a.view(np.int16)), dev(np.ascontiguousarray(b.T).view(np.int16))
    outs = []
    with knobs(GEMMKIT_CUDA_STREAMK=1, GEMMKIT_CUDA_PAIR=0):
        for _ in range(2):
            dc = dev(c0)
            gk.gemm_half_f32(1.5, gk.MatRef.from_row_major(da, m, k),
                             gk.MatRef.new(db, k, n, 1, k), 0.5,
                             gk.MatMut.from_row_major(dc, m, n))
            outs.append(host(dc).reshape(m, n))
    assert np.array_equal(outs[0], outs[1])  # deterministic reduction order
    rows = np.arange(0, m, 37)
    check(outs[0], a, b, 1.5, 0.5, c0, False, rows=rows)


@pytest.mark.parametrize("is_f16", [False, True])
def test_half_pair_odd_shape(is_f16):
    m, k, n = 2341, 300, 2315
    rng = np.random.default_rng(31 + is_f16)
    a = make(rng, (m, k), is_f16)
    b = make(rng, (k, n), is_f16)
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    da, db = dev(a.view(np.int16)), dev(np.ascontiguousarray(b.T).view(np.int16))
    dc = dev(c0)
    gk.gemm_half_f32(1.0, gk.MatRef.from_row_major(da, m, k), gk.MatRef.new(db, k, n, 1, k), -0.5,
                     gk.MatMut.from_row_major(dc, m, n), is_f16=is_f16)
    rows = np.concatenate([np.arange(0, m, 97), [m - 1]])
    check(host(dc).reshape(m, n), a, b, 1.0, -0.5, c0, is_f16, rows=rows)
