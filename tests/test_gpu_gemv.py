"""GPU parity of the small-M streaming kernel (output side <= 64: MMA N of 16, 32 or 64, K cut
between all SMs and summed by the last CTA to arrive): bit-exact against the CPU oracle for i8,
within the stated tolerance for bf16 / f16, and deterministic from call to call."""
import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gpu_util import dev, empty, gather, host, rand_i8

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status():
    gk.set_tile_n(0)
    yield
    assert gk.device_status(0) == 0, "a bounded device wait gave up"


def ptr(t):
    return t.data_ptr()


# (small side, K, large side): widths that select each MMA N and its edges, K tails, large sides
# that are and are not multiples of 128, and a single tile with a long K (many CTAs per tile).
SHAPES = [(1, 4096, 14336), (5, 1000, 3000), (16, 129, 2000), (17, 4096, 1536), (31, 300, 777),
          (32, 8192, 1024), (33, 2048, 640), (63, 555, 1300), (64, 4096, 4096), (3, 65536, 100),
          (16, 1, 300), (2, 200000, 128)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("small_m", [True, False])
def test_gemv_i32_alpha_beta(shape, small_m):
    """i32 out with alpha / beta; the small side is m (A's rows) or n (B's columns)."""
    s, k, big = shape
    m, n = (s, big) if small_m else (big, s)
    rng = np.random.default_rng(s * 7 + k + big + small_m)
    a = rand_i8(rng, (m, k))
    bT = rand_i8(rng, (n, k))
    c0 = rng.integers(-5000, 5000, (m, n)).astype(np.int32)
    want = O.gemm_i8_matrix(3, a, bT.T, -2, c0)
    da, db = dev(a), dev(bT)
    for _ in range(2):  # the second call runs on a fresh counter epoch
        dc = dev(c0)
        gk.gemm_i8(3, gk.MatRef.from_row_major(da, m, k), gk.MatRef.new(db, k, n, 1, k), -2,
                   gk.MatMut.from_row_major(dc, m, n))
        assert np.array_equal(host(dc).reshape(m, n), want)


AXES = [("none", "col"), ("col", "row"), ("row", "col"), ("row", "row"), ("col", "none")]


@pytest.mark.parametrize("axes", AXES, ids=lambda a: f"b{a[0]}-s{a[1]}")
@pytest.mark.parametrize("out_u8", [False, True])
@pytest.mark.parametrize("M", [1, 7, 16, 40])
def test_gemv_prepacked_requant_axes(axes, out_u8, M):
    """Prepacked B with every bias / scale axis (per-row scales run along the MMA N side here)."""
    k, n = 3000, 2500
    rng = np.random.default_rng(M * 31 + out_u8 + len(axes[0]) * 3 + len(axes[1]))
    a = rand_i8(rng, (M, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)
    bias_axis, scale_axis = axes
    nb = {"row": M, "col": n}.get(bias_axis, 0)
    ns = {"row": M, "col": n}.get(scale_axis, 0)
    bias = rng.integers(-2**15, 2**15 + 1, max(nb, 1)).astype(np.int32)
    scales = rng.uniform(1e-4, 1e-3, max(ns, 1)).astype(np.float32)
    zp = 120 if out_u8 else -3
    want = O.requant_matrix(a, bT.T, scales=scales if ns else None,
                            scale_axis=scale_axis if ns else "none",
                            scale=0.0007, bias=bias if nb else None,
                            bias_axis=bias_axis if nb else "none", zp=zp, out_u8=out_u8,
                            relu=True)
    da, dbT = dev(a), dev(bT)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dbT, k, n, 1, k))
    if ns:
        dsc = dev(scales)
        sc = gk.RequantScale.PerRow(dsc) if scale_axis == "row" else gk.RequantScale.PerCol(dsc)
    else:
        sc = gk.RequantScale.PerTensor(0.0007)
    if nb:
        dbias = dev(bias)
        req = gk.Requantize(sc, zp, dbias, gk.AXIS_ROW if bias_axis == "row" else gk.AXIS_COL,
                            True)
    else:
        req = gk.Requantize(sc, zp, None, gk.AXIS_NONE, True)
    dc = empty(M * n, np.uint8 if out_u8 else np.int8)
    gk.gemm_i8_packed_b_requant(M, ptr(da), k, 1, packed, req, ptr(dc), n, 1, out_u8=out_u8)
    assert np.array_equal(host(dc).reshape(M, n), want)


def test_gemv_column_major_out():
    """Small m into a column-major C (the output's unit stride runs along the small side)."""
    m, k, n = 12, 2048, 3000
    rng = np.random.default_rng(5)
    a = rand_i8(rng, (m, k))
    bT = rand_i8(rng, (n, k))
    want = O.gemm_i8_matrix(1, a, bT.T, 0, None)
    dc = empty(m * n, np.int32)
    gk.gemm_i8(1, gk.MatRef.from_row_major(dev(a), m, k), gk.MatRef.new(dev(bT), k, n, 1, k), 0,
               gk.MatMut.from_col_major(dc, m, n))
    assert np.array_equal(gather(host(dc), m, n, 1, m), want)


def _half_check(got, a, b, is_f16):
    ref = O.gemm_half_f64(a, b, 1.0, 0.0, None, is_f16)
    wa = a.view(np.float16).astype(np.float64) if is_f16 else O.bf16_to_f32(a).astype(np.float64)
    wb = b.view(np.float16).astype(np.float64) if is_f16 else O.bf16_to_f32(b).astype(np.float64)
    mag = np.abs(wa) @ np.abs(wb)
    err = np.abs(got.astype(np.float64) - ref)
    assert np.all(err <= 1e-2 * mag + 1e-30), float((err / (mag + 1e-30)).max())


@pytest.mark.parametrize("is_f16", [False, True])
@pytest.mark.parametrize("m", [1, 16, 40])
def test_gemv_half_deterministic(is_f16, m):
    """bf16 / f16 -> f32 small-M: within 1e-2 of the f64 dot, and the cut-K partial sums run in
    a fixed order, so two calls give the same bits."""
    k, n = 4096, 3000
    rng = np.random.default_rng(m + 100 * is_f16)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((k, n)).astype(np.float32)
    if is_f16:
        a, b = x.astype(np.float16).view(np.uint16), w.astype(np.float16).view(np.uint16)
    else:
        a, b = O.f32_to_bf16(x), O.f32_to_bf16(w)
    da = dev(a.view(np.int16))
    dbT = dev(np.ascontiguousarray(b.T).view(np.int16))
    outs = []
    for _ in range(2):
        dc = empty(m * n, np.float32)
        gk.gemm_half_f32(1.0, gk.MatRef.from_row_major(da, m, k), gk.MatRef.new(dbT, k, n, 1, k),
                         0.0, gk.MatMut.from_row_major(dc, m, n), is_f16=is_f16)
        outs.append(host(dc).reshape(m, n))
    assert np.array_equal(outs[0], outs[1])
    _half_check(outs[0], a, b, is_f16)


@pytest.mark.parametrize("shape", [(65, 64, 64), (300, 1000, 9), (1000, 4096, 33)],
                         ids=lambda s: "x".join(map(str, s)))
def test_prepacked_narrow_b(shape):
    """A prepacked B with <= 64 columns puts the packed buffer on the small (MMA N) side: those
    shapes stay with the general kernel, which reads the tiled layout there."""
    m, k, n = shape
    rng = np.random.default_rng(m + k + n)
    a = rand_i8(rng, (m, k))
    bT = rand_i8(rng, (n, k))
    c0 = rng.integers(-100, 100, (m, n)).astype(np.int32)
    want = O.gemm_i8_matrix(2, a, bT.T, 3, c0)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dev(bT), k, n, 1, k))
    dc = dev(np.ascontiguousarray(c0.T).reshape(-1))  # the packed entry wants a column-major C
    gk.gemm_i8_packed_b(2, gk.MatRef.from_row_major(dev(a), m, k), packed, 3,
                        gk.MatMut.from_col_major(dc, m, n))
    assert np.array_equal(gather(host(dc), m, n, 1, m), want)


@pytest.mark.parametrize("M", [1, 4, 16, 64])
@pytest.mark.parametrize("out_u8", [False, True])
def test_gemv_entry(M, out_u8):
    """gk_gemv_i8_requant_unchecked: bit-exact against the oracle and against the packed
    requant entry on the same inputs (both C orientations)."""
    k, n = 2048, 3000
    rng = np.random.default_rng(M * 3 + out_u8)
    a = rand_i8(rng, (M, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)
    scales = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
    bias = rng.integers(-3000, 3000, n).astype(np.int32)
    zp = 128 if out_u8 else -1
    want = O.requant_matrix(a, bT.T, scales=scales, scale_axis="col", bias=bias,
                            bias_axis="col", zp=zp, out_u8=out_u8)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dev(bT), k, n, 1, k))
    req = gk.Requantize(gk.RequantScale.PerCol(dev(scales)), zp, dev(bias), gk.AXIS_COL)
    da = dev(a)
    dt = np.uint8 if out_u8 else np.int8
    for rsc, csc in ((n, 1), (1, M)):
        dc = empty(M * n, dt)
        gk.gemv_i8_requant(M, ptr(da), k, 1, packed, req, ptr(dc), rsc, csc, out_u8=out_u8)
        got = gather(host(dc), M, n, rsc, csc)
        assert np.array_equal(got, want)
        dref = empty(M * n, dt)
        gk.gemm_i8_packed_b_requant(M, ptr(da), k, 1, packed, req, ptr(dref), rsc, csc,
                                    out_u8=out_u8)
        assert np.array_equal(host(dc), host(dref))


@pytest.mark.parametrize("m,n", [(64, 40), (17, 17), (33, 5)])
def test_gemv_entry_packed_side_not_wider(m, n):
    """gk_gemv_i8_requant_unchecked with n <= m <= 64 (both sides small; the general tile
    kernel takes it): bit-exact against the oracle in both C orientations."""
    k = 1000
    rng = np.random.default_rng(m * 100 + n)
    a = rand_i8(rng, (m, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)
    scales = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
    bias = rng.integers(-3000, 3000, n).astype(np.int32)
    want = O.requant_matrix(a, bT.T, scales=scales, scale_axis="col", bias=bias,
                            bias_axis="col", zp=2, relu=True)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dev(bT), k, n, 1, k))
    req = gk.Requantize(gk.RequantScale.PerCol(dev(scales)), 2, dev(bias), gk.AXIS_COL, True)
    da = dev(a)
    for rsc, csc in ((n, 1), (1, m)):
        dc = empty(m * n, np.int8)
        gk.gemv_i8_requant(m, ptr(da), k, 1, packed, req, ptr(dc), rsc, csc)
        assert np.array_equal(gather(host(dc), m, n, rsc, csc), want), (rsc, csc)
