"""GPU parity of the engine's alternative kernel paths: every knob setting the tuner may write
(tile width 192, the CTA-pair kernel off with the stream-K tail off, the small-M kernel off,
launch overlap off), and the 16-warp epilogue form of the CTA-pair kernel (quantized output,
K of one or two 128-byte blocks) on odd shapes in both output orientations. Bit-exact against
the CPU oracle."""
import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gpu_util import dev, empty, gather, host, knobs, rand_i8

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    gk.set_tile_n(0)
    yield
    gk.set_tile_n(0)
    assert gk.device_status(0) == 0, "a bounded device wait gave up"


def ptr(t):
    return t.data_ptr()


def vnni_requant(a, bT, out_u8=False, **req):
    """The oracle's VNNI restatement (bit-identical to the scalar one, tests/test_oracle.py),
    row-major a (m x k) times B = bT^T -> row-major m x n."""
    m, k = a.shape
    n = bT.shape[0]
    pb = O.VnniPacked(np.ascontiguousarray(bT).reshape(-1), 1, k, k, n)
    c = np.empty(m * n, np.uint8 if out_u8 else np.int8)
    O.vnni_requant_packed(O.View(np.ascontiguousarray(a).reshape(-1), m, k, k, 1), pb,
                          O.View(c, m, n, 1, m), out_u8=out_u8, **req)
    return c.reshape(n, m).T


KNOB_SETS = [
    dict(GEMMKIT_CUDA_GEMV_SK=1),
    dict(GEMMKIT_CUDA_PDL=0),
    dict(GEMMKIT_CUDA_PAIR=0, GEMMKIT_CUDA_STREAMK=0),
    dict(GEMMKIT_CUDA_GEMV=0),
    dict(GEMMKIT_CUDA_BN=192),
    dict(GEMMKIT_CUDA_BN=128, GEMMKIT_CUDA_PDL=0),
]


def _kid(d):
    return ",".join(f"{k.replace('GEMMKIT_CUDA_', '')}={v}" for k, v in d.items())


@pytest.mark.parametrize("kv", KNOB_SETS, ids=_kid)
def test_knob_paths_requant_and_i32(kv):
    """Under each knob setting: a large requant product (the pair kernel by default), a
    small-M prepacked product (the streaming kernel by default), an i32 product with beta, and
    three dependent calls issued back to back without a host synchronisation."""
    rng = np.random.default_rng(sum(map(ord, _kid(kv))))
    m, k, n = 1100, 300, 1300
    a = rand_i8(rng, (m, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)
    bias = rng.integers(-2**15, 2**15 + 1, n).astype(np.int32)
    scales = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
    want = vnni_requant(a, bT, scales=scales, scale_axis="col", bias=bias, bias_axis="col",
                        zp=3, relu=True)
    M = 5
    want_small = vnni_requant(a[:M], bT, scales=scales, scale_axis="col", zp=-2)
    c0 = rng.integers(-1000, 1000, (m, n)).astype(np.int32)
    want_i32 = O.gemm_i8_matrix(2, a, bT.T, -3, c0)
    da, dbT, dbias, dsc = dev(a), dev(bT), dev(bias), dev(scales)
    with knobs(**kv):
        packed = gk.prepack_rhs_i8(gk.MatRef.new(dbT, k, n, 1, k))
        req = gk.Requantize(gk.RequantScale.PerCol(dsc), 3, dbias, gk.AXIS_COL, True)
        outs = []
        for _ in range(3):  # chained on one stream, no host synchronisation in between
            dc = empty(m * n, np.int8)
            gk.gemm_i8_packed_b_requant(m, ptr(da), k, 1, packed, req, ptr(dc), 1, m)
            outs.append(dc)
        dsm = empty(M * n, np.int8)
        gk.gemm_i8_packed_b_requant(M, ptr(da), k, 1, packed, gk.Requantize(
            gk.RequantScale.PerCol(dsc), -2), ptr(dsm), n, 1)
        di = dev(c0)
        gk.gemm_i8(2, gk.MatRef.from_row_major(da, m, k), gk.MatRef.new(dbT, k, n, 1, k), -3,
                   gk.MatMut.from_row_major(di, m, n))
    for dc in outs:
        assert np.array_equal(host(dc).reshape(n, m).T, want)
    assert np.array_equal(host(dsm).reshape(M, n), want_small)
    assert np.array_equal(host(di).reshape(m, n), want_i32)


@pytest.mark.parametrize("kv", KNOB_SETS[1:4], ids=_kid)
def test_knob_paths_batched_requant(kv):
    rng = np.random.default_rng(11)
    batch, m, n, k = 24, 512, 512, 128
    a = rand_i8(rng, (batch, m, k))
    bT = rand_i8(rng, (batch, n, k))
    bias = rng.integers(-2**15, 2**15 + 1, (batch, m)).astype(np.int32)
    scales = rng.uniform(1e-4, 1e-3, (batch, n)).astype(np.float32)
    da, dbT, dsc, dbias = dev(a), dev(bT), dev(scales), dev(bias)  # held until the call ends
    req = gk.Requantize(gk.RequantScale.PerCol(dsc), 128, dbias, gk.AXIS_ROW)
    dc = empty(batch * m * n, np.uint8)
    with knobs(**kv):
        gk.gemm_i8_requant_batched(batch, m, k, n, ptr(da), k, 1, m * k, ptr(dbT), 1, k,
                                   n * k, req, m, n, ptr(dc), 1, m, m * n, out_u8=True)
    got = host(dc).reshape(batch, n, m)
    for e in range(batch):
        want = vnni_requant(a[e], bT[e], scales=scales[e], scale_axis="col", bias=bias[e],
                            bias_axis="row", zp=128, out_u8=True)
        assert np.array_equal(got[e].T, want), e


# ---- the 16-warp epilogue form of the CTA-pair kernel -----------------------------------------
# Chosen for quantized outputs when K is one or two 128-byte blocks and the tile is 256 wide;
# these shapes have >= 74 pair tiles, odd edges in M and N, and K not a multiple of 128.

EPI16_SHAPES = [(2341, 200, 2315), (2313, 77, 2339)]


@pytest.mark.parametrize("f32", [1, 0])
@pytest.mark.parametrize("out_u8", [False, True])
@pytest.mark.parametrize("axes", [("col", "col"), ("row", "col"), ("col", "row"), ("row", "row")])
@pytest.mark.parametrize("shape", EPI16_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_pair_epi16_requant(shape, axes, out_u8, f32):
    """With GEMMKIT_CUDA_REQUANT_F32=1 these items take the packed f32 requantize (|acc + bias|
    < 2^22, scales below 1); with 0 the f64 short and general paths."""
    m, k, n = shape
    scale_axis, bias_axis = axes
    rng = np.random.default_rng(m + k + 3 * out_u8 + 7 * len(scale_axis + bias_axis))
    a = rand_i8(rng, (m, k))
    bT = rand_i8(rng, (n, k))
    slen = m if scale_axis == "row" else n
    blen = m if bias_axis == "row" else n
    # scales on both sides of 2^-9, so both requantize paths of the epilogue run
    scales = rng.uniform(1e-4, 6e-3, slen).astype(np.float32)
    bias = rng.integers(-2**15, 2**15 + 1, blen).astype(np.int32)
    zp = (128 if out_u8 else -5) + (rng.integers(0, 2) if scale_axis == "row" else 0)
    want = vnni_requant(a, bT, scales=scales, scale_axis=scale_axis, bias=bias,
                        bias_axis=bias_axis, zp=int(zp), out_u8=out_u8, relu=True)
    da, dbT, dsc, dbias = dev(a), dev(bT), dev(scales), dev(bias)
    sc = gk.RequantScale(0.0, dsc, gk.AXIS_ROW if scale_axis == "row" else gk.AXIS_COL)
    req = gk.Requantize(sc, int(zp), dbias,
                        gk.AXIS_ROW if bias_axis == "row" else gk.AXIS_COL, True)
    for c_row in (True, False):
        dc = empty(m * n, np.uint8 if out_u8 else np.int8)
        rsc, csc = (n, 1) if c_row else (1, m)
        with knobs(GEMMKIT_CUDA_REQUANT_F32=f32):
            gk.gemm_i8_requant_ex_unchecked(m, k, n, ptr(da), k, 1, ptr(dbT), 1, k, req, ptr(dc),
                                            rsc, csc, out_u8=out_u8)
        got = gather(host(dc), m, n, rsc, csc)
        assert np.array_equal(got, want), (c_row, axes)


def _epi16_call(a, bT, req, out_u8):
    """Row-major C, so a per-row scale stays on the kernel's rows (the 16-warp form's case)."""
    m, k = a.shape
    n = bT.shape[0]
    da, dbT = dev(a), dev(bT)
    dc = empty(m * n, np.uint8 if out_u8 else np.int8)
    gk.gemm_i8_requant_ex_unchecked(m, k, n, ptr(da), k, 1, ptr(dbT), 1, k, req, ptr(dc), n, 1,
                                    out_u8=out_u8)
    return host(dc).reshape(m, n)


@pytest.mark.parametrize("edge", ["at_bound", "past_bound"])
def test_pair_epi16_f32_range_bound(edge):
    """The packed f32 requantize needs |acc + bias| < 2^22: A = B = -128 everywhere makes every
    accumulator K * 2^14, and biases of magnitude 2^22 - K * 2^14 - 1 (the f32 path) or
    2^22 - K * 2^14 (the item falls back to the f64 path). Scales near 3e-5 put the results
    across the band; odd zero points; rows with a scale of 1.5 (fallback) in a third call."""
    m, k, n = 2304, 128, 2304
    a = np.full((m, k), -128, np.int8)
    bT = np.full((n, k), -128, np.int8)
    top = (1 << 22) - k * 16384 - (1 if edge == "at_bound" else 0)
    rng = np.random.default_rng(4 + len(edge))
    bias = np.where(rng.random(n) < 0.5, top, -top).astype(np.int32)
    bias[::7] = rng.integers(-1000, 1000, len(bias[::7]))
    dbias = dev(bias)
    for scales, zp, out_u8 in ((rng.uniform(2.5e-5, 3e-5, m), -7, False),
                               (rng.uniform(2.5e-5, 3e-5, m), 129, True),
                               (np.where(rng.random(m) < 0.1, 1.5, 2.9e-5), 3, False)):
        scales = scales.astype(np.float32)
        dsc = dev(scales)
        want = vnni_requant(a, bT, scales=scales, scale_axis="row", bias=bias, bias_axis="col",
                            zp=zp, out_u8=out_u8)
        req = gk.Requantize(gk.RequantScale.PerRow(dsc), zp, dbias, gk.AXIS_COL)
        for f32 in (1, 0):
            with knobs(GEMMKIT_CUDA_REQUANT_F32=f32):
                got = _epi16_call(a, bT, req, out_u8)
            assert np.array_equal(got, want), (edge, zp, f32)


@pytest.mark.parametrize("shape", [(2304, 200, 2304), (1100, 700, 1300), (300, 300, 300),
                                   (8, 4096, 2048)], ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("zp", [-(1 << 30), (1 << 30), (1 << 30) + 1, -2**31, 2**31 - 1])
def test_zero_point_limits(zp, shape):
    """Zero points at and past +-2^30 (the engine clamps zp there; the reference adds it in 64
    bits with saturation), per-tensor scale on both sides of 2^-9, a per-row bias, ReLU, on the
    16-warp form, the 8-warp pair kernel, the tile kernel and the small-M kernel."""
    rng = np.random.default_rng(zp & 0xFFFF)
    m, k, n = shape
    a = rand_i8(rng, (m, k))
    bT = rand_i8(rng, (n, k))
    bias = rng.integers(-2**15, 2**15 + 1, m).astype(np.int32)
    dbias = dev(bias)
    for scale in (3e-4, 0.9, 5e-3):
        want = vnni_requant(a, bT, scale=scale, bias=bias, bias_axis="row", zp=zp, relu=True)
        req = gk.Requantize(gk.RequantScale.PerTensor(scale), zp, dbias, gk.AXIS_ROW, True)
        assert np.array_equal(_epi16_call(a, bT, req, False), want), scale


@pytest.mark.parametrize("sk", [0, 1])
def test_small_m_config5_both_modes(sk):
    """BASELINE config 5 (M = 1, 4, 16 over a 4096 x 14336 prepacked B) with the small-M
    kernel's weight stream in whole tiles and in the even stream-K split, three calls in a row
    (the partial counters' epochs), bit-exact against the oracle."""
    rng = np.random.default_rng(55 + sk)
    k, n = 4096, 14336
    bT = rand_i8(rng, (n, k), -127, 127)
    scales = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
    bias = rng.integers(-2**15, 2**15 + 1, n).astype(np.int32)
    dbT, dsc, dbias = dev(bT), dev(scales), dev(bias)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dbT, k, n, 1, k))
    req = gk.Requantize(gk.RequantScale.PerCol(dsc), -3, dbias, gk.AXIS_COL, True)
    with knobs(GEMMKIT_CUDA_GEMV_SK=sk):
        for M in (1, 4, 16):
            a = rand_i8(rng, (M, k), -127, 127)
            want = vnni_requant(a, bT, scales=scales, scale_axis="col", bias=bias,
                                bias_axis="col", zp=-3, relu=True)
            da = dev(a)
            for _ in range(3):
                dc = empty(M * n, np.int8)
                gk.gemm_i8_packed_b_requant(M, ptr(da), k, 1, packed, req, ptr(dc), n, 1)
                assert np.array_equal(host(dc).reshape(M, n), want), (M, sk)
