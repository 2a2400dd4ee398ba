"""GPU parity of the MN-major right-hand side: a row-major (N-contiguous) i8 B is read by the
tile kernel's TMA as 128 K-rows x BN bytes boxes and fed to tcgen05.mma with the B-transpose
bit, with no transpose pack. Covers gemmkit's row-major A x row-major B call (
1024^3 -> i32), K and N tails, padded leading dimensions, each tile width the path takes
(32, 64, 128, and 192 / 256 capped to 128), requantized outputs, and the same calls with the
path switched off (GEMMKIT_CUDA_MN_B=0: the pack kernel first). Bit-exact against the oracle."""
import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gpu_util import dev, empty, host, knobs, rand_i8

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    gk.set_tile_n(0)
    yield
    gk.set_tile_n(0)
    assert gk.device_status(0) == 0, "a bounded device wait gave up"


def i32_call(a, b, ldb, alpha=1, beta=0, c0=None):
    """C = alpha*A*B + beta*C, A row-major m x k, B row-major k x n at leading dimension ldb."""
    m, k = a.shape
    n = b.shape[1]
    bbuf = np.zeros((k, ldb), np.int8)
    bbuf[:, :n] = b
    da, db = dev(a), dev(bbuf)
    dc = dev(c0) if c0 is not None else empty(m * n, np.int32)
    gk.gemm_i8_unchecked(m, k, n, alpha, da.data_ptr(), k, 1, db.data_ptr(), ldb, 1, beta,
                         dc.data_ptr(), n, 1)
    return host(dc).reshape(m, n)


def test_config1_row_major_b():
    """M = N = K = 1024, row-major A and B, alpha 1, beta 0, i32 out."""
    rng = np.random.default_rng(1)
    a = rand_i8(rng, (1024, 1024))
    b = rand_i8(rng, (1024, 1024))
    want = O.gemm_i8_matrix(1, a, b, 0, None)
    for mn in (1, 0):
        with knobs(GEMMKIT_CUDA_MN_B=mn):
            for _ in range(2):
                assert np.array_equal(i32_call(a, b, 1024), want), mn


# (m, k, n, ldb): K tails (not a multiple of 128), N tails (not a multiple of the tile width),
# padded ldb, K below one block, N just above the small-M bound
SHAPES = [(193, 77, 304, 304), (517, 333, 400, 416), (1000, 1000, 1008, 1024),
          (130, 1500, 80, 96), (2048, 640, 2048, 2048), (300, 5, 144, 160)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_row_major_b_i32(shape):
    m, k, n, ldb = shape
    rng = np.random.default_rng(m + k + n)
    a = rand_i8(rng, (m, k))
    b = rand_i8(rng, (k, n))
    c0 = rng.integers(-2**20, 2**20, (m, n)).astype(np.int32)
    want = O.gemm_i8_matrix(3, a, b, -2, c0)
    for bn in (0, 32, 64, 128, 192, 256):
        gk.set_tile_n(bn)
        assert np.array_equal(i32_call(a, b, ldb, 3, -2, c0.copy()), want), bn


@pytest.mark.parametrize("axes", [("col", "col"), ("row", "row")])
def test_row_major_b_requant(axes):
    """Requantized outputs (u8 and i8, both scale paths) over a row-major B."""
    scale_axis, bias_axis = axes
    rng = np.random.default_rng(len(scale_axis) + 7)
    m, k, n = 777, 300, 912
    a = rand_i8(rng, (m, k))
    b = rand_i8(rng, (k, n))
    slen = m if scale_axis == "row" else n
    blen = m if bias_axis == "row" else n
    scales = rng.uniform(1e-4, 6e-3, slen).astype(np.float32)
    bias = rng.integers(-2**15, 2**15 + 1, blen).astype(np.int32)
    da, db, dsc, dbias = dev(a), dev(b), dev(scales), dev(bias)
    ax = {"row": gk.AXIS_ROW, "col": gk.AXIS_COL}
    for out_u8, zp in ((False, -3), (True, 128)):
        want = O.requant_matrix(a, b, scales=scales, scale_axis=scale_axis, bias=bias,
                                bias_axis=bias_axis, zp=zp, relu=True, out_u8=out_u8)
        req = gk.Requantize(gk.RequantScale(0.0, dsc, ax[scale_axis]), zp, dbias, ax[bias_axis],
                            True)
        for mn in (1, 0):
            dc = empty(m * n, np.uint8 if out_u8 else np.int8)
            with knobs(GEMMKIT_CUDA_MN_B=mn):
                gk.gemm_i8_requant_ex_unchecked(m, k, n, da.data_ptr(), k, 1, db.data_ptr(), n, 1,
                                                req, dc.data_ptr(), n, 1, out_u8=out_u8)
            assert np.array_equal(host(dc).reshape(m, n), want), (out_u8, mn)


def test_row_major_b_stream_k_and_no_pdl():
    """The stream-K tail (partials over K blocks) and launch without overlap, on the MN path."""
    rng = np.random.default_rng(99)
    m, k, n = 1000, 2000, 1040
    a = rand_i8(rng, (m, k))
    b = rand_i8(rng, (k, n))
    want = O.gemm_i8_matrix(1, a, b, 0, None)
    for kv in (dict(GEMMKIT_CUDA_STREAMK=1), dict(GEMMKIT_CUDA_PDL=0)):
        with knobs(**kv):
            assert np.array_equal(i32_call(a, b, n), want), kv
