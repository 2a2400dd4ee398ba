"""GPU parity of the fused i32 epilogue (gk_gemm_i8_fused[_unchecked]): C = act(alpha*A*B +
beta*C + bias) in wrapping i32 arithmetic, bias per row or per column, ReLU or none. Bit-exact
against the oracle (gko_gemm_i8 followed by the bias-then-activation composition) on every
kernel the engine routes an i32 product to: the one-CTA tile kernel, the CTA-pair kernel, the
small-M streaming kernel, the stream-K tail, the pack path and the degenerate fill."""
import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gemmkit_b200 import _lib
from gpu_util import dev, gather, host, knobs, rand_i8

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert gk.device_status(0) == 0, "a bounded device wait gave up"


def run(m, k, n, alpha, beta, a, b, c0, bias, bias_axis, relu, c_row=True, b_col=False):
    """One checked-tier call; returns the row-major result."""
    b_buf = np.ascontiguousarray(b.T).reshape(-1) if b_col else b.reshape(-1)
    da, db = dev(a), dev(b_buf)
    c_buf = c0.reshape(-1) if c_row else np.ascontiguousarray(c0.T).reshape(-1)
    dc = dev(c_buf)
    dbias = dev(bias) if bias is not None else None
    bmat = gk.MatRef.new(db, k, n, 1, k) if b_col else gk.MatRef.from_row_major(db, k, n)
    cmat = gk.MatMut.from_row_major(dc, m, n) if c_row else gk.MatMut.from_col_major(dc, m, n)
    gk.gemm_i8_fused(alpha, gk.MatRef.from_row_major(da, m, k), bmat, beta, cmat, bias=dbias,
                     bias_dim=gk.AXIS_ROW if bias_axis == "row" else gk.AXIS_COL,
                     act=gk.Activation.Relu() if relu else None)
    rsc, csc = (n, 1) if c_row else (1, m)
    return gather(host(dc), m, n, rsc, csc)


def inputs(seed, m, k, n, bias_axis):
    rng = np.random.default_rng(seed)
    a = rand_i8(rng, (m, k))
    b = rand_i8(rng, (k, n))
    c0 = rng.integers(-2**20, 2**20, (m, n)).astype(np.int32)
    blen = m if bias_axis == "row" else n
    bias = rng.integers(-2**31, 2**31, blen, dtype=np.int64).astype(np.int32)  # wraps the sum
    return a, b, c0, bias


# tile kernel (various widths), pair kernel (>= 74 pair tiles), small-M (m or n <= 64)
SHAPES = [(193, 77, 301), (2341, 300, 2315), (16, 1000, 3000), (1500, 640, 40)]


@pytest.mark.parametrize("relu", [False, True])
@pytest.mark.parametrize("bias_axis", ["row", "col", None])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_fused_i32_shapes(shape, bias_axis, relu):
    m, k, n = shape
    a, b, c0, bias = inputs(m + k + n, m, k, n, bias_axis or "row")
    if bias_axis is None:
        bias = None
    for alpha, beta in ((1, 0), (100003, -7)):  # the second wraps alpha*acc
        want = O.gemm_i8_fused_matrix(alpha, a, b, beta, c0, bias, bias_axis or "row", relu)
        for c_row in (True, False):
            got = run(m, k, n, alpha, beta, a, b, c0, bias, bias_axis, relu, c_row=c_row,
                      b_col=not c_row)
            assert np.array_equal(got, want), (alpha, beta, c_row)


@pytest.mark.parametrize("bias_axis", ["row", "col"])
def test_fused_i32_stream_k_tail(bias_axis):
    """A shape whose last wave is cut into stream-K partials: the bias and ReLU are applied
    once, by the CTA that sums the partials."""
    m, k, n = 1000, 1000, 1000
    a, b, c0, bias = inputs(5, m, k, n, bias_axis)
    want = O.gemm_i8_fused_matrix(3, a, b, -2, c0, bias, bias_axis, True)
    with knobs(GEMMKIT_CUDA_STREAMK=1, GEMMKIT_CUDA_PAIR=0):
        for _ in range(2):
            got = run(m, k, n, 3, -2, a, b, c0, bias, bias_axis, True, b_col=True)
            assert np.array_equal(got, want)


def test_fused_i32_strided_pack_path():
    """Operands that are not K-contiguous go through the pack kernel first."""
    rng = np.random.default_rng(12)
    m, k, n = 37, 45, 29
    a = rand_i8(rng, (m, k))
    b = rand_i8(rng, (k, n))
    c0 = rng.integers(-100, 100, (m, n)).astype(np.int32)
    bias = rng.integers(-5000, 5000, n).astype(np.int32)
    want = O.gemm_i8_fused_matrix(2, a, b, 1, c0, bias, "col", True)
    abuf = np.zeros(3 * m * k, np.int8)
    abuf[[i * 3 * k + j * 3 for i in range(m) for j in range(k)]] = a.reshape(-1)
    da, db, dc, dbias = dev(abuf), dev(b), dev(c0), dev(bias)
    gk.gemm_i8_fused_unchecked(m, k, n, 2, da.data_ptr(), 3 * k, 3, db.data_ptr(), n, 1, 1,
                               dc.data_ptr(), n, 1, bias=dbias.data_ptr(), bias_dim=gk.AXIS_COL,
                               act=_lib.ACT_RELU)
    assert np.array_equal(host(dc).reshape(m, n), want)


@pytest.mark.parametrize("k,alpha", [(0, 5), (64, 0)])
def test_fused_i32_degenerate(k, alpha):
    """k == 0 or alpha == 0: C <- act(beta*C + bias)."""
    rng = np.random.default_rng(k + alpha)
    m, n = 70, 50
    c0 = rng.integers(-1000, 1000, (m, n)).astype(np.int32)
    bias = rng.integers(-500, 500, m).astype(np.int32)
    a = rand_i8(rng, (m, max(k, 1)))[:, :k]
    b = rand_i8(rng, (max(k, 1), n))[:k]
    want = O.gemm_i8_fused_matrix(alpha, np.ascontiguousarray(a), np.ascontiguousarray(b), 3,
                                  c0, bias, "row", True)
    da = dev(np.zeros(16, np.int8))
    dc, dbias = dev(c0), dev(bias)
    gk.gemm_i8_fused_unchecked(m, k, n, alpha, da.data_ptr(), max(k, 1), 1, da.data_ptr(), n, 1,
                               3, dc.data_ptr(), n, 1, bias=dbias.data_ptr(),
                               bias_dim=gk.AXIS_ROW, act=_lib.ACT_RELU)
    assert np.array_equal(host(dc).reshape(m, n), want)
