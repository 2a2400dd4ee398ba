"""The producer step (f32 activations -> i8) bit-exact against numpy's f64 arithmetic:
q = saturate_i8(zp + round_half_even(f64(x) / f64(scale))), NaN -> zp; per-row symmetric
scales max|x_r| / 127 in f32. Then quantize -> requantizing GEMM end to end against the
oracle."""
import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gpu_util import dev, empty, host

pytestmark = pytest.mark.gpu


def _want(x, scale, zp):
    with np.errstate(invalid="ignore", over="ignore"):
        q = np.rint(x.astype(np.float64) / np.float64(scale))
    q = np.where(np.isnan(q), 0.0, q)
    return np.clip(q + zp, -128, 127).astype(np.int8)


def test_per_tensor_ties_edges_and_strides():
    rng = np.random.default_rng(1)
    rows, cols = 37, 1000
    x = (rng.standard_normal((rows, cols)) * 40).astype(np.float32)
    x[0, :8] = [0.25, 0.75, 1.25, -0.25, -1.75, 2.25, 1e30, -1e30]  # ties at scale 0.5, saturation
    x[1, :3] = [np.nan, np.inf, -np.inf]
    scale, zp = 0.5, -5
    dq = empty(rows * cols, np.int8)
    gk.quantize_f32_i8(rows, cols, dev(x).data_ptr(), cols, 1, dq.data_ptr(), cols, 1, scale, zp)
    assert np.array_equal(host(dq).reshape(rows, cols), _want(x, scale, zp))
    # a column-major source into a row-major destination
    xc = np.ascontiguousarray(x.T)
    dq2 = empty(rows * cols, np.int8)
    gk.quantize_f32_i8(rows, cols, dev(xc).data_ptr(), 1, rows, dq2.data_ptr(), cols, 1, 0.37, 3)
    assert np.array_equal(host(dq2).reshape(rows, cols), _want(x, np.float32(0.37), 3))


def test_dynamic_per_row_scales():
    rng = np.random.default_rng(2)
    rows, cols = 64, 4096
    x = (rng.standard_normal((rows, cols)) * rng.uniform(0.1, 100, (rows, 1))).astype(np.float32)
    x[5] = 0.0
    dq = empty(rows * cols, np.int8)
    ds = empty(rows, np.float32)
    gk.quantize_f32_i8(rows, cols, dev(x).data_ptr(), cols, 1, dq.data_ptr(), cols, 1,
                       row_scales=ds.data_ptr())
    amax = np.abs(x).max(axis=1)
    want_s = np.where(amax > 0, (amax / np.float32(127)).astype(np.float32), np.float32(1))
    got_s = host(ds)
    assert np.array_equal(got_s, want_s)
    want = np.stack([_want(x[r], want_s[r], 0) for r in range(rows)])
    assert np.array_equal(host(dq).reshape(rows, cols), want)
    assert np.abs(host(dq)).max() <= 127


def test_quantize_feeds_requant_gemm():
    """x (f32) -> i8 with a per-tensor scale -> requantized GEMM over prepacked weights."""
    rng = np.random.default_rng(3)
    m, k, n = 16, 1024, 640
    x = (rng.standard_normal((m, k)) * 3).astype(np.float32)
    wT = rng.integers(-127, 128, (n, k)).astype(np.int8)
    s_x = 0.05
    s_out = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
    xq = _want(x, s_x, 0)
    want = O.requant_matrix(xq, wT.T, scales=s_out, scale_axis="col", zp=0)
    dxq = empty(m * k, np.int8)
    gk.quantize_f32_i8(m, k, dev(x).data_ptr(), k, 1, dxq.data_ptr(), k, 1, s_x, 0)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dev(wT), k, n, 1, k))
    dso = dev(s_out)
    dc = empty(m * n, np.int8)
    gk.gemm_i8_packed_b_requant(m, dxq.data_ptr(), k, 1, packed,
                                gk.Requantize(gk.RequantScale.PerCol(dso), 0), dc.data_ptr(), n, 1)
    assert np.array_equal(host(dxq).reshape(m, k), xq)
    assert np.array_equal(host(dc).reshape(m, n), want)
    assert gk.device_status(0) == 0
