"""The fused float epilogue on the bf16 -> f32 GEMM (gemmkit's gemm_fused semantics,
gemmkit/src/kernel/epilogue.rs:258-330): act(alpha*A*B + beta*C + bias), bias per row or per
column, ReLU or LeakyReLU. Within the path's 1e-2 tolerance against an f64 reference on the
one-CTA tile, CTA-pair and small-M kernels and both orientations; the activation's edge rules
(NaN -> 0) and the degenerate k == 0 rule C <- act(beta*C + bias) exactly."""
import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gpu_util import dev, gather, host

pytestmark = pytest.mark.gpu


def _ref(a, b, alpha, beta, c0, bias, bias_dim, act):
    ref = O.gemm_half_f64(a, b, alpha, beta, c0, False)
    mag = abs(alpha) * (np.abs(O.bf16_to_f32(a).astype(np.float64)) @
                        np.abs(O.bf16_to_f32(b).astype(np.float64)))
    if c0 is not None:
        mag += abs(beta) * np.abs(c0.astype(np.float64))
    if bias is not None:
        bb = bias[:, None] if bias_dim == gk.AXIS_ROW else bias[None, :]
        ref = ref + bb
        mag = mag + np.abs(bb)
    if act is not None and act.kind == gk._lib.ACT_RELU:
        ref = np.maximum(ref, 0.0)
    elif act is not None:
        ref = np.maximum(ref, 0.0) + act.slope * np.minimum(ref, 0.0)
    return ref, mag


@pytest.mark.parametrize("shape", [(200, 333, 129), (2341, 300, 2315), (8, 2048, 3000)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("bias_dim", [gk.AXIS_ROW, gk.AXIS_COL])
@pytest.mark.parametrize("act", ["none", "relu", "leaky"])
@pytest.mark.parametrize("c_col_major", [False, True])
def test_fused_bias_activation(shape, bias_dim, act, c_col_major):
    m, k, n = shape
    rng = np.random.default_rng(m + k + n + bias_dim)
    a = O.f32_to_bf16(rng.standard_normal((m, k)).astype(np.float32))
    b = O.f32_to_bf16(rng.standard_normal((k, n)).astype(np.float32))
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    bias = (rng.standard_normal(m if bias_dim == gk.AXIS_ROW else n) * 4).astype(np.float32)
    activation = {"none": None, "relu": gk.Activation.Relu(),
                  "leaky": gk.Activation.LeakyRelu(0.125)}[act]
    da = dev(a.view(np.int16))
    db = dev(b.view(np.int16))
    if c_col_major:
        dc = dev(np.ascontiguousarray(c0.T).reshape(-1))
        cv = gk.MatMut.from_col_major(dc, m, n)
    else:
        dc = dev(c0)
        cv = gk.MatMut.from_row_major(dc, m, n)
    gk.gemm_half_f32_fused(1.5, gk.MatRef.from_row_major(da, m, k),
                           gk.MatRef.from_row_major(db, k, n), 0.5, cv, bias=dev(bias),
                           bias_dim=bias_dim, act=activation)
    got = gather(host(dc), m, n, 1, m) if c_col_major else host(dc).reshape(m, n)
    rows = np.arange(m) if m <= 256 else np.concatenate([np.arange(0, m, 37), [m - 1]])
    ref, mag = _ref(a[rows], b, 1.5, 0.5, c0[rows],
                    bias[rows] if bias_dim == gk.AXIS_ROW else bias, bias_dim, activation)
    err = np.abs(got[rows].astype(np.float64) - ref)
    assert np.all(err <= 1e-2 * mag + 1e-6), float((err / (mag + 1e-30)).max())
    if act == "relu":
        assert (got >= 0).all()
    assert gk.device_status(0) == 0


def test_fused_relu_maps_nan_to_zero():
    m, k, n = 64, 128, 96
    rng = np.random.default_rng(1)
    a = O.f32_to_bf16(rng.standard_normal((m, k)).astype(np.float32))
    b = O.f32_to_bf16(rng.standard_normal((k, n)).astype(np.float32))
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    c0[3, 5] = np.nan
    dc = dev(c0)
    gk.gemm_half_f32_fused(1.0, gk.MatRef.from_row_major(dev(a.view(np.int16)), m, k),
                           gk.MatRef.from_row_major(dev(b.view(np.int16)), k, n), 1.0,
                           gk.MatMut.from_row_major(dc, m, n), act=gk.Activation.Relu())
    got = host(dc).reshape(m, n)
    assert got[3, 5] == 0.0 and not np.isnan(got).any()


@pytest.mark.parametrize("act", ["relu", "leaky"])
def test_fused_degenerate_k0_exact(act):
    """k == 0: C <- act(beta*C + bias) in f32, element by element (gemmkit's degenerate rule)."""
    m, n = 37, 53
    rng = np.random.default_rng(2)
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    activation = gk.Activation.Relu() if act == "relu" else gk.Activation.LeakyRelu(0.25)
    dc = dev(c0)
    dummy = dev(np.zeros(16, np.int16))
    gk.gemm_half_f32_fused(2.0, gk.MatRef.new(dummy, m, 0, 0, 1), gk.MatRef.new(dummy, 0, n, n, 1),
                           0.75, gk.MatMut.from_row_major(dc, m, n), bias=dev(bias),
                           bias_dim=gk.AXIS_COL, act=activation)
    v = (np.float32(0.75) * c0).astype(np.float32) + bias[None, :]
    v = v.astype(np.float32)
    hi, lo = np.maximum(v, np.float32(0)), np.minimum(v, np.float32(0))
    want = hi if act == "relu" else (hi + np.float32(0.25) * lo).astype(np.float32)
    assert np.array_equal(host(dc).reshape(m, n), want)
