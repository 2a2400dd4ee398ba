"""The tuner end to end on the GPU with its quick shapes: every swept knob gets a profile line,
the engine's knobs are back at their incumbent values afterwards, and the products keep their
parity under the profile the tuner writes (its `export` lines applied as a shell would)."""
import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gemmkit_b200 import tune
from gpu_util import dev, empty, host, rand_i8

pytestmark = pytest.mark.gpu


def test_quick_tune_dry_run():
    before = {n: gk.knob_get(n) for n in gk.knob_names()}
    results, profile = tune.run(["--quick", "--dry-run", "--reps", "3", "--batch-ms", "2",
                                 "--knobs", "GEMMKIT_CUDA_PAIR,GEMMKIT_CUDA_GEMV,GEMMKIT_CUDA_PDL"])
    assert [r.env for r in results] == ["GEMMKIT_CUDA_PAIR", "GEMMKIT_CUDA_GEMV",
                                        "GEMMKIT_CUDA_PDL"]
    for r in results:
        assert all(row.stat.median > 0 for row in r.rows)
        assert f"export {r.env}={r.winner}" in profile
    assert {n: gk.knob_get(n) for n in gk.knob_names()} == before
    assert gk.device_status(0) == 0


def _vnni(a, bT, out_u8=False, **req):
    m, k = a.shape
    n = bT.shape[0]
    pb = O.VnniPacked(np.ascontiguousarray(bT).reshape(-1), 1, k, k, n)
    c = np.empty(m * n, np.uint8 if out_u8 else np.int8)
    O.vnni_requant_packed(O.View(np.ascontiguousarray(a).reshape(-1), m, k, k, 1), pb,
                          O.View(c, m, n, 1, m), out_u8=out_u8, **req)
    return c.reshape(n, m).T


def _parity_checks():
    """A product of every shape class the tuner steers, bit-exact against the oracle."""
    rng = np.random.default_rng(808)
    # large tiles: prepacked B, requant with ReLU
    m, k, n = 1100, 700, 1300
    a = rand_i8(rng, (m, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)
    sc = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
    bias = rng.integers(-2**15, 2**15 + 1, n).astype(np.int32)
    da, dbT, dsc, dbias = dev(a), dev(bT), dev(sc), dev(bias)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dbT, k, n, 1, k))
    req = gk.Requantize(gk.RequantScale.PerCol(dsc), 0, dbias, gk.AXIS_COL, True)
    dc = empty(m * n, np.int8)
    a_ptr = da.data_ptr()
    gk.gemm_i8_packed_b_requant(m, a_ptr, k, 1, packed, req, dc.data_ptr(), 1, m)
    assert np.array_equal(host(dc).reshape(n, m).T, _vnni(a, bT, scales=sc, scale_axis="col",
                                                         bias=bias, bias_axis="col", zp=0,
                                                         relu=True))
    # small M over the same packed weights
    dsm = empty(5 * n, np.int8)
    gk.gemm_i8_packed_b_requant(5, a_ptr, k, 1, packed, req, dsm.data_ptr(), n, 1)
    assert np.array_equal(host(dsm).reshape(5, n), _vnni(a[:5], bT, scales=sc, scale_axis="col",
                                                         bias=bias, bias_axis="col", zp=0,
                                                         relu=True))
    # short K: batched config-4 elements and a K = 200 product
    B, bm, bk, bn = 12, 512, 128, 512
    xa = rand_i8(rng, (B, bm, bk))
    xb = rand_i8(rng, (B, bn, bk))
    xbias = rng.integers(-2**15, 2**15 + 1, (B, bm)).astype(np.int32)
    xsc = rng.uniform(1e-4, 1e-3, (B, bn)).astype(np.float32)
    dxa, dxb, dxbias, dxsc = dev(xa), dev(xb), dev(xbias), dev(xsc)
    xreq = gk.Requantize(gk.RequantScale.PerCol(dxsc), 128, dxbias, gk.AXIS_ROW)
    dxc = empty(B * bm * bn, np.uint8)
    gk.gemm_i8_requant_batched(B, bm, bk, bn, dxa.data_ptr(), bk, 1, bm * bk, dxb.data_ptr(), 1,
                               bk, bn * bk, xreq, bm, bn, dxc.data_ptr(), 1, bm, bm * bn,
                               out_u8=True)
    got = host(dxc).reshape(B, bn, bm)
    for e in range(B):
        assert np.array_equal(got[e].T, _vnni(xa[e], xb[e], scales=xsc[e], scale_axis="col",
                                              bias=xbias[e], bias_axis="row", zp=128,
                                              out_u8=True)), e
    m2, k2, n2 = 2100, 200, 2300
    a2 = rand_i8(rng, (m2, k2))
    b2 = rand_i8(rng, (n2, k2))
    sc2 = rng.uniform(1e-4, 6e-3, m2).astype(np.float32)
    da2, db2, dsc2 = dev(a2), dev(b2), dev(sc2)
    req2 = gk.Requantize(gk.RequantScale.PerRow(dsc2), -3)
    dc2 = empty(m2 * n2, np.int8)
    gk.gemm_i8_requant_ex_unchecked(m2, k2, n2, da2.data_ptr(), k2, 1, db2.data_ptr(), 1, k2,
                                    req2, dc2.data_ptr(), n2, 1)
    assert np.array_equal(host(dc2).reshape(m2, n2),
                          _vnni(a2, b2, scales=sc2, scale_axis="row", zp=-3))
    # row-major A and B -> i32 (B N-contiguous: read MN-major or packed)
    m3, k3, n3 = 1000, 1000, 1000
    a3 = rand_i8(rng, (m3, k3))
    b3 = rand_i8(rng, (k3, n3))
    da3, db3 = dev(a3), dev(b3)
    dc3 = empty(m3 * n3, np.int32)
    gk.gemm_i8_unchecked(m3, k3, n3, 1, da3.data_ptr(), k3, 1, db3.data_ptr(), n3, 1, 0,
                         dc3.data_ptr(), n3, 1)
    assert np.array_equal(host(dc3).reshape(m3, n3), O.gemm_i8_matrix(1, a3, b3, 0, None))


def test_parity_under_tuned_profile():
    """Tune the knobs that choose kernels, forms and ring depths, apply the profile's export
    lines, and check a product of every shape class against the oracle; then restore."""
    before = {n: gk.knob_get(n) for n in gk.knob_names()}
    knobs = ("GEMMKIT_CUDA_BN,GEMMKIT_CUDA_BN_SHORTK,GEMMKIT_CUDA_EPI16,GEMMKIT_CUDA_STAGES,"
             "GEMMKIT_CUDA_GEMV_SK,GEMMKIT_CUDA_GEMV_SPLIT,GEMMKIT_CUDA_MN_B,"
             "GEMMKIT_CUDA_REQUANT_F32")
    results, profile = tune.run(["--quick", "--dry-run", "--reps", "3", "--batch-ms", "2",
                                 "--knobs", knobs])
    exports = [ln.split()[1].split("=") for ln in profile.splitlines()
               if ln.startswith("export ")]
    assert [name for name, _ in exports] == knobs.split(",")
    try:
        for name, value in exports:
            gk.knob_set(name, int(value))
        _parity_checks()
    finally:
        for name in gk.knob_names():
            gk.knob_set(name, -1)
    assert {n: gk.knob_get(n) for n in gk.knob_names()} == before
    assert gk.device_status(0) == 0
