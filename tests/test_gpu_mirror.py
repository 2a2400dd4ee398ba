"""Mirrored outputs on one GPU: the epilogue stores every element of C also at the same offset
from each mirror pointer. Mirrors here are other buffers on the same device (the sharded path
passes peer GPUs' buffers); every mirror must equal C, and C must equal the plain entry's."""
import ctypes as C

import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gemmkit_b200 import _lib
from gpu_util import dev, empty, host, rand_i8

pytestmark = pytest.mark.gpu


def _ptrs(bufs):
    return (C.c_void_p * len(bufs))(*[b.data_ptr() for b in bufs])


@pytest.mark.parametrize("shape", [(1000, 700, 1500), (2341, 300, 2315), (8, 2048, 3000),
                                   (2068, 512, 2660)],
                         ids=lambda s: "x".join(map(str, s)))
def test_half_mirrored_matches_plain(shape):
    """One-CTA tile, CTA-pair and small-M kernels, column-major C, beta != 0. 2068 x 2660 runs
    the CTA-pair kernel with a 16-byte-aligned C: full chunks go through the staged 128-byte
    mirror stores (rows past the edge masked), the ragged last chunk through per-lane stores."""
    m, k, n = shape
    rng = np.random.default_rng(m + n)
    a = O.f32_to_bf16(rng.standard_normal((m, k)).astype(np.float32))
    bT = O.f32_to_bf16(rng.standard_normal((n, k)).astype(np.float32))
    c0 = rng.standard_normal(m * n).astype(np.float32)
    da, db = dev(a.view(np.int16)), dev(bT.view(np.int16))
    lib = _lib.load()
    plain = dev(c0)
    rc = lib.gk_gemm_bf16_f32_unchecked(None, m, k, n, 1.25, da.data_ptr(), k, 1, db.data_ptr(),
                                        1, k, 0.5, plain.data_ptr(), 1, m, _lib.Parallelism(0, 0),
                                        None)
    assert rc == 0, _lib.last_error()
    c = dev(c0)
    mirrors = [empty(m * n, np.float32) for _ in range(3)]
    rc = lib.gk_gemm_half_f32_mirrored_unchecked(None, 0, m, k, n, 1.25, da.data_ptr(), k, 1,
                                                 db.data_ptr(), 1, k, 0.5, c.data_ptr(), 1, m,
                                                 _ptrs(mirrors), 3, None)
    assert rc == 0, _lib.last_error()
    got = host(c)
    assert np.array_equal(got, host(plain))
    for mb in mirrors:
        assert np.array_equal(host(mb), got)
    assert gk.device_status(0) == 0


def test_i8_requant_mirrored_batched_and_packed():
    rng = np.random.default_rng(3)
    batch, m, k, n = 4, 300, 200, 260
    a = rand_i8(rng, (batch, m, k))
    bT = rand_i8(rng, (batch, n, k))
    bias = rng.integers(-2**15, 2**15 + 1, (batch, m)).astype(np.int32)
    scales = rng.uniform(1e-4, 1e-3, (batch, n)).astype(np.float32)
    want = np.stack([O.requant_matrix(a[e], bT[e].T, scales=scales[e], scale_axis="col",
                                      bias=bias[e], bias_axis="row", zp=128, out_u8=True)
                     for e in range(batch)])
    da, db, dbias, dsc = dev(a), dev(bT), dev(bias), dev(scales)
    req = gk.Requantize(gk.RequantScale.PerCol(dsc), 128, dbias, gk.AXIS_ROW)
    lib = _lib.load()
    c = empty(batch * m * n, np.uint8)
    mirror = empty(batch * m * n, np.uint8)
    rc = lib.gk_gemm_i8_requant_mirrored_unchecked(
        None, batch, m, k, n, da.data_ptr(), k, 1, m * k, db.data_ptr(), 1, k, n * k, None,
        C.byref(req.c()), m, n, c.data_ptr(), n, 1, m * n, 1, _ptrs([mirror]), 1, None)
    assert rc == 0, _lib.last_error()
    assert np.array_equal(host(c).reshape(batch, m, n), want)
    assert np.array_equal(host(mirror), host(c))

    # a prepacked B (batch 1), small M: the streaming kernel's epilogue mirrors too
    M, K, N = 5, 1024, 2000
    x = rand_i8(rng, (M, K), -127, 127)
    wT = rand_i8(rng, (N, K), -127, 127)
    s2 = rng.uniform(1e-4, 1e-3, N).astype(np.float32)
    want2 = O.requant_matrix(x, wT.T, scales=s2, scale_axis="col", zp=0)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dev(wT), K, N, 1, K))
    ds2 = dev(s2)
    req2 = gk.Requantize(gk.RequantScale.PerCol(ds2), 0)
    c2, m2 = empty(M * N, np.int8), empty(M * N, np.int8)
    rc = lib.gk_gemm_i8_requant_mirrored_unchecked(
        None, 1, M, K, N, dev(x).data_ptr(), K, 1, 0, None, 0, 0, 0, packed.h,
        C.byref(req2.c()), 0, 0, c2.data_ptr(), N, 1, 0, 0, _ptrs([m2]), 1, None)
    assert rc == 0, _lib.last_error()
    assert np.array_equal(host(c2).reshape(M, N), want2)
    assert np.array_equal(host(m2), host(c2))
    assert gk.device_status(0) == 0
