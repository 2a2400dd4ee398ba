"""The requantize epilogue's short paths against the oracle, bit-exact. An epilogue warp takes
the short path for a tile when every one of its rows has a scale of at most 2^-9 held per row
(or per tensor) and the zero point is even; otherwise the general path. These cases sit on
that boundary: per-row / per-column scales with warps that are all small, warps with one large
scale among small ones, scales of exactly 2^-9, per-tensor scales on both sides of it, even
and odd zero points, bias per row / per column / none with values that wrap the i32
accumulator, ReLU, both C orientations (which decide the kernel frame), and small m (the
small-M kernel) as well as tile-kernel sizes."""
import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gpu_util import dev, empty, gather, host, rand_i8

pytestmark = pytest.mark.gpu

SMALL = 2.0 ** -9


def _scales(rng, length):
    s = rng.uniform(1e-6, SMALL, length).astype(np.float32)
    s[: min(32, length)] = np.float32(SMALL)  # a warp of rows exactly at the bound
    if length > 70:
        s[70] = np.float32(0.02)              # one large scale inside a warp of small ones
    if length > 200:
        s[200:232] = np.float32(0.004)         # a warp of large scales only
    return s


def _bias(rng, length):
    b = rng.integers(-2**15, 2**15 + 1, length).astype(np.int64)
    wrap = rng.random(length) < 0.2            # accumulator + bias wraps modulo 2^32
    b[wrap] = rng.integers(-2**31, 2**31, int(wrap.sum()))
    return b.astype(np.int32)


SCALE_KINDS = ["row", "col", "tensor-small", "tensor-large"]
ZP_CASES = [(False, -128), (True, 128), (False, 5)]  # even i8, even u8, odd i8


@pytest.mark.parametrize("shape", [(300, 200, 260), (8, 1000, 700)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("c_row", [True, False])
@pytest.mark.parametrize("scale_kind", SCALE_KINDS)
@pytest.mark.parametrize("bias_axis", ["row", "col", "none"])
@pytest.mark.parametrize("zp_case", ZP_CASES, ids=lambda z: f"{'u8' if z[0] else 'i8'}{z[1]}")
def test_requant_short_path_boundaries(shape, c_row, scale_kind, bias_axis, zp_case):
    m, k, n = shape
    out_u8, zp = zp_case
    seed = (m * 7 + SCALE_KINDS.index(scale_kind) * 131 + len(bias_axis) * 17 + zp + 1000 * c_row)
    rng = np.random.default_rng(seed & 0xFFFFFFFF)
    relu = (SCALE_KINDS.index(scale_kind) + len(bias_axis)) % 2 == 0
    a = rand_i8(rng, (m, k), -128, 127)
    b = rand_i8(rng, (k, n), -128, 127)
    oreq = dict(zp=zp, out_u8=out_u8, relu=relu)
    ax = {"row": gk.AXIS_ROW, "col": gk.AXIS_COL}
    dbias = None
    if bias_axis != "none":
        bias = _bias(rng, m if bias_axis == "row" else n)
        oreq.update(bias=bias, bias_axis=bias_axis)
        dbias = dev(bias)
    if scale_kind.startswith("tensor"):
        s = SMALL if scale_kind == "tensor-small" else 0.003
        oreq.update(scale=s)
        scale = gk.RequantScale.PerTensor(s)
    else:
        scales = _scales(rng, m if scale_kind == "row" else n)
        oreq.update(scales=scales, scale_axis=scale_kind)
        scale = gk.RequantScale(0.0, dev(scales), ax[scale_kind])
    want = O.requant_matrix(a, b, **oreq)

    req = gk.Requantize(scale, zp, dbias, ax.get(bias_axis, gk.AXIS_ROW), relu)
    dc = empty(m * n, np.uint8 if out_u8 else np.int8)
    rsc, csc = (n, 1) if c_row else (1, m)
    fn = gk.gemm_i8_requant_u8 if out_u8 else gk.gemm_i8_requant
    fn(gk.MatRef.from_row_major(dev(a), m, k), gk.MatRef.new(dev(np.ascontiguousarray(b.T)),
                                                              k, n, 1, k), req,
       gk.MatMut.new(dc, m, n, rsc, csc))
    got = gather(host(dc), m, n, rsc, csc)
    assert np.array_equal(got, want)
    assert gk.device_status(0) == 0
