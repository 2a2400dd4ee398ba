"""GPU parity of the i8 paths (i32, requant i8/u8, prepacked B, batched, small-M) through the
C ABI, bit-exact against the CPU oracle and the golden fixtures of the reference's tests."""
import json
import os

import numpy as np
import pytest

import gemmkit_b200 as gk
import oracle as O
from gpu_util import dev, digest, empty, gather, host, knobs, rand_i8
from refrng import Rng, bias_vec, make_i8, rand_i8 as ref_rand_i8

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


@pytest.fixture(autouse=True)
def _reset_tile():
    gk.set_tile_n(0)
    yield
    gk.set_tile_n(0)
    assert gk.device_status(0) == 0, "a bounded device wait gave up"


def ptr(t):
    return t.data_ptr()


# ---- i8 -> i32 --------------------------------------------------------------------------------

def test_correctness_i8_reference_digests():
    """gemmkit/tests/correctness/int8.rs:11-66 on its own inputs, against the fixture digests."""
    spec = load("model_cases.json")["correctness_i8"]
    for case in spec["cases"]:
        m, k, n, al, be = case["m"], case["k"], case["n"], case["alpha"], case["beta"]
        a = ref_rand_i8(m * k, 0x100 + (m * 7 + k))
        b = ref_rand_i8(k * n, 0x200 + (n * 3 + k)).reshape(k, n)
        bcol = np.ascontiguousarray(b.T).reshape(-1)
        c0 = np.array([(x % 7) - 3 for x in range(m * n)], np.int32)
        da, db, dc = dev(a), dev(bcol), dev(c0)
        gk.gemm_i8(al, gk.MatRef.from_row_major(da, m, k), gk.MatRef.new(db, k, n, 1, k), be,
                   gk.MatMut.from_row_major(dc, m, n))
        assert digest(host(dc)) == case["sha256"], (m, k, n, al, be)


def test_packed_common_reference_digests():
    """gemmkit/tests/i8_packed_common/mod.rs:29-90: prepack (both B layouts) == plain."""
    spec = load("model_cases.json")["i8_packed_common"]
    for case in spec["cases"]:
        m, k, n, al, be = case["m"], case["k"], case["n"], case["alpha"], case["beta"]
        a = ref_rand_i8(m * k, 0x51 + (m * 7 + n))
        b_rm = ref_rand_i8(k * n, 0x62 + (n * 3 + k))
        b_cm = np.ascontiguousarray(b_rm.reshape(k, n).T).reshape(-1)
        c0 = np.array([(x % 7) - 3 for x in range(m * n)], np.int32)
        da = dev(a)
        for bb, rsb, csb in [(b_rm, n, 1), (b_cm, 1, k)]:
            db = dev(bb)
            packed = gk.prepack_rhs_i8(gk.MatRef.new(db, k, n, rsb, csb))
            assert (packed.rows(), packed.cols()) == (k, n)
            dc = dev(c0)
            gk.gemm_i8_packed_b(al, gk.MatRef.from_col_major(da, m, k), packed, be,
                                gk.MatMut.from_col_major(dc, m, n))
            got = host(dc).reshape(n, m).T
            assert digest(got.astype(np.int32)) == case["sha256_rowmajor"], (m, k, n, rsb)
            dplain = dev(c0)
            gk.gemm_i8(al, gk.MatRef.from_col_major(da, m, k), gk.MatRef.new(db, k, n, rsb, csb),
                       be, gk.MatMut.from_col_major(dplain, m, n))
            assert np.array_equal(host(dplain), host(dc))


def test_kat_wraps_on_overflow():
    """gemmkit/tests/correctness/int8.rs:198-238 (alpha = 100000 overflows i32)."""
    case = [c for c in load("kat.json") if c["name"] == "i8_wraps_on_overflow"][0]
    da, db = dev(np.array(case["a_rowmajor"], np.int8)), dev(np.array(case["b_rowmajor"], np.int8))
    dc = dev(np.array(case["c0"], np.int32))
    gk.gemm_i8(case["alpha"], gk.MatRef.from_row_major(da, 2, 2), gk.MatRef.from_row_major(db, 2, 2),
               case["beta"], gk.MatMut.from_row_major(dc, 2, 2))
    assert host(dc).tolist() == case["expect"]


def test_c1_config_1024_row_major():
    """M=N=K=1024, row-major A and B, U[-128,127], alpha=1, beta=0."""
    rng = np.random.default_rng(1)
    m = n = k = 1024
    a = rand_i8(rng, (m, k))
    b = rand_i8(rng, (k, n))
    want = O.acc_i8(a[:96], b)  # oracle on a row slice
    da, db = dev(a), dev(b)
    dc = empty(m * n, np.int32)
    gk.gemm_i8(1, gk.MatRef.from_row_major(da, m, k), gk.MatRef.from_row_major(db, k, n), 0,
               gk.MatMut.from_row_major(dc, m, n))
    got = host(dc).reshape(m, n)
    assert np.array_equal(got[:96], want)
    # the rest through an independent exact path (int64 matmul of the same inputs)
    exact = (a.astype(np.int64) @ b.astype(np.int64)).astype(np.int32)
    assert np.array_equal(got, exact)


@pytest.mark.parametrize("alpha,beta", [(1, 0), (3, -2), (0, 3), (2, 1)])
@pytest.mark.parametrize("layout", ["rr", "rc", "cr", "cc"])
def test_i32_layouts_and_tails(alpha, beta, layout):
    """Odd shapes (k % 16 != 0, n % tile != 0) in every A/B/C orientation, vs the oracle."""
    rng = np.random.default_rng(hash((alpha, beta, layout)) & 0xFFFF)
    m, k, n = 193, 77, 301
    a = rand_i8(rng, (m, k))
    b = rand_i8(rng, (k, n))
    c0 = rng.integers(-1000, 1000, (m, n)).astype(np.int32)
    want = O.gemm_i8_matrix(alpha, a, b, beta, c0)
    a_buf = a.reshape(-1) if layout[0] == "r" else np.ascontiguousarray(a.T).reshape(-1)
    rsa, csa = (k, 1) if layout[0] == "r" else (1, m)
    b_buf = b.reshape(-1) if layout[1] == "r" else np.ascontiguousarray(b.T).reshape(-1)
    rsb, csb = (n, 1) if layout[1] == "r" else (1, k)
    for c_row in (True, False):
        c_buf = c0.reshape(-1) if c_row else np.ascontiguousarray(c0.T).reshape(-1)
        rsc, csc = (n, 1) if c_row else (1, m)
        da, db, dc = dev(a_buf), dev(b_buf), dev(c_buf)
        gk.gemm_i8(alpha, gk.MatRef.new(da, m, k, rsa, csa), gk.MatRef.new(db, k, n, rsb, csb), beta,
                   gk.MatMut.new(dc, m, n, rsc, csc))
        got = gather(host(dc), m, n, rsc, csc)
        assert np.array_equal(got, want), (layout, c_row)


@pytest.mark.parametrize("bn", [16, 32, 64, 128, 192, 256])
def test_every_tile_width(bn):
    rng = np.random.default_rng(bn)
    m, k, n = 260, 300, 530
    a = rand_i8(rng, (m, k))
    b = rand_i8(rng, (k, n))
    want = O.gemm_i8_matrix(1, a, b, 0)
    gk.set_tile_n(bn)
    da, db = dev(a), dev(np.ascontiguousarray(b.T))
    dc = empty(m * n, np.int32)
    gk.gemm_i8(1, gk.MatRef.from_row_major(da, m, k), gk.MatRef.new(db, k, n, 1, k), 0,
               gk.MatMut.from_row_major(dc, m, n))
    assert np.array_equal(host(dc).reshape(m, n), want)


def test_negative_strides_unchecked():
    """gemmkit/tests/correctness/int8.rs:278-316: A walked backwards from its last row."""
    m, k, n = 12, 9, 7
    a = ref_rand_i8(m * k, 5)
    b = ref_rand_i8(k * n, 6)
    cref = O.gemm_i8_matrix(1, a.reshape(m, k), b.reshape(k, n), 0)
    da, db = dev(a), dev(b)
    dc = empty(m * n, np.int32)
    gk.gemm_i8_unchecked(m, k, n, 1, ptr(da) + (m - 1) * k, -k, 1, ptr(db), n, 1, 0, ptr(dc), n, 1)
    got = host(dc).reshape(m, n)
    assert np.array_equal(got, cref[::-1])


def test_degenerate_shapes():
    dc = dev(np.arange(12, dtype=np.int32))
    z = dev(np.zeros(16, np.int8))
    # k == 0: C <- beta*C; alpha == 0 likewise; beta == 0 zero-fills
    gk.gemm_i8_unchecked(3, 0, 4, 1, ptr(z), 0, 1, ptr(z), 4, 1, 3, ptr(dc), 4, 1)
    assert host(dc).tolist() == [3 * x for x in range(12)]
    gk.gemm_i8_unchecked(3, 5, 4, 0, ptr(z), 5, 1, ptr(z), 4, 1, 0, ptr(dc), 4, 1)
    assert host(dc).tolist() == [0] * 12
    # m == 0 / n == 0: nothing is touched
    gk.gemm_i8_unchecked(0, 5, 4, 1, 0, 5, 1, 0, 4, 1, 0, 0, 4, 1)
    gk.gemm_i8_unchecked(3, 5, 0, 1, 0, 5, 1, 0, 4, 1, 0, 0, 4, 1)


# ---- requant --------------------------------------------------------------------------------

@pytest.mark.parametrize("case", load("kat.json"), ids=lambda c: c["name"])
def test_requant_kats(case):
    if case["kind"] != "requant":
        pytest.skip("i32 KAT covered above")
    m, k, n = case["m"], case["k"], case["n"]
    da = dev(np.array(case["a_colmajor"], np.int8))
    db = dev(np.array(case["b"], np.int8))
    dc = empty(m * n, np.uint8 if case["out_u8"] else np.int8)
    req = gk.Requantize(gk.RequantScale.PerTensor(case["scale"]), case["zp"])
    fn = gk.gemm_i8_requant_u8 if case["out_u8"] else gk.gemm_i8_requant
    fn(gk.MatRef.from_col_major(da, m, k), gk.MatRef.from_col_major(db, k, n), req,
       gk.MatMut.from_col_major(dc, m, n))
    assert host(dc).tolist() == case["expect"]


def test_requant_ties_and_saturation_fixture():
    """gemmkit/tests/epilogue/requant.rs:275-320 on its Rng(0x7135) inputs vs the fixture."""
    spec = load("model_cases.json")["requant_ties_and_saturation"]
    rng = Rng(spec["seed"])
    for case in spec["cases"]:
        m, k, n = case["m"], case["k"], case["n"]
        a = make_i8(rng, m * k)
        b = make_i8(rng, k * n)
        bias = bias_vec(rng, m) if case["has_bias"] else None
        row_major = case["tag"] == "sat-"
        da, db = dev(a), dev(b)
        dc = empty(m * n, np.int8)
        dbias = dev(bias) if bias is not None else None
        req = gk.Requantize(gk.RequantScale.PerTensor(case["scale"]), case["zp"], dbias)
        cv = gk.MatMut.from_row_major(dc, m, n) if row_major else gk.MatMut.from_col_major(dc, m, n)
        gk.gemm_i8_requant(gk.MatRef.from_col_major(da, m, k), gk.MatRef.from_col_major(db, k, n),
                           req, cv)
        h = host(dc)
        got = h.reshape(m, n) if row_major else h.reshape(n, m).T
        assert got.reshape(-1).tolist() == case["expect"], (case["tag"], k)


def test_requant_extreme_acc_fixture():
    """requant.rs:486-545: i32-extreme biases, scales up to 1e30, unit and strided C."""
    s = load("model_cases.json")["requant_vector_extreme_acc"]
    m, k, n = s["m"], s["k"], s["n"]
    da = dev(np.array(s["a"], np.int8))
    db = dev(np.array(s["b"], np.int8))
    dbias = dev(np.array(s["bias"], np.int64).astype(np.int32))
    for run in s["runs"]:
        for rsc, csc, size in [(1, m, m * n), (2, 2 * m, 2 * m * n)]:
            dc = dev(np.zeros(size, np.int8))
            req = gk.Requantize(gk.RequantScale.PerTensor(run["scale"]), run["zp"], dbias)
            gk.gemm_i8_requant(gk.MatRef.from_col_major(da, m, k), gk.MatRef.from_col_major(db, k, n),
                               req, gk.MatMut.new(dc, m, n, rsc, csc))
            got = gather(host(dc), m, n, rsc, csc)
            assert got.reshape(-1).tolist() == run["expect"], (run["scale"], run["zp"], rsc)


def test_requant_store_sweep_through_bias():
    """gemmkit/src/simd.rs:743-853 adversarial accumulators, fed through the bias (A = 0)."""
    s = load("model_cases.json")["requant_store_sweep"]
    vals = np.array(s["vals"], np.int64).astype(np.int32)
    m, k, n = len(vals), 32, 40
    da = dev(np.zeros(m * k, np.int8))
    db = dev(np.zeros(k * n, np.int8))
    dbias = dev(vals)
    for g in s["grid"]:
        u8 = g["lo"] == 0
        dc = empty(m * n, np.uint8 if u8 else np.int8)
        req = gk.Requantize(gk.RequantScale.PerTensor(g["scale_f32"]), g["zp"], dbias)
        if u8 and g["zp"] < 0:
            continue  # outside the u8 entry's zero-point range
        fn = gk.gemm_i8_requant_u8 if u8 else gk.gemm_i8_requant
        fn(gk.MatRef.from_row_major(da, m, k), gk.MatRef.from_row_major(db, k, n), req,
           gk.MatMut.from_row_major(dc, m, n))
        got = host(dc).reshape(m, n).view(np.uint8)
        want = np.array(g["expect"], np.uint8)
        assert np.all(got == want[:, None]), (g["scale"], g["zp"], g["lo"])


AXES = [("row", "row"), ("col", "col"), ("row", "col"), ("col", "row"), ("none", "tensor"),
        ("col", "tensor"), ("none", "row")]


@pytest.mark.parametrize("out_u8", [False, True])
@pytest.mark.parametrize("axes", AXES, ids=lambda a: f"b{a[0]}-s{a[1]}")
@pytest.mark.parametrize("c_row", [True, False])
def test_requant_axes_relu(out_u8, axes, c_row):
    rng = np.random.default_rng(hash((out_u8, axes, c_row)) & 0xFFFF)
    m, k, n = 203, 333, 157
    a = rand_i8(rng, (m, k), -127, 127)
    b = rand_i8(rng, (k, n), -127, 127)
    bias_axis, scale_axis = axes
    blen = {"row": m, "col": n}.get(bias_axis, 0)
    slen = {"row": m, "col": n}.get(scale_axis, 0)
    bias = rng.integers(-2**15, 2**15 + 1, max(blen, 1)).astype(np.int32)
    scales = rng.uniform(1e-4, 1e-3, max(slen, 1)).astype(np.float32)
    zp = 7 if out_u8 else -3
    relu = bool(rng.integers(0, 2))
    oreq = dict(zp=zp, out_u8=out_u8, relu=relu)
    if bias_axis != "none":
        oreq.update(bias=bias[:blen], bias_axis=bias_axis)
    if scale_axis == "tensor":
        oreq.update(scale=0.00037)
    else:
        oreq.update(scales=scales[:slen], scale_axis=scale_axis)
    want = O.requant_matrix(a, b, **oreq)

    da, db = dev(a), dev(np.ascontiguousarray(b.T))
    dbias = dev(bias[:blen]) if blen else None
    dsc = dev(scales[:slen]) if slen else None
    ax = {"row": gk.AXIS_ROW, "col": gk.AXIS_COL}
    scale = (gk.RequantScale.PerTensor(0.00037) if scale_axis == "tensor" else
             gk.RequantScale(0.0, dsc, ax[scale_axis]))
    req = gk.Requantize(scale, zp, dbias, ax.get(bias_axis, gk.AXIS_ROW), relu)
    dc = empty(m * n, np.uint8 if out_u8 else np.int8)
    rsc, csc = (n, 1) if c_row else (1, m)
    fn = gk.gemm_i8_requant_u8 if out_u8 else gk.gemm_i8_requant
    fn(gk.MatRef.from_row_major(da, m, k), gk.MatRef.new(db, k, n, 1, k), req,
       gk.MatMut.new(dc, m, n, rsc, csc))
    got = gather(host(dc), m, n, rsc, csc)
    assert np.array_equal(got, want)


def test_requant_degenerate_k0_fixture():
    s = load("model_cases.json")["requant_degenerate_k0"]
    m, n = s["m"], s["n"]
    dc = dev(np.full(m * n, 99, np.int8))
    z = dev(np.zeros(16, np.int8))
    dbias = dev(np.array(s["bias"], np.int32))
    req = gk.Requantize(gk.RequantScale.PerTensor(s["scale"]), s["zp"], dbias)
    gk.gemm_i8_requant_ex_unchecked(m, 0, n, ptr(z), 1, m, ptr(z), 1, 0, req, ptr(dc), 1, m)
    assert host(dc).reshape(n, m).T.tolist() == s["expect"]


def _vnni_requant(a, bT, out_u8=False, **req):
    """The oracle's restatement of gemmkit's VNNI requant path (bit-identical to the scalar
    restatement for every axis mix, tests/test_oracle.py) on all host threads: row-major
    a (m x k) times B = bT^T, returned row-major m x n."""
    m, k = a.shape
    n = bT.shape[0]
    pb = O.VnniPacked(np.ascontiguousarray(bT).reshape(-1), 1, k, k, n)
    c = np.empty(m * n, np.uint8 if out_u8 else np.int8)
    O.vnni_requant_packed(O.View(np.ascontiguousarray(a).reshape(-1), m, k, k, 1), pb,
                          O.View(c, m, n, 1, m), out_u8=out_u8, **req)
    return c.reshape(n, m).T


def test_c2_config_full_size():
    """4096^3, prepacked column-major B, per-column bias and scale, zp 0,
    ReLU, i8 out. Every output against the oracle (gemmkit/tests/epilogue/requant.rs:34-98
    checks every element too), plus the unpacked-B / row-major-C route against the same."""
    rng = np.random.default_rng(2)
    m = n = k = 4096
    a = rand_i8(rng, (m, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)  # B column-major == B^T row-major
    bias = rng.integers(-2**15, 2**15 + 1, n).astype(np.int32)
    scales = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
    da, dbT, dbias, dsc = dev(a), dev(bT), dev(bias), dev(scales)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dbT, k, n, 1, k))
    req = gk.Requantize(gk.RequantScale.PerCol(dsc), 0, dbias, gk.AXIS_COL, True)
    dc = empty(m * n, np.int8)
    gk.gemm_i8_packed_b_requant(m, ptr(da), k, 1, packed, req, ptr(dc), 1, m)
    got = host(dc).reshape(n, m).T
    want = _vnni_requant(a, bT, scales=scales, scale_axis="col", bias=bias, bias_axis="col",
                         zp=0, relu=True)
    assert np.array_equal(got, want)
    rows = np.sort(rng.choice(m, 8, replace=False))  # the scalar restatement on a few rows
    assert np.array_equal(got[rows], O.requant_matrix(
        a[rows], bT.T, scales=scales, scale_axis="col", bias=bias, bias_axis="col", zp=0,
        relu=True))
    dc2 = empty(m * n, np.int8)
    gk.gemm_i8_requant_ex_unchecked(m, k, n, ptr(da), k, 1, ptr(dbT), 1, k, req, ptr(dc2), n, 1)
    assert np.array_equal(host(dc2).reshape(m, n), want)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_c5_small_m_gemv(M):
    """A [M, 4096], prepacked B [4096, 14336], per-column scale, i8 out."""
    rng = np.random.default_rng(M)
    k, n = 4096, 14336
    a = rand_i8(rng, (M, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)
    scales = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
    want = O.requant_matrix(a, bT.T, scales=scales, scale_axis="col", zp=0)
    da, dbT, dsc = dev(a), dev(bT), dev(scales)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dbT, k, n, 1, k))
    req = gk.Requantize(gk.RequantScale.PerCol(dsc), 0)
    dc = empty(M * n, np.int8)
    gk.gemm_i8_packed_b_requant(M, ptr(da), k, 1, packed, req, ptr(dc), n, 1)
    assert np.array_equal(host(dc).reshape(M, n), want)


def _c4_inputs(rng, batch, m, n, k):
    a = rand_i8(rng, (batch, m, k))
    bT = rand_i8(rng, (batch, n, k))
    bias = rng.integers(-2**15, 2**15 + 1, (batch, m)).astype(np.int32)
    scales = rng.uniform(1e-4, 1e-3, (batch, n)).astype(np.float32)
    return a, bT, bias, scales


@pytest.mark.parametrize("batch", [6, 512])
def test_c4_batched(batch):
    """batch of (512x512x128), per-row bias, per-column scale, u8 zp 128.
    Every element of every batch member against the oracle."""
    rng = np.random.default_rng(batch)
    m = n = 512
    k = 128
    a, bT, bias, scales = _c4_inputs(rng, batch, m, n, k)
    da, dbT, dbias, dsc = dev(a), dev(bT), dev(bias), dev(scales)
    req = gk.Requantize(gk.RequantScale.PerCol(dsc), 128, dbias, gk.AXIS_ROW)
    dc = empty(batch * m * n, np.uint8)
    gk.gemm_i8_requant_batched(batch, m, k, n, ptr(da), k, 1, m * k, ptr(dbT), 1, k, n * k, req,
                               m, n, ptr(dc), 1, m, m * n, out_u8=True)
    got = host(dc).reshape(batch, n, m)
    for e in range(batch):
        want = _vnni_requant(a[e], bT[e], scales=scales[e], scale_axis="col", bias=bias[e],
                             bias_axis="row", zp=128, out_u8=True)
        assert np.array_equal(got[e].T, want), e
    e = batch - 1  # and the scalar restatement on one member
    assert np.array_equal(got[e].T, O.requant_matrix(
        a[e], bT[e].T, scales=scales[e], scale_axis="col", bias=bias[e], bias_axis="row",
        zp=128, out_u8=True))


def test_batched_ptr_array_matches_strided():
    rng = np.random.default_rng(9)
    probs, outs, keep = [], [], []
    for (m, k, n) in [(40, 64, 70), (129, 33, 5), (3, 200, 300)]:
        a = rand_i8(rng, (m, k))
        b = rand_i8(rng, (k, n))
        da, db = dev(a), dev(b)
        dc = empty(m * n, np.int8)
        keep += [da, db]
        outs.append((dc, O.requant_matrix(a, b, scale=0.01, zp=1), m, n))
        probs.append(gk.GemmProblem(m, k, n, ptr(da), k, 1, ptr(db), n, 1, ptr(dc), n, 1,
                                    gk.Requantize(gk.RequantScale.PerTensor(0.01), 1)))
    gk.gemm_i8_requant_batched_ptr(probs)
    for dc, want, m, n in outs:
        assert np.array_equal(host(dc).reshape(m, n), want)


def test_general_strided_views():
    """Non-unit strides on every operand (the pack path and the scalar store path)."""
    rng = np.random.default_rng(4)
    m, k, n = 37, 45, 29
    a = rand_i8(rng, (m, k))
    b = rand_i8(rng, (k, n))
    want = O.requant_matrix(a, b, scale=0.02, zp=-5)
    abuf = np.zeros(3 * m * k + 7, np.int8)
    abuf[[i * 3 * k + j * 3 for i in range(m) for j in range(k)]] = a.reshape(-1)
    bbuf = np.zeros(2 * k * n, np.int8)
    bbuf[[i * 2 + j * 2 * k for i in range(k) for j in range(n)]] = b.reshape(-1)
    da, db = dev(abuf), dev(bbuf)
    dc = dev(np.zeros(3 * m * n, np.int8))
    req = gk.Requantize(gk.RequantScale.PerTensor(0.02), -5)
    gk.gemm_i8_requant_ex_unchecked(m, k, n, ptr(da), 3 * k, 3, ptr(db), 2, 2 * k, req, ptr(dc),
                                    3, 3 * m)
    got = gather(host(dc), m, n, 3, 3 * m)
    assert np.array_equal(got, want)


# ---- stream-K tail (tiles cut between CTAs, partials summed by the last arriver) ---------------

SK_SHAPES = [(1000, 1000, 1000), (700, 2000, 300), (2048, 2048, 2304), (16, 4096, 14336 // 4)]


@pytest.mark.parametrize("shape", SK_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_stream_k_i32_beta(shape):
    """Shapes whose last wave is split over all SMs (K blocks >= 4); beta != 0 is applied once,
    by the CTA that finishes each region. Three calls in a row exercise the counter epochs."""
    m, k, n = shape
    rng = np.random.default_rng(m + k + n)
    a = rand_i8(rng, (m, k))
    bT = rand_i8(rng, (n, k))
    c0 = rng.integers(-1000, 1000, (m, n)).astype(np.int32)
    want = O.gemm_i8_matrix(3, a, bT.T, -2, c0)
    da, db = dev(a), dev(bT)
    with knobs(GEMMKIT_CUDA_STREAMK=1, GEMMKIT_CUDA_PAIR=0, GEMMKIT_CUDA_GEMV=0):
        for _ in range(3):
            dc = dev(c0)
            gk.gemm_i8(3, gk.MatRef.from_row_major(da, m, k), gk.MatRef.new(db, k, n, 1, k), -2,
                       gk.MatMut.from_row_major(dc, m, n))
            assert np.array_equal(host(dc).reshape(m, n), want)


@pytest.mark.parametrize("out_u8", [False, True])
@pytest.mark.parametrize("shape", SK_SHAPES[:3], ids=lambda s: "x".join(map(str, s)))
def test_stream_k_requant(shape, out_u8):
    m, k, n = shape
    rng = np.random.default_rng(m * 3 + k + n)
    a = rand_i8(rng, (m, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)
    bias = rng.integers(-2**15, 2**15 + 1, n).astype(np.int32)
    scales = rng.uniform(1e-4, 1e-3, m).astype(np.float32)
    zp = 100 if out_u8 else -7
    want = O.requant_matrix(a, bT.T, scales=scales, scale_axis="row", bias=bias, bias_axis="col",
                            zp=zp, out_u8=out_u8, relu=True)
    da, db, dbias, dsc = dev(a), dev(bT), dev(bias), dev(scales)
    req = gk.Requantize(gk.RequantScale.PerRow(dsc), zp, dbias, gk.AXIS_COL, True)
    with knobs(GEMMKIT_CUDA_STREAMK=1, GEMMKIT_CUDA_PAIR=0):
        for _ in range(2):
            dc = empty(m * n, np.uint8 if out_u8 else np.int8)
            gk.gemm_i8_requant_ex_unchecked(m, k, n, ptr(da), k, 1, ptr(db), 1, k, req, ptr(dc),
                                            n, 1, out_u8=out_u8)
            assert np.array_equal(host(dc).reshape(m, n), want)


@pytest.mark.parametrize("path", ["streaming", "tile+stream-k"])
def test_stream_k_prepacked_gemv_sizes(path):
    """Small-M over a prepacked B of several widths (112, 50 and 7 row tiles), on the streaming
    small-M kernel and on the tile kernel with its stream-K tail."""
    kv = {} if path == "streaming" else dict(GEMMKIT_CUDA_GEMV=0, GEMMKIT_CUDA_STREAMK=1)
    with knobs(**kv):
        _prepacked_gemv_sizes()


def _prepacked_gemv_sizes():
    rng = np.random.default_rng(77)
    for (M, k, n) in [(4, 4096, 14336), (9, 1024, 6400), (1, 8192, 896)]:
        a = rand_i8(rng, (M, k), -127, 127)
        bT = rand_i8(rng, (n, k), -127, 127)
        scales = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
        want = O.requant_matrix(a, bT.T, scales=scales, scale_axis="col", zp=3)
        da, dbT, dsc = dev(a), dev(bT), dev(scales)
        packed = gk.prepack_rhs_i8(gk.MatRef.new(dbT, k, n, 1, k))
        dc = empty(M * n, np.int8)
        gk.gemm_i8_packed_b_requant(M, ptr(da), k, 1, packed, gk.Requantize(
            gk.RequantScale.PerCol(dsc), 3), ptr(dc), n, 1)
        assert np.array_equal(host(dc).reshape(M, n), want), (M, k, n)


# ---- CTA-pair kernel (256 x 256 tiles over two SMs) ------------------------------------------

PAIR_SHAPE = (2341, 300, 2315)  # >= 74 pair tiles, odd edges in every dimension, K % 128 != 0


def test_pair_i32_odd_shape():
    m, k, n = PAIR_SHAPE
    rng = np.random.default_rng(21)
    a = rand_i8(rng, (m, k))
    bT = rand_i8(rng, (n, k))
    c0 = rng.integers(-1000, 1000, (m, n)).astype(np.int32)
    rows = np.sort(rng.choice(m, 48, replace=False))
    want = O.gemm_i8_matrix(-3, a[rows], bT.T, 2, c0[rows])
    da, db, dc = dev(a), dev(bT), dev(c0)
    gk.gemm_i8(-3, gk.MatRef.from_row_major(da, m, k), gk.MatRef.new(db, k, n, 1, k), 2,
               gk.MatMut.from_row_major(dc, m, n))
    got = host(dc).reshape(m, n)
    assert np.array_equal(got[rows], want)
    assert np.array_equal(got[-1], O.gemm_i8_matrix(-3, a[-1:], bT.T, 2, c0[-1:])[0])


@pytest.mark.parametrize("out_u8", [False, True])
def test_pair_requant_odd_shape(out_u8):
    m, k, n = PAIR_SHAPE
    rng = np.random.default_rng(22 + out_u8)
    a = rand_i8(rng, (m, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)
    bias = rng.integers(-2**15, 2**15 + 1, m).astype(np.int32)
    scales = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
    zp = 9 if out_u8 else -4
    rows = np.sort(np.concatenate([rng.choice(m, 40, replace=False), [m - 1]]))
    want = O.requant_matrix(a[rows], bT.T, scales=scales, scale_axis="col", bias=bias[rows],
                            bias_axis="row", zp=zp, out_u8=out_u8, relu=True)
    da, db, dbias, dsc = dev(a), dev(bT), dev(bias), dev(scales)
    req = gk.Requantize(gk.RequantScale.PerCol(dsc), zp, dbias, gk.AXIS_ROW, True)
    for c_row in (True, False):
        dc = empty(m * n, np.uint8 if out_u8 else np.int8)
        rsc, csc = (n, 1) if c_row else (1, m)
        gk.gemm_i8_requant_ex_unchecked(m, k, n, ptr(da), k, 1, ptr(db), 1, k, req, ptr(dc), rsc,
                                        csc, out_u8=out_u8)
        got = gather(host(dc), m, n, rsc, csc)
        assert np.array_equal(got[rows], want), c_row


def test_pair_prepacked_batched_c4_shape():
    """Batched config 4 elements go to the pair kernel (2 x 2 pair tiles each)."""
    rng = np.random.default_rng(23)
    batch, m, n, k = 40, 512, 512, 128
    a, bT, bias, scales = _c4_inputs(rng, batch, m, n, k)
    da, dbT, dbias, dsc = dev(a), dev(bT), dev(bias), dev(scales)
    req = gk.Requantize(gk.RequantScale.PerCol(dsc), 128, dbias, gk.AXIS_ROW)
    dc = empty(batch * m * n, np.uint8)
    gk.gemm_i8_requant_batched(batch, m, k, n, ptr(da), k, 1, m * k, ptr(dbT), 1, k, n * k, req,
                               m, n, ptr(dc), 1, m, m * n, out_u8=True)
    got = host(dc).reshape(batch, n, m)
    for e in (0, 17, batch - 1):
        want = O.requant_matrix(a[e], bT[e].T, scales=scales[e], scale_axis="col",
                                bias=bias[e], bias_axis="row", zp=128, out_u8=True)
        assert np.array_equal(got[e].T, want), e


def test_packed_serialize_round_trip():
    """A packed B stored and loaded back gives the same bytes and the same products."""
    rng = np.random.default_rng(404)
    m, k, n = 200, 300, 500
    a = rand_i8(rng, (m, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)
    scales = rng.uniform(1e-4, 1e-3, n).astype(np.float32)
    want = O.requant_matrix(a, bT.T, scales=scales, scale_axis="col", zp=1)
    packed = gk.prepack_rhs_i8(gk.MatRef.new(dev(bT), k, n, 1, k))
    blob = packed.to_bytes()
    assert blob[:8] == b"GKPACK01" and len(blob) == 64 + 384 * 512
    loaded = gk.PackedRhs.from_bytes(blob)
    assert (loaded.rows(), loaded.cols()) == (k, n)
    assert loaded.to_bytes() == blob
    da, dsc = dev(a), dev(scales)
    req = gk.Requantize(gk.RequantScale.PerCol(dsc), 1)
    for pk in (packed, loaded):
        dc = empty(m * n, np.int8)
        gk.gemm_i8_packed_b_requant(m, ptr(da), k, 1, pk, req, ptr(dc), n, 1)
        assert np.array_equal(host(dc).reshape(m, n), want)
