"""Pin the CPU oracle: it must reproduce every known-answer vector of the reference's tests
and the reference tests' independent model on the reference tests' own inputs. No GPU."""
import hashlib
import json
import os

import numpy as np
import pytest

from model import acc_exact, requant, requant_array
from refrng import Rng, bias_vec, make_i8, rand_i8

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
I8, U8 = (-128, 127), (0, 255)


def load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def digest(arr):
    return hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()


def test_round_ne_f64(oracle_lib):
    o = oracle_lib
    for x, want in [(0.5, 0.0), (1.5, 2.0), (2.5, 2.0), (-0.5, 0.0), (-1.5, -2.0), (-2.5, -2.0),
                    (4503599627370497.0, 4503599627370497.0), (1e300, 1e300), (0.49999999999999994, 0.0)]:
        assert o.round_ne_f64(x) == want
    assert np.isnan(o.round_ne_f64(float("nan")))


@pytest.mark.parametrize("case", load("kat.json"), ids=lambda c: c["name"])
def test_kat(oracle_lib, case):
    o = oracle_lib
    if case["kind"] == "requant":
        m, k, n = case["m"], case["k"], case["n"]
        a = np.array(case["a_colmajor"], np.int8)
        b = np.array(case["b"], np.int8)
        c = np.zeros(m * n, np.uint8 if case["out_u8"] else np.int8)
        o.gemm_i8_requant(o.View(a, m, k, 1, m), o.View(b, k, n, 1, k), o.View(c, m, n, 1, m),
                          scale=case["scale"], zp=case["zp"], out_u8=case["out_u8"])
        assert c.tolist() == case["expect"]
    else:
        m, k, n = case["m"], case["k"], case["n"]
        a = np.array(case["a_rowmajor"], np.int8)
        b = np.array(case["b_rowmajor"], np.int8)
        c = np.array(case["c0"], np.int32)
        o.gemm_i8(case["alpha"], o.View(a, m, k, k, 1), o.View(b, k, n, n, 1), case["beta"],
                  o.View(c, m, n, n, 1))
        assert c.tolist() == case["expect"]


def test_requant_ties_and_saturation(oracle_lib):
    """requant.rs:275-320 on its own Rng(0x7135) stream, all three C orientations/biases."""
    o = oracle_lib
    spec = load("model_cases.json")["requant_ties_and_saturation"]
    rng = Rng(spec["seed"])
    for case in spec["cases"]:
        m, k, n = case["m"], case["k"], case["n"]
        a = make_i8(rng, m * k)
        b = make_i8(rng, k * n)
        bias = bias_vec(rng, m) if case["has_bias"] else None
        row_major = case["tag"] == "sat-"
        c = np.zeros(m * n, np.int8)
        cv = o.View(c, m, n, n, 1) if row_major else o.View(c, m, n, 1, m)
        o.gemm_i8_requant(o.View(a, m, k, 1, m), o.View(b, k, n, 1, k), cv, scale=case["scale"],
                          zp=case["zp"], bias=bias, bias_axis="row")
        got = c.reshape(m, n) if row_major else c.reshape(n, m).T
        assert got.reshape(-1).tolist() == case["expect"], case["tag"]


def test_degenerate_k0(oracle_lib):
    o = oracle_lib
    s = load("model_cases.json")["requant_degenerate_k0"]
    m, n = s["m"], s["n"]
    c = np.full(m * n, 99, np.int8)
    empty = np.zeros(1, np.int8)
    o.gemm_i8_requant(o.View(empty, m, 0, 1, m), o.View(empty, 0, n, 1, 0), o.View(c, m, n, 1, m),
                      scale=s["scale"], zp=s["zp"], bias=np.array(s["bias"]), bias_axis="row")
    assert c.reshape(n, m).T.tolist() == s["expect"]


def test_vector_ties(oracle_lib):
    o = oracle_lib
    s = load("model_cases.json")["requant_vector_ties"]
    a = np.array(s["a"], np.int8)
    m = len(a)
    c = np.zeros(m, np.int8)
    o.gemm_i8_requant(o.View(a, m, 1, 1, m), o.View(np.ones(1, np.int8), 1, 1, 1, 1),
                      o.View(c, m, 1, 1, m), scale=s["scale"], zp=s["zp"])
    assert c.tolist() == s["expect"]


def test_vector_extreme_acc(oracle_lib):
    o = oracle_lib
    s = load("model_cases.json")["requant_vector_extreme_acc"]
    m, k, n = s["m"], s["k"], s["n"]
    a = np.array(s["a"], np.int8)
    b = np.array(s["b"], np.int8)
    bias = np.array(s["bias"], np.int64).astype(np.int32)
    for run in s["runs"]:
        for (rsc, csc, size) in [(1, m, m * n), (2, 2 * m, 2 * m * n)]:
            c = np.zeros(size, np.int8)
            o.gemm_i8_requant(o.View(a, m, k, 1, m), o.View(b, k, n, 1, k),
                              o.View(c, m, n, rsc, csc), scale=run["scale"], zp=run["zp"],
                              bias=bias, bias_axis="row")
            got = np.array([[c[i * rsc + j * csc] for j in range(n)] for i in range(m)])
            assert got.reshape(-1).tolist() == run["expect"], (run["scale"], run["zp"], rsc)


def test_requant_store_sweep(oracle_lib):
    o = oracle_lib
    s = load("model_cases.json")["requant_store_sweep"]
    for g in s["grid"]:
        got = [o.requant_apply(v, 0, g["scale_f32"], g["zp"], g["lo"], g["hi"]) & 0xFF
               for v in s["vals"]]
        assert got == g["expect"], (g["scale"], g["zp"], g["lo"])


def test_correctness_i8_digests(oracle_lib):
    o = oracle_lib
    s = load("model_cases.json")["correctness_i8"]
    for case in s["cases"]:
        m, k, n, al, be = case["m"], case["k"], case["n"], case["alpha"], case["beta"]
        a = rand_i8(m * k, 0x100 + (m * 7 + k))
        b = rand_i8(k * n, 0x200 + (n * 3 + k)).reshape(k, n)
        bcol = np.ascontiguousarray(b.T).reshape(-1)
        c = np.array([(x % 7) - 3 for x in range(m * n)], np.int32)
        o.gemm_i8(al, o.View(a, m, k, k, 1), o.View(bcol, k, n, 1, k), be, o.View(c, m, n, n, 1))
        assert digest(c) == case["sha256"], (m, k, n, al, be)


def test_packed_common_digests_and_vnni_baseline(oracle_lib):
    """i8_packed_common::check shapes: scalar oracle and the threaded VNNI restatement both
    match the exact digests, for row- and column-major B (prepacked) and every (alpha, beta)."""
    o = oracle_lib
    s = load("model_cases.json")["i8_packed_common"]
    for case in s["cases"]:
        m, k, n, al, be = case["m"], case["k"], case["n"], case["alpha"], case["beta"]
        a = rand_i8(m * k, 0x51 + (m * 7 + n))
        b_rm = rand_i8(k * n, 0x62 + (n * 3 + k))
        b_cm = np.ascontiguousarray(b_rm.reshape(k, n).T).reshape(-1)
        c0 = np.array([(x % 7) - 3 for x in range(m * n)], np.int32)
        for (bb, rsb, csb) in [(b_rm, n, 1), (b_cm, 1, k)]:
            c = c0.copy()
            o.gemm_i8(al, o.View(a, m, k, 1, m), o.View(bb, k, n, rsb, csb), be,
                      o.View(c, m, n, 1, m))
            got = c.reshape(n, m).T
            assert digest(got.astype(np.int32)) == case["sha256_rowmajor"]
            pb = o.VnniPacked(bb, rsb, csb, k, n)
            c2 = c0.copy()
            o.vnni_gemm_i8_packed(al, o.View(a, m, k, 1, m), pb, be, o.View(c2, m, n, 1, m),
                                  n_threads=4)
            assert np.array_equal(c, c2)


@pytest.mark.parametrize("out_u8", [False, True])
@pytest.mark.parametrize("axes", [("row", "row"), ("col", "col"), ("row", "col"), ("none", "tensor")])
def test_vnni_requant_matches_scalar(oracle_lib, out_u8, axes):
    """The timed baseline is bit-identical to the scalar restatement for every axis mix."""
    o = oracle_lib
    rng = np.random.default_rng(7)
    m, k, n = 70, 301, 53
    a = rng.integers(-128, 128, (m, k), dtype=np.int8)
    b = rng.integers(-128, 128, (k, n), dtype=np.int8)
    bias_axis, scale_axis = axes
    blen = {"row": m, "col": n}.get(bias_axis, 1)
    slen = {"row": m, "col": n}.get(scale_axis, 1)
    bias = rng.integers(-2**15, 2**15, blen).astype(np.int32)
    scales = rng.uniform(1e-4, 1e-2, slen).astype(np.float32)
    req = dict(zp=7 if out_u8 else -3, out_u8=out_u8, relu=True)
    if bias_axis != "none":
        req.update(bias=bias, bias_axis=bias_axis)
    if scale_axis == "tensor":
        req.update(scale=0.003)
    else:
        req.update(scales=scales, scale_axis=scale_axis)
    want = o.requant_matrix(a, b, **req)
    af = a.reshape(-1)
    bcm = np.ascontiguousarray(b.T).reshape(-1)
    pb = o.VnniPacked(bcm, 1, k, k, n)
    c = np.zeros(m * n, np.uint8 if out_u8 else np.int8)
    o.vnni_requant_packed(o.View(af, m, k, k, 1), pb, o.View(c, m, n, 1, m), n_threads=4, **req)
    assert np.array_equal(c.reshape(n, m).T, want)


def test_relu_is_requant_of_clamped_sum(oracle_lib):
    """ReLU as a raised lower clamp equals requant(max(acc + bias, 0)) (monotone map, scale>0)."""
    rng = np.random.default_rng(3)
    for _ in range(2000):
        v = int(rng.integers(-2**31, 2**31))
        bias = int(rng.integers(-2**15, 2**15))
        scale = float(np.float32(rng.uniform(1e-5, 2.0)))
        zp = int(rng.integers(-128, 128))
        got = oracle_lib.requant_apply(v, bias, scale, zp, -128, 127, True)
        s = v + bias
        s = (s + 2**31) % 2**32 - 2**31
        assert got == requant(max(s, 0), 0, scale, zp, -128, 127)


def test_model_vs_oracle_random(oracle_lib):
    rng = np.random.default_rng(11)
    for _ in range(3000):
        v = int(rng.integers(-2**31, 2**31))
        bias = int(rng.integers(-2**31, 2**31))
        scale = float(np.float32(10.0 ** rng.uniform(-12, 12)))
        zp = int(rng.integers(-128, 256))
        lo, hi = (U8 if zp >= 0 and rng.random() < 0.5 else I8)
        assert oracle_lib.requant_apply(v, bias, scale, zp, lo, hi, 0) == \
            requant(v, bias, scale, zp, lo, hi)


def test_bf16_rounding(oracle_lib):
    o = oracle_lib
    x = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 65504.0, 1e-40, np.inf, -np.inf, np.nan],
                 np.float32)
    h = o.f32_to_bf16(x)
    for xi, hi in zip(x, h):
        assert o.lib().gko_f32_to_bf16(float(xi)) == int(hi)
    # round-half-even on the dropped 16 bits: 1 + 2^-8 is a tie -> even (1.0)
    assert o.bf16_to_f32(o.f32_to_bf16(np.array([1.00390625], np.float32)))[0] == 1.0
    try:
        import torch
        t = torch.from_numpy(x[:-1]).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(t, h[:-1])
    except ImportError:
        pass


def test_half_f64_reference(oracle_lib):
    o = oracle_lib
    rng = np.random.default_rng(5)
    a = o.f32_to_bf16(rng.standard_normal((9, 33)).astype(np.float32))
    b = o.f32_to_bf16(rng.standard_normal((33, 7)).astype(np.float32))
    c = rng.standard_normal((9, 7)).astype(np.float32)
    got = o.gemm_half_f64(a, b, 1.0, 0.5, c)
    want = o.bf16_to_f32(a).astype(np.float64) @ o.bf16_to_f32(b).astype(np.float64) + 0.5 * c
    assert np.allclose(got, want, rtol=1e-12, atol=1e-12)
    cf = np.zeros(9 * 7, np.float32)
    o.cpu_gemm_bf16_f32(1.0, o.View(a.reshape(-1), 9, 33, 33, 1), o.View(b.reshape(-1), 33, 7, 7, 1),
                        0.0, o.View(cf, 9, 7, 7, 1))
    assert np.allclose(cf.reshape(9, 7), o.bf16_to_f32(a).astype(np.float64) @ o.bf16_to_f32(b),
                       rtol=1e-4, atol=1e-4)


def test_acc_matches_model(oracle_lib):
    rng = np.random.default_rng(1)
    a = rng.integers(-128, 128, (17, 40), dtype=np.int8)
    b = rng.integers(-128, 128, (40, 23), dtype=np.int8)
    assert np.array_equal(oracle_lib.acc_i8(a, b), acc_exact(a, b))
    want = requant_array(acc_exact(a, b), 5, np.float32(0.01), 3, -128, 127)
    assert np.array_equal(oracle_lib.requant_matrix(a, b, scale=0.01, zp=3,
                                                    bias=np.full(17, 5), bias_axis="row"), want)
