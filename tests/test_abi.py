"""C-ABI checks that need no GPU: the library loads, exports every entry the header declares,
validates like gemmkit (same messages), and fails loudly (GK_ENODEV) instead of falling back
when there is no sm_100 device."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import gemmkit_b200 as gk
from gemmkit_b200 import _build, _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gemmkit_cuda.h")


@pytest.fixture(scope="module", autouse=True)
def built():
    _build.build()


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(gk_[a-z0-9_]+)\s*\(", src)))


def test_exports_every_declared_symbol():
    lib = C.CDLL(_lib.lib_path())
    syms = declared_symbols()
    assert len(syms) >= 25
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    # and the Python binding declares a signature for every one of them
    assert set(syms) <= set(_lib.SIGNATURES), set(syms) - set(_lib.SIGNATURES)


def test_version():
    assert b"sm_100a" in _lib.load().gk_version()


def host(n, dtype=np.int8):
    arr = np.zeros(n, dtype)
    return (arr.ctypes.data, n), arr


def expect_err(fn, substr, code=gk.GK_EINVAL):
    with pytest.raises(gk.GemmkitError) as ei:
        fn()
    assert substr in str(ei.value), str(ei.value)
    assert ei.value.code == code


def test_shape_mismatch_messages():
    (pa, _), ka = host(16)
    (pb, _), kb = host(16)
    (pc, _), kc = host(16, np.int32)
    a = gk.MatRef((pa, 16), 4, 4, 4, 1)
    b = gk.MatRef((pb, 16), 3, 4, 4, 1)
    c = gk.MatMut((pc, 16), 4, 4, 4, 1)
    expect_err(lambda: gk.gemm_i8(1, a, b, 0, c), "gemmkit: A.cols (4) != B.rows (3)")
    b = gk.MatRef((pb, 16), 4, 4, 4, 1)
    c2 = gk.MatMut((pc, 16), 3, 4, 4, 1)
    expect_err(lambda: gk.gemm_i8(1, a, b, 0, c2), "gemmkit: A.rows (4) != C.rows (3)")
    c3 = gk.MatMut((pc, 16), 4, 3, 4, 1)
    expect_err(lambda: gk.gemm_i8(1, a, b, 0, c3), "gemmkit: B.cols (4) != C.cols (3)")


def test_view_bounds_and_alias_messages():
    (pa, _), ka = host(16)
    (pb, _), kb = host(16)
    (pc, _), kc = host(16, np.int32)
    a_short = gk.MatRef((pa, 15), 4, 4, 4, 1)
    b = gk.MatRef((pb, 16), 4, 4, 4, 1)
    c = gk.MatMut((pc, 16), 4, 4, 4, 1)
    expect_err(lambda: gk.gemm_i8(1, a_short, b, 0, c),
               "gemmkit: A view of 4x4 (strides 4,1) needs 16 elements but slice has 15")
    a_neg = gk.MatRef((pa, 16), 4, 4, -4, 1)
    expect_err(lambda: gk.gemm_i8(1, a_neg, b, 0, c),
               "gemmkit: A view has negative strides or is too large to address; use gemm_unchecked")
    a = gk.MatRef((pa, 16), 4, 4, 4, 1)
    c_alias = gk.MatMut((pc, 16), 4, 4, 0, 1)
    expect_err(lambda: gk.gemm_i8(1, a, b, 0, c_alias), "C view aliases itself (strides 0,1")
    # C overlapping A (byte ranges), as gemmkit's validate_gemm_views
    c_over = gk.MatMut((pa, 4), 2, 2, 2, 1)
    a2 = gk.MatRef((pa, 16), 2, 8, 8, 1)
    b2 = gk.MatRef((pb, 16), 8, 2, 2, 1)
    expect_err(lambda: gk.gemm_i8(1, a2, b2, 0, c_over), "gemmkit: C aliases A or B")


def requant_call(scale=gk.RequantScale.PerTensor(0.5), zp=0, bias=None, u8=False):
    (pa, _), ka = host(16)
    (pb, _), kb = host(16)
    (pc, _), kc = host(16, np.int8)
    a = gk.MatRef((pa, 16), 4, 4, 4, 1)
    b = gk.MatRef((pb, 16), 4, 4, 4, 1)
    c = gk.MatMut((pc, 16), 4, 4, 4, 1)
    req = gk.Requantize(scale, zp, bias)
    fn = gk.gemm_i8_requant_u8 if u8 else gk.gemm_i8_requant
    return lambda: fn(a, b, req, c, sync=False), (ka, kb, kc)


@pytest.mark.parametrize("bad", [0.0, -1.0, float("nan"), float("inf")])
def test_requant_bad_scale(bad):
    """gemmkit/tests/epilogue/requant.rs:578 (expected = "scale")."""
    fn, keep = requant_call(scale=gk.RequantScale.PerTensor(bad))
    want = {0.0: "(0)", -1.0: "(-1)"}.get(bad, "")
    expect_err(fn, f"gemmkit: requantize scale {want}".rstrip() if want else "must be finite and > 0")


def test_requant_bad_zp():
    """requant.rs:599 / :1053 / :1074 (expected = "zero_point")."""
    fn, keep = requant_call(zp=128)
    expect_err(fn, "gemmkit: requantize zero_point (128) out of i8 range [-128, 127]")
    fn, keep = requant_call(zp=-129)
    expect_err(fn, "zero_point (-129) out of i8 range")
    fn, keep = requant_call(zp=256, u8=True)
    expect_err(fn, "gemmkit: requantize zero_point (256) out of u8 range [0, 255]")
    fn, keep = requant_call(zp=-1, u8=True)
    expect_err(fn, "zero_point (-1) out of u8 range")


def test_requant_bad_bias_len_and_overlap():
    """requant.rs:620 / :1095 (expected = "bias length")."""
    bias = np.zeros(3, np.int32)
    fn, keep = requant_call(bias=(bias.ctypes.data, 3))
    expect_err(fn, "gemmkit: requantize bias length (3) != A.rows (4)")
    (pa, _), ka = host(16)
    (pb, _), kb = host(16)
    cbuf = np.zeros(64, np.int8)
    a = gk.MatRef((pa, 16), 4, 4, 4, 1)
    b = gk.MatRef((pb, 16), 4, 4, 4, 1)
    c = gk.MatMut((cbuf.ctypes.data, 16), 4, 4, 4, 1)
    req = gk.Requantize(gk.RequantScale.PerTensor(1.0), 0, (cbuf.ctypes.data + 4, 4))
    expect_err(lambda: gk.gemm_i8_requant(a, b, req, c, sync=False),
               "gemmkit: requantize bias overlaps C")


def test_requant_per_row_scale_len_and_overlap():
    """requant.rs:1461 (expected = "scales length"), :1527 ("scales overlap C")."""
    s = np.ones(3, np.float32)
    fn, keep = requant_call(scale=gk.RequantScale.PerRow((s.ctypes.data, 3)))
    expect_err(fn, "gemmkit: requantize scales length (3) != A.rows (4)")
    (pa, _), ka = host(16)
    (pb, _), kb = host(16)
    cbuf = np.zeros(64, np.int8)
    a = gk.MatRef((pa, 16), 4, 4, 4, 1)
    b = gk.MatRef((pb, 16), 4, 4, 4, 1)
    c = gk.MatMut((cbuf.ctypes.data, 16), 4, 4, 4, 1)
    req = gk.Requantize(gk.RequantScale.PerRow((cbuf.ctypes.data + 8, 4)), 0)
    expect_err(lambda: gk.gemm_i8_requant(a, b, req, c, sync=False),
               "gemmkit: requantize scales overlap C")


def test_packed_b_requires_colmajor_c():
    lib = _lib.load()
    rc = lib.gk_gemm_i8_packed_b_unchecked(None, 1, 4, 0, 4, 1, C.c_void_p(1), 0, 0, 4, 1,
                                           _lib.Parallelism(0, 0), None)
    assert rc == gk.GK_EINVAL
    assert "requires column-major-ish C (|csc| >= |rsc|)" in _lib.last_error()


def test_rust_float_formatting_in_messages():
    for v, txt in [(1e-30, "0.000000000000000000000000000001"), (-2.5, "-2.5"),
                   (float("-inf"), "-inf"), (0.0, "0")]:
        fn, keep = requant_call(scale=gk.RequantScale.PerTensor(v))
        if v > 0:
            continue
        expect_err(fn, f"gemmkit: requantize scale ({txt}) must be finite and > 0")


def test_valid_call_without_gpu_fails_loudly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    (pa, _), ka = host(16)
    (pb, _), kb = host(16)
    (pc, _), kc = host(16, np.int32)
    a = gk.MatRef((pa, 16), 4, 4, 4, 1)
    b = gk.MatRef((pb, 16), 4, 4, 4, 1)
    c = gk.MatMut((pc, 16), 4, 4, 4, 1)
    with pytest.raises(gk.GemmkitError) as ei:
        gk.gemm_i8(1, a, b, 0, c, sync=False)
    assert ei.value.code in (gk.GK_ENODEV,), str(ei.value)
    assert kc.sum() == 0  # nothing computed on the host


def test_empty_problem_is_noop_without_device():
    lib = _lib.load()
    rc = lib.gk_gemm_i8_unchecked(None, 0, 5, 5, 1, None, 0, 0, None, 0, 0, 0, None, 0, 0,
                                  _lib.Parallelism(0, 0), None)
    assert rc == gk.GK_OK


def test_set_tile_n_validation():
    gk.set_tile_n(0)
    with pytest.raises(gk.GemmkitError):
        gk.set_tile_n(48)


def test_mirrored_entries_argument_errors():
    """The mirrored-output extensions reject bad mirror lists before touching a device."""
    import ctypes as C
    lib = _lib.load()
    one = (C.c_void_p * 8)(*([C.c_void_p(16)] * 8))
    rc = lib.gk_gemm_half_f32_mirrored_unchecked(None, 0, 4, 4, 4, 1.0, C.c_void_p(16), 4, 1,
                                                 C.c_void_p(16), 4, 1, 0.0, C.c_void_p(16), 4, 1,
                                                 one, 8, None)
    assert rc == _lib.GK_EINVAL and b"at most 7 mirrored outputs" in lib.gk_last_error()
    rc = lib.gk_gemm_half_f32_mirrored_unchecked(None, 0, 4, 4, 4, 1.0, C.c_void_p(16), 4, 1,
                                                 C.c_void_p(16), 4, 1, 0.0, C.c_void_p(16), 4, 1,
                                                 None, 2, None)
    assert rc == _lib.GK_EINVAL and b"null mirror list" in lib.gk_last_error()
    nulls = (C.c_void_p * 2)(C.c_void_p(16), None)
    rc = lib.gk_gemm_i8_requant_mirrored_unchecked(
        None, 1, 4, 4, 4, C.c_void_p(16), 4, 1, 0, C.c_void_p(16), 4, 1, 0, None,
        C.byref(_lib.RequantC(1.0)), 0, 0, C.c_void_p(16), 4, 1, 0, 0, nulls, 2, None)
    assert rc == _lib.GK_EINVAL and b"null mirrored output 1" in lib.gk_last_error()


def test_ipc_entries_argument_errors():
    import ctypes as C
    lib = _lib.load()
    assert lib.gk_ipc_export(None, None) == _lib.GK_EINVAL
    assert lib.gk_ipc_open(None, None) == _lib.GK_EINVAL
    assert lib.gk_ipc_close(C.c_void_p(12345)) == _lib.GK_EINVAL
    assert b"not opened by gk_ipc_open" in lib.gk_last_error()
    assert lib.gk_ipc_close(None) == _lib.GK_OK


def test_knobs_get_set_and_validation():
    import gemmkit_b200 as gk
    names = gk.knob_names()
    assert names == ["GEMMKIT_CUDA_BN", "GEMMKIT_CUDA_PAIR", "GEMMKIT_CUDA_GEMV",
                     "GEMMKIT_CUDA_PDL", "GEMMKIT_CUDA_STREAMK", "GEMMKIT_CUDA_GEMV_SK",
                     "GEMMKIT_CUDA_BN_SHORTK", "GEMMKIT_CUDA_EPI16", "GEMMKIT_CUDA_STAGES",
                     "GEMMKIT_CUDA_GEMV_SPLIT", "GEMMKIT_CUDA_MN_B", "GEMMKIT_CUDA_REQUANT_F32"]
    base = {n: gk.knob_get(n) for n in names}
    try:
        gk.knob_set("GEMMKIT_CUDA_BN", 128)
        assert gk.knob_get("GEMMKIT_CUDA_BN") == 128
        gk.knob_set("GEMMKIT_CUDA_PAIR", 0)
        assert gk.knob_get("GEMMKIT_CUDA_PAIR") == 0
        with pytest.raises(gk.GemmkitError, match="cannot be 100"):
            gk.knob_set("GEMMKIT_CUDA_BN", 100)
        with pytest.raises(gk.GemmkitError, match="cannot be 2"):
            gk.knob_set("GEMMKIT_CUDA_PDL", 2)
        with pytest.raises(gk.GemmkitError, match="unknown knob"):
            gk.knob_set("GEMMKIT_CUDA_NOPE", 1)
        gk.knob_set("GEMMKIT_CUDA_STAGES", 4)
        assert gk.knob_get("GEMMKIT_CUDA_STAGES") == 4
        with pytest.raises(gk.GemmkitError, match="cannot be 1"):
            gk.knob_set("GEMMKIT_CUDA_STAGES", 1)
        gk.knob_set("GEMMKIT_CUDA_GEMV_SPLIT", 8)
        with pytest.raises(gk.GemmkitError, match="cannot be 9"):
            gk.knob_set("GEMMKIT_CUDA_GEMV_SPLIT", 9)
        gk.knob_set("GEMMKIT_CUDA_BN_SHORTK", 192)
        assert gk.knob_get("GEMMKIT_CUDA_BN_SHORTK") == 192
    finally:
        for n in names:
            gk.knob_set(n, -1)  # drop the overrides
    assert {n: gk.knob_get(n) for n in names} == base


def test_fused_bias_validation_without_gpu():
    """The checked fused entry rejects a bias whose length does not follow its dimension,
    before any device work."""
    a = gk.MatRef.new((16, 6), 2, 3, 3, 1)
    b = gk.MatRef.new((16, 12), 3, 4, 4, 1)
    c = gk.MatMut.new((64, 8), 2, 4, 4, 1)
    with pytest.raises(gk.GemmkitError, match="per-column bias length 3 does not match n = 4"):
        gk.gemm_half_f32_fused(1.0, a, b, 0.0, c, bias=(128, 3), bias_dim=gk.AXIS_COL)
    with pytest.raises(gk.GemmkitError, match="per-row bias length 4 does not match m = 2"):
        gk.gemm_half_f32_fused(1.0, a, b, 0.0, c, bias=(128, 4), bias_dim=gk.AXIS_ROW)
    lib = _lib.load()
    rc = lib.gk_gemm_half_f32_fused_unchecked(None, 0, 2, 3, 4, 1.0, C.c_void_p(16), 3, 1,
                                              C.c_void_p(16), 4, 1, 0.0, C.c_void_p(16), 4, 1,
                                              None, 1, 0, 7, 0.0, _lib.Parallelism(0, 0), None)
    assert rc == _lib.GK_EINVAL and b"unknown activation 7" in lib.gk_last_error()


def test_fused_i32_validation_without_gpu():
    """The fused i32 entries reject a LeakyReLU (its slope is a float), an unknown activation,
    a bias dimension that is neither row nor column, and (checked tier) a bias whose length
    does not follow its dimension -- all before any device work."""
    a = gk.MatRef.new((16, 6), 2, 3, 3, 1)
    b = gk.MatRef.new((16, 12), 3, 4, 4, 1)
    c = gk.MatMut.new((64, 8), 2, 4, 4, 1)
    with pytest.raises(gk.GemmkitError, match="per-column bias length 3 does not match n = 4"):
        gk.gemm_i8_fused(1, a, b, 0, c, bias=(128, 3), bias_dim=gk.AXIS_COL)
    with pytest.raises(gk.GemmkitError, match="per-row bias length 4 does not match m = 2"):
        gk.gemm_i8_fused(1, a, b, 0, c, bias=(128, 4), bias_dim=gk.AXIS_ROW)
    with pytest.raises(gk.GemmkitError, match="no LeakyReLU"):
        gk.gemm_i8_fused(1, a, b, 0, c, act=gk.Activation.LeakyRelu(0.1))
    lib = _lib.load()
    args = (None, 2, 3, 4, 1, C.c_void_p(16), 3, 1, C.c_void_p(16), 4, 1, 0, C.c_void_p(16), 4,
            1)
    rc = lib.gk_gemm_i8_fused_unchecked(*args, None, 1, 0, 9, _lib.Parallelism(0, 0), None)
    assert rc == _lib.GK_EINVAL and b"unknown activation 9" in lib.gk_last_error()
    rc = lib.gk_gemm_i8_fused_unchecked(*args, C.c_void_p(16), 5, 1, 1, _lib.Parallelism(0, 0),
                                        None)
    assert rc == _lib.GK_EINVAL and b"bias dimension" in lib.gk_last_error()
    rc = lib.gk_gemm_i8_fused_unchecked(*args, None, 1, 1, 1, _lib.Parallelism(0, 0), None)
    assert rc == _lib.GK_EINVAL and b"null bias" in lib.gk_last_error()


def test_quantize_argument_errors_without_gpu():
    lib = _lib.load()
    rc = lib.gk_quantize_f32_i8_unchecked(2, 2, C.c_void_p(16), 2, 1, C.c_void_p(16), 2, 1,
                                          -1.0, 0, None, None)
    assert rc == _lib.GK_EINVAL
    rc = lib.gk_quantize_f32_i8_unchecked(2, 2, C.c_void_p(16), 2, 1, C.c_void_p(16), 2, 1,
                                          0.5, 200, None, None)
    assert rc == _lib.GK_EINVAL and b"zero point 200" in lib.gk_last_error()
    assert lib.gk_quantize_f32_i8_unchecked(0, 5, None, 0, 0, None, 0, 0, 1.0, 0, None,
                                            None) == _lib.GK_OK


def test_packed_deserialize_rejects_bad_input_without_gpu():
    """Header checks run before any device work."""
    import struct
    lib = _lib.load()
    out = C.c_void_p()
    assert lib.gk_packed_rhs_deserialize(b"short", 5, None, C.byref(out)) == _lib.GK_EINVAL
    assert b"truncated" in lib.gk_last_error()
    bad = b"NOTPACK!" + bytes(56)
    assert lib.gk_packed_rhs_deserialize(bad, 64, None, C.byref(out)) == _lib.GK_EINVAL
    assert b"bad magic" in lib.gk_last_error()
    hdr = b"GKPACK01" + struct.pack("<7Q", 100, 10, 128, 256, 9, 128 * 256, 0)
    assert lib.gk_packed_rhs_deserialize(hdr, 64, None, C.byref(out)) == _lib.GK_EINVAL
    assert b"unknown layout 9" in lib.gk_last_error()
    hdr = b"GKPACK01" + struct.pack("<7Q", 100, 10, 256, 256, 1, 256 * 256, 0)
    assert lib.gk_packed_rhs_deserialize(hdr, 64, None, C.byref(out)) == _lib.GK_EINVAL
    assert b"inconsistent dimensions" in lib.gk_last_error()
    hdr = b"GKPACK01" + struct.pack("<7Q", 100, 10, 128, 256, 1, 128 * 256, 0)
    assert lib.gk_packed_rhs_deserialize(hdr, 64 + 100, None, C.byref(out)) == _lib.GK_EINVAL
    assert b"truncated" in lib.gk_last_error()


def test_gemv_entry_row_range():
    """gk_gemv_i8_requant_unchecked takes 1 to 64 activation rows; checked before any device
    work, so it needs no GPU."""
    class _NoPack:
        h = None
    req = gk.Requantize(gk.RequantScale.PerTensor(0.01), 0)
    for m in (0, 65):
        expect_err(lambda: gk.gemv_i8_requant(m, 0, 1, 1, _NoPack(), req, 0, 1, 1),
                   "gemv takes 1 to 64 activation rows")
