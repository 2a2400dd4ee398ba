"""ctypes binding of libgemmkit_cuda.so (the C ABI declared in include/gemmkit_cuda.h).

The library is the product; this module only loads it and declares the signatures. It
fails loudly when the library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

from . import _build

GK_OK, GK_EINVAL, GK_ENOMEM, GK_ECUDA, GK_ETIMEOUT, GK_ENODEV = range(6)
AXIS_NONE, AXIS_ROW, AXIS_COL = 0, 1, 2
ACT_NONE, ACT_RELU, ACT_LEAKY_RELU = 0, 1, 2

sz, pd, vp, i32, u32, f32 = C.c_size_t, C.c_ssize_t, C.c_void_p, C.c_int32, C.c_uint32, C.c_float


class Parallelism(C.Structure):
    _fields_ = [("kind", i32), ("threads", i32)]


class MatRefC(C.Structure):
    _fields_ = [("data", vp), ("len", sz), ("rows", sz), ("cols", sz), ("rs", pd), ("cs", pd)]


class MatMutC(C.Structure):
    _fields_ = [("data", vp), ("len", sz), ("rows", sz), ("cols", sz), ("rs", pd), ("cs", pd)]


class RequantC(C.Structure):
    _fields_ = [("scale", f32), ("scales", vp), ("scale_axis", i32), ("zero_point", i32),
                ("bias", vp), ("bias_axis", i32), ("relu", i32), ("scales_len", sz),
                ("bias_len", sz)]


class IpcHandleC(C.Structure):
    _fields_ = [("bytes", C.c_ubyte * 64), ("offset", C.c_uint64)]


class ProblemC(C.Structure):
    _fields_ = [("m", sz), ("k", sz), ("n", sz), ("a", vp), ("rsa", pd), ("csa", pd),
                ("b", vp), ("rsb", pd), ("csb", pd), ("c", vp), ("rsc", pd), ("csc", pd),
                ("req", RequantC)]


SIGNATURES = {
    "gk_version": (C.c_char_p, []),
    "gk_last_error": (C.c_char_p, []),
    "gk_device_status": (i32, [C.c_int, C.c_int, C.POINTER(u32)]),
    "gk_workspace_create": (i32, [C.POINTER(vp)]),
    "gk_workspace_free": (None, [vp]),
    "gk_gemm_i8_unchecked": (i32, [vp, sz, sz, sz, i32, vp, pd, pd, vp, pd, pd, i32, vp, pd, pd,
                                   Parallelism, vp]),
    "gk_gemm_i8": (i32, [vp, i32, MatRefC, MatRefC, i32, MatMutC, Parallelism, vp]),
    "gk_gemm_i8_requant_unchecked": (i32, [vp, sz, sz, sz, vp, pd, pd, vp, pd, pd, f32, vp,
                                           C.c_int, i32, vp, C.c_int, vp, pd, pd, Parallelism,
                                           vp]),
    "gk_gemm_i8_requant_u8_unchecked": (i32, [vp, sz, sz, sz, vp, pd, pd, vp, pd, pd, f32, vp,
                                              C.c_int, i32, vp, C.c_int, vp, pd, pd,
                                              Parallelism, vp]),
    "gk_gemm_i8_requant": (i32, [vp, MatRefC, MatRefC, C.POINTER(RequantC), MatMutC, C.c_int,
                                 Parallelism, vp]),
    "gk_gemm_i8_requant_ex_unchecked": (i32, [vp, sz, sz, sz, vp, pd, pd, vp, pd, pd,
                                              C.POINTER(RequantC), vp, pd, pd, C.c_int,
                                              Parallelism, vp]),
    "gk_prepack_rhs_i8_unchecked": (i32, [vp, pd, pd, sz, sz, vp, C.POINTER(vp)]),
    "gk_prepack_rhs_i8": (i32, [MatRefC, vp, C.POINTER(vp)]),
    "gk_packed_rhs_free": (None, [vp]),
    "gk_packed_rhs_rows": (sz, [vp]),
    "gk_packed_rhs_serialize": (i32, [vp, vp, sz, C.POINTER(sz)]),
    "gk_packed_rhs_deserialize": (i32, [vp, sz, vp, C.POINTER(vp)]),
    "gk_packed_rhs_cols": (sz, [vp]),
    "gk_gemm_i8_packed_b_unchecked": (i32, [vp, i32, sz, vp, pd, pd, vp, i32, vp, pd, pd,
                                            Parallelism, vp]),
    "gk_gemm_i8_packed_b": (i32, [vp, i32, MatRefC, vp, i32, MatMutC, Parallelism, vp]),
    "gk_gemm_i8_packed_b_requant_unchecked": (i32, [vp, sz, vp, pd, pd, vp, C.POINTER(RequantC),
                                                    vp, pd, pd, C.c_int, Parallelism, vp]),
    "gk_gemv_i8_requant_unchecked": (i32, [vp, sz, vp, pd, pd, vp, C.POINTER(RequantC), vp, pd,
                                           pd, C.c_int, vp]),
    "gk_gemm_i8_requant_batched_unchecked": (i32, [vp, sz, sz, sz, sz, vp, pd, pd, pd, vp, pd,
                                                   pd, pd, C.POINTER(RequantC), pd, pd, vp, pd,
                                                   pd, pd, C.c_int, Parallelism, vp]),
    "gk_gemm_i8_requant_batched_ptr_unchecked": (i32, [vp, C.POINTER(ProblemC), sz, C.c_int,
                                                       Parallelism, vp]),
    "gk_gemm_bf16_f32_unchecked": (i32, [vp, sz, sz, sz, f32, vp, pd, pd, vp, pd, pd, f32, vp,
                                         pd, pd, Parallelism, vp]),
    "gk_gemm_f16_f32_unchecked": (i32, [vp, sz, sz, sz, f32, vp, pd, pd, vp, pd, pd, f32, vp,
                                        pd, pd, Parallelism, vp]),
    "gk_gemm_half_f32": (i32, [vp, C.c_int, f32, MatRefC, MatRefC, f32, MatMutC, Parallelism,
                               vp]),
    "gk_gemm_half_f32_batched_unchecked": (i32, [vp, C.c_int, sz, sz, sz, sz, f32, vp, pd, pd,
                                                 pd, vp, pd, pd, pd, f32, vp, pd, pd, pd,
                                                 Parallelism, vp]),
    "gk_gemm_i8_noalloc_unchecked": (i32, [sz, sz, sz, i32, vp, pd, pd, vp, pd, pd, i32, vp, pd,
                                           pd, vp]),
    "gk_ipc_export": (i32, [vp, C.POINTER(IpcHandleC)]),
    "gk_ipc_open": (i32, [C.POINTER(IpcHandleC), C.POINTER(vp)]),
    "gk_ipc_close": (i32, [vp]),
    "gk_gemm_half_f32_mirrored_unchecked": (i32, [vp, C.c_int, sz, sz, sz, f32, vp, pd, pd, vp,
                                                  pd, pd, f32, vp, pd, pd, C.POINTER(vp),
                                                  C.c_int, vp]),
    "gk_gemm_i8_requant_mirrored_unchecked": (i32, [vp, sz, sz, sz, sz, vp, pd, pd, pd, vp, pd,
                                                    pd, pd, vp, C.POINTER(RequantC), pd, pd, vp,
                                                    pd, pd, pd, C.c_int, C.POINTER(vp), C.c_int,
                                                    vp]),
    "gk_gemm_half_f32_fused_unchecked": (i32, [vp, C.c_int, sz, sz, sz, f32, vp, pd, pd, vp, pd,
                                               pd, f32, vp, pd, pd, vp, C.c_int, C.c_int,
                                               C.c_int, f32, Parallelism, vp]),
    "gk_gemm_half_f32_fused": (i32, [vp, C.c_int, f32, MatRefC, MatRefC, f32, MatMutC, vp, sz,
                                     C.c_int, C.c_int, f32, Parallelism, vp]),
    "gk_gemm_i8_fused_unchecked": (i32, [vp, sz, sz, sz, i32, vp, pd, pd, vp, pd, pd, i32, vp, pd,
                                         pd, vp, C.c_int, C.c_int, C.c_int, Parallelism, vp]),
    "gk_gemm_i8_fused": (i32, [vp, i32, MatRefC, MatRefC, i32, MatMutC, vp, sz, C.c_int, C.c_int,
                               Parallelism, vp]),
    "gk_quantize_f32_i8_unchecked": (i32, [sz, sz, vp, pd, pd, vp, pd, pd, f32, i32, vp, vp]),
    "gk_set_tile_n": (i32, [C.c_int]),
    "gk_knob_names": (C.c_char_p, []),
    "gk_knob_get": (i32, [C.c_char_p, C.POINTER(C.c_int64)]),
    "gk_knob_set": (i32, [C.c_char_p, C.c_int64]),
    "gk_selftest_wait_timeout": (i32, [C.c_uint64, vp]),
}

_lib = None


def lib_path() -> str:
    return _build.LIB


def load() -> C.CDLL:
    """Load the engine library (built in-tree). Raises if it is missing or incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise RuntimeError(
            f"gemmkit_b200: CUDA engine library not found at {path}; "
            "build it with `python -m gemmkit_b200._build` (there is no CPU fallback)")
    L = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    return load().gk_last_error().decode()
