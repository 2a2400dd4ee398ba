"""numpy front end of the CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference legs import
this package, and only as the checker or the timed CPU baseline. The product library
(gemmkit_b200, libgemmkit_cuda.so) never imports it.

The C sources restate gemmkit's algorithm (Rust, v0.1.2); each C function cites the gemmkit
file:line it follows. Parity pin: tests/test_oracle.py checks these functions against the
known-answer vectors hard-coded in the reference's own tests (tests/golden/kat.json) and the
reference tests' independent ``round_ties_even`` model on their own xorshift* inputs.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build as _build

AXIS = {"none": 0, "row": 1, "col": 2}

_lib = None


class Requant(C.Structure):
    _fields_ = [("scale", C.c_float), ("scales", C.c_void_p), ("scale_axis", C.c_int32),
                ("zp", C.c_int32), ("bias", C.c_void_p), ("bias_axis", C.c_int32),
                ("relu", C.c_int32), ("out_u8", C.c_int32)]


class PackedRhs(C.Structure):
    _fields_ = [("buf", C.c_void_p), ("colsum", C.c_void_p), ("k", C.c_size_t),
                ("n", C.c_size_t), ("k_pad", C.c_size_t), ("n_pad", C.c_size_t)]


def lib():
    global _lib
    if _lib is None:
        path = _build.LIB
        if not os.path.exists(path):
            path = _build.build()
        L = C.CDLL(path)
        sz, pd, vp, i32 = C.c_size_t, C.c_ssize_t, C.c_void_p, C.c_int32
        L.gko_round_ne_f64.restype = C.c_double
        L.gko_round_ne_f64.argtypes = [C.c_double]
        L.gko_requant_apply.restype = i32
        L.gko_requant_apply.argtypes = [i32, i32, C.c_float, i32, i32, i32, i32]
        L.gko_gemm_i8.argtypes = [sz, sz, sz, i32, vp, pd, pd, vp, pd, pd, i32, vp, pd, pd]
        L.gko_gemm_i8_requant.argtypes = [sz, sz, sz, vp, pd, pd, vp, pd, pd,
                                          C.POINTER(Requant), vp, pd, pd]
        L.gko_acc_i8.argtypes = [sz, sz, sz, vp, pd, pd, vp, pd, pd, vp]
        L.gko_f32_to_bf16.restype = C.c_uint16
        L.gko_f32_to_bf16.argtypes = [C.c_float]
        L.gko_bf16_to_f32.restype = C.c_float
        L.gko_bf16_to_f32.argtypes = [C.c_uint16]
        L.gko_f16_to_f32.restype = C.c_float
        L.gko_f16_to_f32.argtypes = [C.c_uint16]
        L.gko_gemm_half_f64.argtypes = [C.c_int, sz, sz, sz, C.c_double, vp, pd, pd, vp, pd, pd,
                                        C.c_double, vp, pd, pd, vp]
        L.gko_cpu_has_vnni.restype = C.c_int
        L.gko_threads.restype = C.c_int
        L.gko_threads.argtypes = [C.c_int]
        L.gko_vnni_prepack.restype = C.c_int
        L.gko_vnni_prepack.argtypes = [vp, pd, pd, sz, sz, C.POINTER(PackedRhs)]
        L.gko_vnni_packed_free.argtypes = [C.POINTER(PackedRhs)]
        L.gko_vnni_gemm_i8_requant_packed.argtypes = [sz, vp, pd, pd, C.POINTER(PackedRhs),
                                                      C.POINTER(Requant), vp, pd, pd, C.c_int]
        L.gko_vnni_gemm_i8_packed.argtypes = [sz, i32, vp, pd, pd, C.POINTER(PackedRhs), i32,
                                              vp, pd, pd, C.c_int]
        L.gko_cpu_gemm_bf16_f32.argtypes = [sz, sz, sz, C.c_float, vp, pd, pd, vp, pd, pd,
                                            C.c_float, vp, pd, pd, C.c_int]
        _lib = L
    return _lib


def _ptr(x: np.ndarray | None, off: int = 0):
    if x is None:
        return None
    return x.ctypes.data + off * x.itemsize


def round_ne_f64(x: float) -> float:
    return lib().gko_round_ne_f64(float(x))


def requant_apply(v: int, bias: int, scale: float, zp: int, lo: int, hi: int,
                  relu: bool = False) -> int:
    return lib().gko_requant_apply(int(v), int(bias), float(scale), int(zp), int(lo), int(hi),
                                   int(relu))


class View:
    """A strided view (gemmkit MatRef / MatMut): element (i, j) at ``base + i*rs + j*cs``
    of the flat array ``buf``; ``base`` lets negative strides start mid-buffer."""

    def __init__(self, buf: np.ndarray, rows: int, cols: int, rs: int, cs: int, base: int = 0):
        self.buf, self.rows, self.cols, self.rs, self.cs, self.base = buf, rows, cols, rs, cs, base

    def ptr(self):
        return _ptr(self.buf, self.base)


def gemm_i8(alpha: int, a: View, b: View, beta: int, c: View) -> None:
    lib().gko_gemm_i8(a.rows, a.cols, b.cols, alpha, a.ptr(), a.rs, a.cs, b.ptr(), b.rs, b.cs,
                      beta, c.ptr(), c.rs, c.cs)


def make_requant(scale=1.0, scales=None, scale_axis="none", zp=0, bias=None, bias_axis="none",
                 relu=False, out_u8=False) -> tuple[Requant, list]:
    keep = []
    if scales is not None:
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        keep.append(scales)
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.int32)
        keep.append(bias)
    r = Requant(float(scale), _ptr(scales), AXIS[scale_axis] if scales is not None else 0,
                int(zp), _ptr(bias), AXIS[bias_axis] if bias is not None else 0, int(relu),
                int(out_u8))
    return r, keep


def gemm_i8_requant(a: View, b: View, c: View, **req) -> None:
    r, keep = make_requant(**req)
    lib().gko_gemm_i8_requant(a.rows, a.cols, b.cols, a.ptr(), a.rs, a.cs, b.ptr(), b.rs, b.cs,
                              C.byref(r), c.ptr(), c.rs, c.cs)
    del keep


def acc_i8(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Exact wrapping i32 accumulator of row-major a (m x k) times row-major b (k x n)."""
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), dtype=np.int32)
    lib().gko_acc_i8(m, k, n, _ptr(a), k, 1, _ptr(b), n, 1, _ptr(out))
    return out


def requant_matrix(a: np.ndarray, b: np.ndarray, *, out_u8=False, **req) -> np.ndarray:
    """Row-major requantized product of row-major a (m x k) and b (k x n)."""
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), dtype=np.uint8 if out_u8 else np.int8)
    gemm_i8_requant(View(a.reshape(-1), m, k, k, 1), View(b.reshape(-1), k, n, n, 1),
                    View(out.reshape(-1), m, n, n, 1), out_u8=out_u8, **req)
    return out


def gemm_i8_matrix(alpha: int, a: np.ndarray, b: np.ndarray, beta: int,
                   c: np.ndarray | None = None) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    m, k = a.shape
    n = b.shape[1]
    out = np.zeros((m, n), dtype=np.int32) if c is None else np.array(c, dtype=np.int32)
    gemm_i8(alpha, View(a.reshape(-1), m, k, k, 1), View(b.reshape(-1), k, n, n, 1), beta,
            View(out.reshape(-1), m, n, n, 1))
    return out


def gemm_i8_fused_matrix(alpha: int, a: np.ndarray, b: np.ndarray, beta: int,
                         c: np.ndarray | None = None, bias: np.ndarray | None = None,
                         bias_axis: str = "row", relu: bool = False) -> np.ndarray:
    """act(alpha*A*B + beta*C + bias) for the fused i32 epilogue (an engine extension): the
    scalar restatement of int32_epilogue (gko_gemm_i8) followed by the bias-then-activation
    composition of gemmkit's FusedEpi::apply (gemmkit/src/kernel/epilogue.rs:300-330), here in
    wrapping i32: v + bias mod 2^32, then ReLU as max(v, 0)."""
    out = gemm_i8_matrix(alpha, a, b, beta, c).astype(np.int64)
    if bias is not None:
        bv = np.asarray(bias, dtype=np.int64)
        out = out + (bv[:, None] if bias_axis == "row" else bv[None, :])
        out = ((out + 2**31) % 2**32) - 2**31
    if relu:
        out = np.maximum(out, 0)
    return out.astype(np.int32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16), NaN kept quiet."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u.astype(np.uint64) + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def gemm_half_f64(a: np.ndarray, b: np.ndarray, alpha: float, beta: float,
                  c: np.ndarray | None, is_f16: bool = False) -> np.ndarray:
    """f64 reference of alpha*A*B + beta*C for row-major uint16 bit-pattern operands."""
    a = np.ascontiguousarray(a, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), dtype=np.float64)
    cc = None if c is None else np.ascontiguousarray(c, dtype=np.float32)
    lib().gko_gemm_half_f64(int(is_f16), m, k, n, alpha, _ptr(a), k, 1, _ptr(b), n, 1, beta,
                            _ptr(cc), n, 1, _ptr(out))
    return out


# ---- timed CPU baseline -------------------------------------------------------------------

def has_vnni() -> bool:
    return bool(lib().gko_cpu_has_vnni())


def threads(t: int = 0) -> int:
    return lib().gko_threads(t)


class VnniPacked:
    """gemmkit's VNNI prepacked RHS (k-quad interleave, NR = 12) built by the C baseline."""

    def __init__(self, b: np.ndarray, rsb: int, csb: int, k: int, n: int):
        self._keep = b
        self.p = PackedRhs()
        if lib().gko_vnni_prepack(_ptr(b), rsb, csb, k, n, C.byref(self.p)) != 0:
            raise MemoryError("oracle prepack failed")
        self.k, self.n = k, n

    def __del__(self):
        if getattr(self, "p", None) is not None and self.p.buf:
            lib().gko_vnni_packed_free(C.byref(self.p))


def vnni_requant_packed(a: View, pb: VnniPacked, c: View, n_threads: int = 0, **req) -> None:
    r, keep = make_requant(**req)
    lib().gko_vnni_gemm_i8_requant_packed(a.rows, a.ptr(), a.rs, a.cs, C.byref(pb.p), C.byref(r),
                                          c.ptr(), c.rs, c.cs, n_threads)
    del keep


def vnni_gemm_i8_packed(alpha: int, a: View, pb: VnniPacked, beta: int, c: View,
                        n_threads: int = 0) -> None:
    lib().gko_vnni_gemm_i8_packed(a.rows, alpha, a.ptr(), a.rs, a.cs, C.byref(pb.p), beta,
                                  c.ptr(), c.rs, c.cs, n_threads)


def cpu_gemm_bf16_f32(alpha: float, a: View, b: View, beta: float, c: View,
                      n_threads: int = 0) -> None:
    lib().gko_cpu_gemm_bf16_f32(a.rows, a.cols, b.cols, alpha, a.ptr(), a.rs, a.cs, b.ptr(),
                                b.rs, b.cs, beta, c.ptr(), c.rs, c.cs, n_threads)
