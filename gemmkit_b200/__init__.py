"""gemmkit_b200 -- gemmkit's quantized-inference GEMM path on NVIDIA B200 (sm_100a).

A Python mirror of gemmkit's Rust API (gemmkit/src/lib.rs:98-148 re-exports) over the C ABI of
``libgemmkit_cuda.so``: the same entry names, argument meaning, view rules and ``gemmkit:``
error messages (raised as :class:`GemmkitError` where gemmkit panics). Matrices are views
over flat CUDA tensors; calls are enqueued on the current torch stream, and the checked
entries synchronise like gemmkit's blocking calls unless ``sync=False``.

All arithmetic runs in the engine's sm_100a kernels; there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Optional, Sequence

from . import _lib
from ._lib import (AXIS_COL, AXIS_NONE, AXIS_ROW, GK_EINVAL, GK_ENODEV, GK_ENOMEM, GK_ETIMEOUT,
                   GK_OK, MatMutC, MatRefC, ProblemC, RequantC)

__all__ = [
    "GemmkitError", "Parallelism", "MatRef", "MatMut", "Workspace", "RequantScale", "Requantize",
    "PackedRhs", "gemm_i8", "gemm_i8_with", "gemm_i8_unchecked", "gemm_i8_requant",
    "gemv_i8_requant",
    "gemm_i8_requant_u8", "gemm_i8_requant_unchecked", "gemm_i8_requant_u8_unchecked",
    "prepack_rhs_i8", "prepack_rhs_i8_unchecked", "gemm_i8_packed_b", "gemm_i8_packed_b_unchecked",
    "gemm_i8_packed_b_requant", "gemm_i8_requant_batched", "gemm_i8_requant_batched_ptr",
    "gemm_half_f32", "gemm_bf16_f32_unchecked", "gemm_f16_f32_unchecked",
    "gemm_half_f32_batched", "gemm_half_f32_fused", "gemm_i8_fused", "gemm_i8_fused_unchecked", "Activation", "quantize_f32_i8", "gemm_i8_noalloc_unchecked", "set_tile_n", "knob_names", "knob_get",
    "knob_set", "device_status", "selftest_wait_timeout",
]


class GemmkitError(RuntimeError):
    """A rejected call: the engine's status code plus gemmkit's message."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def _check(rc: int) -> None:
    if rc != GK_OK:
        raise GemmkitError(rc, _lib.last_error())


# ---- Parallelism (gemmkit/src/parallel.rs:25-39) -------------------------------------------

class Parallelism:
    """Accepted for API parity; the device engine always uses the whole GPU."""

    def __init__(self, kind: int = 0, threads: int = 0):
        self.kind, self.threads = kind, threads

    @staticmethod
    def Serial() -> "Parallelism":
        return Parallelism(0, 0)

    @staticmethod
    def Rayon(n: int = 0) -> "Parallelism":
        return Parallelism(1, n)

    def c(self) -> _lib.Parallelism:
        return _lib.Parallelism(self.kind, self.threads)


SERIAL = Parallelism.Serial()


def _stream(stream):
    if stream is not None:
        return C.c_void_p(int(stream))
    try:
        import torch
        if torch.cuda.is_available():
            return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    except ImportError:
        pass
    return C.c_void_p(0)


def _sync(stream) -> None:
    import torch
    if torch.cuda.is_available():
        if stream is None:
            torch.cuda.current_stream().synchronize()
        else:
            torch.cuda.synchronize()


# ---- views (gemmkit/src/api.rs:99-186) -------------------------------------------------------

def _flat(data):
    """(pointer, length in elements) of a flat tensor / (ptr, len) pair."""
    if isinstance(data, tuple):
        return int(data[0]), int(data[1])
    return int(data.data_ptr()), int(data.numel())


class MatRef:
    """An immutable strided view: element (i, j) at data[i*rs + j*cs] (gemmkit MatRef)."""

    def __init__(self, data, rows: int, cols: int, rs: int, cs: int):
        self.data, self.rows, self.cols, self.rs, self.cs = data, rows, cols, rs, cs

    @classmethod
    def new(cls, data, rows, cols, rs, cs):
        return cls(data, rows, cols, rs, cs)

    @classmethod
    def from_row_major(cls, data, rows, cols):
        return cls(data, rows, cols, cols, 1)

    @classmethod
    def from_col_major(cls, data, rows, cols):
        return cls(data, rows, cols, 1, rows)

    def c(self) -> MatRefC:
        p, n = _flat(self.data)
        return MatRefC(p, n, self.rows, self.cols, self.rs, self.cs)

    def ptr(self) -> int:
        return _flat(self.data)[0]


class MatMut(MatRef):
    """A mutable strided view (gemmkit MatMut), the output C."""

    def c(self) -> MatMutC:
        p, n = _flat(self.data)
        return MatMutC(p, n, self.rows, self.cols, self.rs, self.cs)


class Workspace:
    """gemmkit::Workspace: reusable device scratch for operand packs (one per stream)."""

    def __init__(self):
        h = C.c_void_p()
        _check(_lib.load().gk_workspace_create(C.byref(h)))
        self.h = h

    def __del__(self):
        try:
            if getattr(self, "h", None) is not None and self.h.value:
                _lib.load().gk_workspace_free(self.h)
                self.h = None
        except Exception:  # interpreter shutdown
            pass


def _ws(ws: Optional[Workspace]):
    return ws.h if ws is not None else None


# ---- requant descriptors (gemmkit/src/api/int8.rs:185-209) ---------------------------------

@dataclass
class RequantScale:
    """PerTensor(s) or PerRow(vector) as gemmkit; PerCol(vector) is the extension."""
    value: float = 1.0
    vector: object = None
    axis: int = AXIS_NONE

    @staticmethod
    def PerTensor(s: float) -> "RequantScale":
        return RequantScale(float(s), None, AXIS_NONE)

    @staticmethod
    def PerRow(v) -> "RequantScale":
        return RequantScale(0.0, v, AXIS_ROW)

    @staticmethod
    def PerCol(v) -> "RequantScale":
        return RequantScale(0.0, v, AXIS_COL)


@dataclass
class Requantize:
    """gemmkit::Requantize plus the extension fields ``bias_axis`` and ``relu``."""
    scale: RequantScale
    zero_point: int = 0
    bias: object = None
    bias_axis: int = AXIS_ROW
    relu: bool = False

    def c(self) -> RequantC:
        key = (self.scale.value, self.scale.axis, id(self.scale.vector), self.zero_point,
               id(self.bias), self.bias_axis, self.relu)
        cached = self.__dict__.get("_c_cache")
        if cached is not None and cached[0] == key:
            return cached[1]
        r = self._build_c()
        self.__dict__["_c_cache"] = (key, r)
        return r

    def _build_c(self) -> RequantC:
        r = RequantC()
        r.scale = self.scale.value
        r.scale_axis = self.scale.axis
        if self.scale.vector is not None:
            p, n = _flat(self.scale.vector)
            r.scales, r.scales_len = p, n
        r.zero_point = int(self.zero_point)
        if self.bias is not None:
            p, n = _flat(self.bias)
            r.bias, r.bias_len, r.bias_axis = p, n, self.bias_axis
        r.relu = 1 if self.relu else 0
        return r


# ---- i8 -> i32 ----------------------------------------------------------------------------

def gemm_i8_with(ws, alpha: int, a: MatRef, b: MatRef, beta: int, c: MatMut,
                 par: Parallelism = SERIAL, stream=None, sync: bool = True) -> None:
    """gemm_i8_with (gemmkit/src/api/int8.rs:38): C(i32) <- alpha*A*B + beta*C, wrapping."""
    _check(_lib.load().gk_gemm_i8(_ws(ws), alpha, a.c(), b.c(), beta, c.c(), par.c(),
                                  _stream(stream)))
    if sync:
        _sync(stream)


def gemm_i8(alpha: int, a: MatRef, b: MatRef, beta: int, c: MatMut,
            par: Parallelism = SERIAL, stream=None, sync: bool = True) -> None:
    """gemm_i8 (gemmkit/src/api/int8.rs:22)."""
    gemm_i8_with(None, alpha, a, b, beta, c, par, stream, sync)


def gemm_i8_unchecked(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc,
                      par: Parallelism = SERIAL, ws=None, stream=None) -> None:
    """gemm_i8_unchecked (gemmkit/src/api/int8.rs:86): raw device pointers (ints)."""
    _check(_lib.load().gk_gemm_i8_unchecked(_ws(ws), m, k, n, alpha, a, rsa, csa, b, rsb, csb,
                                            beta, c, rsc, csc, par.c(), _stream(stream)))


# ---- requant ------------------------------------------------------------------------------

def _requant(a, b, req, c, out_u8, par, ws, stream, sync):
    r = req.c()
    _check(_lib.load().gk_gemm_i8_requant(_ws(ws), a.c(), b.c(), C.byref(r), c.c(), int(out_u8),
                                          par.c(), _stream(stream)))
    if sync:
        _sync(stream)


def gemm_i8_requant(a: MatRef, b: MatRef, req: Requantize, c: MatMut,
                    par: Parallelism = SERIAL, ws=None, stream=None, sync: bool = True) -> None:
    """gemm_i8_requant (gemmkit/src/api/int8.rs:230): i8 output, clamp band [-128, 127]."""
    _requant(a, b, req, c, False, par, ws, stream, sync)


def gemm_i8_requant_u8(a: MatRef, b: MatRef, req: Requantize, c: MatMut,
                       par: Parallelism = SERIAL, ws=None, stream=None, sync: bool = True) -> None:
    """gemm_i8_requant_u8 (gemmkit/src/api/int8.rs:479): u8 output, clamp band [0, 255]."""
    _requant(a, b, req, c, True, par, ws, stream, sync)


def gemm_i8_requant_unchecked(m, k, n, a, rsa, csa, b, rsb, csb, scale, row_scales,
                              has_row_scales, zero_point, bias, has_bias, c, rsc, csc,
                              par: Parallelism = SERIAL, ws=None, stream=None) -> None:
    """gemm_i8_requant_unchecked (gemmkit/src/api/int8.rs:347)."""
    _check(_lib.load().gk_gemm_i8_requant_unchecked(
        _ws(ws), m, k, n, a, rsa, csa, b, rsb, csb, scale, row_scales, int(has_row_scales),
        zero_point, bias, int(has_bias), c, rsc, csc, par.c(), _stream(stream)))


def gemm_i8_requant_u8_unchecked(m, k, n, a, rsa, csa, b, rsb, csb, scale, row_scales,
                                 has_row_scales, zero_point, bias, has_bias, c, rsc, csc,
                                 par: Parallelism = SERIAL, ws=None, stream=None) -> None:
    """gemm_i8_requant_u8_unchecked (gemmkit/src/api/int8.rs:562)."""
    _check(_lib.load().gk_gemm_i8_requant_u8_unchecked(
        _ws(ws), m, k, n, a, rsa, csa, b, rsb, csb, scale, row_scales, int(has_row_scales),
        zero_point, bias, int(has_bias), c, rsc, csc, par.c(), _stream(stream)))


def gemm_i8_requant_ex_unchecked(m, k, n, a, rsa, csa, b, rsb, csb, req: Requantize, c, rsc,
                                 csc, out_u8=False, par: Parallelism = SERIAL, ws=None,
                                 stream=None) -> None:
    r = req.c()
    _check(_lib.load().gk_gemm_i8_requant_ex_unchecked(
        _ws(ws), m, k, n, a, rsa, csa, b, rsb, csb, C.byref(r), c, rsc, csc, int(out_u8),
        par.c(), _stream(stream)))


# ---- prepacked B (gemmkit/src/api/packed.rs) ----------------------------------------------

class PackedRhs:
    """gemmkit::PackedRhs<i8>: B packed once on the device (K-major tile layout)."""

    def __init__(self, handle: C.c_void_p):
        self.h = handle

    def rows(self) -> int:
        return _lib.load().gk_packed_rhs_rows(self.h)

    def cols(self) -> int:
        return _lib.load().gk_packed_rhs_cols(self.h)

    def to_bytes(self) -> bytes:
        """Extension: the serialized packed B (header + device-ready bytes)."""
        lib = _lib.load()
        need = C.c_size_t()
        _check(lib.gk_packed_rhs_serialize(self.h, None, 0, C.byref(need)))
        buf = C.create_string_buffer(need.value)
        _check(lib.gk_packed_rhs_serialize(self.h, buf, need.value, C.byref(need)))
        return buf.raw

    @staticmethod
    def from_bytes(data: bytes, stream=None) -> "PackedRhs":
        """Extension: a packed B loaded back from `to_bytes` output onto the current device."""
        h = C.c_void_p()
        _check(_lib.load().gk_packed_rhs_deserialize(data, len(data), _stream(stream),
                                                     C.byref(h)))
        return PackedRhs(h)

    def __del__(self):
        try:
            if getattr(self, "h", None) is not None and self.h.value:
                _lib.load().gk_packed_rhs_free(self.h)
                self.h = None
        except Exception:  # interpreter shutdown: the library may already be unloaded
            pass


def prepack_rhs_i8(b: MatRef, stream=None, sync: bool = True) -> PackedRhs:
    """prepack_rhs_i8 (gemmkit/src/api/packed.rs:372)."""
    h = C.c_void_p()
    _check(_lib.load().gk_prepack_rhs_i8(b.c(), _stream(stream), C.byref(h)))
    if sync:
        _sync(stream)
    return PackedRhs(h)


def prepack_rhs_i8_unchecked(b: int, rsb: int, csb: int, k: int, n: int, stream=None) -> PackedRhs:
    """prepack_rhs_i8_unchecked (gemmkit/src/api/packed.rs:386)."""
    h = C.c_void_p()
    _check(_lib.load().gk_prepack_rhs_i8_unchecked(b, rsb, csb, k, n, _stream(stream),
                                                   C.byref(h)))
    return PackedRhs(h)


def gemm_i8_packed_b(alpha: int, a: MatRef, packed: PackedRhs, beta: int, c: MatMut,
                     par: Parallelism = SERIAL, ws=None, stream=None, sync: bool = True) -> None:
    """gemm_i8_packed_b (gemmkit/src/api/packed.rs:473)."""
    _check(_lib.load().gk_gemm_i8_packed_b(_ws(ws), alpha, a.c(), packed.h, beta, c.c(), par.c(),
                                           _stream(stream)))
    if sync:
        _sync(stream)


def gemm_i8_packed_b_unchecked(alpha, m, a, rsa, csa, packed: PackedRhs, beta, c, rsc, csc,
                               par: Parallelism = SERIAL, ws=None, stream=None) -> None:
    """gemm_i8_packed_b_unchecked (gemmkit/src/api/packed.rs:584)."""
    _check(_lib.load().gk_gemm_i8_packed_b_unchecked(_ws(ws), alpha, m, a, rsa, csa, packed.h,
                                                     beta, c, rsc, csc, par.c(), _stream(stream)))


def gemm_i8_packed_b_requant(m, a, rsa, csa, packed: PackedRhs, req: Requantize, c, rsc, csc,
                             out_u8=False, par: Parallelism = SERIAL, ws=None,
                             stream=None) -> None:
    """Extension: requantized product with a prepacked B (raw device pointers)."""
    r = req.c()
    _check(_lib.load().gk_gemm_i8_packed_b_requant_unchecked(
        _ws(ws), m, a, rsa, csa, packed.h, C.byref(r), c, rsc, csc, int(out_u8), par.c(),
        _stream(stream)))


def gemv_i8_requant(m, a, rsa, csa, packed: PackedRhs, req: Requantize, c, rsc, csc,
                    out_u8=False, ws=None, stream=None) -> None:
    """The decode-step GEMV: gemm_i8_packed_b_requant for 1 <= m <= 64 activation rows on the
    small-M streaming kernel (gemmkit's internal small-shape route,
    gemmkit/src/special/small_mn.rs:834-1060, given an entry of its own)."""
    r = req.c()
    _check(_lib.load().gk_gemv_i8_requant_unchecked(
        _ws(ws), m, a, rsa, csa, packed.h, C.byref(r), c, rsc, csc, int(out_u8),
        _stream(stream)))


# ---- batched (extension of gemmkit/src/api/batched.rs to i8) ------------------------------

def gemm_i8_requant_batched(batch, m, k, n, a, rsa, csa, a_bs, b, rsb, csb, b_bs,
                            req: Requantize, bias_bs, scales_bs, c, rsc, csc, c_bs,
                            out_u8=False, par: Parallelism = SERIAL, ws=None,
                            stream=None) -> None:
    r = req.c()
    _check(_lib.load().gk_gemm_i8_requant_batched_unchecked(
        _ws(ws), batch, m, k, n, a, rsa, csa, a_bs, b, rsb, csb, b_bs, C.byref(r), bias_bs,
        scales_bs, c, rsc, csc, c_bs, int(out_u8), par.c(), _stream(stream)))


@dataclass
class GemmProblem:
    """One pointer-array batch element (gemmkit GemmProblem, gemmkit/src/dispatch.rs:135)."""
    m: int
    k: int
    n: int
    a: int
    rsa: int
    csa: int
    b: int
    rsb: int
    csb: int
    c: int
    rsc: int
    csc: int
    req: Requantize = field(default_factory=lambda: Requantize(RequantScale.PerTensor(1.0)))


def gemm_i8_requant_batched_ptr(problems: Sequence[GemmProblem], out_u8=False,
                                par: Parallelism = SERIAL, ws=None, stream=None) -> None:
    arr = (ProblemC * len(problems))()
    for i, p in enumerate(problems):
        arr[i] = ProblemC(p.m, p.k, p.n, p.a, p.rsa, p.csa, p.b, p.rsb, p.csb, p.c, p.rsc, p.csc,
                          p.req.c())
    _check(_lib.load().gk_gemm_i8_requant_batched_ptr_unchecked(
        _ws(ws), arr, len(problems), int(out_u8), par.c(), _stream(stream)))


# ---- half -> f32 ----------------------------------------------------------------------------

def gemm_half_f32(alpha: float, a: MatRef, b: MatRef, beta: float, c: MatMut, is_f16=False,
                  par: Parallelism = SERIAL, ws=None, stream=None, sync: bool = True) -> None:
    """bf16 / f16 inputs, f32 accumulate and output: C <- alpha*A*B + beta*C."""
    _check(_lib.load().gk_gemm_half_f32(_ws(ws), int(is_f16), alpha, a.c(), b.c(), beta, c.c(),
                                        par.c(), _stream(stream)))
    if sync:
        _sync(stream)


class Activation:
    """gemmkit::Activation (gemmkit/src/api.rs:63): ReLU or LeakyReLU(slope)."""

    def __init__(self, kind: int, slope: float = 0.0):
        self.kind, self.slope = kind, slope

    @staticmethod
    def Relu() -> "Activation":
        return Activation(_lib.ACT_RELU)

    @staticmethod
    def LeakyRelu(slope: float) -> "Activation":
        return Activation(_lib.ACT_LEAKY_RELU, float(slope))


def gemm_half_f32_fused(alpha: float, a: MatRef, b: MatRef, beta: float, c: MatMut, bias=None,
                        bias_dim: int = AXIS_ROW, act: Optional[Activation] = None, is_f16=False,
                        par: Parallelism = SERIAL, ws=None, stream=None,
                        sync: bool = True) -> None:
    """gemm_fused (gemmkit/src/api/fused.rs) on bf16 / f16 inputs with f32 output:
    C <- act(alpha*A*B + beta*C + bias), the bias per row (AXIS_ROW, length m) or per column
    (AXIS_COL, length n)."""
    bp, bn = _flat(bias) if bias is not None else (0, 0)
    _check(_lib.load().gk_gemm_half_f32_fused(
        _ws(ws), int(is_f16), alpha, a.c(), b.c(), beta, c.c(), C.c_void_p(bp or None), bn,
        bias_dim, act.kind if act else _lib.ACT_NONE, act.slope if act else 0.0, par.c(),
        _stream(stream)))
    if sync:
        _sync(stream)


def gemm_i8_fused(alpha: int, a: MatRef, b: MatRef, beta: int, c: MatMut, bias=None,
                  bias_dim: int = AXIS_ROW, act: Optional[Activation] = None,
                  par: Parallelism = SERIAL, ws=None, stream=None, sync: bool = True) -> None:
    """The i8 -> i32 GEMM with a fused integer epilogue (extension; gemmkit's gemm_fused is
    float-only): C <- act(alpha*A*B + beta*C + bias), wrapping i32 arithmetic, the i32 bias
    per row (AXIS_ROW, length m) or per column (AXIS_COL, length n), act None or ReLU."""
    bp, bn = _flat(bias) if bias is not None else (0, 0)
    _check(_lib.load().gk_gemm_i8_fused(
        _ws(ws), int(alpha), a.c(), b.c(), int(beta), c.c(), C.c_void_p(bp or None), bn,
        bias_dim, act.kind if act else _lib.ACT_NONE, par.c(), _stream(stream)))
    if sync:
        _sync(stream)


def gemm_i8_fused_unchecked(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc,
                            bias=None, bias_dim: int = AXIS_ROW, act: int = 0,
                            par: Parallelism = SERIAL, ws=None, stream=None) -> None:
    """Raw-pointer tier of gemm_i8_fused (device pointers as ints; bias a device pointer or
    None; act one of _lib.ACT_NONE / _lib.ACT_RELU)."""
    _check(_lib.load().gk_gemm_i8_fused_unchecked(
        _ws(ws), m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc,
        C.c_void_p(bias) if bias else None, bias_dim, 1 if bias else 0, act, par.c(),
        _stream(stream)))


def quantize_f32_i8(rows, cols, x, rsx, csx, q, rsq, csq, scale: float = 1.0,
                    zero_point: int = 0, row_scales=None, stream=None) -> None:
    """Extension: f32 -> i8 activations (raw device pointers). Per-tensor scale / zero point,
    or per-row symmetric scales written to `row_scales` (a device pointer) when given."""
    _check(_lib.load().gk_quantize_f32_i8_unchecked(
        rows, cols, C.c_void_p(x), rsx, csx, C.c_void_p(q), rsq, csq, float(scale),
        int(zero_point), C.c_void_p(row_scales) if row_scales else None, _stream(stream)))


def gemm_bf16_f32_unchecked(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc,
                            par: Parallelism = SERIAL, ws=None, stream=None) -> None:
    _check(_lib.load().gk_gemm_bf16_f32_unchecked(_ws(ws), m, k, n, alpha, a, rsa, csa, b, rsb,
                                                  csb, beta, c, rsc, csc, par.c(),
                                                  _stream(stream)))


def gemm_f16_f32_unchecked(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc,
                           par: Parallelism = SERIAL, ws=None, stream=None) -> None:
    _check(_lib.load().gk_gemm_f16_f32_unchecked(_ws(ws), m, k, n, alpha, a, rsa, csa, b, rsb,
                                                 csb, beta, c, rsc, csc, par.c(),
                                                 _stream(stream)))


def gemm_half_f32_batched(is_f16, batch, m, k, n, alpha, a, rsa, csa, a_bs, b, rsb, csb, b_bs,
                          beta, c, rsc, csc, c_bs, par: Parallelism = SERIAL, ws=None,
                          stream=None) -> None:
    _check(_lib.load().gk_gemm_half_f32_batched_unchecked(
        _ws(ws), int(is_f16), batch, m, k, n, alpha, a, rsa, csa, a_bs, b, rsb, csb, b_bs, beta,
        c, rsc, csc, c_bs, par.c(), _stream(stream)))


# ---- i8 -> i32 without allocation ---------------------------------------------------------

NOALLOC_SCRATCH_BYTES = 16 << 20


def gemm_i8_noalloc_unchecked(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc,
                              stream=None) -> None:
    """gemm_i8_unchecked for callers that must not allocate device memory: operand packs use
    the library's fixed 16 MiB device scratch (shared by all calls; order calls on one
    stream). Raises GemmkitError(GK_EINVAL) when the packs need more than that."""
    _check(_lib.load().gk_gemm_i8_noalloc_unchecked(m, k, n, alpha, a, rsa, csa, b, rsb, csb,
                                                    beta, c, rsc, csc, _stream(stream)))


# ---- misc -----------------------------------------------------------------------------------

def set_tile_n(bn: int) -> None:
    """Force the MMA tile width (16/32/64/128/192/256) on this thread; 0 drops the override
    (the GEMMKIT_CUDA_BN knob, by default chosen per shape)."""
    _check(_lib.load().gk_set_tile_n(bn))


def knob_names() -> list[str]:
    """The engine's knobs (gemmkit's tuning knobs, gemmkit/src/tuning.rs:585-690)."""
    return _lib.load().gk_knob_names().decode().split(",")


def knob_get(name: str) -> int:
    """The value in effect: the run-time override, else the environment, else the default."""
    v = C.c_int64()
    _check(_lib.load().gk_knob_get(name.encode(), C.byref(v)))
    return int(v.value)


def knob_set(name: str, value: int) -> None:
    """Process-wide run-time override of a knob; a negative value drops the override."""
    _check(_lib.load().gk_knob_set(name.encode(), int(value)))


def device_status(device: int = 0, clear: bool = True) -> int:
    v = C.c_uint32()
    _check(_lib.load().gk_device_status(device, int(clear), C.byref(v)))
    return v.value


def selftest_wait_timeout(timeout_ns: int, stream=None) -> int:
    """Run the bounded-wait self test; returns the status code (GK_ETIMEOUT expected)."""
    return _lib.load().gk_selftest_wait_timeout(timeout_ns, _stream(stream))
