"""Shared helpers for the GPU parity tests (device buffers from numpy, oracle slices)."""
from __future__ import annotations

import contextlib
import hashlib

import numpy as np


def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def dev(arr: np.ndarray):
    """A flat CUDA tensor holding a copy of ``arr`` (C order)."""
    torch = torch_cuda()
    return torch.from_numpy(np.ascontiguousarray(arr).reshape(-1).copy()).cuda()


def empty(n: int, dtype) -> "object":
    torch = torch_cuda()
    tdt = {np.int8: torch.int8, np.uint8: torch.uint8, np.int32: torch.int32,
           np.float32: torch.float32, np.uint16: torch.int16}[dtype]
    return torch.empty(n, dtype=tdt, device="cuda")


def host(t, dtype=None) -> np.ndarray:
    torch = torch_cuda()
    torch.cuda.synchronize()
    a = t.cpu().numpy()
    return a.view(dtype) if dtype is not None else a


def digest(arr: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()


def gather(buf: np.ndarray, rows: int, cols: int, rs: int, cs: int, base: int = 0) -> np.ndarray:
    """The logical rows x cols matrix of a strided view into a flat buffer."""
    i = np.arange(rows)[:, None]
    j = np.arange(cols)[None, :]
    return buf[base + i * rs + j * cs]


def rand_i8(rng, shape, lo=-128, hi=127):
    return rng.integers(lo, hi + 1, size=shape, dtype=np.int64).astype(np.int8)


@contextlib.contextmanager
def knobs(**values):
    """Run a block with engine knobs overridden (e.g. knobs(GEMMKIT_CUDA_STREAMK=1)); the
    overrides are dropped afterwards."""
    import gemmkit_b200 as gk
    for name, v in values.items():
        gk.knob_set(name, v)
    try:
        yield
    finally:
        for name in values:
            gk.knob_set(name, -1)
