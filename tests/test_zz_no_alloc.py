"""gk_gemm_i8_noalloc_unchecked: the i8 -> i32 product for callers that must not allocate
device memory (their own allocator owns the GPU budget, or a cudaMalloc / cudaFree could
synchronise the device in the middle of a latency-critical loop). It packs operands into the
library's fixed 16 MiB device scratch instead of a workspace. This file is collected last on
purpose, so a failure here comes after every other test has run."""
import ctypes as C

import numpy as np
import pytest

import gemmkit_b200 as gk
from gemmkit_b200 import _lib
import oracle as O
from gpu_util import dev, host, rand_i8

pytestmark = pytest.mark.gpu


def noalloc(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc):
    import torch
    return _lib.load().gk_gemm_i8_noalloc_unchecked(
        m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc,
        C.c_void_p(torch.cuda.current_stream().cuda_stream))


def existing(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc):
    import torch
    return _lib.load().gk_gemm_i8_unchecked(
        None, m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc,
        _lib.Parallelism(0, 0), C.c_void_p(torch.cuda.current_stream().cuda_stream))


def case(seed, m, k, n):
    """Row-major B (packed through the scratch) and an A with a 3-element row gap."""
    rng = np.random.default_rng(seed)
    a = rand_i8(rng, (m, k + 3))  # rsa = k + 3: not 16-byte aligned rows -> packed too
    b = rand_i8(rng, (k, n))
    c0 = rng.integers(-50, 50, (m, n)).astype(np.int32)
    return a, b, c0


def test_noalloc_matches_existing_entry_two_calls_in_a_row():
    import torch
    shapes = [(300, 200, 260), (97, 515, 1031)]
    inputs = [case(40 + i, *s) for i, s in enumerate(shapes)]
    args, refs, outs = [], [], []
    for (m, k, n), (a, b, c0) in zip(shapes, inputs):
        da, db = dev(a), dev(b)
        dref, dout = dev(c0), dev(c0)
        call = (m, k, n, 3, da.data_ptr(), k + 3, 1, db.data_ptr(), n, 1, -2)
        args.append((da, db, dref, dout))
        assert existing(*call, dref.data_ptr(), n, 1) == gk.GK_OK, _lib.last_error()
        refs.append(dref)
        outs.append((call, dout, n))
    torch.cuda.synchronize()
    free_before = None
    for i, (call, dout, n) in enumerate(outs):  # two no-alloc calls back to back
        assert noalloc(*call, dout.data_ptr(), n, 1) == gk.GK_OK, _lib.last_error()
        if i == 0:
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before  # no device memory taken by call 2
    for (m, k, n), (a, b, c0), dref, (_, dout, _) in zip(shapes, inputs, refs, outs):
        got = host(dout).reshape(m, n)
        assert np.array_equal(got, host(dref).reshape(m, n))  # integer path: bit-exact
        want = O.gemm_i8_matrix(3, a[:, :k], b, -2, c0)  # the CPU oracle (gemmkit's semantics)
        assert np.array_equal(got, want)
    assert gk.device_status(0) == 0


def test_noalloc_rejects_packs_beyond_its_scratch():
    # B row-major 4096 x 4096 needs a 16 MiB transpose pack, A (padded rows) another 16 MiB
    m = k = n = 4096
    z = dev(np.zeros(m * (k + 1), np.int8))
    c = dev(np.zeros(16, np.int32))
    rc = noalloc(m, k, n, 1, z.data_ptr(), k + 1, 1, z.data_ptr(), n, 1, 0, c.data_ptr(), n, 1)
    assert rc == gk.GK_EINVAL
    msg = _lib.last_error()
    assert "fixed scratch holds 16777216 bytes" in msg, msg
