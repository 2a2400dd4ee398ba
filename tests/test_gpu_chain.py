"""Back-to-back dependent calls on one stream, no host synchronisation in between: every
kernel may start before the previous one has finished (programmatic dependent launch), so
these chains check that each one reads its inputs and writes its outputs only after the
previous kernel is done. Two requantized chains are interleaved (a decode-like one with 8
rows on the small-M kernel, a prefill-like one with 1184 rows on the tile kernels), and each
chain ping-pongs between two buffers, so a kernel overwrites the buffer the kernel before it
was reading. Bit-exact against the oracle chain."""
import numpy as np
import pytest
import torch

import gemmkit_b200 as gk
import oracle as O
from gpu_util import dev, empty, host, rand_i8

pytestmark = pytest.mark.gpu

# k -> n per step; with 1184 rows the 256 -> 4096 step runs on the CTA-pair kernel, the others
# on the one-CTA kernel; with 8 rows every step runs on the small-M kernel (cluster-split K
# for the narrow ones)
WIDTHS = [256, 4096, 256, 2048, 512]


def _weights(rng):
    ws = []
    for k, n in zip(WIDTHS[:-1], WIDTHS[1:]):
        wT = rand_i8(rng, (n, k), -127, 127)
        scales = rng.uniform(2e-4, 6e-4, n).astype(np.float32)
        bias = rng.integers(-3000, 3000, n).astype(np.int32)
        ws.append((k, n, wT, scales, bias))
    return ws


def _oracle_chain(x, ws):
    for k, n, wT, scales, bias in ws:
        x = O.requant_matrix(x, wT.T, scales=scales, scale_axis="col", bias=bias,
                             bias_axis="col", zp=0, relu=True)
    return x


def test_interleaved_dependent_chains():
    rng = np.random.default_rng(2024)
    ws = _weights(rng)
    dev_ws = []
    for k, n, wT, scales, bias in ws:
        packed = gk.prepack_rhs_i8(gk.MatRef.new(dev(wT), k, n, 1, k))
        dsc, dbias = dev(scales), dev(bias)
        req = gk.Requantize(gk.RequantScale.PerCol(dsc), 0, dbias, gk.AXIS_COL, True)
        dev_ws.append((k, n, packed, req, dsc, dbias))
    chains = {}
    for name, m in (("decode", 8), ("prefill", 1184)):
        x0 = rand_i8(rng, (m, WIDTHS[0]), -127, 127)
        bufs = [empty(m * max(WIDTHS), np.int8), empty(m * max(WIDTHS), np.int8)]
        bufs[0][: m * WIDTHS[0]].copy_(torch.from_numpy(x0.reshape(-1)))
        chains[name] = (m, x0, bufs)
    torch.cuda.synchronize()
    for step, (k, n, packed, req, _, _) in enumerate(dev_ws):
        for name in ("decode", "prefill"):
            m, _, bufs = chains[name]
            src, dst = bufs[step % 2], bufs[(step + 1) % 2]
            gk.gemm_i8_packed_b_requant(m, src.data_ptr(), k, 1, packed, req, dst.data_ptr(), n,
                                        1)
    torch.cuda.synchronize()
    assert gk.device_status(0) == 0
    last = len(dev_ws) % 2
    for name in ("decode", "prefill"):
        m, x0, bufs = chains[name]
        want = _oracle_chain(x0, ws)
        got = host(bufs[last])[: m * WIDTHS[-1]].reshape(m, WIDTHS[-1])
        assert np.array_equal(got, want), name


def test_dependent_gemv_after_large_gemm():
    """A large requantized GEMM whose output rows feed a small-M call right behind it."""
    rng = np.random.default_rng(7)
    m, k, n, n2 = 768, 2048, 1024, 4096
    a = rand_i8(rng, (m, k), -127, 127)
    bT = rand_i8(rng, (n, k), -127, 127)
    w2T = rand_i8(rng, (n2, n), -127, 127)
    s1 = rng.uniform(2e-4, 5e-4, n).astype(np.float32)
    s2 = rng.uniform(2e-4, 5e-4, n2).astype(np.float32)
    y1 = O.requant_matrix(a, bT.T, scales=s1, scale_axis="col", zp=0)
    want = O.requant_matrix(y1[-4:], w2T.T, scales=s2, scale_axis="col", zp=0)
    p1 = gk.prepack_rhs_i8(gk.MatRef.new(dev(bT), k, n, 1, k))
    p2 = gk.prepack_rhs_i8(gk.MatRef.new(dev(w2T), n, n2, 1, n))
    ds1, ds2 = dev(s1), dev(s2)
    da = dev(a)
    dy1 = empty(m * n, np.int8)
    dy2 = empty(4 * n2, np.int8)
    r1 = gk.Requantize(gk.RequantScale.PerCol(ds1), 0)
    r2 = gk.Requantize(gk.RequantScale.PerCol(ds2), 0)
    for _ in range(3):
        gk.gemm_i8_packed_b_requant(m, da.data_ptr(), k, 1, p1, r1, dy1.data_ptr(), n, 1)
        gk.gemm_i8_packed_b_requant(4, dy1.data_ptr() + (m - 4) * n, n, 1, p2, r2,
                                    dy2.data_ptr(), n2, 1)
    torch.cuda.synchronize()
    assert np.array_equal(host(dy2).reshape(4, n2), want)
