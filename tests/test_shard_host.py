"""Host logic of the sharded paths on CPU, world size 2 over gloo: the column / batch
partitions, the block offsets each rank computes into, and the gather that replicates C.
The device GEMM of each block is replaced by a numpy / oracle computation of the same block,
so these run without a GPU; the kernels themselves are covered by tests/test_gpu_shard.py."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _split_cases():
    from gemmkit_b200.shard import _split
    for total in (0, 1, 5, 127, 128, 129, 700, 4096, 8192, 8193):
        for parts in (1, 2, 3, 4, 8):
            for align in (1, 128):
                spans = [_split(total, parts, i, align) for i in range(parts)]
                yield total, parts, align, spans


def test_split_covers_and_aligns():
    for total, parts, align, spans in _split_cases():
        assert spans[0][0] == 0 and spans[-1][1] == total
        for (a, b), (c, _) in zip(spans, spans[1:]):
            assert b == c  # contiguous, no overlap
        for lo, hi in spans:
            assert lo <= hi
            assert lo % align == 0 or lo == total
        if total >= parts * align:
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 2 * align  # balanced up to the alignment


def _worker(rank, port, results):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from gemmkit_b200.shard import Replicated, ShardGroup
        import oracle as O
        g = ShardGroup()
        out = {}

        # -- column-sharded wide GEMM, replicated through the gather route ------------------
        for (m, k, n) in [(64, 96, 512), (48, 40, 700)]:  # equal and unequal blocks
            rng = np.random.default_rng(m + n)
            A = rng.standard_normal((m, k)).astype(np.float32)
            B = rng.standard_normal((k, n)).astype(np.float32)
            C0 = rng.standard_normal((m, n)).astype(np.float32)
            alpha, beta = 1.5, -0.5
            c = Replicated(torch.from_numpy(np.asfortranarray(C0).ravel(order="F").copy()),
                           [None] * WORLD, [])

            def block(is_f16, mm, kk, nr, al, a_ptr, rsa, csa, b_ptr, rsb, csb, be, c_ptr, ldc,
                      mirrors, stream):
                n0 = (c_ptr - c.ptr()) // (mm * 4)
                blk = al * (A @ B[:, n0:n0 + nr]) + be * C0[:, n0:n0 + nr]
                c.tensor[n0 * mm:(n0 + nr) * mm] = torch.from_numpy(
                    np.asfortranarray(blk).ravel(order="F").astype(np.float32))
                assert mirrors == []  # the gather route stores locally only

            g._gemm_block_half = block
            n0, n1 = g.gemm_half_f32_cols(m, k, n, alpha, 0, k, 1, 0, n, 1, beta, c,
                                          replicate=True, route="nccl", stream=0)
            want = (alpha * (A @ B) + beta * C0).ravel(order="F")
            out[f"cols_{m}x{k}x{n}"] = (bool(np.allclose(c.tensor.numpy(), want, rtol=1e-5,
                                                         atol=1e-5)), (n0, n1))

        # -- batch-sharded requantized GEMM, bit-exact through the oracle --------------------
        batch, m, k, n = 5, 16, 32, 24
        rng = np.random.default_rng(9)
        a = rng.integers(-128, 128, (batch, m, k)).astype(np.int8)
        b = rng.integers(-128, 128, (batch, k, n)).astype(np.int8)
        bias = rng.integers(-2**15, 2**15, (batch, m)).astype(np.int32)
        scales = rng.uniform(1e-4, 1e-3, (batch, n)).astype(np.float32)
        want = np.stack([O.requant_matrix(a[e], b[e], scales=scales[e], scale_axis="col",
                                          bias=bias[e], bias_axis="row", zp=128, out_u8=True)
                         for e in range(batch)]).reshape(-1)
        c = Replicated(torch.zeros(batch * m * n, dtype=torch.uint8), [None] * WORLD, [])
        seen = []

        def rblock(nb, mm, kk, nn, a_ptr, rsa, csa, a_bs, b_ptr, rsb, csb, b_bs, rq, bias_bs,
                   scales_bs, c_ptr, rsc, csc, c_bs, out_u8, mirrors, stream):
            e0 = (c_ptr - c.ptr()) // c_bs
            assert a_ptr == e0 * a_bs and b_ptr == e0 * b_bs  # operands offset like C
            seen.append((e0, nb))
            for e in range(e0, e0 + nb):
                c.tensor[e * c_bs:(e + 1) * c_bs] = torch.from_numpy(O.requant_matrix(
                    a[e], b[e], scales=scales[e], scale_axis="col", bias=bias[e],
                    bias_axis="row", zp=128, out_u8=True).reshape(-1))

        g._gemm_block_requant = rblock

        class Req:  # the Requantize descriptor shape the shard call reads
            def c(self):
                import gemmkit_b200._lib as L
                r = L.RequantC()
                r.scale = 1.0
                r.scales = 1000  # offsets are checked, not dereferenced
                r.bias = 2000
                r.zero_point = 128
                return r

        b0, b1 = g.gemm_i8_requant_batched_shard(
            batch, m, k, n, 0, k, 1, m * k, 0, n, 1, k * n, Req(), m, n, c.ptr(), n, 1, m * n,
            True, c=c, replicate=True, route="nccl", stream=0)
        out["batch"] = (bool(np.array_equal(c.tensor.numpy(), want)), (b0, b1), seen)
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_sharded_host_logic_gloo():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0, "a rank failed"
    res = dict(results)
    assert set(res) == set(range(WORLD))
    for key in ("cols_64x96x512", "cols_48x40x700"):
        spans = [res[r][key][1] for r in range(WORLD)]
        assert all(res[r][key][0] for r in range(WORLD)), key
        assert spans[0][0] == 0 and spans[-1][1] == int(key.split("x")[-1])
    assert all(res[r]["batch"][0] for r in range(WORLD))
    spans = [res[r]["batch"][1] for r in range(WORLD)]
    assert spans == [(0, 2), (2, 5)]
