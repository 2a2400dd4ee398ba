"""The sharded paths on 2 GPUs (one process per GPU, NCCL with NVLS off): the column-sharded
bf16 -> f32 GEMM with C replicated through the GEMM's own peer stores ("nvlink") and through
an NCCL all-gather ("nccl"), and the batch-sharded requantized i8 GEMM. Every rank checks the
whole replicated C: against the f64 reference within the stated 1e-2 tolerance for bf16, bit
for bit against the oracle for i8, and the two routes against each other bit for bit.
Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    out = {}
    try:
        import gemmkit_b200 as gk
        import oracle as O
        from gemmkit_b200.shard import ShardGroup
        g = ShardGroup()

        # ---- column-sharded bf16 GEMM, C column-major m x n, replicated ------------------
        m, k, n = 1024, 768, 1408  # 1408 = 11 tiles: uneven blocks (640 / 768 columns)
        rng = np.random.default_rng(11)  # the same inputs on every rank
        A = O.f32_to_bf16(rng.standard_normal((m, k)).astype(np.float32))
        B = O.f32_to_bf16(rng.standard_normal((k, n)).astype(np.float32))
        C0 = rng.standard_normal((m, n)).astype(np.float32)
        alpha, beta = 1.0, 0.5
        dA = torch.from_numpy(A.view(np.int16)).cuda()
        dBT = torch.from_numpy(np.ascontiguousarray(B.T).view(np.int16)).cuda()  # n x k
        c0_cm = torch.from_numpy(np.asfortranarray(C0).ravel(order="F").copy()).cuda()
        got = {}
        for route in ("nvlink", "nccl"):
            c = g.replicated_empty(m * n, torch.float32)
            c.tensor.copy_(c0_cm)
            torch.cuda.synchronize()
            g.fence()
            n0, n1 = g.col_range(n)
            g.gemm_half_f32_cols(m, k, n, alpha, dA.data_ptr(), k, 1,
                                 dBT.data_ptr() + n0 * k * 2, 1, k, beta, c,
                                 replicate=True, route=route)
            torch.cuda.synchronize()
            got[route] = c.tensor.cpu().numpy().reshape(n, m).T.copy()
            g.fence()
            torch.cuda.synchronize()
            c.close()
        ref = O.gemm_half_f64(A, B, alpha, beta, C0, False)
        mag = np.abs(O.bf16_to_f32(A).astype(np.float64)) @ np.abs(
            O.bf16_to_f32(B).astype(np.float64)) + abs(beta) * np.abs(C0.astype(np.float64))
        err = np.abs(got["nvlink"].astype(np.float64) - ref)
        out["cols_tol"] = bool(np.all(err <= 1e-2 * mag + 1e-30))
        out["cols_routes_equal"] = bool(np.array_equal(got["nvlink"], got["nccl"]))

        # ---- batch-sharded requantized i8 GEMM, replicated ---------------------------------
        batch, bm, bk, bn = 6, 256, 128, 384
        rng = np.random.default_rng(5)
        a = rng.integers(-128, 128, (batch, bm, bk)).astype(np.int8)
        bT = rng.integers(-128, 128, (batch, bn, bk)).astype(np.int8)
        bias = rng.integers(-2**15, 2**15 + 1, (batch, bm)).astype(np.int32)
        scales = rng.uniform(1e-4, 1e-3, (batch, bn)).astype(np.float32)
        want = np.stack([O.requant_matrix(a[e], bT[e].T, scales=scales[e], scale_axis="col",
                                          bias=bias[e], bias_axis="row", zp=128, out_u8=True)
                         for e in range(batch)])
        da = torch.from_numpy(a.reshape(-1)).cuda()
        db = torch.from_numpy(bT.reshape(-1)).cuda()
        dbias = torch.from_numpy(bias.reshape(-1)).cuda()
        dsc = torch.from_numpy(scales.reshape(-1)).cuda()
        req = gk.Requantize(gk.RequantScale.PerCol(dsc), 128, dbias, gk.AXIS_ROW)
        for route in ("nvlink", "nccl"):
            c = g.replicated_empty(batch * bm * bn, torch.uint8)
            c.tensor.zero_()
            torch.cuda.synchronize()
            g.fence()
            g.gemm_i8_requant_batched_shard(batch, bm, bk, bn, da.data_ptr(), bk, 1, bm * bk,
                                            db.data_ptr(), 1, bk, bn * bk, req, bm, bn,
                                            c.ptr(), bn, 1, bm * bn, True, c=c, replicate=True,
                                            route=route)
            torch.cuda.synchronize()
            res = c.tensor.cpu().numpy().reshape(batch, bm, bn)
            out[f"batch_{route}"] = bool(np.array_equal(res, want))
            g.fence()
            torch.cuda.synchronize()
            c.close()
        out["status"] = gk.device_status(rank)
    except Exception as e:  # reported to the parent, which fails the test
        out["error"] = repr(e)
    finally:
        results[rank] = out
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_sharded_paths_two_gpus():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = dict(results)
    assert set(res) == set(range(WORLD)), res
    for r in range(WORLD):
        o = res[r]
        assert "error" not in o, o
        assert o["cols_tol"] and o["cols_routes_equal"], o
        assert o["batch_nvlink"] and o["batch_nccl"], o
        assert o["status"] == 0, o
