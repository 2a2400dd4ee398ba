"""One problem across the GPUs of a node, one process per GPU (no counterpart in gemmkit, which
is single-process; this is the multi-GPU form of its wide and batched GEMMs).

* Column sharding of one wide GEMM (C = alpha*A*B + beta*C, bf16/f16 -> f32): every rank holds
  A (replicated) and its own block of B's columns [n0, n1), and computes C[:, n0:n1]. C is
  column-major, so a block of columns is one contiguous slab. When the caller wants C
  replicated on every rank, the GEMM's epilogue stores each output tile into every rank's C
  (peer stores over NVLink through CUDA IPC mappings, the ``"nvlink"`` route) -- the
  all-gather is fused into the GEMM and overlaps its math tile by tile -- or, on the
  ``"nccl"`` route, the block is computed locally and NCCL all-gathers the blocks.
* Batch sharding of a batched requantized i8 GEMM: rank r takes batch elements [b0, b1) (each
  with its own bias / scales); no collective unless the caller wants C replicated (same two
  routes).

After a replicated call every rank's stream waits on an NCCL all-reduce of one element, which
completes only once every rank's GEMM (and with it every peer store) is done.

All ranks must make the same calls in the same order (they are collectives).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _lib


def _split(total: int, parts: int, index: int, align: int) -> tuple[int, int]:
    """[lo, hi) of part `index` of `total` cut into `parts` near-equal runs whose boundaries
    are multiples of `align` (the last part takes the remainder)."""
    units = -(-total // align)
    lo = min(total, (units * index // parts) * align)
    hi = total if index == parts - 1 else min(total, (units * (index + 1) // parts) * align)
    return lo, hi


@dataclass
class Replicated:
    """A device buffer allocated on every rank with the same size, with the other ranks'
    copies mapped into this process (peers[r] is None for this rank)."""
    tensor: object          # torch.Tensor, this rank's copy
    peers: list             # device addresses of every rank's copy, as seen from this process
    opened: list            # addresses this process opened (closed by close())

    def ptr(self) -> int:
        return self.tensor.data_ptr()

    def close(self):
        lib = _lib.load()
        for p in self.opened:
            lib.gk_ipc_close(C.c_void_p(p))
        self.opened = []


class ShardGroup:
    """The ranks of a torch.distributed process group (NCCL on GPUs; gloo for the host-logic
    tests), one GPU per rank."""

    TILE = 128  # column / batch boundaries fall on tile boundaries

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self._flag = None

    # ---- partitions ---------------------------------------------------------------------
    def col_range(self, n: int, rank: int | None = None) -> tuple[int, int]:
        return _split(n, self.world, self.rank if rank is None else rank, self.TILE)

    def batch_range(self, batch: int, rank: int | None = None) -> tuple[int, int]:
        return _split(batch, self.world, self.rank if rank is None else rank, 1)

    # ---- replicated buffers -------------------------------------------------------------
    def replicated_empty(self, numel: int, dtype) -> Replicated:
        """Allocate `numel` elements on every rank and map every other rank's copy here."""
        import torch
        t = torch.empty(numel, dtype=dtype, device="cuda")
        lib = _lib.load()
        h = _lib.IpcHandleC()
        rc = lib.gk_ipc_export(C.c_void_p(t.data_ptr()), C.byref(h))
        if rc != 0:
            raise RuntimeError(_lib.last_error())
        mine = (bytes(h.bytes), int(h.offset))
        allh = [None] * self.world
        self.dist.all_gather_object(allh, mine, group=self.group)
        peers, opened = [], []
        for r, (hb, off) in enumerate(allh):
            if r == self.rank:
                peers.append(None)
                continue
            ph = _lib.IpcHandleC()
            C.memmove(ph.bytes, hb, 64)
            ph.offset = off
            p = C.c_void_p()
            rc = lib.gk_ipc_open(C.byref(ph), C.byref(p))
            if rc != 0:
                raise RuntimeError(_lib.last_error())
            peers.append(p.value)
            opened.append(p.value)
        return Replicated(t, peers, opened)

    # ---- completion ---------------------------------------------------------------------
    def fence(self):
        """Stream-ordered barrier: the current stream continues only once every rank has
        reached this point in its stream (NCCL all-reduce of one element)."""
        import torch
        if self._flag is None:
            dev = "cuda" if torch.cuda.is_available() else "cpu"
            self._flag = torch.zeros(1, dtype=torch.float32, device=dev)
        work = self.dist.all_reduce(self._flag, group=self.group, async_op=True)
        work.wait()

    # ---- column-sharded wide GEMM ---------------------------------------------------------
    def _gemm_block_half(self, is_f16, m, k, nr, alpha, a_ptr, rsa, csa, b_ptr, rsb, csb, beta,
                         c_ptr, ldc, mirrors, stream):
        lib = _lib.load()
        if mirrors:
            arr = (C.c_void_p * len(mirrors))(*mirrors)
            rc = lib.gk_gemm_half_f32_mirrored_unchecked(
                None, int(is_f16), m, k, nr, alpha, C.c_void_p(a_ptr), rsa, csa,
                C.c_void_p(b_ptr), rsb, csb, beta, C.c_void_p(c_ptr), 1, ldc, arr, len(mirrors),
                C.c_void_p(stream))
        else:
            fn = lib.gk_gemm_f16_f32_unchecked if is_f16 else lib.gk_gemm_bf16_f32_unchecked
            rc = fn(None, m, k, nr, alpha, C.c_void_p(a_ptr), rsa, csa, C.c_void_p(b_ptr), rsb,
                    csb, beta, C.c_void_p(c_ptr), 1, ldc, _lib.Parallelism(0, 0),
                    C.c_void_p(stream))
        if rc != 0:
            raise RuntimeError(_lib.last_error())

    def gemm_half_f32_cols(self, m: int, k: int, n: int, alpha: float, a_ptr: int, rsa: int,
                           csa: int, b_block_ptr: int, rsb: int, csb: int, beta: float,
                           c: Replicated, *, is_f16: bool = False, replicate: bool = True,
                           route: str = "nvlink", stream=None) -> tuple[int, int]:
        """This rank's columns [n0, n1) of C (m x n, column-major, ld = m, in the replicated
        buffer `c`) = alpha * A(m x k) * B[:, n0:n1] + beta * C[:, n0:n1]. `b_block_ptr`
        addresses B[0, n0] of this rank's block with strides (rsb, csb) in elements. With
        `replicate`, every rank's C holds the whole product afterwards. Returns (n0, n1)."""
        import torch
        n0, n1 = self.col_range(n)
        st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        off = n0 * m * 4
        mirrors = []
        if replicate and route == "nvlink":
            mirrors = [p + off for p in c.peers if p is not None]
        if n1 > n0:
            self._gemm_block_half(is_f16, m, k, n1 - n0, alpha, a_ptr, rsa, csa, b_block_ptr,
                                  rsb, csb, beta, c.ptr() + off, m, mirrors, st)
        if replicate:
            if route == "nccl":
                self._all_gather_cols(c.tensor, m, n)
            else:
                self.fence()
        return n0, n1

    def _all_gather_cols(self, c_full, m: int, n: int):
        """NCCL route: gather every rank's column block of the column-major C in place."""
        self._gather_spans(c_full, [(lo * m, hi * m) for lo, hi in
                                    (self.col_range(n, r) for r in range(self.world))])

    def _gather_spans(self, flat, spans):
        """Every rank's span [lo, hi) of `flat` from its owner into every rank's `flat`. Equal
        spans laid end to end gather in place; otherwise each span is padded to the longest
        (all-gather needs equal counts) and copied back into place."""
        import torch
        sizes = [hi - lo for lo, hi in spans]
        contiguous = all(spans[i][1] == spans[i + 1][0] for i in range(len(spans) - 1))
        lo, hi = spans[self.rank]
        if len(set(sizes)) == 1 and contiguous:
            self.dist.all_gather_into_tensor(flat[spans[0][0]:spans[-1][1]],
                                             flat[lo:hi].clone(), group=self.group)
            return
        big = max(sizes)
        send = torch.zeros(big, dtype=flat.dtype, device=flat.device)
        send[: hi - lo].copy_(flat[lo:hi])
        recv = torch.empty(big * self.world, dtype=flat.dtype, device=flat.device)
        self.dist.all_gather_into_tensor(recv, send, group=self.group)
        for r, (a, b) in enumerate(spans):
            if r != self.rank and b > a:
                flat[a:b].copy_(recv[r * big: r * big + (b - a)])

    # ---- batch-sharded requantized GEMM ---------------------------------------------------
    def gemm_i8_requant_batched_shard(self, batch: int, m: int, k: int, n: int, a_ptr: int,
                                      rsa: int, csa: int, a_bs: int, b_ptr: int, rsb: int,
                                      csb: int, b_bs: int, req, bias_bs: int, scales_bs: int,
                                      c_ptr: int, rsc: int, csc: int, c_bs: int, out_u8: bool,
                                      c: Replicated | None = None, replicate: bool = False,
                                      route: str = "nvlink", stream=None) -> tuple[int, int]:
        """This rank's batch elements [b0, b1) of a strided batched requantized i8 GEMM
        (arguments as gk_gemm_i8_requant_batched_unchecked, for the whole batch). With
        `replicate` (C must then be the replicated buffer `c`, c_ptr == c.ptr()), every
        rank's C holds every element afterwards. Returns (b0, b1)."""
        import torch
        b0, b1 = self.batch_range(batch)
        st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        rq = req.c()
        rq_local = _lib.RequantC()
        C.memmove(C.byref(rq_local), C.byref(rq), C.sizeof(rq))
        if rq_local.bias:
            rq_local.bias = rq_local.bias + b0 * bias_bs * 4
        if rq_local.scales:
            rq_local.scales = rq_local.scales + b0 * scales_bs * 4
        mirrors = []
        if replicate and route == "nvlink":
            if c is None or c_ptr != c.ptr():
                raise ValueError("replicate needs C in a replicated buffer")
            mirrors = [p + b0 * c_bs for p in c.peers if p is not None]
        if b1 > b0:
            self._gemm_block_requant(b1 - b0, m, k, n, a_ptr + b0 * a_bs, rsa, csa, a_bs,
                                     b_ptr + b0 * b_bs, rsb, csb, b_bs, rq_local, bias_bs,
                                     scales_bs, c_ptr + b0 * c_bs, rsc, csc, c_bs, out_u8,
                                     mirrors, st)
        if replicate:
            if route == "nccl":
                self._all_gather_batch(c.tensor, batch, c_bs)
            else:
                self.fence()
        return b0, b1

    def _gemm_block_requant(self, nb, m, k, n, a_ptr, rsa, csa, a_bs, b_ptr, rsb, csb, b_bs,
                            rq, bias_bs, scales_bs, c_ptr, rsc, csc, c_bs, out_u8, mirrors,
                            stream):
        lib = _lib.load()
        arr = (C.c_void_p * len(mirrors))(*mirrors) if mirrors else None
        rc = lib.gk_gemm_i8_requant_mirrored_unchecked(
            None, nb, m, k, n, C.c_void_p(a_ptr), rsa, csa, a_bs, C.c_void_p(b_ptr), rsb, csb,
            b_bs, None, C.byref(rq), bias_bs, scales_bs, C.c_void_p(c_ptr), rsc, csc, c_bs,
            int(out_u8), arr, len(mirrors), C.c_void_p(stream))
        if rc != 0:
            raise RuntimeError(_lib.last_error())

    def _all_gather_batch(self, c_full, batch: int, c_bs: int):
        self._gather_spans(c_full, [(lo * c_bs, hi * c_bs) for lo, hi in
                                    (self.batch_range(batch, r) for r in range(self.world))])
