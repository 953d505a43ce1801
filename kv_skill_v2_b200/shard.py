"""Chunk-sharded read of one large Library across the GPUs of one node (the long-document decode of BASELINE
config 5: one Library of 2048 chunks x 512 slots, 8 query tokens, every chunk read).

The reference reads one Library on one device (xenc/injector.py:149-157, 231-273). Its dense read is
    r = sum_c w_c r_c,   w = softmax_c(l_c),  l_c = route_temp * q . S_c           (xenc/injector.py:220-229)
which regroups by chunk shard g (chunks [lo_g, hi_g)) as
    M_g = max_{c in g} l_c,  Z_g = sum_{c in g} e^(l_c - M_g),  A_g = sum_{c in g} e^(l_c - M_g) r_c
    r   = sum_g e^(M_g - M) A_g / sum_g e^(M_g - M) Z_g,         M = max_g M_g.
So each rank keeps its chunk shard of K and S in its own HBM, computes its partial (M_g, Z_g, A_g) with
ops.route_lse + ops.read_multi into one flat block, the blocks are exchanged, and ops.shard_merge combines them.
On GPUs with one process per GPU of one node the exchange goes over NVLink peer memory (PeerExchange: each rank's
block pushed straight into every rank's exchange buffer, the merge waiting on per-block flags); otherwise one
all-gather over the process group lays the blocks end to end in rank order. Every rank takes the same exchange
steps in the same order.

The compute is pluggable (`compute=`) so that the orchestration -- the partition, the block layout, the
collective -- is testable on CPU ranks (gloo) with the oracle standing in for the kernels; the product path
uses CudaShardCompute, and there is no CPU path.
"""

from __future__ import annotations

import contextlib
import ctypes
import socket
from typing import Optional

import torch
import torch.distributed as dist

from . import _native as N
from . import ops


def partition_chunks(n_chunks: int, world: int) -> list:
    """Even contiguous chunk ranges [(lo, hi)] per rank; the first n_chunks % world ranks get one more chunk."""
    n_chunks, world = int(n_chunks), int(world)
    if world <= 0:
        raise ValueError(f"world={world} must be positive")
    if n_chunks < world:
        raise ValueError(f"{n_chunks} chunks cannot be sharded over {world} ranks (every shard needs a chunk)")
    base, extra = divmod(n_chunks, world)
    out, lo = [], 0
    for g in range(world):
        hi = lo + base + (1 if g < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def shard_pages(pages: ops.Pages, lo: int, hi: int) -> ops.Pages:
    """The view of chunks [lo, hi) of every Library in `pages` (page table, counts and keys sliced; the slot pool
    is shared, so nothing is copied)."""
    nco = None
    if pages.n_chunks_of is not None:
        nco = (pages.n_chunks_of - lo).clamp(0, hi - lo).to(torch.int32)
    return ops.Pages(slots=pages.slots, page_of=pages.page_of[:, lo:hi].contiguous(),
                     n_valid=pages.n_valid[:, lo:hi].contiguous(), S=pages.S[:, lo:hi].contiguous(), n_chunks_of=nco,
                     vslots=pages.vslots)


class CudaShardCompute:
    """The kernels: route_lse + the many-query read into a block, shard_merge of the gathered blocks."""

    def __init__(self, route_temp: float = 10.0, read_temp: float = 12.0, read_softmax: bool = True):
        self.route_temp, self.read_temp, self.read_softmax = float(route_temp), float(read_temp), bool(read_softmax)

    def partial(self, q: torch.Tensor, pages: ops.Pages, rows_per_lib: int, header: torch.Tensor,
                acc: torch.Tensor) -> None:
        w, _ = ops.route_lse(q, pages.S, rows_per_lib=rows_per_lib, route_temp=self.route_temp,
                             n_chunks_of=pages.n_chunks_of, header_out=header)
        ops.read_weighted(q, pages, w, rows_per_lib=rows_per_lib, read_temp=self.read_temp,
                          read_softmax=self.read_softmax, out=acc)

    def partial_from_hidden(self, h: torch.Tensor, w_in: torch.Tensor, w_prep, pages: ops.Pages, rows_per_lib: int,
                            header: torch.Tensor, acc: torch.Tensor) -> torch.Tensor:
        """The input projection of the hidden rows h fused with the shard's routing (one pass after the GEMM),
        then the read; returns q."""
        q, w, _ = ops.project_in_route_lse(h, w_in, S=pages.S, rows_per_lib=rows_per_lib,
                                           route_temp=self.route_temp, n_chunks_of=pages.n_chunks_of,
                                           header_out=header, w_prep=w_prep)
        ops.read_weighted(q, pages, w, rows_per_lib=rows_per_lib, read_temp=self.read_temp,
                          read_softmax=self.read_softmax, out=acc)
        return q

    def merge(self, gathered: torch.Tensor, world: int, n_rows: int, d_s: int, out: torch.Tensor) -> None:
        ops.shard_merge(gathered, world, n_rows, d_s, out=out)


class PeerExchange:
    """The partial blocks of a chunk-sharded read over NVLink peer memory (xencb_shard_push /
    xencb_shard_merge_wait): every rank allocates an exchange buffer (xencb_exch_alloc), the CUDA IPC handles are
    swapped once over the process group and each rank maps the others' buffers (xencb_exch_open). A step pushes
    this rank's block into slot `rank` of every buffer with plain peer stores and raises that slot's flag; the merge
    waits for the flags (bounded) and combines the blocks. The epochs live in a small device state, so a step
    captured in a CUDA graph replays. close() (collective) unmaps and frees."""

    def __init__(self, per: int, world: int, rank: int, device: torch.device, group=None):
        """Collective. Every rank takes the same steps whatever fails locally; `ok` is True only when every rank
        mapped every buffer (otherwise nothing stays allocated and the caller uses the all-gather)."""
        L = N.lib()
        self.per, self.world, self.rank, self.group = int(per), int(world), int(rank), group
        self.device = torch.device(device)
        self.ptr, self.opened = None, []
        ok = True
        handle = ctypes.create_string_buffer(64)
        nbytes = L.xencb_exch_bytes(self.world, self.per)
        if nbytes == 0:
            ok = False
        else:
            ptr = ctypes.c_void_p()
            with self._on_device():
                ok = L.xencb_exch_alloc(nbytes, ctypes.byref(ptr), ctypes.cast(handle, ctypes.c_void_p)) == N.OK
            self.ptr = ptr.value if ok else None
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw if ok else None, group=group)
        peers = []
        if ok and all(h is not None for h in handles):
            for g, h in enumerate(handles):
                if g == self.rank:
                    peers.append(self.ptr)
                    continue
                pp = ctypes.c_void_p()
                hb = ctypes.create_string_buffer(bytes(h), 64)
                with self._on_device():
                    if L.xencb_exch_open(ctypes.cast(hb, ctypes.c_void_p), ctypes.byref(pp)) != N.OK:
                        ok = False
                        break
                peers.append(pp.value)
                self.opened.append(pp.value)
        else:
            ok = False
        votes = [None] * self.world
        dist.all_gather_object(votes, ok, group=group)
        self.ok = all(votes)
        if not self.ok:
            self._release()
        else:
            self.peers_dev = torch.tensor(peers, dtype=torch.int64, device=self.device)
            self.state = torch.zeros(4, dtype=torch.int32, device=self.device)
        dist.barrier(group=group)  # every buffer is mapped everywhere (or released everywhere) before going on

    def push(self, block: torch.Tensor) -> None:
        N.call("xencb_shard_push", ops._ptr(block), self.per, ops._ptr(self.peers_dev), self.world, self.rank,
               ops._ptr(self.state), ops._stream(self.device))

    def merge(self, n_rows: int, d_s: int, out: torch.Tensor) -> torch.Tensor:
        N.call("xencb_shard_merge_wait", ctypes.c_void_p(self.ptr), self.world, int(n_rows), int(d_s),
               ops._ptr(self.state), ops._ptr(out), ops._stream(self.device))
        return out

    def _on_device(self):
        return torch.cuda.device(self.device) if self.device.type == "cuda" else contextlib.nullcontext()

    def _release(self) -> None:
        L = N.lib()
        with self._on_device():
            for pp in self.opened:
                L.xencb_exch_close(ctypes.c_void_p(pp))
            self.opened = []
            if self.ptr:
                L.xencb_exch_free(ctypes.c_void_p(self.ptr))
            self.ptr = None

    def close(self) -> None:
        """Collective: no rank unmaps or frees while another may still push into its buffer."""
        if self.ptr is None:
            return
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._release()


def _one_gpu_per_rank(device: torch.device, group=None) -> bool:
    """Every rank of `group` on its own GPU of this node (the peer exchange's precondition)."""
    me = (socket.gethostname(), str(torch.cuda.get_device_properties(device).uuid))
    world = dist.get_world_size(group)
    seen = [None] * world
    dist.all_gather_object(seen, me, group=group)
    return len({h for h, _ in seen}) == 1 and len({u for _, u in seen}) == world


class ShardedRead:
    """r [n_rows, d_s] of the whole Library from this rank's chunk shard `pages` (one Library, or several with
    rows_per_lib rows each). Buffers are allocated once, so a step is CUDA-graph capturable (the all-gather
    included, on NCCL)."""

    def __init__(self, pages: ops.Pages, n_rows: int, *, rows_per_lib: Optional[int] = None, group=None,
                 compute=None, device=None, exchange: str = "auto"):
        self.pages = pages
        self.n_rows = int(n_rows)
        self.rows_per_lib = int(rows_per_lib or n_rows)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.compute = compute or CudaShardCompute()
        self.d_s = int(pages.S.shape[-1])
        device = torch.device(device) if device is not None else pages.S.device
        per = self.n_rows * 4 + self.n_rows * self.d_s
        self.block = torch.zeros(per, dtype=torch.float32, device=device)
        self.gathered = torch.zeros(self.world * per, dtype=torch.float32, device=device)
        self.r = torch.empty(self.n_rows, self.d_s, dtype=torch.float32, device=device)
        self.header, self.acc = ops.shard_views(self.block, self.n_rows, self.d_s)
        # exchange: "peer" (NVLink peer memory), "collective" (all-gather), or "auto" (peer when every rank has
        # its own GPU of one node and the kernels are the CUDA ones)
        if exchange not in ("auto", "peer", "collective"):
            raise ValueError(f"ShardedRead: exchange={exchange!r} is not one of auto, peer, collective")
        self.peer = None
        want_peer = (self.world > 1 and exchange != "collective" and device.type == "cuda"
                     and isinstance(self.compute, CudaShardCompute))
        if want_peer and _one_gpu_per_rank(device, group):
            pe = PeerExchange(per, self.world, self.rank, device, group)
            self.peer = pe if pe.ok else None
        if self.peer is None and exchange == "peer" and self.world > 1:
            raise ValueError("ShardedRead: exchange='peer' needs CUDA kernels, one GPU per rank on one node and "
                             "peer mappings of the exchange buffers")
        self.exchange_kind = "peer" if self.peer is not None else ("collective" if self.world > 1 else "none")

    def partial_from_hidden(self, h: torch.Tensor, w_in: torch.Tensor, w_prep=None) -> torch.Tensor:
        """This rank's block from the hidden rows h [n_rows, d_m]: q = project_in(h) (rms, L2) fused with the
        routing, then the read (CUDA kernels only). Returns the block."""
        if not isinstance(self.compute, CudaShardCompute):
            raise TypeError("ShardedRead.partial_from_hidden needs the CUDA kernels")
        self.compute.partial_from_hidden(h, w_in, w_prep, self.pages, self.rows_per_lib, self.header, self.acc)
        return self.block

    def partial(self, q: torch.Tensor) -> torch.Tensor:
        """This rank's block (headers, accumulators) for query rows q [n_rows, d_s]."""
        if tuple(q.shape) != (self.n_rows, self.d_s):
            raise ValueError(f"ShardedRead: q must be [{self.n_rows}, {self.d_s}], got {tuple(q.shape)}")
        self.compute.partial(q, self.pages, self.rows_per_lib, self.header, self.acc)
        return self.block

    def exchange(self) -> None:
        """Every rank's block to every rank: pushed over peer memory, or one all-gather into `gathered`."""
        if self.peer is not None:
            self.peer.push(self.block)
        elif self.world > 1:
            dist.all_gather_into_tensor(self.gathered, self.block, group=self.group)

    def merge(self) -> torch.Tensor:
        if self.peer is not None:
            return self.peer.merge(self.n_rows, self.d_s, self.r)
        src = self.gathered if self.world > 1 else self.block
        self.compute.merge(src, self.world, self.n_rows, self.d_s, self.r)
        return self.r

    def close(self) -> None:
        """Collective when the exchange is on peer memory: unmaps and frees the exchange buffers."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def __call__(self, q: torch.Tensor) -> torch.Tensor:
        self.partial(q)
        self.exchange()
        return self.merge()
