"""Host logic of the chunk-sharded read on CPU ranks (gloo, world size 2 and 3).

Each rank builds the same seeded Library, keeps its chunk range (partition_chunks), and runs ShardedRead with
the numpy oracle standing in for the kernels (partial = oracle.shard_partials written into the rank's block,
merge = oracle.merge_shards over the gathered blocks). The all-gather is the real torch.distributed collective,
so the test checks the partition, the block layout and the gather order end to end: the merged read must equal
the oracle's unsharded dense read."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kv_skill_v2_b200 import ops
from kv_skill_v2_b200.shard import ShardedRead, partition_chunks, shard_pages
from oracle import xenc_oracle as X


def test_partition_chunks_covers_evenly():
    for C in (1, 2, 7, 8, 48, 2048, 2049):
        for world in (1, 2, 3, 4, 8):
            if C < world:
                with pytest.raises(ValueError):
                    partition_chunks(C, world)
                continue
            parts = partition_chunks(C, world)
            assert parts[0][0] == 0 and parts[-1][1] == C
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1


def test_shard_pages_slices_tables_not_slots():
    C, N, d = 10, 4, 8
    slots = torch.zeros(2 * C, N, d, dtype=torch.float16)
    pages = ops.Pages(slots=slots, page_of=torch.arange(2 * C, dtype=torch.int32).view(2, C),
                      n_valid=torch.full((2, C), N, dtype=torch.int32), S=torch.randn(2, C, d),
                      n_chunks_of=torch.tensor([10, 6], dtype=torch.int32))
    sp = shard_pages(pages, 4, 8)
    assert sp.slots is slots
    assert sp.page_of.tolist() == [[4, 5, 6, 7], [14, 15, 16, 17]]
    assert torch.equal(sp.S, pages.S[:, 4:8])
    assert sp.n_chunks_of.tolist() == [4, 2]
    assert shard_pages(pages, 8, 10).n_chunks_of.tolist() == [2, 0]


C, N, D, T = 12, 16, 32, 5


def _library():
    rng = np.random.default_rng(0)
    K = rng.standard_normal((C, N, D)).astype(np.float32)
    K /= np.linalg.norm(K, axis=-1, keepdims=True)
    M = np.ones((C, N), bool)
    M[-1, 9:] = False
    M[3, 1:] = False
    q = rng.standard_normal((T, D)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    return K, M, q


class OracleCompute:
    """Test stand-in for CudaShardCompute: the oracle's shard partial and merge on CPU tensors."""

    def __init__(self, K, M, softmax):
        self.K, self.M, self.softmax = K, M, softmax
        self.lo = self.hi = None

    def partial(self, q, pages, rows_per_lib, header, acc):
        Kl, Ml = self.K[self.lo:self.hi], self.M[self.lo:self.hi]
        Mx, Z, A = X.shard_partials(q.numpy(), Kl, Ml, X.summaries(Kl, Ml), 10.0, 12.0, self.softmax)
        header.zero_()
        header[:, 0] = torch.from_numpy(Mx)
        header[:, 1] = torch.from_numpy(Z)
        acc.copy_(torch.from_numpy(A))

    def merge(self, gathered, world, n_rows, d_s, out):
        per = n_rows * 4 + n_rows * d_s
        parts = []
        for g in range(world):
            blk = gathered[g * per:(g + 1) * per]
            hdr, acc = ops.shard_views(blk, n_rows, d_s)
            parts.append((hdr[:, 0].numpy(), hdr[:, 1].numpy(), acc.numpy()))
        out.copy_(torch.from_numpy(X.merge_shards(parts)))


def _rank_main(rank, world, port, softmax, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        K, M, q = _library()
        lo, hi = partition_chunks(C, world)[rank]
        comp = OracleCompute(K, M, softmax)
        comp.lo, comp.hi = lo, hi
        pages = ops.Pages(slots=torch.zeros(1, N, D, dtype=torch.float16),
                          page_of=torch.arange(hi - lo, dtype=torch.int32).view(1, -1),
                          n_valid=torch.from_numpy(M[lo:hi].sum(-1).astype(np.int32)).view(1, -1),
                          S=torch.from_numpy(X.summaries(K[lo:hi], M[lo:hi])).view(1, hi - lo, D))
        sr = ShardedRead(pages, T, compute=comp, device="cpu")
        assert sr.world == world and sr.rank == rank
        r = sr(torch.from_numpy(q)).clone()
        # every rank ends with the same merged read
        allr = [torch.empty_like(r) for _ in range(world)]
        dist.all_gather(allr, r)
        if rank == 0:
            np.save(result_path, torch.stack(allr).numpy())
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("softmax", [True, False])
def test_sharded_read_gloo_matches_unsharded_oracle(tmp_path, world, softmax):
    out = tmp_path / "r.npy"
    mp.start_processes(_rank_main, args=(world, _free_port(), softmax, str(out)), nprocs=world, join=True,
                       start_method="spawn")
    got = np.load(out)
    K, M, q = _library()
    w, _, _ = X.route(q, X.summaries(K, M), 10.0, 0)
    ref = X.read(q, K, M, w, 12.0, softmax)
    for g in range(world):
        assert np.abs(got[g] - ref).max() <= 1e-5 * np.abs(ref).max(), g


class _FakeExchLib:
    """Stands in for libxencb's exchange entry points on CPU ranks: allocation and mapping succeed or fail as
    told, and every successful call is recorded, so the collective set-up of PeerExchange is checked without a
    GPU."""

    def __init__(self, fail_alloc=False, fail_open=False):
        self.fail_alloc, self.fail_open = fail_alloc, fail_open
        self.calls = []

    def xencb_exch_bytes(self, world, per):
        return 256 + 2 * world * per * 4

    def xencb_exch_alloc(self, nbytes, ptr_ref, handle):
        if self.fail_alloc:
            return 2
        import ctypes
        self.calls.append("alloc")
        ctypes.cast(ptr_ref, ctypes.POINTER(ctypes.c_void_p))[0] = 0x1000
        return 0

    def xencb_exch_open(self, handle, ptr_ref):
        if self.fail_open:
            return 2
        import ctypes
        self.calls.append("open")
        ctypes.cast(ptr_ref, ctypes.POINTER(ctypes.c_void_p))[0] = 0x2000
        return 0

    def xencb_exch_close(self, p):
        self.calls.append("close")
        return 0

    def xencb_exch_free(self, p):
        self.calls.append("free")
        return 0


def _exch_rank(rank, world, port, failing_rank, mode, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kv_skill_v2_b200 import _native as N
        from kv_skill_v2_b200.shard import PeerExchange
        fake = _FakeExchLib(fail_alloc=(mode == "alloc" and rank == failing_rank),
                            fail_open=(mode == "open" and rank == failing_rank))
        N.lib = lambda: fake  # this spawned process only
        pe = PeerExchange(per=40, world=world, rank=rank, device=torch.device("cpu"))
        held = "alloc" in fake.calls and "free" not in fake.calls
        with open(f"{result_path}.{rank}", "w") as f:
            f.write(f"{int(pe.ok)} {int(held)} {fake.calls.count('open')} {fake.calls.count('close')}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["none", "alloc", "open"])
def test_peer_exchange_setup_agrees_across_ranks(tmp_path, mode):
    """One rank failing to allocate or to map a peer buffer makes every rank give the peer exchange up (and free
    what it holds) instead of leaving the ranks on different exchanges; without failures every rank maps the
    others' buffers and keeps its own."""
    world, failing = 3, 1
    out = tmp_path / "r"
    mp.start_processes(_exch_rank, args=(world, _free_port(), failing, mode, str(out)), nprocs=world, join=True,
                       start_method="spawn")
    res = [open(f"{out}.{r}").read().split() for r in range(world)]
    assert {r[0] for r in res} == ({"1"} if mode == "none" else {"0"})
    for r in res:
        if mode == "none":
            assert r[1] == "1" and r[2] == str(world - 1)
        else:
            assert r[1] == "0" and r[2] == r[3]  # nothing left allocated, every opened mapping closed
