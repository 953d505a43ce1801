"""The partial-block exchange of the chunk-sharded read over peer memory (xencb_shard_push /
xencb_shard_merge_wait, kv_skill_v2_b200.shard.PeerExchange).

On one GPU the ranks are emulated in one process: each "rank" has its own exchange buffer and epoch state on the
same device, the pushes of all ranks run before the merges in one stream (no kernel waits on a kernel that runs
beside it), and every merge must equal ops.shard_merge of the blocks laid end to end, bit for bit, over several
steps (the two halves of the buffer alternate). A merge whose peer never pushed runs its bounded wait out and
reports XENCB_DEV_TIMEOUT. With two or more GPUs, two processes (NCCL) check ShardedRead's peer exchange against
its all-gather exchange, eagerly and replayed from a CUDA graph."""

from __future__ import annotations

import ctypes
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _blocks(G, n_rows, d_s, seed, dev):
    """G shard blocks [n_rows * 4 headers (M, Z, 0, 0), n_rows * d_s accumulators]; some rows empty (Z = 0)."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for s in range(G):
        hdr = torch.zeros(n_rows, 4)
        hdr[:, 0] = torch.randn(n_rows, generator=g) * 3
        hdr[:, 1] = torch.rand(n_rows, generator=g) + 0.5
        if s == 1:
            hdr[0, 1] = 0.0  # shard 1 holds nothing for row 0
        acc = torch.randn(n_rows, d_s, generator=g)
        out.append(torch.cat([hdr.reshape(-1), acc.reshape(-1)]).to(dev))
    return out


def _emulated(G, per, dev):
    from kv_skill_v2_b200 import _native as N
    nbytes = N.lib().xencb_exch_bytes(G, per)
    assert nbytes > 0
    bufs = [torch.zeros(nbytes // 4, dtype=torch.int32, device=dev) for _ in range(G)]
    peers = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    states = [torch.zeros(4, dtype=torch.int32, device=dev) for _ in range(G)]
    return bufs, peers, states


def _push(block, per, peers, G, rank, state, dev):
    from kv_skill_v2_b200 import _native as N, ops
    N.call("xencb_shard_push", ops._ptr(block), per, ops._ptr(peers), G, rank, ops._ptr(state), ops._stream(dev))


def _merge(buf, G, n_rows, d_s, state, out, dev):
    from kv_skill_v2_b200 import _native as N, ops
    N.call("xencb_shard_merge_wait", ops._ptr(buf), G, n_rows, d_s, ops._ptr(state), ops._ptr(out), ops._stream(dev))


@pytest.mark.parametrize("G,n_rows,d_s", [(1, 3, 64), (2, 8, 2560), (4, 5, 300), (8, 8, 2560)])
def test_push_merge_equals_shard_merge(dev, G, n_rows, d_s):
    from kv_skill_v2_b200 import ops
    per = n_rows * 4 + n_rows * d_s
    bufs, peers, states = _emulated(G, per, dev)
    for step in range(3):  # epochs 1, 2, 3: both halves of the buffers, then the first again
        blocks = _blocks(G, n_rows, d_s, seed=100 * step + G, dev=dev)
        for rank in range(G):
            _push(blocks[rank], per, peers, G, rank, states[rank], dev)
        ref = ops.shard_merge(torch.cat(blocks), G, n_rows, d_s)
        for rank in range(G):
            out = torch.empty(n_rows, d_s, device=dev)
            _merge(bufs[rank], G, n_rows, d_s, states[rank], out, dev)
            assert torch.equal(out, ref), (step, rank)
        assert int(states[0][0]) == step + 1 and int(states[0][1]) == step + 1 and int(states[0][2]) == 0
    assert ops.device_status(dev) == 0


def test_merge_without_peer_push_times_out(dev):
    """Rank 1 never pushes: rank 0's merge runs its bounded wait out (about 1.5 s), reports XENCB_DEV_TIMEOUT
    and returns; the context stays usable."""
    from kv_skill_v2_b200 import _native as N, ops
    G, n_rows, d_s = 2, 2, 64
    per = n_rows * 4 + n_rows * d_s
    bufs, peers, states = _emulated(G, per, dev)
    blocks = _blocks(G, n_rows, d_s, seed=7, dev=dev)
    _push(blocks[0], per, peers, G, 0, states[0], dev)
    out = torch.empty(n_rows, d_s, device=dev)
    _merge(bufs[0], G, n_rows, d_s, states[0], out, dev)
    st = ops.device_status(dev)  # synchronises, reads and clears
    assert st & N.DEV_TIMEOUT
    assert ops.device_status(dev) == 0
    torch.ones(4, device=dev).sum().item()  # the device still answers


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    from kv_skill_v2_b200 import ops
    from kv_skill_v2_b200.shard import ShardedRead, partition_chunks
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        C, N, d_s, T = 16, 64, 256, 8
        lo, hi = partition_chunks(C, world)[rank]
        g = torch.Generator().manual_seed(3 + lo)
        slots = torch.nn.functional.normalize(torch.randn(hi - lo, N, d_s, generator=g), dim=-1).half().to(dev)
        po = torch.arange(hi - lo, dtype=torch.int32, device=dev).view(1, -1)
        nv = torch.full((1, hi - lo), N, dtype=torch.int32, device=dev)
        pages = ops.Pages(slots=slots, page_of=po, n_valid=nv, S=ops.summaries(slots, po, nv))
        q = torch.nn.functional.normalize(torch.randn(T, d_s, generator=torch.Generator().manual_seed(9)), dim=-1)
        q = q.to(dev)
        a = ShardedRead(pages, T, rows_per_lib=T, exchange="peer")
        b = ShardedRead(pages, T, rows_per_lib=T, exchange="collective")
        ok = a.exchange_kind == "peer"
        for _ in range(3):
            ra = a(q).clone()
            rb = b(q).clone()
            ok = ok and torch.equal(ra, rb)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            a.partial(q)
            a.exchange()
            a.merge()
        for _ in range(3):
            gr.replay()
            ok = ok and torch.equal(a.r, rb)
        torch.cuda.synchronize(dev)
        ok = ok and ops.device_status(dev) == 0
        del gr
        a.close()
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_peer_exchange_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_two_rank_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        assert (tmp_path / f"rank{r}").read_text() == "ok"
