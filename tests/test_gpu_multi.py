"""Many-query read (read_multi), dense shard routing (route_lse) and the shard merge, against the oracle.

The many-query read is the dense read of a Library queried by several tokens at once (xenc/injector.py:239-265
with T > 1); the shard partials regroup the routing softmax by chunk shard (oracle.shard_partials /
merge_shards). Cases cover: chunks cut into pieces that straddle CTA ranges (open partials), CTAs whose range
spans several query groups (several fold slots), partial query groups (T not a multiple of 8), ragged chunks,
chunk counts per Library, f16 / bf16 slots, softmax and linear reads, dense and top-k weights."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import xenc_oracle as X
from tests._fixtures import TOL, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _status_clean(dev):
    from kv_skill_v2_b200 import ops
    assert ops.device_status(dev) == 0, "a kernel flagged a device status bit"


def _libraries(n_lib, C, N, d, seed, ragged=True):
    """Unit-row slots [n_lib, C, N, d] (float32 values exactly representable in f16) and n_valid [n_lib, C]."""
    g = torch.Generator().manual_seed(seed)
    K = torch.randn(n_lib, C, N, d, generator=g)
    K = (K / K.norm(dim=-1, keepdim=True)).half().float()
    nv = torch.full((n_lib, C), N, dtype=torch.int32)
    if ragged:
        nv[:, -1] = torch.randint(1, N + 1, (n_lib,), generator=g, dtype=torch.int32)
        if C > 2:
            nv[:, C // 2] = torch.randint(1, N + 1, (n_lib,), generator=g, dtype=torch.int32)
    return K, nv


def _pages(K, nv, dev, slot_dtype, n_chunks_of=None):
    from kv_skill_v2_b200 import ops
    n_lib, C, N, d = K.shape
    slots = K.reshape(n_lib * C, N, d).to(slot_dtype).to(dev).contiguous()
    page_of = torch.arange(n_lib * C, dtype=torch.int32, device=dev).view(n_lib, C)
    nv_d = nv.to(dev)
    S = ops.summaries(slots, page_of, nv_d)
    nco = None if n_chunks_of is None else torch.tensor(n_chunks_of, dtype=torch.int32, device=dev)
    return ops.Pages(slots=slots, page_of=page_of, n_valid=nv_d, S=S, n_chunks_of=nco)


def _oracle_rows(q, K, nv, w, T, softmax, n_chunks_of=None):
    """Per Library, the oracle's read for its T rows (chunks past the Library's count excluded)."""
    n_lib, C, N, d = K.shape
    R = q.shape[0]
    out = np.zeros((R, d), np.float32)
    for lib in range((R + T - 1) // T):
        rows = slice(lib * T, min(R, lib * T + T))
        nc = C if n_chunks_of is None else n_chunks_of[lib]
        Kl = K[lib, :nc].numpy()
        M = np.arange(N)[None, :] < nv[lib, :nc].numpy()[:, None]
        out[rows] = X.read(q[rows], Kl, M, w[rows, :nc], 12.0, softmax)
    return out


CASES = [
    # (n_lib, T, C, N, d_s, top_k, n_chunks_of): pieces and CTA ranges differ per case
    (1, 8, 5, 96, 64, 0, None),        # 15 units on 15 CTAs: every chunk cut in 3 open pieces
    (1, 3, 40, 96, 256, 0, None),      # partial query group, complete + open chunks
    (3, 11, 40, 96, 256, 2, None),     # two groups per Library (8 + 3 rows), top-k weights
    (2, 8, 24, 160, 2560, 0, [24, 17]),  # the config-5 width (16-column tiles x 16 per warp), chunk counts
    (400, 1, 4, 32, 64, 0, None),      # CTAs spanning several groups (several fold slots each)
    (6, 5, 9, 200, 2048, 3, None),     # the config-2 width, ragged, top-k
]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("slot_dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("softmax", [True, False])
def test_read_multi_matches_oracle(dev, case, slot_dtype, softmax):
    from kv_skill_v2_b200 import ops
    n_lib, T, C, N, d, top_k, nco = case
    K, nv = _libraries(n_lib, C, N, d, seed=n_lib * 131 + C)
    if slot_dtype == torch.bfloat16:
        K = K.bfloat16().float()
    pages = _pages(K, nv, dev, slot_dtype, nco)
    R = n_lib * T
    g = torch.Generator().manual_seed(7)
    q = torch.nn.functional.normalize(torch.randn(R, d, generator=g), dim=-1)
    _, _, w, _ = ops.route(q.to(dev), pages.S, rows_per_lib=T, top_k=top_k, route_temp=10.0,
                           n_chunks_of=pages.n_chunks_of)
    if ops.multi_supported(pages, R, T):
        r = ops.read_multi(q.to(dev), pages, w, rows_per_lib=T, read_temp=12.0, read_softmax=softmax)
    else:  # bf16 at d_s 2560: query fragments and two stages do not fit on chip -> the decode kernel
        assert slot_dtype == torch.bfloat16 and d > 2048
        with pytest.raises(NotImplementedError):
            ops.read_multi(q.to(dev), pages, w, rows_per_lib=T)
        r = ops.read_weighted(q.to(dev), pages, w, rows_per_lib=T, read_temp=12.0, read_softmax=softmax)
    ref = _oracle_rows(q.numpy(), K, nv, w.cpu().numpy(), T, softmax, nco)
    assert rel_err(r, ref) < TOL, case
    _status_clean(dev)


def test_read_multi_equals_decode_read(dev):
    """Same weights through both read kernels (the decode read takes each row's chunks as separate items)."""
    from kv_skill_v2_b200 import ops
    K, nv = _libraries(2, 16, 128, 512, seed=5)
    pages = _pages(K, nv, dev, torch.float16)
    g = torch.Generator().manual_seed(1)
    q = torch.nn.functional.normalize(torch.randn(12, 512, generator=g), dim=-1).to(dev)
    for top_k in (0, 4):
        idx, wk, w, _ = ops.route(q, pages.S, rows_per_lib=6, top_k=top_k, route_temp=10.0)
        a = ops.read_multi(q, pages, w, rows_per_lib=6)
        b = ops.read_decode(q, pages, idx, wk, rows_per_lib=6)
        assert rel_err(a, b) < 5e-4  # both within TOL of the oracle; P is rounded at different points
    _status_clean(dev)


def test_read_weighted_f32_slots_use_decode_kernel(dev):
    from kv_skill_v2_b200 import ops
    K, nv = _libraries(1, 6, 64, 100, seed=9)
    pages = _pages(K, nv, dev, torch.float32)
    q = torch.nn.functional.normalize(torch.randn(5, 100), dim=-1)
    _, _, w, _ = ops.route(q.to(dev), pages.S, rows_per_lib=5, top_k=0, route_temp=10.0)
    with pytest.raises(NotImplementedError):
        ops.read_multi(q.to(dev), pages, w, rows_per_lib=5)
    r = ops.read_weighted(q.to(dev), pages, w, rows_per_lib=5)
    ref = _oracle_rows(q.numpy(), K, nv, w.cpu().numpy(), 5, True)
    assert rel_err(r, ref) < TOL
    _status_clean(dev)


@pytest.mark.parametrize("bounds", [[0, 48], [0, 24, 48], [0, 7, 30, 48], [0, 12, 24, 36, 48], [0, 1, 47, 48]])
@pytest.mark.parametrize("softmax", [True, False])
def test_shards_merge_to_the_whole_read(dev, bounds, softmax):
    """Chunk shards of one Library (uneven, down to one chunk): route_lse + read_multi per shard, blocks laid end
    to end as an all-gather leaves them, shard_merge -> the unsharded dense read of the oracle; the headers match
    oracle.shard_partials."""
    from kv_skill_v2_b200 import ops
    C, N, d, T = 48, 128, 512, 8
    K, nv = _libraries(1, C, N, d, seed=21)
    g = torch.Generator().manual_seed(2)
    q = torch.nn.functional.normalize(torch.randn(T, d, generator=g), dim=-1)
    G = len(bounds) - 1
    parts = torch.empty(G, T * 4 + T * d, dtype=torch.float32, device=dev)
    for i in range(G):
        lo, hi = bounds[i], bounds[i + 1]
        pages = _pages(K[:, lo:hi], nv[:, lo:hi], dev, torch.float16)
        hdr, acc = ops.shard_views(parts[i], T, d)
        w, _ = ops.route_lse(q.to(dev), pages.S, rows_per_lib=T, route_temp=10.0, header_out=hdr)
        ops.read_multi(q.to(dev), pages, w, rows_per_lib=T, read_softmax=softmax, out=acc)
        Kl = K[0, lo:hi].numpy()
        M = np.arange(N)[None, :] < nv[0, lo:hi].numpy()[:, None]
        Mx, Z, A = X.shard_partials(q.numpy(), Kl, M, X.summaries(Kl, M), 10.0, 12.0, softmax)
        assert rel_err(hdr[:, 0], Mx) < 1e-5 and rel_err(hdr[:, 1], Z) < 1e-4
        assert rel_err(acc, A) < TOL
    r = ops.shard_merge(parts, G, T, d)
    Kl = K[0].numpy()
    M = np.arange(N)[None, :] < nv[0].numpy()[:, None]
    w_full, _, _ = X.route(q.numpy(), X.summaries(Kl, M), 10.0, 0)
    ref = X.read(q.numpy(), Kl, M, w_full, 12.0, softmax)
    assert rel_err(r, ref) < TOL
    _status_clean(dev)


def test_config5_shape_shards_agree(dev):
    """BASELINE config-5 width and chunk size on a 256-chunk Library (131,072 slots, 8 queries): the merge of
    2, 4 and 8 emulated shards equals the single-shard read, and a sample of chunks checks the oracle."""
    from kv_skill_v2_b200 import ops
    C, N, d, T = 256, 512, 2560, 8
    g = torch.Generator(device=dev).manual_seed(0)
    K = torch.randn(C, N, d, generator=g, device=dev)
    K = (K / K.norm(dim=-1, keepdim=True)).half()
    nv = torch.full((1, C), N, dtype=torch.int32, device=dev)
    q = torch.nn.functional.normalize(torch.randn(T, d, generator=g, device=dev), dim=-1)

    def part(lo, hi, block):
        pg = torch.arange(hi - lo, dtype=torch.int32, device=dev).view(1, -1)
        slots, nvs = K[lo:hi].contiguous(), nv[:, lo:hi].contiguous()
        pages = ops.Pages(slots=slots, page_of=pg, n_valid=nvs, S=ops.summaries(slots, pg, nvs))
        hdr, acc = ops.shard_views(block, T, d)
        w, _ = ops.route_lse(q, pages.S, rows_per_lib=T, route_temp=10.0, header_out=hdr)
        ops.read_multi(q, pages, w, rows_per_lib=T, out=acc)

    results = {}
    for G in (1, 2, 4, 8):
        parts = torch.empty(G, T * 4 + T * d, dtype=torch.float32, device=dev)
        step = C // G
        for i in range(G):
            part(i * step, (i + 1) * step, parts[i])
        results[G] = ops.shard_merge(parts, G, T, d)
    for G in (2, 4, 8):
        assert rel_err(results[G], results[1]) < 5e-4, G  # f16 rounding of P at other piece boundaries
    # oracle on the first 16 chunks as their own Library
    sub = K[:16].float().cpu().numpy()
    M = np.ones((16, N), bool)
    w16, _, _ = X.route(q.cpu().numpy(), X.summaries(sub, M), 10.0, 0)
    parts = torch.empty(1, T * 4 + T * d, dtype=torch.float32, device=dev)
    part(0, 16, parts[0])
    r16 = ops.shard_merge(parts, 1, T, d)
    assert rel_err(r16, X.read(q.cpu().numpy(), sub, M, w16, 12.0, True)) < TOL
    _status_clean(dev)
