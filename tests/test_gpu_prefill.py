"""Prefill (registration) read on the tensor cores (BASELINE config 3's path): two tcgen05 GEMMs, scores with the
chunk softmax folded into f16 weights P, then r = P K. Checked against the oracle's dense read
(xenc/injector.py:239-265) on seeded inputs: tokens per Library not a multiple of the 128-token tile, page sizes
below / above 256 and not a multiple of 64 (one or two MMAs per chunk), ragged chunks, chunk counts per Library,
dense and top-k routing weights, softmax and linear reads; and at config-3 shapes on a sample of tokens."""

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


def _build(n_lib, C, N, d, seed, dev, n_chunks_of=None):
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(seed)
    K = torch.randn(n_lib, C, N, d, generator=g)
    K = (K / K.norm(dim=-1, keepdim=True)).half()
    nv = torch.full((n_lib, C), N, dtype=torch.int32)
    nv[:, -1] = torch.randint(1, N + 1, (n_lib,), generator=g, dtype=torch.int32)
    if C > 2:
        nv[:, 1] = torch.randint(1, N + 1, (n_lib,), generator=g, dtype=torch.int32)
    # rows past n_valid are zero, as the Library pads them
    mask = torch.arange(N).view(1, 1, N) < nv.view(n_lib, C, 1)
    K = K * mask.unsqueeze(-1).half()
    slots = K.reshape(n_lib * C, N, d).to(dev).contiguous()
    page_of = torch.arange(n_lib * C, dtype=torch.int32, device=dev).view(n_lib, C)
    S = ops.summaries(slots, page_of, nv.to(dev))
    nco = None if n_chunks_of is None else torch.tensor(n_chunks_of, dtype=torch.int32, device=dev)
    pages = ops.Pages(slots=slots, page_of=page_of, n_valid=nv.to(dev), S=S, n_chunks_of=nco)
    return pages, K.float().numpy(), nv.numpy()


CASES = [
    # (n_lib, T, C, page_rows, d_s, top_k, n_chunks_of)
    (1, 128, 4, 64, 64, 0, None),
    (2, 200, 6, 96, 128, 0, None),       # T not a multiple of 128, page_rows not a multiple of 64
    (1, 256, 5, 512, 256, 0, None),      # 512 score columns per chunk: two N=256 MMAs
    (2, 130, 3, 320, 64, 2, None),       # 320 columns (256 + 64), top-k weights
    (3, 64, 7, 128, 512, 3, [7, 4, 6]),  # chunk counts per Library
    (2, 300, 4, 256, 128, 2, [4, 3]),    # 256 columns: CTA pairs with an odd tile count, chunk counts per Library
]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("softmax", [True, False])
def test_prefill_matches_oracle(dev, case, softmax):
    from kv_skill_v2_b200 import ops
    n_lib, T, C, N, d, top_k, nco = case
    pages, K, nv = _build(n_lib, C, N, d, seed=n_lib * 17 + C, dev=dev, n_chunks_of=nco)
    g = torch.Generator().manual_seed(3)
    R = n_lib * T
    q = torch.nn.functional.normalize(torch.randn(R, d, generator=g), dim=-1)
    _, _, w, _ = ops.route(q.to(dev), pages.S, rows_per_lib=T, top_k=top_k, route_temp=10.0,
                           n_chunks_of=pages.n_chunks_of)
    r = ops.read_prefill(q.to(dev), pages, w, rows_per_lib=T, read_temp=12.0, read_softmax=softmax)
    wn = w.cpu().numpy()
    ref = np.zeros((R, d), np.float32)
    for lib in range(n_lib):
        nc = C if nco is None else nco[lib]
        rows = slice(lib * T, lib * T + T)
        M = np.arange(N)[None, :] < nv[lib, :nc][:, None]
        ref[rows] = X.read(q.numpy()[rows], K[lib, :nc], M, wn[rows, :nc], 12.0, softmax)
    assert rel_err(r, ref) < TOL, case
    assert ops.device_status(dev) == 0


def test_prefill_agrees_with_many_query_read(dev):
    from kv_skill_v2_b200 import ops
    pages, _, _ = _build(2, 8, 256, 256, seed=5, dev=dev)
    q = torch.nn.functional.normalize(torch.randn(2 * 300, 256, generator=torch.Generator().manual_seed(9)), dim=-1)
    _, _, w, _ = ops.route(q.to(dev), pages.S, rows_per_lib=300, top_k=0, route_temp=10.0)
    a = ops.read_prefill(q.to(dev), pages, w, rows_per_lib=300)
    b = ops.read_multi(q.to(dev), pages, w, rows_per_lib=300)
    assert rel_err(a, b) < 1e-3  # f16 q in the score product vs split f16 q; both within TOL of the oracle


def test_prefill_config3_shapes_sample(dev):
    """One config-3 document: T = 2048 tokens, 128 chunks x 512 fp16 slots, d_s 2048, every chunk read; 16 sampled
    tokens against the oracle's dense read."""
    from kv_skill_v2_b200 import ops
    C, N, d, T = 128, 512, 2048, 2048
    gd = torch.Generator(device=dev).manual_seed(0)
    slots = torch.randn(C, N, d, generator=gd, device=dev)
    slots = (slots / slots.norm(dim=-1, keepdim=True)).half()
    nv = torch.full((1, C), N, dtype=torch.int32, device=dev)
    nv[0, -1] = 300
    slots[-1, 300:] = 0
    po = torch.arange(C, dtype=torch.int32, device=dev).view(1, C)
    pages = ops.Pages(slots=slots, page_of=po, n_valid=nv, S=ops.summaries(slots, po, nv))
    q = torch.nn.functional.normalize(torch.randn(T, d, generator=gd, device=dev), dim=-1)
    _, _, w, _ = ops.route(q, pages.S, rows_per_lib=T, top_k=0, route_temp=10.0)
    r = ops.read_prefill(q, pages, w, rows_per_lib=T)
    idx = torch.randperm(T, generator=torch.Generator().manual_seed(1))[:16].sort().values
    K = slots.float().cpu().numpy()
    M = np.arange(N)[None, :] < nv[0].cpu().numpy()[:, None]
    ref = X.read(q[idx.to(dev)].cpu().numpy(), K, M, w[idx.to(dev)].cpu().numpy(), 12.0, True)
    assert rel_err(r[idx.to(dev)], ref) < TOL
    assert ops.device_status(dev) == 0


def test_route_logits_tiled_for_many_rows(dev):
    """Libraries with >= 64 rows take the shared-memory-tiled logits kernel; its logits, weights and index sets
    match the oracle's routing (xenc/injector.py:220-229), with chunk counts per Library."""
    from kv_skill_v2_b200 import ops
    from tests._fixtures import topk_sets
    g = torch.Generator().manual_seed(12)
    n_lib, T, C, d = 3, 150, 70, 96
    S = torch.nn.functional.normalize(torch.randn(n_lib, C, d, generator=g), dim=-1)
    q = torch.nn.functional.normalize(torch.randn(n_lib * T, d, generator=g), dim=-1)
    nco = [70, 33, 64]
    for top_k in (0, 4):
        idx, wk, w, lg = ops.route(q.to(dev), S.to(dev), rows_per_lib=T, top_k=top_k, route_temp=10.0,
                                   n_chunks_of=torch.tensor(nco, dtype=torch.int32, device=dev), want_logits=True)
        for lib in range(n_lib):
            rows = slice(lib * T, lib * T + T)
            nc = nco[lib]
            ref_l = (q[rows].numpy() @ S[lib, :nc].numpy().T) * 10.0
            assert rel_err(lg[rows, :nc], ref_l) < 1e-5
            assert torch.isinf(lg[rows, nc:]).all()
            wo, _, _ = X.route(q[rows].numpy(), S[lib, :nc].numpy(), 10.0, top_k)
            assert topk_sets(w[rows, :nc]) == topk_sets(wo)
            assert rel_err(w[rows, :nc], wo) < 1e-5



@pytest.mark.parametrize("T", [390, 256])
def test_prefill_pair_read_matches_single(dev, T):
    """The read as CTA pairs (cta_group::2, d_s in 512-column slices) gives the single-CTA kernel's r."""
    import os
    from kv_skill_v2_b200 import ops
    pages, _, _ = _build(2, 5, 192, 1024, seed=T, dev=dev)
    q = torch.nn.functional.normalize(torch.randn(2 * T, 1024, generator=torch.Generator().manual_seed(4)), dim=-1)
    _, _, w, _ = ops.route(q.to(dev), pages.S, rows_per_lib=T, top_k=3, route_temp=10.0)
    a = ops.read_prefill(q.to(dev), pages, w, rows_per_lib=T)
    os.environ["XENCB_PREFILL_PAIR"] = "0"
    try:
        b = ops.read_prefill(q.to(dev), pages, w, rows_per_lib=T)
    finally:
        del os.environ["XENCB_PREFILL_PAIR"]
    assert rel_err(a, b) < 1e-6
    assert ops.device_status(dev) == 0
