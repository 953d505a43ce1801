"""Parity of the CUDA path (through the C ABI) with the reference's outputs and the oracle.

Bar: routing index sets identical per token; outputs within max|out - ref| <= 2e-3 * max|ref|.
Golden cases come from the reference's own code (tests/golden/make_golden.py); larger cases use seeded
synthetic inputs checked against the numpy oracle; BASELINE config-2 shapes are checked on a sample of
documents plus size-independent properties."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import xenc_oracle as X
from tests._fixtures import GOLDEN, TOL, TinyReader, load_case, rel_err, topk_sets

pytestmark = pytest.mark.gpu

READ_CASES = ["cfg1_softmax_top2", "cfg1_dense", "cfg1_linear_top2", "cfg1_topk_eq_C", "cfg1_linear_dense",
              "small_ragged_top2", "small_ragged_linear", "small_ragged_dense_t3", "one_chunk", "odd_dims_top3"]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _status_clean(dev):
    from kv_skill_v2_b200 import ops
    assert ops.device_status(dev) == 0, "a kernel flagged a device status bit"


def _pages_from_case(c, dev, slot_dtype=torch.float16):
    from kv_skill_v2_b200 import ops
    K = torch.from_numpy(c["K"]).to(dev)
    C = K.shape[0]
    nv = torch.from_numpy(c["n_valid"].astype(np.int32)).to(dev).view(1, C)
    page_of = torch.arange(C, dtype=torch.int32, device=dev).view(1, C)
    slots = K.to(slot_dtype).contiguous()
    S = ops.summaries(slots, page_of, nv)
    return ops.Pages(slots=slots, page_of=page_of, n_valid=nv, S=S)


# ------------------------------------------------------------------------------------------------ ops level
@pytest.mark.parametrize("name", READ_CASES)
@pytest.mark.parametrize("slot_dtype", [torch.float16, torch.float32])
def test_read_path_matches_reference(dev, name, slot_dtype):
    from kv_skill_v2_b200 import ops
    c = load_case(name)
    pages = _pages_from_case(c, dev, slot_dtype)
    assert rel_err(pages.S[0], c["S"]) < 1e-5
    h = torch.from_numpy(c["h"]).to(dev)
    h2 = h.reshape(-1, h.shape[-1])
    W_in = torch.from_numpy(c["W_in"]).t().contiguous().to(dev)    # nn.Linear layout [d_s, d_m]
    W_out = torch.from_numpy(c["W_out"]).t().contiguous().to(dev)  # [d_m, d_s]
    q, _, _, _ = ops.project_in(h2, W_in)
    assert rel_err(q, c["q"].reshape(q.shape)) < 1e-4
    R = q.shape[0]
    idx, wk, w, _ = ops.route(q, pages.S, rows_per_lib=R, top_k=int(c["top_k"]), route_temp=float(c["route_temp"]))
    w_ref = c["w"].reshape(w.shape)
    assert topk_sets(w) == topk_sets(w_ref), "routing index sets differ from the reference"
    assert rel_err(w, w_ref) < 1e-4
    r = ops.read_decode(q, pages, idx, wk, rows_per_lib=R, read_temp=float(c["read_temp"]),
                        read_softmax=bool(c["read_softmax"]))
    assert rel_err(r, c["r"].reshape(r.shape)) < TOL
    delta, _, _ = ops.project_out(r, W_out, h2)
    assert rel_err(delta, c["delta"].reshape(delta.shape)) < TOL
    _status_clean(dev)


@pytest.mark.parametrize("kernel", ["auto", "simt"])
@pytest.mark.parametrize("slot_dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("softmax", [True, False])
def test_read_ragged_rows_both_kernels(dev, monkeypatch, kernel, slot_dtype, softmax):
    """Valid-row counts around the 16-row group and 64-row stage edges, every slot type, both read kernels
    (tensor-core for f16/bf16 when d_s % 16 == 0, SIMT otherwise or when forced), against the oracle."""
    from kv_skill_v2_b200 import ops
    if kernel == "simt":
        monkeypatch.setenv("XENCB_READ_SIMT", "1")
    g = torch.Generator().manual_seed(21)
    ns = [1, 15, 16, 17, 63, 64, 65, 200, 511]
    C, N, d_s, R = len(ns), 512, 512, 12
    K = torch.randn(C, N, d_s, generator=g)
    K = (K / K.norm(dim=-1, keepdim=True)).to(slot_dtype)
    for c, n in enumerate(ns):
        K[c, n:] = 0
    Kf = K.float().numpy()
    M = np.arange(N)[None, :] < np.array(ns)[:, None]
    q = torch.nn.functional.normalize(torch.randn(R, d_s, generator=g), dim=-1)
    S = torch.from_numpy(X.summaries(Kf, M)).to(dev).view(1, C, d_s)
    pages = ops.Pages(slots=K.to(dev).contiguous(), page_of=torch.arange(C, dtype=torch.int32, device=dev).view(1, C),
                      n_valid=torch.tensor(ns, dtype=torch.int32, device=dev).view(1, C), S=S)
    for top_k in (0, 3):
        idx, wk, w, _ = ops.route(q.to(dev), pages.S, rows_per_lib=R, top_k=top_k, route_temp=10.0)
        r = ops.read_decode(q.to(dev), pages, idx, wk, rows_per_lib=R, read_temp=12.0, read_softmax=softmax)
        ref = X.read(q.numpy(), Kf, M, w.cpu().numpy(), 12.0, softmax)
        assert rel_err(r, ref) < TOL, (kernel, slot_dtype, softmax, top_k)
    _status_clean(dev)


@pytest.mark.parametrize("slot_dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("softmax", [True, False])
@pytest.mark.parametrize("masked", [0.0, 0.75, 1.0])
def test_read_decode_sparse_matches_dense(dev, slot_dtype, softmax, masked):
    """The sparse plan (128-row pieces, only the pieces that hold rows listed on the device) against the dense
    plan and the oracle: a share of the rows masked out (weight 0, as the selector's row mask does; they read
    nothing), ragged chunks around the 16- and 64-row edges, every row its own Library. float32 slots take the
    CUDA-core read, where the sparse entry runs the dense plan."""
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(31)
    B, C, N, d_s, k = 24, 16, 512, 256, 4
    ns = torch.randint(1, N + 1, (B, C), generator=g)
    ns.view(-1)[:8] = torch.tensor([1, 15, 16, 17, 63, 64, 65, 512])
    K = torch.randn(B * C, N, d_s, generator=g)
    K = (K / K.norm(dim=-1, keepdim=True)).to(slot_dtype)
    M = np.arange(N)[None, :] < ns.view(-1, 1).numpy()
    K[torch.from_numpy(~M)] = 0
    Kf = K.float().numpy()
    q = torch.nn.functional.normalize(torch.randn(B, d_s, generator=g), dim=-1)
    page_of = torch.arange(B * C, dtype=torch.int32).view(B, C)
    S = torch.from_numpy(np.stack([X.summaries(Kf[b * C:(b + 1) * C], M[b * C:(b + 1) * C]) for b in range(B)]))
    pages = ops.Pages(slots=K.to(dev).contiguous(), page_of=page_of.to(dev), n_valid=ns.to(torch.int32).to(dev),
                      S=S.to(dev))
    row_w = (torch.rand(B, generator=g) >= masked).float()
    idx, wk, w, _ = ops.route(q.to(dev), pages.S, rows_per_lib=1, top_k=k, route_temp=10.0, row_w=row_w.to(dev))
    r_dense = ops.read_decode(q.to(dev), pages, idx, wk, rows_per_lib=1, read_temp=12.0, read_softmax=softmax)
    r_sparse = ops.read_decode(q.to(dev), pages, idx, wk, rows_per_lib=1, read_temp=12.0, read_softmax=softmax,
                               sparse=True)
    live = row_w > 0
    assert (r_sparse.cpu()[~live] == 0).all() and (r_dense.cpu()[~live] == 0).all()
    if live.any():
        assert rel_err(r_sparse[live.to(dev)], r_dense[live.to(dev)]) < TOL
        wn = w.cpu().numpy()
        ref = np.stack([X.read(q[b:b + 1].numpy(), Kf[b * C:(b + 1) * C], M[b * C:(b + 1) * C], wn[b:b + 1], 12.0,
                               softmax)[0] for b in range(B) if live[b]])
        assert rel_err(r_sparse[live.to(dev)], ref) < TOL
    # 96 pairs: the tensor-core kernel builds the piece list itself; the separate compaction kernel lists the same
    # pieces in the same order, so the two agree bit for bit
    import os
    os.environ["XENCB_READ_PLAN_KERNEL"] = "1"
    try:
        r_listed = ops.read_decode(q.to(dev), pages, idx, wk, rows_per_lib=1, read_temp=12.0, read_softmax=softmax,
                                   sparse=True)
    finally:
        del os.environ["XENCB_READ_PLAN_KERNEL"]
    assert torch.equal(r_listed, r_sparse)
    _status_clean(dev)


def test_route_ties_go_to_lower_index(dev):
    from kv_skill_v2_b200 import ops
    S = torch.zeros(1, 6, 8, device=dev)
    S[0, :, 0] = torch.tensor([0.5, 0.9, 0.9, 0.1, 0.9, 0.2])
    q = torch.zeros(3, 8, device=dev)
    q[:, 0] = 1.0
    idx, wk, w, _ = ops.route(q, S, rows_per_lib=3, top_k=2, route_temp=10.0)
    assert idx.tolist() == [[1, 2]] * 3
    assert torch.allclose(wk, torch.full_like(wk, 0.5))
    assert (w > 0).sum(-1).tolist() == [2, 2, 2]


def test_route_chunks_per_library(dev):
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(3)
    S = torch.nn.functional.normalize(torch.randn(2, 5, 16, generator=g), dim=-1).to(dev)
    q = torch.nn.functional.normalize(torch.randn(4, 16, generator=g), dim=-1).to(dev)
    n_of = torch.tensor([3, 5], dtype=torch.int32, device=dev)
    for top_k in (0, 2, 4):
        idx, wk, w, _ = ops.route(q, S, rows_per_lib=2, top_k=top_k, route_temp=10.0, n_chunks_of=n_of)
        assert (w[:2, 3:] == 0).all(), "chunks beyond a Library's count must get no weight"
        assert torch.allclose(w.sum(-1), torch.ones(4, device=dev), atol=1e-6)
        for row in range(4):
            lib = row // 2
            wo, _, _ = X.route(q[row:row + 1].cpu().numpy(), S[lib, : int(n_of[lib])].cpu().numpy(), 10.0, top_k)
            assert topk_sets(w[row:row + 1, : int(n_of[lib])]) == topk_sets(wo)


@pytest.mark.parametrize("C", [1, 7, 20, 64, 100, 128, 129, 300])
@pytest.mark.parametrize("d_s", [30, 256, 2052])
def test_route_decode_shapes(dev, C, d_s):
    """Decode routing (few rows per Library): up to 128 chunks one fused launch (a cluster per row, or per 64 / C
    rows), more chunks the logits + top-k pair. Against the oracle: logits, the kept index list in (value desc,
    index asc) order, the weights; ragged chunk counts per Library and rows of weight 0."""
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(100 + C + d_s)
    rows_per_lib, n_lib = 3, 5
    R = rows_per_lib * n_lib - 1  # the last Library has one row fewer
    S = torch.nn.functional.normalize(torch.randn(n_lib, C, d_s, generator=g), dim=-1)
    q = torch.nn.functional.normalize(torch.randn(R, d_s, generator=g), dim=-1)
    n_of = torch.tensor([C, max(1, C - 3), max(1, C // 2), 1, C], dtype=torch.int32)
    row_w = torch.ones(R)
    row_w[4] = 0.0
    for top_k in (0, 1, 5, 40):
        idx, wk, w, lg = ops.route(q.to(dev), S.to(dev), rows_per_lib=rows_per_lib, top_k=top_k, route_temp=10.0,
                                   n_chunks_of=n_of.to(dev), want_logits=True, row_w=row_w.to(dev))
        idx, wk, w, lg = idx.cpu().numpy(), wk.cpu().numpy(), w.cpu().numpy(), lg.cpu().numpy()
        assert idx.shape == (R, ops.route_k(top_k, C))
        for row in range(R):
            lib = row // rows_per_lib
            nc = int(n_of[lib])
            wo, lo, io = X.route(q[row:row + 1].numpy(), S[lib, :nc].numpy(), 10.0, top_k)
            assert np.abs(lg[row, :nc] - lo[0]).max() <= 1e-5 * max(1.0, np.abs(lo).max()), (C, d_s, row)
            assert (lg[row, nc:] == -np.inf).all()
            assert topk_sets(w[row:row + 1, :nc]) == topk_sets(wo), (C, d_s, top_k, row)
            assert (w[row, nc:] == 0).all()
            assert np.abs(w[row, :nc] - wo[0]).max() < 1e-5
            kept = min(top_k, nc) if 0 < top_k < nc else nc
            if row_w[row] == 0:
                assert (idx[row] == -1).all() and (wk[row] == 0).all()
                continue
            if 0 < top_k < nc:
                assert idx[row, :kept].tolist() == io[0, :kept].tolist(), (C, d_s, top_k, row)
            else:
                assert idx[row, :nc].tolist() == list(range(nc))
            assert (idx[row, kept:] == -1).all()
            assert np.abs(wk[row, :kept] - w[row, idx[row, :kept]]).max() == 0
    _status_clean(dev)


def test_batched_documents_match_reference(dev):
    """Each row reads its own Library (a paged pool of 4 documents) -- checked per document against
    reference runs of the single-Library read."""
    from kv_skill_v2_b200 import ops
    c = load_case("batch_docs_top2")
    K = torch.from_numpy(c["K"]).to(dev)  # [B, C, N, d]
    B, C, N, d = K.shape
    slots = K.reshape(B * C, N, d).half().contiguous()
    page_of = torch.arange(B * C, dtype=torch.int32, device=dev).view(B, C)
    nv = torch.from_numpy(c["n_valid"].astype(np.int32)).to(dev)
    pages = ops.Pages(slots=slots, page_of=page_of, n_valid=nv, S=ops.summaries(slots, page_of, nv))
    h = torch.from_numpy(c["h"]).to(dev).reshape(B, -1)
    q, _, _, _ = ops.project_in(h, torch.from_numpy(c["W_in"]).t().contiguous().to(dev))
    idx, wk, w, _ = ops.route(q, pages.S, rows_per_lib=1, top_k=2, route_temp=10.0)
    assert topk_sets(w) == topk_sets(c["w"].reshape(B, C))
    r = ops.read_decode(q, pages, idx, wk, rows_per_lib=1)
    assert rel_err(r, c["r"].reshape(B, d)) < TOL
    _status_clean(dev)


def test_selector_kernels_match_reference(dev):
    from kv_skill_v2_b200 import ops
    c = dict(np.load(__import__("tests._fixtures", fromlist=["GOLDEN"]).GOLDEN / "selector.npz"))
    for st in (0, 1):
        for k in (1, 2, 3):
            key = f"st{st}_k{k}"
            hs = torch.from_numpy(c[f"{key}_h"]).to(dev)
            z = ops.selector_logits(hs[0].reshape(-1, hs.shape[-1]), torch.from_numpy(c[f"{key}_u_w"]).to(dev),
                                    torch.from_numpy(c[f"{key}_u_b"]).to(dev), rms=True)
            assert rel_err(z, c[f"{key}_z"].reshape(z.shape)) < 1e-4
            w = ops.selector_weights(z, k, bool(st))
            assert topk_sets(w) == topk_sets(c[f"{key}_w"])
            assert rel_err(w, c[f"{key}_w"].reshape(w.shape)) < 1e-4
            for i in range(len(c["cand"])):
                delta = torch.from_numpy(c[f"{key}_delta"][i]).to(dev)
                out = ops.selector_apply(delta, hs[i], w, i, float(c[f"{key}_log_alpha"]))
                assert rel_err(out, c[f"{key}_out"][i]) < 1e-4
    _status_clean(dev)


@pytest.mark.parametrize("dims", [(37, 264, 136), (5, 5120, 2052), (3, 6148, 6144)])
@pytest.mark.parametrize("hdt", [torch.float32, torch.bfloat16, torch.float16])
def test_projections_with_gate_selector_mask(dev, hdt, dims):
    """project_in / project_out against the oracle with bias, gate, selector rescale, position mask and a
    low-precision hidden state (cast, residual add and mag term in h's dtype). Widths cover the one-CTA-per-row
    reduce kernels with 1, 2 and 3 float4 columns per thread and, past 6144 columns, the chunked kernels."""
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(7)
    R, d_m, d_s = dims
    h = (torch.randn(R, d_m, generator=g) * 2).to(hdt)
    W_in = torch.randn(d_s, d_m, generator=g) * 0.05
    b_in = torch.randn(d_s, generator=g) * 0.1
    gate_w = torch.randn(d_m, generator=g) * 0.1
    W_out = torch.randn(d_m, d_s, generator=g) * 0.05
    b_out = torch.randn(d_m, generator=g) * 0.1
    sel_col = torch.rand(R, generator=g)
    pm = (torch.rand(R, generator=g) > 0.3).float()
    r = torch.randn(R, d_s, generator=g)
    hf = h.float().numpy()
    hn = X.rms_norm(hf)
    q_ref = X.query(hn, W_in.t().numpy(), b_in.numpy())
    g_ref = X.gate(hn, gate_w.numpy(), 0.25)[:, 0]
    q, gate, rstd, _ = ops.project_in(h.to(dev), W_in.to(dev), b_in.to(dev), gate_w=gate_w.to(dev), gate_b=0.25)
    assert rel_err(q, q_ref) < 1e-4 and rel_err(gate, g_ref) < 1e-5
    d = 0.7 * g_ref[:, None] * (r.numpy() @ W_out.t().numpy() + b_out.numpy())
    d = X.selector_apply(d, hf, sel_col.numpy(), -2.0) * pm.numpy()[:, None]
    d_h = torch.from_numpy(d.astype(np.float32)).to(hdt)
    delta, h_new, rel = ops.project_out(r.to(dev), W_out.to(dev), h.to(dev), b_out=b_out.to(dev), scale=0.7,
                                        gate=gate, sel_w=sel_col.to(dev), log_alpha=-2.0, pos_mask=pm.to(dev),
                                        want_delta=True, h_out=torch.empty_like(h.to(dev)), want_rel=True)
    assert delta.dtype == hdt and h_new.dtype == hdt
    tol = TOL if hdt == torch.float32 else 1e-2
    assert rel_err(delta.float(), d_h.float()) < tol
    assert rel_err(h_new.float(), (h.float() + d_h.float()).to(hdt).float()) < tol
    assert rel_err(rel, X.rel_norm(d_h.float().numpy(), hf)) < tol
    _status_clean(dev)


@pytest.mark.parametrize("shape", [(64, 4096, 2048), (200, 520, 264), (7, 96, 16), (130, 30, 44), (64, 2048, 4096)])
@pytest.mark.parametrize("hdt", [torch.float32, torch.bfloat16])
def test_projection_gemm_fp32_faithful(dev, shape, hdt):
    """The projection GEMM (tensor-core 3xTF32 when d_in % 4 == 0, CUDA-core fallback otherwise) against a
    float64 product: relative error well inside float32-level accuracy (1e-5 of the largest entry)."""
    from kv_skill_v2_b200 import ops
    M, K, N = shape
    g = torch.Generator().manual_seed(M + K + N)
    h = torch.randn(M, K, generator=g).to(hdt)
    W = torch.randn(N, K, generator=g) * 0.05
    y, _, _, _ = ops.project_in(h.to(dev), W.to(dev), rms=False, l2=False)
    ref = h.double() @ W.double().t()
    assert rel_err(y, ref) < 1e-5, shape
    _status_clean(dev)


@pytest.mark.parametrize("shape", [(64, 4096, 2048), (200, 520, 264), (8, 96, 16), (130, 40, 44), (64, 2048, 4096),
                                   (1, 64, 128), (1000, 256, 136)])
@pytest.mark.parametrize("hdt", [torch.float32, torch.bfloat16, torch.float16])
def test_projection_gemm_f16x3_fp32_faithful(dev, shape, hdt):
    """The 3xF16 GEMM (weights split once by weights_prep, rows split per call with their own power-of-two scale)
    against a float64 product: the same 1e-5 bar as 3xTF32, for row counts and widths that leave partial tiles,
    and for inputs whose rows span very different magnitudes."""
    from kv_skill_v2_b200 import ops
    M, K, N = shape
    g = torch.Generator().manual_seed(M + K + N + 7)
    h = torch.randn(M, K, generator=g) * torch.logspace(-3, 3, M).view(M, 1)  # rows from 1e-3 to 1e3
    h = h.to(hdt)
    W = torch.randn(N, K, generator=g) * 0.05
    Wd = W.to(dev)
    prep = ops.weights_prep(Wd)
    y, _, _, _ = ops.project_in(h.to(dev), Wd, rms=False, l2=False, w_prep=prep, prefer_prep=True)
    ref = h.double() @ W.double().t()
    # per-row relative error (rows have different scales)
    err = ((y.double().cpu() - ref).abs().amax(1) / ref.abs().amax(1).clamp_min(1e-300)).max().item()
    assert err < 1e-5, (shape, err)
    # project_out through the same prepared form of its weight
    Wo = torch.randn(K, N, generator=g) * 0.05
    Wod = Wo.to(dev)
    r = torch.randn(M, N, generator=g)
    hh = torch.zeros(M, K, dtype=torch.float32)
    d, _, _ = ops.project_out(r.to(dev), Wod, hh.to(dev), w_prep=ops.weights_prep(Wod) if N % 8 == 0 else None,
                              prefer_prep=True)
    ref_o = r.double() @ Wo.double().t()
    assert rel_err(d, ref_o) < 1e-5, shape
    _status_clean(dev)


@pytest.mark.parametrize("nk", [(200, 520), (128, 64), (4096, 2048), (44, 40)])
def test_weights_prep_tile_layout(dev, nk):
    """weights_prep's layout: a 256-byte head (max |w|, 1/s), then per 128-row band and 64-column block the
    128 x 64 f16 tile of hi = rn(w s) and the one of lo = rn(w s - hi), bands outer, zeros past n and k."""
    from kv_skill_v2_b200 import ops
    n, k = nk
    g = torch.Generator().manual_seed(n + k)
    W = torch.randn(n, k, generator=g) * 0.05
    prep = ops.weights_prep(W.to(dev)).cpu()
    NT, KB = (n + 127) // 128, (k + 63) // 64
    assert prep.numel() == 256 + NT * KB * 2 * 128 * 64 * 2
    head = prep[:8].view(torch.float32)
    assert head[0].item() == W.abs().max().item()
    s = 1.0 / head[1].item()
    assert s == 2.0 ** round(np.log2(s))  # a power of two
    tiles = prep[256:].view(torch.float16).view(NT, KB, 2, 128, 64)
    full = tiles.permute(2, 0, 3, 1, 4).reshape(2, NT * 128, KB * 64)  # [hi | lo][band row][block column]
    v = W * s
    hi = v.half()
    lo = (v - hi.float()).half()
    assert torch.equal(full[0, :n, :k], hi) and torch.equal(full[1, :n, :k], lo)
    assert not full[:, n:, :].any() and not full[:, :, k:].any()
    _status_clean(dev)


def test_injector_f16x3_matches_tf32_path(dev):
    """The hooked model with the 3xF16 projections (default) and with 3xTF32 (gemm_f16x3 = False) agree with the
    reference's output; the per-layer CUDA graphs are keyed by the weights' versions, so an in-place weight change
    is seen by the next step."""
    from kv_skill_v2_b200 import CAND, LayerSelector, Library, LibraryInjector, ModelInterface
    c = load_case("hooked")
    d_m = c["x"].shape[-1]
    reader = TinyReader(d_m, 10)
    with torch.no_grad():
        for i, blk in enumerate(reader.model.layers):
            blk.weight.copy_(torch.from_numpy(c[f"blk{i}_w"]))
            blk.bias.copy_(torch.from_numpy(c[f"blk{i}_b"]))
    reader = reader.to(dev).eval().requires_grad_(False)
    layers = [int(x) for x in c["layers"]]
    d_s = c[f"K_{layers[0]}"].shape[-1]
    chunks = [{"K": {float(r): torch.from_numpy(c[f"K_{li}"][i, :n]) for r, li in zip(CAND, layers)}}
              for i, n in enumerate(c["n"])]
    lib = Library(chunks, layers, CAND)
    itf = ModelInterface(d_m, d_s, layers)
    with torch.no_grad():
        itf.A.weight.copy_(torch.from_numpy(c["A_w"]))
        itf.B.weight.copy_(torch.from_numpy(c["B_w"]))
        itf.gate_w.copy_(torch.from_numpy(c["gate_w"]))
        itf.gate_b.copy_(torch.from_numpy(c["gate_b"]))
        itf.log_gain.copy_(torch.from_numpy(c["log_gain"]))
    itf = itf.to(dev).requires_grad_(False)
    x = torch.from_numpy(c["x"]).to(dev)
    outs = []
    for f16x3 in (True, False):
        inj = LibraryInjector(reader, itf, top_k=4)
        inj.gemm_f16x3 = f16x3
        inj.load_library(lib)
        with torch.no_grad():
            y1 = reader(x)
            y2 = reader(x)  # replayed from the captured graphs
        assert rel_err(y1, c["out_sel0"]) < TOL and rel_err(y2, c["out_sel0"]) < TOL
        outs.append(y2)
        if f16x3:
            with torch.no_grad():
                itf.B.weight.mul_(2.0)   # in place: the next step must use the new weights
                y3 = reader(x)
                itf.B.weight.mul_(0.5)
                y4 = reader(x)
            assert not torch.allclose(y3, y2, atol=1e-6, rtol=0)  # the doubled write weights took effect
            assert rel_err(y4, y2) < 1e-5
        inj.detach()
    assert rel_err(outs[0], outs[1]) < 1e-5
    _status_clean(dev)


def test_low_rank_query_two_calls(dev):
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(8)
    h = torch.randn(9, 96, generator=g)
    A1, A2 = torch.randn(16, 96, generator=g) * 0.1, torch.randn(48, 16, generator=g) * 0.1
    t, _, _, _ = ops.project_in(h.to(dev), A1.to(dev), rms=True, l2=False)
    q, _, _, _ = ops.project_in(t, A2.to(dev), rms=False, l2=True)
    ref = X.l2(X.rms_norm(h.numpy()) @ A1.t().numpy() @ A2.t().numpy())
    assert rel_err(q, ref) < 1e-4


# ------------------------------------------------------------------------------------------------ API level
def test_injector_branch_cfg1(dev):
    from kv_skill_v2_b200 import Library, LibraryInjector, LinearInterface
    c = load_case("cfg1_softmax_top2")
    reader = TinyReader(8, 8).to(dev)
    li = 4
    rows = [torch.from_numpy(c["K"][i, :n]).float() for i, n in enumerate(c["n_valid"])]
    lib = Library([{"K": {0.5: r}} for r in rows], [li], [0.5])
    itf = LinearInterface(torch.from_numpy(c["W_in"]), torch.from_numpy(c["W_out"]), [li]).to(dev)
    for top_k, name in ((2, "cfg1_softmax_top2"), (0, "cfg1_dense")):
        ref = load_case(name)
        inj = LibraryInjector(reader, itf, top_k=top_k)
        inj.load_library(lib)
        with torch.no_grad():
            delta = inj._branch(torch.from_numpy(c["h"]).to(dev), li)
        assert topk_sets(inj.last_route) == topk_sets(ref["w"])
        assert rel_err(delta, ref["delta"]) < TOL
        inj.detach()


def test_hooked_model_with_interface_and_selector(dev):
    """Full hook path: ModelInterface (gate, gain, B), LayerSelector over 8 candidate depths, top-4 routing;
    the model output and mag terms match the reference's hooked forward."""
    from kv_skill_v2_b200 import CAND, LayerSelector, Library, LibraryInjector, ModelInterface
    c = load_case("hooked")
    d_m = c["x"].shape[-1]
    L = 10
    reader = TinyReader(d_m, L)
    with torch.no_grad():
        for i, blk in enumerate(reader.model.layers):
            blk.weight.copy_(torch.from_numpy(c[f"blk{i}_w"]))
            blk.bias.copy_(torch.from_numpy(c[f"blk{i}_b"]))
    reader = reader.to(dev).eval().requires_grad_(False)
    layers = [int(x) for x in c["layers"]]
    d_s = c[f"K_{layers[0]}"].shape[-1]
    chunks = [{"K": {float(r): torch.from_numpy(c[f"K_{li}"][i, :n]) for r, li in zip(CAND, layers)}}
              for i, n in enumerate(c["n"])]
    lib = Library(chunks, layers, CAND)
    itf = ModelInterface(d_m, d_s, layers)
    with torch.no_grad():
        itf.A.weight.copy_(torch.from_numpy(c["A_w"]))
        itf.B.weight.copy_(torch.from_numpy(c["B_w"]))
        itf.gate_w.copy_(torch.from_numpy(c["gate_w"]))
        itf.gate_b.copy_(torch.from_numpy(c["gate_b"]))
        itf.log_gain.copy_(torch.from_numpy(c["log_gain"]))
    itf = itf.to(dev).requires_grad_(False)
    sel = LayerSelector(d_m, layers, k=2, alpha_init=0.05)
    with torch.no_grad():
        sel.u.weight.copy_(torch.from_numpy(c["u_w"]))
        sel.u.bias.copy_(torch.from_numpy(c["u_b"]))
        sel.log_alpha.fill_(float(c["log_alpha"]))
    sel = sel.to(dev).requires_grad_(False)
    x = torch.from_numpy(c["x"]).to(dev)
    with torch.no_grad():
        assert rel_err(reader(x), c["bare"]) < 1e-5
    for use_sel in (0, 1):
        inj = LibraryInjector(reader, itf, top_k=4, selector=sel if use_sel else None)
        inj.load_library(lib)
        with torch.no_grad():
            y = reader(x)
        assert rel_err(y, c[f"out_sel{use_sel}"]) < TOL
        mags = np.array([float(m) for m in inj.mag_terms], np.float32)
        assert mags.shape == c[f"mag_sel{use_sel}"].shape
        assert np.abs(mags - c[f"mag_sel{use_sel}"]).max() <= TOL * np.abs(c[f"mag_sel{use_sel}"]).max()
        if use_sel:
            assert topk_sets(sel.weights()) == topk_sets(c["sel_w"])
        inj.detach()
    _status_clean(dev)


def test_noop_at_init_and_unload(dev):
    from kv_skill_v2_b200 import DEPTHS, Library, LibraryInjector, injection_layers, make_interface, rho_layer_map
    reader = TinyReader(40, 8).to(dev).requires_grad_(False)
    layers = injection_layers(reader, DEPTHS)
    itf = make_interface(40, 24, layers).to(dev).requires_grad_(False)
    g = torch.Generator().manual_seed(9)
    rmap = rho_layer_map(reader, DEPTHS)
    lib = Library([{"K": {r: torch.nn.functional.normalize(torch.randn(n, 24, generator=g), dim=-1)
                          for r in DEPTHS}} for n in (5, 9, 3)], [rmap[r] for r in DEPTHS], DEPTHS)
    x = torch.randn(2, 7, 40, generator=g).to(dev)
    with torch.no_grad():
        bare = reader(x)
    inj = LibraryInjector(reader, itf, top_k=2)
    inj.load_library(lib)
    with torch.no_grad():
        assert torch.equal(reader(x), bare), "zero-init B must be a no-op"
    assert len(inj.mag_terms) == len(layers) and all(float(m) == 0 for m in inj.mag_terms)
    inj.unload()
    assert inj.mag_terms == [] and inj.last_route is None
    inj.detach()


def test_duck_selector_and_forward_only_guard(dev):
    from kv_skill_v2_b200 import DEPTHS, Library, LibraryInjector, LinearInterface, injection_layers, rho_layer_map

    class Halver:
        def __init__(self):
            self.resets, self.applied = 0, []

        def reset(self):
            self.resets += 1

        def apply(self, delta, h, li):
            self.applied.append(li)
            return 0.5 * delta

    reader = TinyReader(32, 8).to(dev).requires_grad_(False)
    layers = injection_layers(reader, DEPTHS)
    g = torch.Generator().manual_seed(10)
    itf = LinearInterface(torch.randn(32, 32, generator=g) * 0.3, torch.randn(32, 32, generator=g) * 0.3,
                          layers).to(dev).requires_grad_(False)
    rmap = rho_layer_map(reader, DEPTHS)
    lib = Library([{"K": {r: torch.nn.functional.normalize(torch.randn(6, 32, generator=g), dim=-1)
                          for r in DEPTHS}} for _ in range(3)], [rmap[r] for r in DEPTHS], DEPTHS)
    x = torch.randn(2, 7, 32, generator=g).to(dev)
    base = LibraryInjector(reader, itf)
    base.load_library(lib)
    with torch.no_grad():
        full = reader(x)
    base.detach()
    sel = Halver()
    inj = LibraryInjector(reader, itf, selector=sel)
    inj.load_library(lib)
    with torch.no_grad():
        reader(x)
        reader(x)
        halved = reader(x)
    assert sel.resets == 3 and sel.applied == layers * 3
    assert (halved - full).abs().max() > 1e-4
    inj.detach()
    itf.requires_grad_(True)
    inj = LibraryInjector(reader, itf)
    inj.load_library(lib)
    with pytest.raises(RuntimeError, match="forward-only"):
        reader(x)
    inj.detach()


# ------------------------------------------------------------------------------------------------ full size
def _cfg2_sample(dev, n_docs=8, seed=0):
    """BASELINE config-2 shapes (C=64 x 512 slots, d_s=2048, d_m=4096, top-4, T=1) for n_docs documents."""
    g = torch.Generator(device=dev).manual_seed(seed)
    C, N, d_s, d_m = 64, 512, 2048, 4096
    slots = torch.randn(n_docs * C, N, d_s, generator=g, device=dev)
    slots = (slots / slots.norm(dim=-1, keepdim=True)).half()
    nv = torch.full((n_docs, C), N, dtype=torch.int32, device=dev)
    nv[:, -1] = torch.randint(1, N + 1, (n_docs,), generator=g, device=dev, dtype=torch.int32)
    page_of = torch.arange(n_docs * C, dtype=torch.int32, device=dev).view(n_docs, C)
    h = torch.randn(n_docs, d_m, generator=g, device=dev)
    W_in = torch.randn(d_s, d_m, generator=g, device=dev) * 0.02
    W_out = torch.randn(d_m, d_s, generator=g, device=dev) * 0.02
    return slots, nv, page_of, h, W_in, W_out


def test_config2_sample_matches_oracle(dev):
    from kv_skill_v2_b200 import ops
    slots, nv, page_of, h, W_in, W_out = _cfg2_sample(dev, n_docs=6)
    S = ops.summaries(slots, page_of, nv)
    pages = ops.Pages(slots=slots, page_of=page_of, n_valid=nv, S=S)
    q, _, _, _ = ops.project_in(h, W_in)
    idx, wk, w, _ = ops.route(q, S, rows_per_lib=1, top_k=4, route_temp=10.0)
    r = ops.read_decode(q, pages, idx, wk, rows_per_lib=1)
    delta, _, _ = ops.project_out(r, W_out, h)
    for b in range(h.shape[0]):
        K = slots[b * 64:(b + 1) * 64].float().cpu().numpy()
        M = np.arange(K.shape[1])[None, :] < nv[b].cpu().numpy()[:, None]
        S_ref = X.summaries(K, M)
        assert rel_err(S[b], S_ref) < 1e-5
        out = X.branch(h[b:b + 1].cpu().numpy(), W_in.t().cpu().numpy(), W_out.t().cpu().numpy(), K, M, S_ref,
                       top_k=4)
        assert topk_sets(w[b:b + 1]) == topk_sets(out["w"])
        assert rel_err(r[b], out["r"][0]) < TOL
        assert rel_err(delta[b], out["delta"][0]) < TOL
    _status_clean(dev)


def test_config2_properties(dev):
    """Size-independent properties at full config-2 scale: weights sum to 1 with exactly k nonzeros, a
    one-hot routing reproduces the single-chunk read, and reading with weights (a, 1-a) is linear."""
    from kv_skill_v2_b200 import ops
    slots, nv, page_of, h, W_in, _ = _cfg2_sample(dev, n_docs=64, seed=1)
    S = ops.summaries(slots, page_of, nv)
    pages = ops.Pages(slots=slots, page_of=page_of, n_valid=nv, S=S)
    q, _, _, _ = ops.project_in(h, W_in)
    idx, wk, w, _ = ops.route(q, S, rows_per_lib=1, top_k=4, route_temp=10.0)
    assert ((w > 0).sum(-1) == 4).all() and torch.allclose(w.sum(-1), torch.ones(64, device=dev), atol=1e-5)
    r = ops.read_decode(q, pages, idx, wk, rows_per_lib=1)
    parts = []
    for j in range(4):
        one = torch.zeros_like(wk)
        one[:, j] = 1.0
        parts.append(ops.read_decode(q, pages, idx, one, rows_per_lib=1))
    lin = sum(wk[:, j:j + 1] * parts[j] for j in range(4))
    assert rel_err(r, lin) < 1e-5
    # a chunk read is a convex combination of unit rows: norm <= 1
    assert (parts[0].norm(dim=-1) <= 1.0 + 1e-4).all()
    _status_clean(dev)


def test_injector_cuda_graph_cache(dev):
    """The hook path replayed from a CUDA graph gives the eager path's results; outputs of successive forwards
    stay independent; changing the Library or a scalar the graph captured re-captures."""
    from kv_skill_v2_b200 import LibraryInjector, LinearInterface, PagedLibrary, ops
    g = torch.Generator().manual_seed(21)
    B, C, N, d_s, d_m = 4, 6, 64, 128, 256
    K = torch.nn.functional.normalize(torch.randn(B * C, N, d_s, generator=g), dim=-1).half().to(dev)
    po = torch.arange(B * C, dtype=torch.int32, device=dev).view(B, C)
    nv = torch.full((B, C), N, dtype=torch.int32, device=dev)
    plib = PagedLibrary({1: ops.Pages(slots=K, page_of=po, n_valid=nv, S=ops.summaries(K, po, nv))})
    itf = LinearInterface(torch.randn(d_m, d_s, generator=g) * 0.05, torch.randn(d_s, d_m, generator=g) * 0.05,
                          [1]).to(dev).requires_grad_(False)
    reader = TinyReader(d_m, 3).to(dev).eval().requires_grad_(False)
    xs = [torch.randn(B, 1, d_m, generator=g).to(dev) for _ in range(3)]
    outs = {}
    for graphs in (False, True):
        inj = LibraryInjector(reader, itf, top_k=2, cuda_graphs=graphs)
        inj.load_library(plib)
        with torch.no_grad():
            outs[graphs] = [reader(x) for x in xs]
            if graphs:
                assert len({k[0] for k in inj._graphs}) == 1  # one captured configuration (per input buffer)
                inj.gain_scale = 0.5
                half = reader(xs[0])
                assert len({k[0] for k in inj._graphs}) == 2
                inj.gain_scale = 1.0
                inj.load_library(plib)
                assert len(inj._graphs) == 0
                again = reader(xs[1])
        inj.detach()
    for a, b in zip(outs[False], outs[True]):
        assert torch.allclose(a, b, rtol=0, atol=1e-6)
    assert not torch.allclose(outs[True][0], outs[True][1])
    assert torch.allclose(again, outs[False][1], rtol=0, atol=1e-6)
    assert not torch.allclose(half, outs[True][0])
    _status_clean(dev)


def test_injector_graphs_on_caller_buffers(dev):
    """The first few input buffers a hooked layer sees get graphs captured on the buffers themselves (no copy-in);
    further ones share a graph with a copy-in. Refilling the buffers in place between steps, as a serving loop
    does, gives the eager path's results every time."""
    from kv_skill_v2_b200 import LibraryInjector, LinearInterface, PagedLibrary, ops
    from kv_skill_v2_b200.injector import _PTR_GRAPHS

    class IdReader(torch.nn.Module):  # the hooked block returns its input: the hook sees the caller's buffer
        def __init__(self):
            super().__init__()
            self.layers = torch.nn.ModuleList([torch.nn.Identity(), torch.nn.Identity()])
            self._p = torch.nn.Parameter(torch.zeros(1), requires_grad=False)  # the injector finds the device here

        def forward(self, x):
            for blk in self.layers:
                x = blk(x)
            return x

    g = torch.Generator().manual_seed(23)
    B, C, N, d_s, d_m = 4, 6, 64, 128, 256
    K = torch.nn.functional.normalize(torch.randn(B * C, N, d_s, generator=g), dim=-1).half().to(dev)
    po = torch.arange(B * C, dtype=torch.int32, device=dev).view(B, C)
    nv = torch.full((B, C), N, dtype=torch.int32, device=dev)
    plib = PagedLibrary({1: ops.Pages(slots=K, page_of=po, n_valid=nv, S=ops.summaries(K, po, nv))})
    itf = LinearInterface(torch.randn(d_m, d_s, generator=g) * 0.05, torch.randn(d_s, d_m, generator=g) * 0.05,
                          [1]).to(dev).requires_grad_(False)
    reader = IdReader().to(dev)
    n_buf = _PTR_GRAPHS + 2
    bufs = [torch.empty(B, 1, d_m, device=dev) for _ in range(n_buf)]
    rounds = [[torch.randn(B, 1, d_m, generator=g).to(dev) for _ in range(n_buf)] for _ in range(2)]
    ref = LibraryInjector(reader, itf, top_k=2, cuda_graphs=False)
    ref.load_library(plib)
    with torch.no_grad():
        want = [[reader(x.clone()) for x in r] for r in rounds]
    ref.detach()
    inj = LibraryInjector(reader, itf, top_k=2)
    inj.load_library(plib)
    with torch.no_grad():
        for r, xr in enumerate(rounds):
            for i, x in enumerate(xr):
                bufs[i].copy_(x)
                y = reader(bufs[i])
                assert torch.allclose(y, want[r][i], rtol=0, atol=1e-6), (r, i)
    on_buffer = [k for k in inj._graphs if k[1] is not None]
    assert len(on_buffer) == _PTR_GRAPHS and any(k[1] is None for k in inj._graphs)
    inj.detach()
    _status_clean(dev)


def test_bounded_wait_gives_up_and_context_stays_usable(dev):
    """Failure detection without a fault: a wait on an mbarrier phase that nothing completes gives up after its
    cycle limit, raises XENCB_DEV_TIMEOUT in the status word, and the next read on the same context is correct."""
    from kv_skill_v2_b200 import ops
    assert ops.device_status(dev) == 0
    assert ops.wait_selftest(dev, limit_cycles=2_000_000) == 0
    st = ops.device_status(dev)
    assert st & 1, f"status {st}: XENCB_DEV_TIMEOUT expected"
    assert ops.device_status(dev) == 0  # read-and-clear
    c = load_case("cfg1_softmax_top2")
    pages = _pages_from_case(c, dev)
    q = torch.from_numpy(c["q"]).to(dev).reshape(-1, c["q"].shape[-1])
    R = q.shape[0]
    idx, wk, _, _ = ops.route(q, pages.S, rows_per_lib=R, top_k=2, route_temp=float(c["route_temp"]))
    r = ops.read_decode(q, pages, idx, wk, rows_per_lib=R, read_temp=float(c["read_temp"]))
    assert rel_err(r, c["r"].reshape(r.shape)) < TOL
    _status_clean(dev)


@pytest.mark.parametrize("case", [
    # (n_lib, rows_per_lib, C, d_s, d_m, top_k, h dtype, gate, bias, n_chunks_of, row mask)
    (64, 1, 64, 2048, 4096, 4, torch.float32, False, False, False, False),   # config-2 shapes
    (8, 1, 32, 512, 640, 4, torch.float32, True, True, False, True),         # gate, bias, selector row mask
    (5, 3, 8, 256, 512, 0, torch.bfloat16, True, False, True, False),        # dense, chunk counts per Library
    (3, 2, 70, 384, 256, 5, torch.float16, False, True, True, True),
])
def test_project_in_route_matches_the_two_calls(dev, case):
    """xencb_project_in_route gives project_in's q and route's logits, index sets, weights and dense weights
    bit for bit (the same sums in the same order), with and without gate, bias, per-Library chunk counts and a
    selector row mask."""
    from kv_skill_v2_b200 import ops
    n_lib, rpl, C, d_s, d_m, top_k, hdt, use_gate, use_bias, use_nco, use_mask = case
    g = torch.Generator().manual_seed(C + d_s)
    R = n_lib * rpl
    h = torch.randn(R, d_m, generator=g).to(dev, hdt)
    W = (torch.randn(d_s, d_m, generator=g) * 0.02).to(dev)
    b = (torch.randn(d_s, generator=g) * 0.01).to(dev) if use_bias else None
    gate_w = (torch.randn(d_m, generator=g) * 0.02).to(dev) if use_gate else None
    gate_b = torch.tensor([0.3], device=dev)
    S = torch.nn.functional.normalize(torch.randn(n_lib, C, d_s, generator=g), dim=-1).to(dev)
    nco = torch.randint(1, C + 1, (n_lib,), generator=g, dtype=torch.int32).to(dev) if use_nco else None
    row_w = (torch.rand(R, generator=g) > 0.5).float().to(dev) if use_mask else None
    prep = ops.weights_prep(W)
    q0, g0, r0, _ = ops.project_in(h, W, b, gate_w=gate_w, gate_b=gate_b, w_prep=prep)
    i0, k0, w0, l0 = ops.route(q0, S, rows_per_lib=rpl, top_k=top_k, route_temp=10.0, n_chunks_of=nco,
                               want_logits=True, row_w=row_w)
    q1, g1, r1, i1, k1, w1, l1 = ops.project_in_route(h, W, b, S=S, rows_per_lib=rpl, top_k=top_k, route_temp=10.0,
                                                      n_chunks_of=nco, row_w=row_w, want_logits=True,
                                                      gate_w=gate_w, gate_b=gate_b, w_prep=prep)
    assert torch.equal(q0, q1) and torch.equal(r0, r1)
    assert (g0 is None and g1 is None) or torch.equal(g0, g1)
    assert torch.equal(l0, l1), "routing logits differ"
    assert torch.equal(i0, i1) and torch.equal(k0, k1) and torch.equal(w0, w1)
    _status_clean(dev)


@pytest.mark.parametrize("case", [
    # (n_lib, rows_per_lib, C, d_s, d_m, use_nco)
    (1, 8, 256, 2560, 5120, False),    # one rank's config-5 shard at 8 GPUs: up to 18 CTAs per row
    (1, 8, 2048, 2560, 1024, False),   # the whole config-5 Library: 114 chunks per CTA
    (3, 4, 5, 256, 512, True),         # fewer chunks than CTAs, per-Library chunk counts
    (1, 64, 16, 128, 256, False),      # rows_per_lib >= 64: the two calls
])
def test_project_in_route_lse_matches_the_two_calls(dev, case):
    """xencb_project_in_route_lse gives project_in's q and route_lse's unnormalised weights and (max, sum) headers
    bit for bit (the same sums in the same order), so a sharded read that uses it merges as before."""
    from kv_skill_v2_b200 import ops
    n_lib, rpl, C, d_s, d_m, use_nco = case
    g = torch.Generator().manual_seed(C + d_s + rpl)
    R = n_lib * rpl
    h = torch.randn(R, d_m, generator=g).to(dev)
    W = (torch.randn(d_s, d_m, generator=g) * 0.02).to(dev)
    S = torch.nn.functional.normalize(torch.randn(n_lib, C, d_s, generator=g), dim=-1).to(dev)
    nco = torch.randint(1, C + 1, (n_lib,), generator=g, dtype=torch.int32).to(dev) if use_nco else None
    prep = ops.weights_prep(W)
    q0, _, _, _ = ops.project_in(h, W, w_prep=prep)
    w0, h0 = ops.route_lse(q0, S, rows_per_lib=rpl, route_temp=10.0, n_chunks_of=nco)
    q1, w1, h1 = ops.project_in_route_lse(h, W, S=S, rows_per_lib=rpl, route_temp=10.0, n_chunks_of=nco,
                                          w_prep=prep)
    assert torch.equal(q0, q1)
    assert torch.equal(w0, w1) and torch.equal(h0, h1)
    _status_clean(dev)


@pytest.mark.parametrize("name", ["attn_record_top2", "attn_record_linear", "attn_force", "attn_force_norm"])
def test_attention_diagnostics_against_reference(dev, name):
    """record_attn (last_attn[li]: the last position's route-weighted slot attention of batch row 0) and force_attn
    (a given [C, N] addressing replacing the computed one, with and without force_norm_match) through
    LibraryInjector, against the reference's own LibraryInjector run (xenc/injector.py:246-262)."""
    from kv_skill_v2_b200 import Library, LibraryInjector, LinearInterface
    c = load_case(name)
    base = dict(np.load(GOLDEN / "attn_record_top2.npz"))
    li = int(base["layer"])
    K, nv = base["K"], base["n_valid"]
    lib = Library([{"K": {0.5: torch.from_numpy(K[i, :n]).float()}} for i, n in enumerate(nv)], [li], [0.5])
    reader = TinyReader(8, 8).to(dev)
    itf = LinearInterface(torch.from_numpy(base["W_in"]), torch.from_numpy(base["W_out"]), [li]).to(dev)
    inj = LibraryInjector(reader, itf, top_k=int(c["top_k"]), read_softmax=bool(c["read_softmax"]),
                          read_temp=float(c["read_temp"]), route_temp=float(c["route_temp"]))
    inj.load_library(lib)
    inj.record_attn = True
    if name.startswith("attn_force"):
        inj.force_attn = {li: torch.from_numpy(base["force"])}
        inj.force_norm_match = bool(c["force_norm_match"])
    with torch.no_grad():
        delta = inj._branch(torch.from_numpy(base["h"]).to(dev), li)
    assert topk_sets(inj.last_route) == topk_sets(c["w"])
    assert inj.last_attn[li].device.type == "cpu" and tuple(inj.last_attn[li].shape) == c["last_attn"].shape
    assert rel_err(inj.last_attn[li], c["last_attn"]) < (TOL if name == "attn_force_norm" else 1e-5)
    assert rel_err(delta, c["delta"]) < TOL
    inj.force_attn = {li: torch.zeros(3, 3)}
    with pytest.raises(ValueError, match="force_attn"):
        with torch.no_grad():
            inj._branch(torch.from_numpy(base["h"]).to(dev), li)
    inj.detach()
    _status_clean(dev)
