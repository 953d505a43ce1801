"""D8 top-k slot-selection read on the GPU (xenc/topk_read.py): the selection-score, top-k and gathered-read
kernels against the oracle, and TopKLibraryInjector against the reference's own outputs (tests/golden/topk_*.npz,
made by the reference's TopKLibraryInjector on the same tiny attention reader).

Bar: selected slot sets identical (and in the same score order where scores are distinct); scores within 1e-5;
outputs within max|out - ref| <= 2e-3 * max|ref|."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import xenc_oracle as X
from tests._fixtures import TOL, TinyAttnReader, load_case, rel_err

pytestmark = pytest.mark.gpu

LAYERS, SEL, DEP = [1, 3, 5, 7], 3, [0.2, 0.4, 0.6, 0.8]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _status_clean(dev):
    from kv_skill_v2_b200 import ops
    assert ops.device_status(dev) == 0, "a kernel flagged a device status bit"


# ------------------------------------------------------------------------------------------------ kernels
@pytest.mark.parametrize("keys_dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("geom", [(2, 2, 8), (8, 4, 128), (1, 16, 64), (4, 1, 32), (4, 2, 64)])  # (n_kv, groups, hd)
@pytest.mark.parametrize("mode", [("last", "max"), ("last", "mean"), ("all_max", "mean"), ("all_mean", "max")])
def test_select_scores_against_oracle(dev, keys_dtype, geom, mode):
    from kv_skill_v2_b200 import ops
    n_kv, groups, hd = geom
    query, pool = mode
    g = torch.Generator().manual_seed(n_kv * 100 + hd)
    C, N, B = 5, 40, 3
    T = 1 if query == "last" else 6
    nv = torch.tensor([[40, 17, 1, 40, 33]], dtype=torch.int32)
    keys = torch.randn(1, C * N, n_kv, hd, generator=g).to(keys_dtype)
    q = torch.randn(B, T, n_kv * groups, hd, generator=g)
    sc = ops.select_scores(q.to(dev), keys.to(dev), nv.to(dev), page_rows=N, rows_per_lib=B, query_pool=
                           "mean" if query == "all_mean" else "max", head_pool=pool)
    valid = (np.arange(N)[None, :] < nv.numpy()[0][:, None]).reshape(-1)
    ref = X.topk_select_scores(q.permute(0, 2, 1, 3).numpy(), keys[0].float().numpy(), valid, query=query,
                               pool=pool)
    got = sc.cpu().numpy()
    assert np.array_equal(np.isfinite(got), np.isfinite(ref))
    fin = np.isfinite(ref)
    assert np.abs(got[fin] - ref[fin]).max() <= 1e-5 * max(1.0, np.abs(ref[fin]).max())
    _status_clean(dev)


@pytest.mark.parametrize("qmag", [1e-5, 1.0, 3e3])
@pytest.mark.parametrize("pool", ["max", "mean"])
def test_select_scores_tensor_core_path(dev, qmag, pool):
    """One position with f16 keys takes the tensor-core kernel (q split into f16 hi + lo after a power-of-two scale
    per KV head): several 128-slot tiles, a ragged last tile, invalid rows, a KV head whose q is all zero, and q
    magnitudes far from 1; scores within 1e-5 of the oracle and the same top-k sets as the FMA path."""
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(int(qmag * 10) + 7)
    n_kv, groups, hd, C, N, B = 8, 4, 128, 7, 96, 4
    nv = torch.tensor([[96, 95, 1, 64, 33, 96, 17]], dtype=torch.int32)
    keys = (torch.randn(1, C * N, n_kv, hd, generator=g) * 2).half()
    q = torch.randn(B, 1, n_kv * groups, hd, generator=g) * qmag
    q[1, 0, 4:8] = 0.0  # KV head 1 of row 1: all-zero queries
    sc = ops.select_scores(q.to(dev), keys.to(dev), nv.to(dev), page_rows=N, rows_per_lib=B, head_pool=pool)
    valid = (np.arange(N)[None, :] < nv.numpy()[0][:, None]).reshape(-1)
    ref = X.topk_select_scores(q.permute(0, 2, 1, 3).numpy(), keys[0].float().numpy(), valid, query="last",
                               pool=pool)
    got = sc.cpu().numpy()
    assert np.array_equal(np.isfinite(got), np.isfinite(ref))
    fin = np.isfinite(ref)
    assert np.abs(got[fin] - ref[fin]).max() <= 1e-5 * np.abs(ref[fin]).max()
    import os
    os.environ["XENCB_SELECT_SIMT"] = "1"
    try:
        sc2 = ops.select_scores(q.to(dev), keys.to(dev), nv.to(dev), page_rows=N, rows_per_lib=B, head_pool=pool)
    finally:
        del os.environ["XENCB_SELECT_SIMT"]
    k = 64
    i1, _ = ops.select_topk(sc, k)
    i2, _ = ops.select_topk(sc2, k)
    for r in range(B):
        a, b = set(i1[r].tolist()), set(i2[r].tolist())
        if a != b:  # only a near-tie at the k-th score may differ
            s = np.sort(ref[r][fin[r]])[::-1]
            assert s[k - 1] - s[k] <= 2e-5 * np.abs(s).max(), (r, a ^ b)
    _status_clean(dev)


def test_select_scores_several_libraries(dev):
    """Rows of Library b score Library b's keys; chunks past a Library's count are invalid."""
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(3)
    n_lib, C, N, n_kv, hd, groups = 3, 4, 16, 2, 16, 2
    keys = torch.randn(n_lib, C * N, n_kv, hd, generator=g).half()
    nv = torch.randint(1, N + 1, (n_lib, C), generator=g, dtype=torch.int32)
    nco = torch.tensor([4, 2, 3], dtype=torch.int32)
    q = torch.randn(n_lib * 2, 1, n_kv * groups, hd, generator=g)
    sc = ops.select_scores(q.to(dev), keys.to(dev), nv.to(dev), page_rows=N, rows_per_lib=2,
                           n_chunks_of=nco.to(dev)).cpu().numpy()
    for b in range(n_lib):
        valid = (np.arange(N)[None, :] < nv[b].numpy()[:, None])
        valid[int(nco[b]):] = False
        ref = X.topk_select_scores(q[2 * b:2 * b + 2].permute(0, 2, 1, 3).numpy(), keys[b].float().numpy(),
                                   valid.reshape(-1))
        got = sc[2 * b:2 * b + 2]
        assert np.array_equal(np.isfinite(got), np.isfinite(ref))
        fin = np.isfinite(ref)
        assert np.abs(got[fin] - ref[fin]).max() <= 1e-5 * np.abs(ref[fin]).max()
    _status_clean(dev)


@pytest.mark.parametrize("S,k", [(48, 7), (1000, 1), (4096, 64), (65536, 64), (65536, 2048), (300, 300),
                                 (32768, 64), (32767, 2048), (1023, 5)])
def test_select_topk_exact(dev, S, k):
    """Exact top-k in score order, ties to the lower slot, -inf slots last: against a lexicographic sort."""
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(S + k)
    s = torch.randn(3, S, generator=g)
    s[0] = torch.round(s[0] * 4) / 4              # many exact ties
    s[1, S // 2:] = float("-inf")                 # invalid slots
    s[2] = torch.randn(S, generator=g).abs() * -1  # all negative
    kk = min(k, S // 2) if S > 1 else k
    idx, val = ops.select_topk(s.to(dev), kk)
    ref = X.topk_select(s.numpy(), kk)
    assert np.array_equal(idx.cpu().numpy(), ref)
    assert np.array_equal(val.cpu().numpy(), np.take_along_axis(s.numpy(), ref, -1))
    _status_clean(dev)


def _read_case(dev, slot_dtype, untied, k, T, n_sets, n_lib, softmax, seed=0):
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(seed)
    C, N, d = 6, 64, 256
    K = torch.nn.functional.normalize(torch.randn(n_lib, C, N, d, generator=g), dim=-1).to(slot_dtype)
    V = (torch.randn(n_lib, C, N, d, generator=g) * 0.5).to(slot_dtype) if untied else K
    slots = K.reshape(n_lib * C, N, d).to(dev).contiguous()
    vslots = V.reshape(n_lib * C, N, d).to(dev).contiguous() if untied else None
    page_of = torch.arange(n_lib * C, dtype=torch.int32, device=dev).view(n_lib, C)
    pages = ops.Pages(slots=slots, page_of=page_of, n_valid=torch.full((n_lib, C), N, dtype=torch.int32,
                                                                        device=dev),
                      S=torch.zeros(n_lib, C, d, device=dev), vslots=vslots)
    idx = torch.stack([torch.randperm(C * N, generator=g)[:k] for _ in range(n_sets)]).to(torch.int32)
    q = torch.nn.functional.normalize(torch.randn(n_sets * T, d, generator=g), dim=-1)
    r, attn = ops.topk_read(q.to(dev), pages, idx.to(dev), read_softmax=softmax, want_attn=True)
    ref_r, ref_a = [], []
    for b in range(n_sets):
        lib = b if n_lib > 1 else 0
        rr, aa = X.topk_read(q[b * T:(b + 1) * T].numpy()[None], K[lib].float().reshape(C * N, d).numpy(),
                             idx[b:b + 1].numpy(), read_softmax=softmax,
                             Vf=V[lib].float().reshape(C * N, d).numpy())
        ref_r.append(rr[0]), ref_a.append(aa[0])
    return r, attn, np.concatenate(ref_r), np.concatenate(ref_a)


@pytest.mark.parametrize("slot_dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("softmax", [True, False])
@pytest.mark.parametrize("untied", [False, True])
def test_topk_read_against_oracle(dev, slot_dtype, softmax, untied):
    r, attn, ref_r, ref_a = _read_case(dev, slot_dtype, untied, k=64, T=11, n_sets=2, n_lib=1, softmax=softmax)
    assert rel_err(r, ref_r) < TOL
    assert rel_err(attn, ref_a) < TOL
    _status_clean(dev)


@pytest.mark.parametrize("k,T,n_sets,n_lib", [(1, 1, 1, 1), (7, 19, 3, 3), (2048, 2, 1, 1), (300, 8, 4, 1)])
def test_topk_read_shapes(dev, k, T, n_sets, n_lib):
    """One slot, several Libraries with one index set each, the largest k, partial row blocks."""
    r, attn, ref_r, ref_a = _read_case(dev, torch.float16, False, k=k, T=T, n_sets=n_sets, n_lib=n_lib,
                                       softmax=True, seed=k)
    assert rel_err(r, ref_r) < TOL
    assert np.allclose(attn.sum(-1).cpu().numpy(), 1.0, atol=1e-5)
    _status_clean(dev)


# ------------------------------------------------------------------------------------------------ injector
def _setup(c, dev):
    from kv_skill_v2_b200 import Library, ModelInterface
    from kv_skill_v2_b200.topk_read import attach_sel_keys
    m = TinyAttnReader(32, 8, 2, 8, 2).load_arrays(c).to(dev).eval().requires_grad_(False)
    n = [int(v) for v in c["n"]]
    chunks = [{"K": {r: torch.from_numpy(c[f"K_{li}"][i, :n[i]]) for r, li in zip(DEP, LAYERS)}}
              for i in range(len(n))]
    lib = Library(chunks, LAYERS, DEP)
    ac = {"chunks": [{"K": {0.25: torch.from_numpy(c["sel_K"][i, :n[i]])}} for i in range(len(n))]}
    lib = attach_sel_keys(lib, ac, 0.25)
    itf = ModelInterface(32, 24, LAYERS)
    with torch.no_grad():
        itf.A.weight.copy_(torch.from_numpy(c["A_w"]))
        itf.B.weight.copy_(torch.from_numpy(c["B_w"]))
        itf.gate_w.copy_(torch.from_numpy(c["gate_w"]))
        itf.gate_b.copy_(torch.from_numpy(c["gate_b"]))
        itf.log_gain.copy_(torch.from_numpy(c["log_gain"]))
    return m, lib, itf.to(dev).requires_grad_(False)


def _inj(m, itf, c, lib):
    from kv_skill_v2_b200.topk_read import TopKLibraryInjector, TopKSelector
    sel = TopKSelector(m, SEL, k=int(c["k"]), pool=str(c["pool"]), query=str(c["query"]))
    inj = TopKLibraryInjector(m, itf, sel, read_temp=12.0, read_softmax=bool(c["read_softmax"]))
    inj.load_library(lib)
    inj.sel_pos = int(c["sel_pos"])
    return inj


def test_topk_injector_golden_last_softmax(dev):
    """model(x) (top-level hook) and logits(x) (block-0 hook) with record_attn, against the reference."""
    c = load_case("topk_last_softmax")
    m, lib, itf = _setup(c, dev)
    inj = _inj(m, itf, c, lib)
    x = torch.from_numpy(c["x"]).to(dev)
    with torch.no_grad():
        y = m(x)
        assert np.array_equal(inj.last_idx.cpu().numpy(), c["idx_call"])
        sc = inj.tk.last_scores.cpu().numpy()
        fin = np.isfinite(c["scores_call"])
        assert np.array_equal(np.isfinite(sc), fin)
        assert np.abs(sc[fin] - c["scores_call"][fin]).max() < 1e-5
        assert rel_err(y, c["out_call"]) < TOL
        mags = np.array([float(t) for t in inj.mag_terms], np.float32)
        assert np.abs(mags - c["mag_call"]).max() <= TOL * np.abs(c["mag_call"]).max()
        inj.record_attn = True
        lg = m.logits(x)
    assert inj.n_select_passes == int(c["passes"])
    assert np.array_equal(inj.last_idx.cpu().numpy(), c["idx"])
    assert rel_err(lg, c["logits"]) < TOL
    for li in LAYERS:
        A = inj.last_attn[li]
        assert A.shape == c[f"attn_{li}"].shape
        assert rel_err(A, c[f"attn_{li}"]) < TOL
    inj.detach()
    _status_clean(dev)


@pytest.mark.parametrize("name", ["topk_allmean_linear", "topk_batch2_allmax"])
def test_topk_injector_golden_modes(dev, name):
    c = load_case(name)
    m, lib, itf = _setup(c, dev)
    inj = _inj(m, itf, c, lib)
    x = torch.from_numpy(c["x"]).to(dev)
    with torch.no_grad():
        lg = m.logits(x)
    assert np.array_equal(inj.last_idx.cpu().numpy(), c["idx"])
    sc = inj.tk.last_scores.cpu().numpy()
    fin = np.isfinite(c["scores"])
    assert np.abs(sc[fin] - c["scores"][fin]).max() < 1e-5
    assert rel_err(lg, c["logits"]) < TOL
    inj.detach()
    _status_clean(dev)


def test_topk_full_k_equals_library_read_and_decode_reuse(dev):
    """k >= valid slots: the read is LibraryInjector's and no selection pass runs; a genuine selection runs once
    per multi-token forward and single-token forwards reuse it (xenc tests/test_topk_read.py (b), (d))."""
    from kv_skill_v2_b200 import LibraryInjector
    from kv_skill_v2_b200.topk_read import TopKLibraryInjector, TopKSelector
    c = load_case("topk_last_softmax")
    m, lib, itf = _setup(c, dev)
    x = torch.from_numpy(c["x"]).to(dev)
    ref_inj = LibraryInjector(m, itf, read_temp=12.0)
    ref_inj.load_library(lib)
    with torch.no_grad():
        ref = m.logits(x)
    ref_inj.detach()
    inj = TopKLibraryInjector(m, itf, TopKSelector(m, SEL, k=10_000), read_temp=12.0)
    inj.load_library(lib)
    with torch.no_grad():
        out = m.logits(x)
    assert inj.n_select_passes == 0
    assert rel_err(out, ref) < 1e-5
    inj.detach()

    inj = TopKLibraryInjector(m, itf, TopKSelector(m, SEL, k=4), read_temp=12.0)
    inj.load_library(lib)
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        m.logits(torch.randn(1, 8, 32, generator=g).to(dev))
        assert inj.n_select_passes == 1
        idx0 = inj.last_idx.clone()
        m.logits(torch.randn(1, 1, 32, generator=g).to(dev))
        m(torch.randn(1, 1, 32, generator=g).to(dev))
        assert inj.n_select_passes == 1 and torch.equal(inj.last_idx, idx0)
        m(torch.randn(1, 8, 32, generator=g).to(dev))
        assert inj.n_select_passes == 2
        inj.enabled = False
        m(torch.randn(1, 8, 32, generator=g).to(dev))
        assert inj.n_select_passes == 2
    inj.detach()
    _status_clean(dev)


@pytest.mark.parametrize("k,n_sets,n_lib", [(1, 1, 1), (3, 5, 5), (64, 64, 64), (301, 5, 1), (2048, 2, 2)])
@pytest.mark.parametrize("softmax", [True, False])
@pytest.mark.parametrize("untied", [False, True])
def test_topk_read_decode_cluster(dev, k, n_sets, n_lib, softmax, untied):
    """One query row per index set: the 4-CTA cluster form (k split across the cluster, some CTAs with no rows
    when k < 4), against the oracle."""
    r, attn, ref_r, ref_a = _read_case(dev, torch.float16, untied, k=k, T=1, n_sets=n_sets, n_lib=n_lib,
                                       softmax=softmax, seed=k + n_sets)
    assert rel_err(r, ref_r) < TOL
    assert rel_err(attn, ref_a) < TOL
    _status_clean(dev)
