"""Library build on the device (xencb_library_build) against the reference's own Library (tests/golden/library.npz,
made by the reference's Library.__init__ / _summaries / centering) and the oracle's build_library.

Bar: uncentred slots bit-exact (a copy of the cache's rows, zeros after each chunk), valid-row counts exact,
centred slots and S within 1e-6 absolute (float32 arithmetic in another order). A doc-cache build on the device
(PagedLibrary.from_doc_caches) equals the host build (PagedLibrary.from_libraries of Library.from_doc_cache)
and reads the same."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import xenc_oracle as X
from tests._fixtures import GOLDEN, TOL, TinyReader, load_case, rel_err, unit_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _status(dev):
    from kv_skill_v2_b200 import ops
    return ops.device_status(dev)


@pytest.mark.parametrize("centered", [False, True])
def test_build_matches_reference_library(dev, centered):
    from kv_skill_v2_b200 import ops
    c = dict(np.load(GOLDEN / "library.npz"))
    n = [int(x) for x in c["n"]]
    for li in [int(x) for x in c["layers"]]:
        rows = torch.cat([torch.from_numpy(c[f"rows_{li}"][i, :n[i]]) for i in range(len(n))]).to(dev)
        mu = torch.from_numpy(c[f"mu_{li}"]).to(dev) if centered else None
        slots, nv, S = ops.library_build(rows, n, mu=mu, slot_dtype=torch.float32)
        K_ref = c[f"Kc_{li}"] if centered else c[f"K_{li}"]
        S_ref = c[f"Sc_{li}"] if centered else c[f"S_{li}"]
        assert nv.tolist() == n
        got = slots.cpu().numpy()
        if centered:
            assert np.abs(got - K_ref).max() <= 1e-6
        else:
            assert np.array_equal(got, K_ref)
        assert np.abs(S.cpu().numpy() - S_ref).max() <= 1e-6
    assert _status(dev) == 0


@pytest.mark.parametrize("rows_dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("slot_dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("centered", [False, True])
def test_build_ragged_against_oracle(dev, rows_dtype, slot_dtype, centered):
    """Ragged chunks (an empty one, one-row, full pages) at a BASELINE width, split across CTAs."""
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(11)
    d, pr = 2048, 512
    counts = [512, 1, 0, 300, 17, 512, 64, 255]
    chunks = [(torch.randn(n, d, generator=g) / d ** 0.5).to(rows_dtype) for n in counts]
    mu = (torch.randn(d, generator=g) * 0.01) if centered else None
    rows = torch.cat(chunks).to(dev)
    slots, nv, S = ops.library_build(rows, counts, page_rows=pr, mu=None if mu is None else mu.to(dev),
                                     slot_dtype=slot_dtype)
    K_ref, M_ref, S_ref = X.build_library([ch.float().numpy() for ch in chunks],
                                          None if mu is None else mu.numpy())
    K_pad = np.zeros((len(counts), pr, d), np.float32)
    K_pad[:, :K_ref.shape[1]] = K_ref
    assert nv.tolist() == counts
    got = slots.float().cpu().numpy()
    if slot_dtype == torch.float32:
        tol = 1e-6 if centered else 0.0
        assert np.abs(got - K_pad).max() <= tol
    else:
        exp = torch.from_numpy(K_pad).to(slot_dtype).float().numpy()
        if centered:  # float32 results one ulp apart may round to neighbouring f16 / bf16 values
            assert np.abs(got - exp).max() <= (1e-3 if slot_dtype == torch.float16 else 8e-3) * np.abs(exp).max()
        elif rows_dtype == slot_dtype or rows_dtype == torch.float32:
            assert np.array_equal(got, exp)
        else:  # f16 <-> bf16: one rounding of the row value
            assert np.abs(got - exp).max() <= 8e-3 * np.abs(exp).max()
    assert np.abs(S.cpu().numpy() - S_ref).max() <= 1e-6
    assert _status(dev) == 0


def test_build_into_shared_pool_pages(dev):
    """Chunks written to chosen pages of an existing pool (other pages untouched)."""
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(3)
    counts = [5, 9, 2]
    rows = unit_rows(16, 64, g).half().to(dev)
    pool = torch.full((6, 16, 64), 7.0, dtype=torch.float16, device=dev)
    page_of = torch.tensor([4, 1, 2], dtype=torch.int32, device=dev)
    slots, nv, S = ops.library_build(rows, counts, page_rows=16, slots=pool, page_of=page_of)
    assert slots.data_ptr() == pool.data_ptr()
    assert torch.equal(pool[4, :5], rows[:5]) and torch.equal(pool[1, :9], rows[5:14])
    assert torch.equal(pool[2, :2], rows[14:16])
    assert bool((pool[4, 5:] == 0).all()) and bool((pool[2, 2:] == 0).all())
    assert bool((pool[0] == 7).all()) and bool((pool[3] == 7).all()) and bool((pool[5] == 7).all())
    assert _status(dev) == 0


def test_build_bad_row_range_is_flagged(dev):
    """A row range that leaves the row buffer builds an empty chunk and raises XENCB_DEV_BADROWS (the kernel
    checks the range before reading any row)."""
    from kv_skill_v2_b200 import _native as N
    from kv_skill_v2_b200 import ops
    rows = torch.ones(10, 64, dtype=torch.float16, device=dev)
    start = torch.tensor([0, 4, 40], dtype=torch.int64, device=dev)  # chunk 1 claims rows [4, 40) of 10
    slots = torch.full((2, 64, 64), 3.0, dtype=torch.float16, device=dev)
    page_of = torch.arange(2, dtype=torch.int32, device=dev)
    nv = torch.full((2,), -1, dtype=torch.int32, device=dev)
    S = torch.empty(2, 64, dtype=torch.float32, device=dev)
    ws_bytes = N.lib().xencb_library_build_workspace(2, 64, 64)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    N.call("xencb_library_build", ops._ptr(rows), N.F16, 10, ops._ptr(start), 2, 64, None, ops._ptr(slots), N.F16,
           2, 64 * 64, 64, ops._ptr(page_of), ops._ptr(nv), ops._ptr(S), ops._ptr(ws), ws.numel(),
           ops._stream(dev))
    st = _status(dev)
    assert st & 8, f"status {st}: XENCB_DEV_BADROWS expected"
    assert nv.tolist() == [4, 0]
    assert bool((slots[1] == 0).all()) and bool((S[1] == 0).all())
    assert torch.equal(slots[0, :4], rows[:4])


def _doc_cache(g, counts, d, depths, untied=False, doc="d"):
    chunks = []
    for i, n in enumerate(counts):
        ch = {"K": {r: unit_rows(n, d, g).half() for r in depths}, "n_tokens": n, "start": 32 * i}
        if untied:
            ch["V"] = {r: (torch.randn(n, d, generator=g) * 0.3).half() for r in depths}
        chunks.append(ch)
    return {"chunks": chunks, "d_s": d, "doc_id": doc, "encoder": "tiny", "chunk_tokens": 32, "depths": depths}


@pytest.mark.parametrize("untied", [False, True])
@pytest.mark.parametrize("centered", [False, True])
def test_from_doc_caches_equals_host_build(dev, untied, centered):
    from kv_skill_v2_b200 import DEPTHS, Library, PagedLibrary, ops
    g = torch.Generator().manual_seed(5)
    reader = TinyReader(40, 8)
    d = 64
    caches = [_doc_cache(g, cs, d, DEPTHS, untied, f"doc{b}") for b, cs in enumerate(((32, 32, 26), (7, 32)))]
    center = {r: torch.randn(d, generator=g) * 0.05 for r in DEPTHS} if centered else None
    dt = torch.float16  # centred float32 rows are rounded to float16 slots too (Library.pages "auto")
    pl_dev = PagedLibrary.from_doc_caches(caches, reader, device=dev, center=center)
    libs = [Library.from_doc_cache(c, reader, center=center) for c in caches]
    pl_host = PagedLibrary.from_libraries(libs, dev, slot_dtype=dt)
    assert pl_dev.layers == pl_host.layers and pl_dev.n_lib == 2 and pl_dev.n_chunks == 3
    assert (pl_dev.V is not None) == untied
    for li in pl_dev.layers:
        a, b = pl_dev.pages(li), pl_host.pages(li)
        assert a.slots.dtype == dt
        assert torch.equal(a.n_valid, b.n_valid) and torch.equal(a.n_chunks_of, b.n_chunks_of)
        for lb in range(2):
            for cc in range(int(a.n_chunks_of[lb])):
                n = int(a.n_valid[lb, cc])
                pa, pb = int(a.page_of[lb, cc]), int(b.page_of[lb, cc])
                ka, kb = a.slots[pa, :n].float(), b.slots[pb, :n].float()
                if centered:
                    assert (ka - kb).abs().max().item() <= (1e-3 if dt == torch.float16 else 1e-6)
                else:
                    assert torch.equal(ka, kb)
                if untied:
                    assert torch.equal(a.vslots[pa, :n], b.vslots[pb, :n])
        assert (a.S - b.S).abs().max().item() <= 1e-6
        q = torch.nn.functional.normalize(torch.randn(2, d, generator=g), dim=-1).to(dev)
        idx, wk, _, _ = ops.route(q, a.S, rows_per_lib=1, top_k=2, route_temp=10.0, n_chunks_of=a.n_chunks_of)
        r_a = ops.read_decode(q, a, idx, wk, rows_per_lib=1)
        r_b = ops.read_decode(q, b, idx, wk, rows_per_lib=1)
        assert rel_err(r_a, r_b.cpu().numpy()) < (TOL if centered else 1e-6)
    assert _status(dev) == 0


def test_device_build_serves_untied_centered_golden(dev):
    """The reference's untied + centred case built on the device reads the reference's r."""
    from kv_skill_v2_b200 import ops
    c = load_case("untied_centered_linear")
    n = [int(x) for x in c["n_valid"]]
    rows = torch.cat([torch.from_numpy(c["K"][i, :n[i]]) for i in range(len(n))]).to(dev)
    vrows = torch.cat([torch.from_numpy(c["V"][i, :n[i]]) for i in range(len(n))]).to(dev)
    slots, nv, S = ops.library_build(rows, n, page_rows=128, mu=torch.from_numpy(c["center"]).to(dev),
                                     slot_dtype=torch.float16)
    vslots, _, _ = ops.library_build(vrows, n, page_rows=128, slot_dtype=torch.float16, want_summaries=False)
    assert np.abs(S.cpu().numpy() - c["S"]).max() <= 1e-6
    C = len(n)
    pages = ops.Pages(slots=slots, page_of=torch.arange(C, dtype=torch.int32, device=dev).view(1, C),
                      n_valid=nv.view(1, C), S=S.view(1, C, -1), vslots=vslots)
    h = torch.from_numpy(c["h"]).to(dev).reshape(-1, c["h"].shape[-1])
    q, _, _, _ = ops.project_in(h, torch.from_numpy(c["W_in"]).t().contiguous().to(dev))
    R = q.shape[0]
    idx, wk, w, _ = ops.route(q, pages.S, rows_per_lib=R, top_k=int(c["top_k"]), route_temp=float(c["route_temp"]))
    r = ops.read_decode(q, pages, idx, wk, rows_per_lib=R, read_temp=float(c["read_temp"]),
                        read_softmax=bool(c["read_softmax"]))
    assert rel_err(r, c["r"].reshape(R, -1)) < TOL
    assert _status(dev) == 0
