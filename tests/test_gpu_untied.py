"""Untied values (harvest="attn": chunks with a separate V; xenc/library.py:46, 61-65) and centered Libraries
(K = L2(K - mu) on valid rows, V untouched; xenc/library.py:56-58) through the CUDA read kernels.

The reference's untied read scores with K and sums V (xenc/injector.py:211-218, 263-265). Golden cases come from
the reference's own _branch (tests/golden/make_golden.py gen_untied); larger seeded cases run the decode,
many-query and prefill kernels against the oracle. Bar: routing sets identical, outputs within
max|out - ref| <= 2e-3 * max|ref| (values and keys are rounded to float16 slots for the tensor-core read)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import xenc_oracle as X
from tests._fixtures import TOL, load_case, rel_err, topk_sets

pytestmark = pytest.mark.gpu

CASES = ["untied_top2", "untied_centered_linear"]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _status_clean(dev):
    from kv_skill_v2_b200 import ops
    assert ops.device_status(dev) == 0, "a kernel flagged a device status bit"


def _library(c, li=3):
    """The case's chunks as a Library (raw K rows, V rows, the centering mean when the case has one)."""
    from kv_skill_v2_b200 import Library
    n = c["n_valid"]
    chunks = [{"K": {0.5: torch.from_numpy(c["K"][i, :n[i]]).float()},
               "V": {0.5: torch.from_numpy(c["V"][i, :n[i]]).float()}} for i in range(len(n))]
    center = {0.5: torch.from_numpy(c["center"])} if "center" in c else None
    return Library(chunks, [li], [0.5], center=center)


@pytest.mark.parametrize("name", CASES)
def test_untied_golden_all_read_kernels(dev, name):
    """Decode (top-k), many-query and prefill reads of the reference's untied / centered cases."""
    from kv_skill_v2_b200 import ops
    c = load_case(name)
    lib = _library(c)
    assert lib.V is not None
    if "center" in c:
        assert rel_err(lib.K[3], c["K_lib"]) < 1e-6
    pages = lib.pages(3, dev)
    assert pages.vslots is not None and pages.vslots.dtype == pages.slots.dtype == torch.float16
    assert rel_err(pages.S[0], c["S"]) < 1e-5
    h = torch.from_numpy(c["h"]).to(dev).reshape(-1, c["h"].shape[-1])
    W_in = torch.from_numpy(c["W_in"]).t().contiguous().to(dev)
    W_out = torch.from_numpy(c["W_out"]).t().contiguous().to(dev)
    q, _, _, _ = ops.project_in(h, W_in)
    R = q.shape[0]
    idx, wk, w, _ = ops.route(q, pages.S, rows_per_lib=R, top_k=int(c["top_k"]), route_temp=float(c["route_temp"]))
    w_ref = c["w"].reshape(w.shape)
    assert topk_sets(w) == topk_sets(w_ref)
    kw = dict(rows_per_lib=R, read_temp=float(c["read_temp"]), read_softmax=bool(c["read_softmax"]))
    r_ref = c["r"].reshape(R, -1)
    r = ops.read_decode(q, pages, idx, wk, **kw)
    assert rel_err(r, r_ref) < TOL
    delta, _, _ = ops.project_out(r, W_out, h)
    assert rel_err(delta, c["delta"].reshape(delta.shape)) < TOL
    r_m = ops.read_multi(q, pages, w, **kw)
    assert rel_err(r_m, r_ref) < TOL
    r_p = ops.read_prefill(q, pages, w, **kw)
    assert rel_err(r_p, r_ref) < TOL
    _status_clean(dev)


def test_untied_injector_branch(dev):
    """The LibraryInjector branch over an untied Library gives the reference's delta."""
    from kv_skill_v2_b200 import LibraryInjector, LinearInterface
    from tests._fixtures import TinyReader
    c = load_case("untied_top2")
    lib = _library(c, li=4)
    reader = TinyReader(8, 8).to(dev)
    itf = LinearInterface(torch.from_numpy(c["W_in"]), torch.from_numpy(c["W_out"]), [4]).to(dev)
    inj = LibraryInjector(reader, itf, top_k=2)
    inj.load_library(lib)
    with torch.no_grad():
        delta = inj._branch(torch.from_numpy(c["h"]).to(dev), 4)
    assert topk_sets(inj.last_route) == topk_sets(c["w"])
    assert rel_err(delta, c["delta"]) < TOL
    inj.detach()
    _status_clean(dev)


def _synthetic(n_lib, C, N, d, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    K = torch.randn(n_lib, C, N, d, generator=g)
    K = (K / K.norm(dim=-1, keepdim=True)).to(dtype).float()
    V = (torch.randn(n_lib, C, N, d, generator=g) * 0.5).to(dtype).float()
    nv = torch.full((n_lib, C), N, dtype=torch.int32)
    # valid-row counts at and around the 16-row group edges and a one-row chunk
    edges = [1, 15, 16, 17, 31, 33, N - 1, N]
    for b in range(n_lib):
        for j, e in enumerate(edges[:C]):
            nv[b, (j * 3 + b) % C] = min(max(e, 1), N)
    return K, V, nv


def _pages(K, V, nv, dev, dtype):
    from kv_skill_v2_b200 import ops
    n_lib, C, N, d = K.shape
    slots = K.reshape(n_lib * C, N, d).to(dtype).to(dev).contiguous()
    vslots = V.reshape(n_lib * C, N, d).to(dtype).to(dev).contiguous()
    page_of = torch.arange(n_lib * C, dtype=torch.int32, device=dev).view(n_lib, C)
    nv_d = nv.to(dev)
    return ops.Pages(slots=slots, page_of=page_of, n_valid=nv_d, S=ops.summaries(slots, page_of, nv_d),
                     vslots=vslots)


def _oracle(q, K, V, nv, w, T, softmax):
    n_lib, C, N, d = K.shape
    out = []
    for b in range(n_lib):
        M = (np.arange(N)[None, :] < nv[b].numpy()[:, None])
        rows = slice(b * T, (b + 1) * T)
        out.append(X.read(q[rows], K[b].numpy(), M, w[rows], read_temp=12.0, read_softmax=softmax,
                          V=V[b].numpy()))
    return np.concatenate(out, 0)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("softmax", [True, False])
@pytest.mark.parametrize("d", [64, 256])
def test_untied_synthetic_decode_and_multi(dev, dtype, softmax, d):
    """Two Libraries, ragged chunks, top-3 decode read and the dense many-query read against the oracle."""
    from kv_skill_v2_b200 import ops
    n_lib, C, N, T = 2, 8, 200, 11
    K, V, nv = _synthetic(n_lib, C, N, d, 31 + d, dtype)
    pages = _pages(K, V, nv, dev, dtype)
    g = torch.Generator().manual_seed(7)
    q = torch.nn.functional.normalize(torch.randn(n_lib * T, d, generator=g), dim=-1)
    qd = q.to(dev)
    idx, wk, w, _ = ops.route(qd, pages.S, rows_per_lib=T, top_k=3, route_temp=10.0)
    ref_top = _oracle(q.numpy(), K, V, nv, w.cpu().numpy(), T, softmax)
    r = ops.read_decode(qd, pages, idx, wk, rows_per_lib=T, read_temp=12.0, read_softmax=softmax)
    assert rel_err(r, ref_top) < TOL
    r_m = ops.read_multi(qd, pages, w, rows_per_lib=T, read_temp=12.0, read_softmax=softmax)
    assert rel_err(r_m, ref_top) < TOL
    wd = torch.softmax(torch.randn(n_lib * T, C, generator=g), -1)
    ref_dense = _oracle(q.numpy(), K, V, nv, wd.numpy(), T, softmax)
    r_d = ops.read_multi(qd, pages, wd.to(dev), rows_per_lib=T, read_temp=12.0, read_softmax=softmax)
    assert rel_err(r_d, ref_dense) < TOL
    if dtype == torch.float16 and d % 64 == 0:
        r_p = ops.read_prefill(qd, pages, wd.to(dev), rows_per_lib=T, read_temp=12.0, read_softmax=softmax)
        assert rel_err(r_p, ref_dense) < TOL
    _status_clean(dev)


def test_untied_with_values_equal_keys_matches_tied(dev):
    """vslots = a copy of slots gives the tied read (the value stage reads the same rows as the key stage)."""
    from kv_skill_v2_b200 import ops
    K, _, nv = _synthetic(1, 6, 130, 128, 5, torch.float16)
    tied = _pages(K, K, nv, dev, torch.float16)
    untied = ops.Pages(slots=tied.slots, page_of=tied.page_of, n_valid=tied.n_valid, S=tied.S,
                       vslots=tied.slots.clone())
    tied = ops.Pages(slots=tied.slots, page_of=tied.page_of, n_valid=tied.n_valid, S=tied.S)
    q = torch.nn.functional.normalize(torch.randn(5, 128, generator=torch.Generator().manual_seed(3)), dim=-1).to(dev)
    idx, wk, w, _ = ops.route(q, tied.S, rows_per_lib=5, top_k=2, route_temp=10.0)
    a = ops.read_decode(q, tied, idx, wk, rows_per_lib=5)
    b = ops.read_decode(q, untied, idx, wk, rows_per_lib=5)
    assert rel_err(b, a) < 1e-5
    a = ops.read_multi(q, tied, w, rows_per_lib=5)
    b = ops.read_multi(q, untied, w, rows_per_lib=5)
    assert rel_err(b, a) < 1e-5
    _status_clean(dev)


def test_untied_float32_slots_are_refused(dev):
    """The untied read runs on the tensor cores only: float32 pools raise NotImplementedError, no fallback."""
    from kv_skill_v2_b200 import ops
    K, V, nv = _synthetic(1, 3, 40, 64, 9, torch.float16)
    pages = _pages(K, V, nv, dev, torch.float32)
    q = torch.nn.functional.normalize(torch.randn(2, 64), dim=-1).to(dev)
    idx, wk, _, _ = ops.route(q, pages.S, rows_per_lib=2, top_k=2, route_temp=10.0)
    with pytest.raises(NotImplementedError):
        ops.read_decode(q, pages, idx, wk, rows_per_lib=2)


def test_centered_library_reads_float16_slots_against_oracle(dev):
    """A centred tied Library (K = L2(K - mu), xenc/library.py:56-58: float32 rows that float16 does not hold
    exactly) is stored as float16 slots by default, so it is read by the tensor-core kernel; S comes from the
    float32 rows. Routing matches the oracle's exactly and the read is within the path's tolerance of the oracle's
    float32 read; slot_dtype=torch.float32 keeps float32 slots."""
    from kv_skill_v2_b200 import Library, ops
    from oracle import xenc_oracle as X
    g = torch.Generator().manual_seed(31)
    d, counts = 256, (64, 40, 64, 17, 64)
    rows = [torch.randn(n, d, generator=g) for n in counts]
    mu = torch.randn(d, generator=g) * 0.3
    lib = Library([{"K": {0.5: r}} for r in rows], [3], [0.5], center={0.5: mu})
    K_ref, M_ref, S_ref = X.build_library([r.numpy() for r in rows], mu.numpy())
    pages = lib.pages(3, dev)
    assert pages.slots.dtype == torch.float16
    assert lib.pages(3, dev, slot_dtype=torch.float32).slots.dtype == torch.float32
    assert rel_err(pages.S[0], S_ref) < 1e-5
    q = torch.nn.functional.normalize(torch.randn(6, d, generator=g), dim=-1)
    w_ref, _, _ = X.route(q.numpy(), S_ref, 10.0, 2)
    r_ref = X.read(q.numpy(), K_ref, M_ref, w_ref, 12.0, True)
    qd = q.to(dev)
    idx, wk, w, _ = ops.route(qd, pages.S, rows_per_lib=6, top_k=2, route_temp=10.0)
    assert topk_sets(w) == topk_sets(w_ref)
    r = ops.read_decode(qd, pages, idx, wk, rows_per_lib=6)
    assert rel_err(r, r_ref) < TOL
    _status_clean(dev)
