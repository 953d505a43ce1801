"""Host-side logic of the xenc-compatible API, on CPU (no kernel is launched here).

Library construction is checked against the reference's own Library outputs (tests/golden/library.npz);
interface save/load, param groups and counts, selector and injector argument validation follow the
reference's tests (tests/test_library.py, test_interface.py, test_selector.py of xenc)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from kv_skill_v2_b200 import (DEPTHS, DepthCollisionError, LayerSelector, Library, LibraryInjector, LinearInterface,
                              PagedLibrary, count_params, injection_layers, interface_param_groups, load_interface,
                              make_interface, rho_layer_map, save_interface)
from tests._fixtures import GOLDEN, TinyReader, unit_rows


def _golden_library():
    c = dict(np.load(GOLDEN / "library.npz"))
    layers = [int(x) for x in c["layers"]]
    depths = [float(x) for x in c["depths"]]
    chunks = []
    for i, n in enumerate(c["n"]):
        chunks.append({"K": {depths[j]: torch.from_numpy(c[f"rows_{li}"][i, :n].astype(np.float32))
                             for j, li in enumerate(layers)}})
    mu = {depths[j]: torch.from_numpy(c[f"mu_{li}"]) for j, li in enumerate(layers)}
    return c, layers, depths, chunks, mu


def test_library_matches_reference_build():
    c, layers, depths, chunks, mu = _golden_library()
    lib = Library(chunks, layers, depths)
    assert lib.layers == layers and lib.n_chunks == len(c["n"]) and lib.d_s == 24
    for li in layers:
        assert torch.equal(lib.K[li], torch.from_numpy(c[f"K_{li}"]))
        assert torch.equal(lib.mask[li], torch.from_numpy(c[f"mask_{li}"]))
        assert torch.allclose(lib.S[li], torch.from_numpy(c[f"S_{li}"]), atol=1e-6)
        assert lib.n_valid(li).tolist() == [int(x) for x in c["n"]]
    libc = Library(chunks, layers, depths, center=mu)
    for li in layers:
        assert torch.allclose(libc.K[li], torch.from_numpy(c[f"Kc_{li}"]), atol=1e-6)
        assert torch.allclose(libc.S[li], torch.from_numpy(c[f"Sc_{li}"]), atol=1e-6)
    sub = lib.subset([1, 3])
    for li in layers:
        assert torch.equal(sub.K[li], torch.from_numpy(c[f"Ksub_{li}"]))
        assert torch.equal(sub.mask[li], torch.from_numpy(c[f"masksub_{li}"]))
        assert torch.allclose(sub.S[li], torch.from_numpy(c[f"Ssub_{li}"]), atol=1e-6)


def test_library_guards_and_subset_rebuild():
    with pytest.raises(ValueError):
        Library([], [2], [0.5])
    g = torch.Generator().manual_seed(0)
    ch = [{"K": {0.5: unit_rows(n, 16, g)}} for n in (6, 12, 3, 9)]
    with pytest.raises(ValueError):
        Library(ch, [1, 2], [0.5])
    lib = Library(ch, [4], [0.5])
    for i in range(4):
        a, b = lib.subset([i]), Library([ch[i]], [4], [0.5])
        assert torch.equal(a.K[4], b.K[4]) and torch.equal(a.mask[4], b.mask[4])
        assert torch.allclose(a.S[4], b.S[4], atol=1e-6)
    with pytest.raises(ValueError):
        lib.subset([])


def test_from_doc_cache_ragged():
    g = torch.Generator().manual_seed(1)
    reader = TinyReader(40, 8)
    chunks = [{"K": {r: unit_rows(n, 24, g).half() for r in DEPTHS}, "n_tokens": n, "start": 32 * i}
              for i, n in enumerate((32, 32, 26))]
    cache = {"chunks": chunks, "d_s": 24, "doc_id": "dd", "encoder": "tiny", "chunk_tokens": 32, "depths": DEPTHS}
    lib = Library.from_doc_cache(cache, reader)
    assert lib.n_chunks == 3 and lib.d_s == 24 and lib.layers == injection_layers(reader, DEPTHS)
    assert lib.mask[lib.layers[0]].sum(-1).tolist() == [32, 32, 26]
    assert lib.K[lib.layers[0]].dtype == torch.float32
    assert [m["start"] for m in lib.chunk_meta] == [0, 32, 64]


def test_rho_layer_map_collision():
    assert rho_layer_map(8, DEPTHS) == {0.25: 2, 0.5: 4, 0.75: 6, 1.0: 7}
    with pytest.raises(DepthCollisionError):
        rho_layer_map(3, DEPTHS)


def test_pages_layout_and_empty_chunk_rejected():
    g = torch.Generator().manual_seed(2)
    ch = [{"K": {0.5: unit_rows(n, 16, g)}} for n in (5, 9)]
    lib = Library(ch, [4], [0.5])
    p = lib.pages(4, "cpu")
    assert p.slots.dtype == torch.float16  # exact in fp16 -> stored as fp16
    assert p.page_of.tolist() == [[0, 1]] and p.n_valid.tolist() == [[5, 9]] and p.S.shape == (1, 2, 16)
    lib.mask[4][0] = False
    lib._page_cache = {}
    with pytest.raises(ValueError):
        lib.pages(4, "cpu")
    assert lib.pages(4, "cpu", require_nonempty=False).n_valid.tolist() == [[0, 9]]


def test_paged_library_from_libraries():
    g = torch.Generator().manual_seed(3)
    libs = [Library([{"K": {0.5: unit_rows(n, 16, g)}} for n in ns], [4], [0.5]) for ns in ((5, 9), (3, 4, 7))]
    pl = PagedLibrary.from_libraries(libs, "cpu")
    p = pl.pages(4)
    assert pl.n_lib == 2 and pl.n_chunks == 3 and pl.d_s == 16
    assert p.page_of.tolist() == [[0, 1, 0], [2, 3, 4]]
    assert p.n_valid.tolist() == [[5, 9, 0], [3, 4, 7]]
    assert p.n_chunks_of.tolist() == [2, 3]
    assert torch.equal(p.slots[3, :4].float(), libs[1].K[4][1, :4])


def test_untied_pages_and_paged_value_pools():
    """Untied chunks give a value pool beside the key pool (same layout, float16); a tied Library stacked with an
    untied one contributes its keys as values; float32 untied pools are refused."""
    g = torch.Generator().manual_seed(4)
    ch = [{"K": {0.5: unit_rows(n, 16, g)}, "V": {0.5: torch.randn(n, 16, generator=g)}} for n in (5, 9)]
    lib = Library(ch, [4], [0.5])
    assert lib.V is not None
    p = lib.pages(4, "cpu")
    assert p.vslots is not None and p.vslots.shape == p.slots.shape and p.vslots.dtype == torch.float16
    assert torch.equal(p.vslots[1, :9], lib.V[4][1, :9].half())
    assert torch.equal(p.slots[0, :5], lib.K[4][0, :5].half())
    with pytest.raises(NotImplementedError):
        lib.pages(4, "cpu", slot_dtype=torch.float32)
    tied = Library([{"K": {0.5: unit_rows(n, 16, g)}} for n in (3, 4)], [4], [0.5])
    pl = PagedLibrary.from_libraries([lib, tied], "cpu")
    q = pl.pages(4)
    assert pl.V is not None and q.vslots.shape == q.slots.shape
    assert torch.equal(q.vslots[0, :5], lib.V[4][0, :5].half())
    assert torch.equal(q.vslots[3, :4], q.slots[3, :4])  # the tied Library's values are its keys
    assert PagedLibrary.from_libraries([tied], "cpu").V is None


def test_interface_save_load_roundtrip(tmp_path):
    for with_sel in (False, True):
        for rank in (0, 8):
            torch.manual_seed(1)
            itf = make_interface(40, 24, [2, 4, 6, 7], rank=rank)
            with torch.no_grad():
                for p_ in itf.parameters():
                    p_.add_(torch.randn(p_.shape) * 0.1)
            sel = LayerSelector(40, [2, 4, 6, 7], k=2, alpha_init=0.05) if with_sel else None
            path = str(tmp_path / f"itf_{with_sel}_{rank}.pt")
            save_interface(itf, path, selector=sel, extra={"step": 7})
            itf2, sel2, extra = load_interface(path, 40, 24, [2, 4, 6, 7])
            assert extra == {"step": 7} and (sel2 is None) == (sel is None)
            for k, v in itf.state_dict().items():
                assert torch.equal(v, itf2.state_dict()[k])
            if sel is not None:
                assert sel2.cand_layers == sel.cand_layers and sel2.k == sel.k
    with pytest.raises(ValueError):
        load_interface(path, 40, 32, [2, 4, 6, 7])
    with pytest.raises(ValueError):
        make_interface(40, 24, [2, 2])


def test_param_groups_and_counts():
    for rank in (0, 8):
        itf = make_interface(40, 24, [2, 4, 6, 7], rank=rank)
        sel = LayerSelector(40, [2, 4, 6, 7], k=2)
        for s, slr in ((None, None), (sel, None), (sel, 1e-3)):
            groups = interface_param_groups(itf, 2e-4, selector=s, selector_lr=slr)
            ids = [id(p) for g in groups for p in g["params"]]
            expect = [id(p) for p in itf.parameters()] + ([id(p) for p in s.parameters()] if s is not None else [])
            assert len(ids) == len(set(ids)) == len(expect) and set(ids) == set(expect)
        ga = [g for g in interface_param_groups(itf, 2e-4, lr_A=2e-3) if g["name"] == "interface_A"][0]
        assert {id(p) for p in ga["params"]} == {id(p) for p in itf.A.parameters()}
        c = count_params(itf, sel)
        assert c["total"] == c["interface"] + c["selector"]
        assert c["selector"] == 40 * 4 + 4 + 1
        assert c["A"] + c["B"] + c["gate_gain"] == c["interface"]


def test_selector_validation():
    with pytest.raises(ValueError):
        LayerSelector(40, [3, 3, 5], k=1)
    with pytest.raises(ValueError):
        LayerSelector(40, [3, 5], k=3)
    with pytest.raises(ValueError):
        LayerSelector(40, [3, 5], k=1, alpha_init=0.0)
    sel = LayerSelector(40, [9, 3, 5, 7], k=2)
    assert sel.cand_layers == [3, 5, 7, 9] and sel.pos[7] == 2 and sel.first_layer == 3
    assert sel.config() == {"d_m": 40, "cand_layers": [3, 5, 7, 9], "k": 2, "straight_through": False}


def test_injector_guards_and_no_cpu_path():
    reader = TinyReader(32, 8)
    layers = injection_layers(reader, DEPTHS)
    g = torch.Generator().manual_seed(4)
    W_in, W_out = torch.randn(32, 24, generator=g), torch.randn(24, 32, generator=g)
    itf = LinearInterface(W_in, W_out, layers)
    rmap = rho_layer_map(reader, DEPTHS)
    lib = Library([{"K": {r: unit_rows(n, 24, g) for r in DEPTHS}} for n in (5, 9, 3)],
                  [rmap[r] for r in DEPTHS], DEPTHS)
    inj = LibraryInjector(reader, itf, top_k=2)
    bad = Library([{"K": {r: unit_rows(4, 16, g) for r in DEPTHS}}], [rmap[r] for r in DEPTHS], DEPTHS)
    with pytest.raises(ValueError):
        inj.load_library(bad)
    partial = Library([{"K": {r: unit_rows(4, 24, g) for r in DEPTHS[:2]}}], [rmap[r] for r in DEPTHS[:2]],
                      DEPTHS[:2])
    with pytest.raises(KeyError):
        inj.load_library(partial)
    inj.load_library(lib)
    with torch.no_grad(), pytest.raises(RuntimeError, match="no CPU path"):
        reader(torch.randn(2, 5, 32))
    inj.unload()
    with torch.no_grad():
        reader(torch.randn(2, 5, 32))  # unloaded: the bare model runs
    inj.detach()


def test_topk_library_keys_gold_hit_and_no_cpu_path():
    """D8 host logic (xenc tests/test_topk_read.py (c), (e)): sel_K follows subset, misaligned harvests raise,
    gold-hit statistics against brute force, and the selection has no CPU path."""
    import math
    from itertools import combinations

    from kv_skill_v2_b200.topk_read import TopKLibrary, TopKSelector, attach_sel_keys
    from tests._fixtures import TinyAttnReader

    g = torch.Generator().manual_seed(9)
    depths, layers = [0.2, 0.4, 0.6, 0.8], [1, 3, 5, 7]
    ns = (16, 16, 9)
    lib = Library([{"K": {r: unit_rows(n, 24, g) for r in depths}} for n in ns], layers, depths)
    lib = attach_sel_keys(lib, {"chunks": [{"K": {0.25: torch.randn(n, 16, generator=g)}} for n in ns]}, 0.25)
    assert isinstance(lib, TopKLibrary) and lib.sel_K.shape == (3, 16, 16)
    sub = lib.subset([2, 0])
    assert isinstance(sub, TopKLibrary) and sub.sel_K.shape[:2] == sub.mask[layers[0]].shape
    assert torch.equal(sub.sel_K[1], lib.sel_K[0, : sub.sel_K.shape[1]])
    bad = Library([{"K": {r: unit_rows(n, 24, g) for r in depths}} for n in ns], layers, depths)
    with pytest.raises(ValueError):
        attach_sel_keys(bad, {"chunks": [{"K": {0.25: torch.zeros(5, 16)}}] * 3}, 0.25)

    m = TinyAttnReader(32, 8, 2, 8, 2)
    sel = TopKSelector(m, 3, k=3)
    n = 10
    sel.valid = torch.ones(n, dtype=torch.bool)
    sel.last_scores = torch.arange(n, dtype=torch.float32).flip(0).unsqueeze(0)
    gold = torch.zeros(n, dtype=torch.bool)
    gold[[4, 7]] = True
    st = sel.gold_hit(gold, ks=[3, 5])
    assert st["n_gold"] == 2 and st["best_rank"] == 4
    assert st[3]["hit"] == 0.0 and st[5]["hit"] == 1.0 and st[5]["n_gold_sel"] == 1
    for k in (3, 5):
        brute = sum(any(i in (4, 7) for i in cmb) for cmb in combinations(range(n), k)) / math.comb(n, k)
        assert abs(st[k]["chance_any"] - brute) < 1e-9
        assert abs(st[k]["chance_frac"] - k * 2 / n) < 1e-12
    assert sel.gold_hit(torch.zeros(n, dtype=torch.bool)) == {}

    sel.set_keys(lib.sel_K, lib.mask[layers[0]])
    assert sel.n_valid == 41 and sel.keys.shape == (48, 2, 8)
    with pytest.raises(RuntimeError, match="CPU"):
        sel.select_from_input(torch.randn(1, 5, 32))
