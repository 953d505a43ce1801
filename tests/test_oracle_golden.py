"""Pin the numpy oracle to the golden fixtures produced by the reference's own code.

The fixtures under tests/golden/ were written by tests/golden/make_golden.py, which ran the reference's
unchanged xenc.library / xenc.injector / xenc.selector. Every oracle function used as a checker for the
CUDA path is compared here first. CPU only."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import xenc_oracle as X

G = Path(__file__).resolve().parent / "golden"
READ_CASES = ["cfg1_softmax_top2", "cfg1_dense", "cfg1_linear_top2", "cfg1_topk_eq_C", "cfg1_linear_dense",
              "small_ragged_top2", "small_ragged_linear", "small_ragged_dense_t3", "one_chunk", "odd_dims_top3"]


def load_case(name: str) -> dict:
    """Golden case with its inputs (cases that share inputs name the case that holds them)."""
    rec = dict(np.load(G / f"{name}.npz"))
    if "inputs" in rec:
        base = dict(np.load(G / f"{str(rec.pop('inputs'))}.npz"))
        for k in ("K", "n_valid", "h", "W_in", "W_out"):
            rec[k] = base[k]
    return rec


def rel_err(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def topk_sets(w: np.ndarray) -> list:
    return [frozenset(np.flatnonzero(row > 0).tolist()) for row in w.reshape(-1, w.shape[-1])]


@pytest.mark.parametrize("name", READ_CASES)
def test_oracle_branch_matches_reference(name):
    c = load_case(name)
    K = c["K"].astype(np.float32)
    M = np.arange(K.shape[1])[None, :] < c["n_valid"][:, None]
    S = X.summaries(K, M)
    assert rel_err(S, c["S"]) < 1e-6
    assert np.array_equal(M, c["mask"])
    h = c["h"].reshape(-1, c["h"].shape[-1])
    out = X.branch(h, c["W_in"], c["W_out"], K, M, S, read_temp=float(c["read_temp"]),
                   route_temp=float(c["route_temp"]), top_k=int(c["top_k"]), read_softmax=bool(c["read_softmax"]))
    assert rel_err(out["q"], c["q"].reshape(out["q"].shape)) < 1e-5
    w_ref = c["w"].reshape(out["w"].shape)
    assert topk_sets(out["w"]) == topk_sets(w_ref), "routing index sets must be identical"
    assert rel_err(out["w"], w_ref) < 1e-5
    assert rel_err(out["r"], c["r"].reshape(out["r"].shape)) < 1e-5
    assert rel_err(out["delta"], c["delta"].reshape(out["delta"].shape)) < 1e-5


def test_oracle_batch_docs_matches_reference():
    c = load_case("batch_docs_top2")
    for b in range(c["K"].shape[0]):
        K = c["K"][b].astype(np.float32)
        M = np.arange(K.shape[1])[None, :] < c["n_valid"][b][:, None]
        out = X.branch(c["h"][b], c["W_in"], c["W_out"], K, M, X.summaries(K, M), top_k=2)
        assert topk_sets(out["w"]) == topk_sets(c["w"][b])
        assert rel_err(out["r"], c["r"][b]) < 1e-5
        assert rel_err(out["delta"], c["delta"][b]) < 1e-5


def test_oracle_topk_every_row_has_k_nonzeros():
    c = load_case("cfg1_softmax_top2")
    nz = (c["w"] > 0).sum(-1)
    assert (nz == 2).all()
    assert np.allclose(c["w"].sum(-1), 1.0, atol=1e-6)


def test_oracle_selector_matches_reference():
    c = dict(np.load(G / "selector.npz"))
    for st in (0, 1):
        for k in (1, 2, 3):
            key = f"st{st}_k{k}"
            h0 = c[f"{key}_h"][0]
            z = X.selector_logits(X.rms_norm(h0), c[f"{key}_u_w"], c[f"{key}_u_b"])
            assert rel_err(z, c[f"{key}_z"]) < 1e-5
            w = X.selector_weights(z, k, straight_through=bool(st))
            assert np.array_equal(w > 0, c[f"{key}_w"] > 0)
            assert rel_err(w, c[f"{key}_w"]) < 1e-5
            for i in range(len(c["cand"])):
                out = X.selector_apply(c[f"{key}_delta"][i], c[f"{key}_h"][i], w[..., i], float(c[f"{key}_log_alpha"]))
                assert rel_err(out, c[f"{key}_out"][i]) < 1e-5


def test_oracle_library_matches_reference():
    c = dict(np.load(G / "library.npz"))
    for li in c["layers"]:
        rows = c[f"rows_{li}"].astype(np.float32)
        chunk_rows = [rows[i, :n] for i, n in enumerate(c["n"])]
        K, M, S = X.build_library(chunk_rows)
        assert np.array_equal(K, c[f"K_{li}"]) and np.array_equal(M, c[f"mask_{li}"])
        assert rel_err(S, c[f"S_{li}"]) < 1e-6
        Kc, Mc, Sc = X.build_library(chunk_rows, center_mu=c[f"mu_{li}"])
        assert rel_err(Kc, c[f"Kc_{li}"]) < 1e-6 and rel_err(Sc, c[f"Sc_{li}"]) < 1e-6
        Ks, Ms, Ss = X.subset(K, M, [1, 3])
        assert np.array_equal(Ks, c[f"Ksub_{li}"]) and np.array_equal(Ms, c[f"masksub_{li}"])
        assert rel_err(Ss, c[f"Ssub_{li}"]) < 1e-6


def test_oracle_shard_merge_equals_dense_read():
    c = load_case("cfg1_dense")
    K = c["K"].astype(np.float32)
    M = np.arange(K.shape[1])[None, :] < c["n_valid"][:, None]
    S = X.summaries(K, M)
    q = c["q"].reshape(-1, c["q"].shape[-1])
    parts = [X.shard_partials(q, K[a:b], M[a:b], S[a:b], 10.0, 12.0) for a, b in ((0, 3), (3, 5), (5, 8))]
    r = X.merge_shards(parts)
    assert rel_err(r, c["r"].reshape(r.shape)) < 1e-5


@pytest.mark.parametrize("name", ["untied_top2", "untied_centered_linear"])
def test_untied_values_and_centering(name):
    """Untied V (the read weights V, the scores and summaries use K) and a centered Library
    (K = L2(K - mu) on valid rows, V untouched): the oracle against the reference's own _branch."""
    c = load_case(name)
    K, n = c["K"].astype(np.float32), c["n_valid"]
    M = np.arange(K.shape[1])[None, :] < n[:, None]
    if "center" in c:
        K = X.build_library([K[i, :n[i]] for i in range(len(n))], c["center"])[0]
        assert np.abs(K - c["K_lib"]).max() < 1e-6
    S = X.summaries(K, M)
    assert np.abs(S - c["S"]).max() < 1e-6
    h = c["h"].reshape(-1, c["h"].shape[-1])
    out = X.branch(h, c["W_in"], c["W_out"], K, M, S, read_temp=float(c["read_temp"]),
                   route_temp=float(c["route_temp"]), top_k=int(c["top_k"]), read_softmax=bool(c["read_softmax"]),
                   V=c["V"].astype(np.float32))
    assert topk_sets(out["w"]) == topk_sets(c["w"].reshape(out["w"].shape))
    assert rel_err(out["r"], c["r"].reshape(out["r"].shape)) < 1e-5
    assert rel_err(out["delta"], c["delta"].reshape(out["delta"].shape)) < 1e-5


# ------------------------------------------------------------------------------------------------ D8 top-k read
TOPK_CASES = ["topk_last_softmax", "topk_allmean_linear", "topk_batch2_allmax"]


def _topk_oracle_forward(c):
    """The reference's hooked D8 forward restated with the oracle: the selection from the bare reader's queries
    at layer 3, then at each injection layer h + gain * sigmoid(hn . gate_w + gate_b) * B (topk_read(A hn))."""
    import torch
    from kv_skill_v2_b200.topk_read import attn_geometry, reader_queries
    from tests._fixtures import TinyAttnReader

    m = TinyAttnReader(32, 8, 2, 8, 2).load_arrays(c).eval()
    layers, sel_layer = [1, 3, 5, 7], 3
    x = torch.from_numpy(c["x"])
    att = m.model.layers[sel_layer].self_attn
    cap = {}
    hook = att.register_forward_pre_hook(lambda mod, a: cap.setdefault("x", a[0].detach().clone()))
    with torch.no_grad():
        m(x)
    hook.remove()
    T = x.shape[1]
    pos = T + int(c["sel_pos"]) if int(c["sel_pos"]) < 0 else int(c["sel_pos"])
    with torch.no_grad():
        q_sel = reader_queries(att, cap["x"][:, : pos + 1], attn_geometry(att)).numpy()
    n = c["n"]
    C, N = len(n), c[f"K_{layers[0]}"].shape[1]
    valid = (np.arange(N)[None, :] < n[:, None]).reshape(-1)
    keys = c["sel_K"].reshape(C * N, 2, 8)
    scores = X.topk_select_scores(q_sel, keys, valid, query=str(c["query"]), pool=str(c["pool"]))
    k = min(int(c["k"]), int(valid.sum()))
    idx = X.topk_select(scores, k)

    pos_of = {li: i for i, li in enumerate(layers)}

    def inject(mod, args, out, li):
        h = out.detach().numpy()
        B, Tq, d = h.shape
        hn = X.rms_norm(h.reshape(-1, d))
        q = X.l2(hn @ c["A_w"].T).reshape(B, Tq, -1)
        r, _ = X.topk_read(q, c[f"K_{li}"].reshape(C * N, -1), idx, read_softmax=bool(c["read_softmax"]))
        p = pos_of[li]
        g = 1.0 / (1.0 + np.exp(-(hn @ c["gate_w"] + c["gate_b"][p])))
        delta = np.exp(c["log_gain"][p]) * g.reshape(B, Tq, 1) * (r @ c["B_w"].T)
        return torch.from_numpy((h + delta).astype(np.float32))

    hs = [m.model.layers[li].register_forward_hook(lambda mod, a, o, li=li: inject(mod, a, o, li)) for li in layers]
    with torch.no_grad():
        lg = m.logits(x).numpy()
    for hd in hs:
        hd.remove()
    return scores, idx, lg


@pytest.mark.parametrize("name", TOPK_CASES)
def test_topk_oracle_matches_reference(name):
    """Selection scores, the selected slot sets (in score order) and the hooked model's logits of the reference's
    TopKLibraryInjector, restated with the oracle (selection query / pool modes, softmax and linear reads, two
    batch rows with their own selections)."""
    c = load_case(name)
    scores, idx, lg = _topk_oracle_forward(c)
    ref_scores = c["scores_call"] if "scores_call" in c else c["scores"]
    fin = np.isfinite(ref_scores)
    assert np.array_equal(fin, np.isfinite(scores))
    assert np.abs(scores[fin] - ref_scores[fin]).max() < 1e-5
    assert [set(r) for r in idx.tolist()] == [set(r) for r in c["idx"].tolist()]
    assert np.array_equal(idx, c["idx"]), "selection order (score descending) differs"
    assert rel_err(lg, c["logits"]) < 1e-5


ATTN_CASES = ["attn_record_top2", "attn_record_linear", "attn_force", "attn_force_norm"]


@pytest.mark.parametrize("name", ATTN_CASES)
def test_attention_diagnostics_oracle_matches_reference(name):
    """record_attn's last_attn and force_attn's read (with and without force_norm_match) of the reference's
    LibraryInjector (xenc/injector.py:246-262), restated with X.route_attn / X.forced_read."""
    c = load_case(name)
    base = dict(np.load(G / "attn_record_top2.npz"))  # the inputs every case shares, the forced addressing too
    K = base["K"].astype(np.float32)
    C, N, _ = K.shape
    M = np.arange(N)[None, :] < base["n_valid"][:, None]
    h = base["h"]
    B, T, d_m = h.shape
    q = X.query(X.rms_norm(h.reshape(-1, d_m)), base["W_in"])
    w, _, _ = X.route(q, X.summaries(K, M), float(c["route_temp"]), int(c["top_k"]))
    assert topk_sets(w) == topk_sets(c["w"].reshape(-1, C))
    aw = X.route_attn(q, K, M, w, float(c["read_temp"]), bool(c["read_softmax"]))
    if name.startswith("attn_force"):
        r, aw = X.forced_read(base["force"], K, aw, bool(c["force_norm_match"]))
    else:
        r = (aw.reshape(B * T, C * N) @ K.reshape(C * N, -1)).astype(np.float32)
    assert rel_err(aw[T - 1], c["last_attn"]) < 1e-5  # batch row 0, last position
    assert rel_err(r, c["r"].reshape(B * T, -1)) < 1e-5
    assert rel_err(r @ base["W_out"], c["delta"].reshape(B * T, -1)) < 1e-5
