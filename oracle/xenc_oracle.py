"""CPU oracle for the xenc Library read -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain numpy (float32, the reference's arithmetic type), the algorithm of the
reference's Library read path (Rickyzhaoweihan/KV_skill_v2, package `xenc`). It exists to CHECK the CUDA
product path and to serve as the timed CPU baseline. Only `tests/`, `__graft_entry__.smoke()` and
`bench.py` (its `cpu_baseline` leg and `--impl reference`) may import it. The product package
`kv_skill_v2_b200` never imports it and has no CPU fallback.

Pinning. The reference is Python; its own `xenc.library`, `xenc.injector` and `xenc.selector` were run
unchanged (with a minimal stand-in for the un-vendored `deltaskill` package) by
`tests/golden/make_golden.py`, which wrote the fixtures under `tests/golden/`. `tests/test_oracle_golden.py`
checks every function here against them. One piece stays UNPINNED: `rms_norm` lives in the un-vendored
`deltaskill.derive` (called at xenc/injector.py:235 and xenc/selector.py:100); it is restated as
`x * rsqrt(mean(x^2) + 1e-6)` without a weight, the RMS idiom the reference uses itself at
xenc/p5_copy.py:101 and xenc/d13_read.py:179. The golden generator uses the same assumption, so the fixtures
pin everything downstream of `rms_norm`, not `rms_norm` itself.

Conventions: arrays are float32 unless named otherwise; `K` is [C, N, d_s] (tied K = V), `mask` is [C, N]
bool, `S` is [C, d_s]; hidden states are [B, T, d_m] or [R, d_m].
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
EPS = 1e-6  # xenc/library.py:22, xenc/injector.py:197,333, xenc/selector.py:28


# ----------------------------------------------------------------------------------------------- helpers
def l2(x: np.ndarray) -> np.ndarray:
    """x / (||x|| + 1e-6) along the last dim (xenc/library.py:21-22, xenc/injector.py:197)."""
    x = np.asarray(x, dtype=F32)
    n = np.sqrt(np.sum(x * x, axis=-1, keepdims=True, dtype=F32), dtype=F32)
    return (x / (n + F32(EPS))).astype(F32)


def rms_norm(x: np.ndarray, eps: float = EPS) -> np.ndarray:
    """UNPINNED restatement of deltaskill.derive.rms_norm (see module docstring)."""
    x = np.asarray(x, dtype=F32)
    ms = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    return (x * (F32(1.0) / np.sqrt(ms + F32(eps), dtype=F32))).astype(F32)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """Numerically-stable softmax; all -inf rows give NaN exactly as torch.softmax does."""
    x = np.asarray(x, dtype=F32)
    m = np.max(x, axis=axis, keepdims=True)
    with np.errstate(invalid="ignore"):
        e = np.exp(x - m, dtype=F32)
        return (e / np.sum(e, axis=axis, keepdims=True, dtype=F32)).astype(F32)


def topk_indices(x: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest entries along the last dim, ties broken toward the LOWER index.

    torch.topk leaves the order of equal values unspecified; the reference only uses the index SET
    (scattered into a keep-mask, xenc/injector.py:226-227), so lower-index-wins is one valid choice and the
    one the CUDA router implements. Result is sorted by (value desc, index asc)."""
    x = np.asarray(x, dtype=F32)
    order = np.argsort(-x, axis=-1, kind="stable")
    return order[..., :k]


# ----------------------------------------------------------------------------------------------- Library
def build_library(chunk_rows: list, center_mu: np.ndarray | None = None):
    """Pad one depth of C chunks into (K [C,N_max,d_s], mask [C,N_max], S [C,d_s]).

    xenc/library.py:47-67 (padding, mask, optional centering L2(K - mu) on valid rows only) and
    xenc/library.py:69-74 (S = L2(sum of valid rows / max(count,1)))."""
    if not chunk_rows:
        raise ValueError("Library needs at least one chunk")  # xenc/library.py:32-33
    n = [int(r.shape[0]) for r in chunk_rows]
    d = int(chunk_rows[0].shape[-1])
    C, N = len(chunk_rows), max(n)
    K = np.zeros((C, N, d), dtype=F32)
    M = np.zeros((C, N), dtype=bool)
    for c, r in enumerate(chunk_rows):
        K[c, : n[c]] = np.asarray(r, dtype=F32)
        M[c, : n[c]] = True
    if center_mu is not None:
        K = np.where(M[..., None], l2(K - np.asarray(center_mu, dtype=F32)), F32(0)).astype(F32)
    return K, M, summaries(K, M)


def summaries(K: np.ndarray, M: np.ndarray) -> np.ndarray:
    """S[c] = L2(mean of chunk c's valid rows) (xenc/library.py:69-74)."""
    s = np.sum(K * M[..., None].astype(F32), axis=1, dtype=F32)
    cnt = np.maximum(M.sum(1, keepdims=True), 1).astype(F32)
    return l2(s / cnt)


def subset(K: np.ndarray, M: np.ndarray, idx) -> tuple:
    """Chunks `idx`, re-trimmed to their longest valid row count (xenc/library.py:103-123)."""
    idx = [int(i) for i in idx]
    if not idx:
        raise ValueError("empty subset")
    Ms = M[idx]
    n = int(Ms.sum(-1).max())
    Ks = K[idx][:, :n].copy()
    Ms = Ms[:, :n].copy()
    return Ks, Ms, summaries(Ks, Ms)


# ----------------------------------------------------------------------------------------------- interface
def query(hn: np.ndarray, W_in: np.ndarray, b_in: np.ndarray | None = None) -> np.ndarray:
    """q = L2(hn @ W_in (+ b)) -- itf_query for a full-rank A (xenc/injector.py:54-58).
    `W_in` is [d_m, d_s] (so hn @ W_in); a torch nn.Linear weight is its transpose."""
    q = np.asarray(hn, dtype=F32) @ np.asarray(W_in, dtype=F32)
    if b_in is not None:
        q = q + np.asarray(b_in, dtype=F32)
    return l2(q)


def gate(hn: np.ndarray, gate_w: np.ndarray, gate_b: float) -> np.ndarray:
    """sigmoid(hn . gate_w + gate_b[pos]) -> [..., 1] (xenc/injector.py:61-65)."""
    z = np.asarray(hn, dtype=F32) @ np.asarray(gate_w, dtype=F32) + F32(gate_b)
    return (F32(1) / (F32(1) + np.exp(-z, dtype=F32)))[..., None].astype(F32)


# ----------------------------------------------------------------------------------------------- routing
def route(q: np.ndarray, S: np.ndarray, route_temp: float = 10.0, top_k: int = 0):
    """LibraryInjector.route (xenc/injector.py:220-229).

    logit = (q . S_c) * route_temp; if 0 < top_k < C keep the top_k logits (others -inf); softmax over C.
    Returns (w [..., C], logit [..., C], keep-index set [..., k] sorted by (value desc, index asc))."""
    logit = (np.asarray(q, dtype=F32) @ np.asarray(S, dtype=F32).T).astype(F32) * F32(route_temp)
    C = logit.shape[-1]
    if top_k and top_k < C:
        idx = topk_indices(logit, top_k)
        keep = np.zeros(logit.shape, dtype=bool)
        np.put_along_axis(keep, idx, True, axis=-1)
        masked = np.where(keep, logit, F32(-np.inf)).astype(F32)
    else:
        idx = topk_indices(logit, C)
        masked = logit
    return softmax(masked, -1), logit, idx


# ----------------------------------------------------------------------------------------------- read
def read(q: np.ndarray, K: np.ndarray, M: np.ndarray, w: np.ndarray, read_temp: float = 12.0,
         read_softmax: bool = True, V: np.ndarray | None = None) -> np.ndarray:
    """The masked two-level read of LibraryInjector._branch (xenc/injector.py:239-245, 263-265).

    a = q . K (dense over ALL C*N slots, as the reference does); softmax(a * read_temp) within each chunk
    over its valid slots (or linear: a * M / sqrt(n_c)); aw = a * w_c; r = aw @ V with V = K (tied) unless
    the Library has untied values (xenc/injector.py:211-218). q: [R, d_s]; w: [R, C]. Returns r [R, d_s]."""
    q = np.asarray(q, dtype=F32)
    C, N, d = K.shape
    Kf = K.reshape(C * N, d)
    a = (q @ Kf.T).reshape(q.shape[0], C, N).astype(F32)
    if read_softmax:
        a = softmax(np.where(M[None], a * F32(read_temp), F32(-np.inf)), -1)
    else:
        n = np.maximum(M.sum(-1), 1).astype(F32)
        a = (np.where(M[None], a, F32(0)) / np.sqrt(n, dtype=F32)[None, :, None]).astype(F32)
    aw = (a * np.asarray(w, dtype=F32)[..., None]).astype(F32)
    Vf = Kf if V is None else np.asarray(V, dtype=F32).reshape(C * N, d)
    return (aw.reshape(q.shape[0], C * N) @ Vf).astype(F32)


def route_attn(q: np.ndarray, K: np.ndarray, M: np.ndarray, w: np.ndarray, read_temp: float = 12.0,
               read_softmax: bool = True) -> np.ndarray:
    """The route-weighted slot attention aw = a * w of LibraryInjector._branch (xenc/injector.py:239-245):
    [R, C, N]; record_attn keeps aw of the last position of batch row 0 (:259-260)."""
    q = np.asarray(q, dtype=F32)
    C, N, d = K.shape
    a = (q @ K.reshape(C * N, d).T).reshape(q.shape[0], C, N).astype(F32)
    if read_softmax:
        a = softmax(np.where(M[None], a * F32(read_temp), F32(-np.inf)), -1)
    else:
        n = np.maximum(M.sum(-1), 1).astype(F32)
        a = (np.where(M[None], a, F32(0)) / np.sqrt(n, dtype=F32)[None, :, None]).astype(F32)
    return (a * np.asarray(w, dtype=F32)[..., None]).astype(F32)


def forced_read(fa: np.ndarray, K: np.ndarray, aw: np.ndarray | None = None, norm_match: bool = False,
                V: np.ndarray | None = None):
    """force_attn (xenc/injector.py:246-258): the given addressing fa [C, N] replaces aw for every token; with
    force_norm_match it is scaled per token so that ||fa @ K|| = ||aw @ K||. Returns (r [R, d_s], aw_used
    [R, C, N]); R is aw's row count (1 when aw is None)."""
    fa = np.asarray(fa, dtype=F32)
    C, N, d = K.shape
    Kf = K.reshape(C * N, d)
    R = 1 if aw is None else aw.shape[0]
    use = np.broadcast_to(fa, (R, C, N)).astype(F32)
    if norm_match:
        r0 = aw.reshape(R, C * N) @ Kf
        r1 = use.reshape(R, C * N) @ Kf
        scale = np.linalg.norm(r0, axis=-1, keepdims=True) / (np.linalg.norm(r1, axis=-1, keepdims=True) + F32(EPS))
        use = (use * scale.astype(F32)[:, :, None]).astype(F32)
    Vf = Kf if V is None else np.asarray(V, dtype=F32).reshape(C * N, d)
    return (use.reshape(R, C * N) @ Vf).astype(F32), use


def branch(h: np.ndarray, W_in: np.ndarray, W_out: np.ndarray, K: np.ndarray, M: np.ndarray,
           S: np.ndarray, read_temp: float = 12.0, route_temp: float = 10.0, top_k: int = 0,
           read_softmax: bool = True, b_in=None, b_out=None, gate_w=None, gate_b: float = 0.0,
           gain: float = 1.0, gain_scale: float = 1.0, V: np.ndarray | None = None):
    """LibraryInjector._branch without a selector (xenc/injector.py:231-267).

    Interface: q = L2(rms_norm(h) @ W_in + b_in); g = sigmoid(hn.gate_w + gate_b) or 1 when gate_w is None;
    delta = gain_scale * gain * g * (r @ W_out + b_out). h: [R, d_m].
    Returns dict(hn, q, w, idx, r, delta)."""
    hn = rms_norm(h)
    q = query(hn, W_in, b_in)
    w, logit, idx = route(q, S, route_temp, top_k)
    r = read(q, K, M, w, read_temp, read_softmax, V)
    out = r @ np.asarray(W_out, dtype=F32)
    if b_out is not None:
        out = out + np.asarray(b_out, dtype=F32)
    g = gate(hn, gate_w, gate_b) if gate_w is not None else F32(1)
    delta = (F32(gain_scale) * F32(gain) * g * out).astype(F32)
    return {"hn": hn, "q": q, "w": w, "logit": logit, "idx": idx, "r": r.astype(F32), "delta": delta}


# ----------------------------------------------------------------------------------------------- selector
def selector_weights(z: np.ndarray, k: int, straight_through: bool = False) -> np.ndarray:
    """LayerSelector._weights_from_logits, forward value (xenc/selector.py:59-67): top-k of the logits,
    softmax over the kept ones, zeros elsewhere; straight-through forward is uniform 1/k on the kept."""
    z = np.asarray(z, dtype=F32)
    idx = topk_indices(z, k)
    v = np.take_along_axis(z, idx, -1)
    vals = np.full(v.shape, F32(1.0 / k), dtype=F32) if straight_through else softmax(v, -1)
    w = np.zeros_like(z)
    np.put_along_axis(w, idx, vals, axis=-1)
    return w


def selector_logits(hn0: np.ndarray, u_w: np.ndarray, u_b: np.ndarray) -> np.ndarray:
    """z = hn0 @ u.weight.T + u.bias (xenc/selector.py:69-74); u_w is [n_cand, d_m] (nn.Linear layout)."""
    return (np.asarray(hn0, dtype=F32) @ np.asarray(u_w, dtype=F32).T + np.asarray(u_b, dtype=F32)).astype(F32)


def selector_apply(delta: np.ndarray, h: np.ndarray, w_pos: np.ndarray, log_alpha: float) -> np.ndarray:
    """LayerSelector.apply after the weights exist (xenc/selector.py:106-110):
    rel = ||d|| / (||h|| + eps); d = d / (rel + eps) * exp(log_alpha); out = w[..., pos] * d."""
    d = np.asarray(delta, dtype=F32)
    hf = np.asarray(h, dtype=F32)
    rel = np.sqrt(np.sum(d * d, -1, keepdims=True, dtype=F32)) / (
        np.sqrt(np.sum(hf * hf, -1, keepdims=True, dtype=F32)) + F32(EPS))
    d = d / (rel + F32(EPS)) * np.exp(F32(log_alpha), dtype=F32)
    return (np.asarray(w_pos, dtype=F32)[..., None] * d).astype(F32)


def rel_norm(delta: np.ndarray, h: np.ndarray) -> np.ndarray:
    """Per-token ||delta|| / (||h|| + 1e-6), the hook's mag term before `.mean()` (xenc/injector.py:192-193)."""
    d = np.asarray(delta, dtype=F32)
    hf = np.asarray(h, dtype=F32)
    return (np.sqrt(np.sum(d * d, -1, dtype=F32)) / (np.sqrt(np.sum(hf * hf, -1, dtype=F32)) + F32(EPS))).astype(F32)


# ----------------------------------------------------------------------------------------------- shards
def shard_partials(q: np.ndarray, K: np.ndarray, M: np.ndarray, S: np.ndarray, route_temp: float,
                   read_temp: float, read_softmax: bool = True):
    """Per-shard routing-LSE triple for a dense (top_k = 0) read over a chunk shard.

    With w = softmax_c(l_c) over ALL chunks, r = sum_c w_c r_c splits over shards as
    (Mx = max_c l_c, Z = sum_c e^(l_c - Mx), A = sum_c e^(l_c - Mx) r_c); this is the same two-level
    formula as xenc/injector.py:239-265 regrouped by chunk, and merge_shards() recombines exactly."""
    logit = (np.asarray(q, dtype=F32) @ S.T).astype(F32) * F32(route_temp)
    Mx = logit.max(-1)
    e = np.exp(logit - Mx[:, None], dtype=F32)
    Z = e.sum(-1, dtype=F32)
    # read() with weights e (unnormalised) sums e_c * r_c over the shard's chunks in one pass
    A = read(q, K, M, e, read_temp, read_softmax)
    return Mx.astype(F32), Z.astype(F32), A.astype(F32)


def merge_shards(parts: list) -> np.ndarray:
    """Combine per-shard (Mx, Z, A) triples: r = sum_g e^(Mx_g - M) A_g / sum_g e^(Mx_g - M) Z_g."""
    Mx = np.max(np.stack([p[0] for p in parts]), 0)
    num = sum(np.exp(p[0] - Mx, dtype=F32)[:, None] * p[2] for p in parts)
    den = sum(np.exp(p[0] - Mx, dtype=F32) * p[1] for p in parts)
    return (num / den[:, None]).astype(F32)


__all__ = ["l2", "rms_norm", "softmax", "topk_indices", "build_library", "summaries", "subset", "query",
           "gate", "route", "read", "route_attn", "forced_read", "branch", "selector_weights", "selector_logits", "selector_apply",
           "rel_norm", "shard_partials", "merge_shards"]


# ----------------------------------------------------------------------------------------------- D8 top-k read
def topk_select_scores(q: np.ndarray, keys: np.ndarray, valid: np.ndarray, query: str = "last",
                       pool: str = "max") -> np.ndarray:
    """TopKSelector.head_scores + pool_scores (xenc/topk_read.py:215-239).

    q [B, n_q, T, hd]; keys [S, n_kv, hd]; valid [S] bool. Query head h scores KV head h // groups (GQA);
    positions pooled per `query` (last | all_max | all_mean), heads per `pool` (max | mean); invalid = -inf."""
    q = np.asarray(q, F32)
    B, n_q, T, hd = q.shape
    keys = np.asarray(keys, F32)
    n_kv = keys.shape[1]
    groups = n_q // n_kv
    qh = q.reshape(B, n_kv, groups, T, hd)
    s = np.einsum("bkgtd,skd->bkgts", qh, keys).reshape(B, n_q, T, -1).astype(F32)
    if query == "last":
        s = s[:, :, -1]
    elif query == "all_max":
        s = s.max(2)
    elif query == "all_mean":
        s = s.mean(2, dtype=F32)
    else:
        raise ValueError(f"unknown selection query {query}")
    s = s.max(1) if pool == "max" else s.mean(1, dtype=F32)
    return np.where(np.asarray(valid, bool)[None, :], s, F32(-np.inf)).astype(F32)


def topk_select(scores: np.ndarray, k: int) -> np.ndarray:
    """sc.topk(k).indices (xenc/topk_read.py:254): per row the k largest, sorted descending; ties (which
    torch.topk leaves unordered) go to the lower slot here. -> [B, k] int64."""
    scores = np.asarray(scores, F32)
    order = np.lexsort((np.arange(scores.shape[-1])[None, :].repeat(scores.shape[0], 0), -scores), axis=-1)
    return order[:, :k].astype(np.int64)


def topk_read(q: np.ndarray, Kf: np.ndarray, idx: np.ndarray, read_temp: float = 12.0,
              read_softmax: bool = True, Vf: np.ndarray | None = None):
    """The read of TopKLibraryInjector._branch (xenc/topk_read.py:392-405, 412).

    q [B, T, d_s]; Kf [C*N, d_s] (the padded Library flattened); idx [B, k] (or [1, k], broadcast over B).
    a = q . Kf[idx]; softmax(a * read_temp) over k, or a / sqrt(k); r = a @ Vf[idx]. -> (r [B, T, d_s], a)."""
    q = np.asarray(q, F32)
    Kf = np.asarray(Kf, F32)
    Vf = Kf if Vf is None else np.asarray(Vf, F32)
    idx = np.asarray(idx)
    if idx.shape[0] != q.shape[0]:
        idx = np.repeat(idx[:1], q.shape[0], 0)
    Ks, Vs = Kf[idx], Vf[idx]                                   # [B, k, d_s]
    a = np.einsum("btd,bkd->btk", q, Ks).astype(F32)
    if read_softmax:
        a = softmax(a * F32(read_temp), -1)
    else:
        a = (a / F32(idx.shape[-1] ** 0.5)).astype(F32)
    return np.einsum("btk,bkd->btd", a, Vs).astype(F32), a
