"""D8: question-dependent top-k slot selection inside the read branch (xenc/topk_read.py).

Two slot-aligned harvests of one document: selection keys `sel_K` [C, N, n_kv * hd] (the encoder's attention keys
at a full-attention layer) and the residual Library read by the injector. Once per multi-token forward the
reader's own queries at its selection layer (last prompt position by default) score every valid slot,
    s_slot = pool_h (q_h . k_{h / groups, slot})          (GQA, max over heads by default)
and the k best slots are kept (`last_idx`, sorted by score). Every injection layer then reads only those slots:
    a = softmax(read_temp * K_sel q) (or K_sel q / sqrt(k)),   r = a @ V_sel,   h' = h + gain * g * B r
through the registered interface; single-token (decode) forwards reuse the index set. k >= the number of valid
slots makes the read exactly LibraryInjector's.

Scoring (xencb_select_scores), the top-k (xencb_select_topk) and the gathered read (xencb_topk_read) are CUDA
kernels; the selection pre-pass that produces the queries runs the reader itself up to the selection layer,
as the reference does (xenc/topk_read.py:300-373).
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import ops
from .depth import decoder_layers, key_for, rho_layer_map
from .injector import LibraryInjector, _on
from .library import Library
from .selector import LayerSelector


# ------------------------------------------------------------------------------------------------ geometry
def attn_geometry(att) -> dict:
    """{hd, n_kv, groups, n_q, gated} of an attention module with q_proj / k_proj (xenc/topk_read.py:40-50)."""
    hd = int(getattr(att, "head_dim"))
    n_kv = att.k_proj.out_features // hd
    groups = int(getattr(att, "num_key_value_groups", 1))
    n_q = n_kv * groups
    gated = att.q_proj.out_features == 2 * n_q * hd
    if not gated and att.q_proj.out_features != n_q * hd:
        raise ValueError(f"q_proj out {att.q_proj.out_features} inconsistent with {n_q} heads x {hd}")
    return {"hd": hd, "n_kv": n_kv, "groups": groups, "n_q": n_q, "gated": gated}


def reader_queries(att, x: torch.Tensor, geo: dict) -> torch.Tensor:
    """The attention module's own pre-RoPE queries (after q_norm when it has one) -> [B, n_q, T, hd]
    (xenc/topk_read.py:53-63; a gated q_proj carries [query | gate] per head)."""
    B, T, _ = x.shape
    hd = geo["hd"]
    qg = att.q_proj(x)
    if geo["gated"]:
        q = qg.view(B, T, -1, 2 * hd)[..., :hd]
    else:
        q = qg.view(B, T, -1, hd)
    if hasattr(att, "q_norm"):
        q = att.q_norm(q)
    return q.transpose(1, 2)


class _StopSelect(Exception):
    pass


def _attn_module(block):
    att = getattr(block, "self_attn", None)
    return att if att is not None and hasattr(att, "k_proj") and hasattr(att, "v_proj") else None


def attn_layer_map(model, depths) -> dict:
    """depth -> the first full-attention layer at or after rho_layer_map(depth), else the last one before it
    (xenc/depth_skill.py:130-141)."""
    blocks = decoder_layers(model)
    full = [i for i, b in enumerate(blocks) if _attn_module(b) is not None]
    if not full:
        raise ValueError("the model has no self-attention module with k_proj / v_proj")
    out = {}
    for rho, li in rho_layer_map(model, depths).items():
        after = [j for j in full if j >= li]
        out[rho] = after[0] if after else full[-1]
    return out


def sel_layer_for(model, sel_rho: float) -> int:
    return int(attn_layer_map(model, [float(sel_rho)])[float(sel_rho)])


def load_sel_kmap(path: str, sel_rho: float) -> dict:
    """A fitted key map {"W": [d_dst, d_src], "b": [d_dst]} at sel_rho (xenc/topk_read.py:168-172)."""
    blob = torch.load(path, map_location="cpu", weights_only=False)
    e = blob["maps"][key_for(blob["maps"], sel_rho)]
    return {"W": e["Wk"].float(), "b": e["bk"].float()}


# ------------------------------------------------------------------------------------------------ library
class TopKLibrary(Library):
    """A residual Library plus `sel_K` [C, N, d_k]: the slot-aligned attention keys used for selection."""

    sel_K: torch.Tensor

    def subset(self, idx) -> "TopKLibrary":
        new = super().subset(idx)
        idx = [int(i) for i in (idx if hasattr(idx, "__iter__") else [idx])]
        n = next(iter(new.K.values())).shape[1]
        new.__class__ = TopKLibrary
        new.sel_K = self.sel_K.index_select(0, torch.tensor(idx, device=self.sel_K.device))[:, :n].clone()
        return new

    def to(self, device=None, dtype=None) -> "TopKLibrary":
        super().to(device=device, dtype=dtype)
        self.sel_K = self.sel_K.to(device=device, dtype=dtype)
        return self


def attach_sel_keys(lib: Library, attn_cache: dict, sel_rho: float) -> TopKLibrary:
    """Turn `lib` (in place) into a TopKLibrary whose sel_K holds the attention cache's keys at sel_rho, padded to
    lib's [C, N] (xenc/topk_read.py:93-113). ValueError when the two harvests are not slot-aligned."""
    chunks = attn_cache["chunks"]
    C, N = next(iter(lib.mask.values())).shape
    if len(chunks) != C:
        raise ValueError(f"attn cache has {len(chunks)} chunks, residual library {C}")
    rows = [c["K"][key_for(c["K"], sel_rho)] for c in chunks]
    n_lib = next(iter(lib.mask.values())).sum(-1).tolist()
    for c, r in enumerate(rows):
        if r.shape[0] != int(n_lib[c]):
            raise ValueError(f"chunk {c}: attn cache {r.shape[0]} slots vs residual {int(n_lib[c])} (not aligned)")
    d_k = rows[0].shape[-1]
    dev = next(iter(lib.K.values())).device
    S = torch.zeros(C, N, d_k, dtype=torch.float32, device=dev)
    for c, r in enumerate(rows):
        S[c, : r.shape[0]] = r.to(device=dev, dtype=torch.float32)
    lib.__class__ = TopKLibrary
    lib.sel_K = S
    return lib


# ------------------------------------------------------------------------------------------------ selector
class TopKSelector:
    """Captures the reader's queries at `sel_layer` and scores them against the loaded selection keys
    (xenc/topk_read.py:176-255). keys [S, n_kv, hd] float32 (flat over C * N; invalid slots masked);
    last_idx [B, k] int64 sorted by score; last_scores [B, S] (invalid = -inf)."""

    def __init__(self, model, sel_layer: int, k: int = 64, pool: str = "max", query: str = "last",
                 kmap: Optional[dict] = None):
        blocks = decoder_layers(model)
        att = getattr(blocks[sel_layer], "self_attn", None)
        if att is None or not hasattr(att, "q_proj"):
            raise ValueError(f"selection layer {sel_layer} has no softmax self-attention with q_proj")
        if pool not in ("max", "mean"):
            raise ValueError(f"unknown selection pool {pool}")
        if query not in ("last", "all_max", "all_mean"):
            raise ValueError(f"unknown selection query {query}")
        self.model, self.sel_layer, self.att = model, int(sel_layer), att
        self.geo = attn_geometry(att)
        self.k, self.pool, self.query = int(k), pool, query
        self.kmap = kmap
        self.keys: Optional[torch.Tensor] = None      # [S, n_kv, hd]
        self.valid: Optional[torch.Tensor] = None     # [S] bool
        self.pos: int = -1
        self.last_idx: Optional[torch.Tensor] = None  # [B, k] int64
        self.last_scores: Optional[torch.Tensor] = None
        self.last_head_scores: Optional[torch.Tensor] = None
        self.keep_heads = False
        self.armed = False
        self._idx32: Optional[torch.Tensor] = None    # the index set as the read kernel takes it
        self._grid: Optional[tuple] = None            # (C, N) of the slot grid
        self._dev_keys: Optional[torch.Tensor] = None
        self._n_valid: Optional[torch.Tensor] = None
        self._n_valid_total = 0

    # ---- keys
    def set_keys(self, sel_K: torch.Tensor, valid: torch.Tensor) -> None:
        """sel_K [C, N, d_k] slot-aligned with valid [C, N] (rows 0..n_c-1 of each chunk)."""
        C, N = valid.shape
        K = sel_K.reshape(-1, sel_K.shape[-1]).float()
        if self.kmap is not None:
            K = K @ self.kmap["W"].to(K).T + self.kmap["b"].to(K)
        g = self.geo
        if K.shape[-1] != g["n_kv"] * g["hd"]:
            raise ValueError(f"selection keys d={K.shape[-1]} != reader KV dim {g['n_kv'] * g['hd']} "
                             "(cross-model selection needs a key map)")
        self.keys = K.reshape(-1, g["n_kv"], g["hd"])
        self.valid = valid.reshape(-1).bool()
        nv = valid.sum(-1).to(torch.int32)
        prefix = torch.arange(N, device=valid.device).view(1, N) < nv.view(C, 1).to(valid.device)
        if not torch.equal(prefix, valid.bool()):
            raise ValueError("selection needs each chunk's valid slots to be its first rows (a Library mask)")
        self._grid = (C, N)
        self._n_valid = nv.view(1, C)
        self._n_valid_total = int(nv.sum())
        self._dev_keys = None
        self._idx32 = None

    def _device_keys(self, dev: torch.device):
        if self._dev_keys is None or self._dev_keys.device != dev:
            K = self.keys.to(dev)
            h = K.half()
            # float16 keys when that is exact (attention caches store float16 rows), else float32
            self._dev_keys = (h if torch.equal(h.float(), K) else K).unsqueeze(0).contiguous()
            self._n_valid = self._n_valid.to(dev)
        return self._dev_keys, self._n_valid

    def clear(self) -> None:
        self.keys = self.valid = self.last_idx = self.last_scores = self.last_head_scores = None
        self._idx32 = self._dev_keys = None

    @property
    def n_valid(self) -> int:
        return self._n_valid_total if self.valid is not None else 0

    # ---- scoring
    def head_scores(self, q: torch.Tensor) -> torch.Tensor:
        """q [B, n_q, T, hd] -> per-head scores [B, n_q, T, S] (a diagnostic: the selection itself runs the
        pooled kernel)."""
        g = self.geo
        K = _on(self.keys, q)
        B, _, T, hd = q.shape
        qh = q.float().reshape(B, g["n_kv"], g["groups"], T, hd)
        return torch.einsum("bkgtd,skd->bkgts", qh, K).reshape(B, g["n_q"], T, -1)

    def pool_scores(self, s: torch.Tensor, query: Optional[str] = None, pool: Optional[str] = None) -> torch.Tensor:
        """[B, n_q, T, S] -> [B, S]: positions per `query`, heads per `pool` (for per-head diagnostics)."""
        query, pool = query or self.query, pool or self.pool
        if query == "last":
            s = s[:, :, -1]
        elif query == "all_max":
            s = s.amax(2)
        elif query == "all_mean":
            s = s.mean(2)
        else:
            raise ValueError(f"unknown selection query {query}")
        s = s.amax(1) if pool == "max" else s.mean(1)
        return s.masked_fill(~_on(self.valid, s).unsqueeze(0), float("-inf"))

    def select_from_input(self, x: torch.Tensor) -> torch.Tensor:
        """x = the input of the selection layer's attention [B, T, d] -> last_idx [B, k]."""
        if self.keys is None:
            raise RuntimeError("TopKSelector: no selection keys loaded")
        T = x.shape[1]
        pos = self.pos if self.pos >= 0 else T + self.pos
        q = reader_queries(self.att, x[:, : pos + 1], self.geo)       # [B, n_q, pos+1, hd]
        if self.keep_heads:
            self.last_head_scores = self.head_scores(q).detach()
        if self.query == "last":
            q = q[:, :, -1:]
        dev = q.device
        keys, nv = self._device_keys(dev)
        C, N = self._grid
        qk = q.detach().float().transpose(1, 2).contiguous()          # [B, T', n_q, hd]
        sc = ops.select_scores(qk, keys, nv, page_rows=N, rows_per_lib=qk.shape[0],
                               query_pool="mean" if self.query == "all_mean" else "max", head_pool=self.pool)
        k = min(self.k, self.n_valid)
        idx, _ = ops.select_topk(sc, k)
        self.last_scores = sc
        self._idx32 = idx
        self.last_idx = idx.long()
        return self.last_idx

    # ---- stats
    def gold_hit(self, gold_flat: torch.Tensor, ks=None) -> dict:
        """gold_flat [C * N] bool -> {n_valid, n_gold, best_rank, best_rank_frac, k: {hit, n_gold_sel, chance_any,
        chance_frac}} for batch row 0 (xenc/topk_read.py:257-283); {} when no valid slot is gold."""
        sc = self.last_scores[0].float().cpu()
        v = self.valid.cpu()[: sc.numel()]
        gold = gold_flat.reshape(-1).bool().cpu()[: sc.numel()] & v
        n, ng = int(v.sum()), int(gold.sum())
        if ng == 0:
            return {}
        order = torch.sort(sc, descending=True, stable=True).indices
        rank = torch.empty_like(order)
        rank[order] = torch.arange(order.numel())
        best = int(rank[gold].min())
        out = {"n_valid": n, "n_gold": ng, "best_rank": best, "best_rank_frac": best / max(n - 1, 1)}
        for k in (ks or [self.k]):
            k = min(int(k), n)
            hits = int(gold[order[:k]].sum())
            # P(a random k-subset of the n valid slots holds >= 1 of the ng gold ones) = 1 - C(n-ng, k) / C(n, k)
            if n - ng >= k:
                log_p = (math.lgamma(n - ng + 1) - math.lgamma(n - ng - k + 1)
                         - math.lgamma(n + 1) + math.lgamma(n - k + 1))
                chance = 1.0 - math.exp(log_p)
            else:
                chance = 1.0
            out[k] = {"hit": float(hits > 0), "n_gold_sel": hits, "chance_any": chance, "chance_frac": k * ng / n}
        return out


# ------------------------------------------------------------------------------------------------ injector
class TopKLibraryInjector(LibraryInjector):
    """LibraryInjector whose read is restricted to the selector's top-k slots (xenc/topk_read.py:288-413)."""

    def __init__(self, model, interface, selector: TopKSelector, read_softmax: bool = True, read_temp: float = 12.0,
                 route_temp: float = 10.0, top_k: int = 0, layer_selector=None, read_fp32: bool = True,
                 slot_dtype="auto", cuda_graphs: bool = True):
        self.tk = selector
        self._selecting = False
        self._sel_this_forward = False
        self.sel_pos = -1              # prompt position whose query selects (training: -(m + 1))
        self.n_select_passes = 0
        super().__init__(model, interface, read_softmax=read_softmax, read_temp=read_temp, route_temp=route_temp,
                         top_k=top_k, selector=layer_selector, read_fp32=read_fp32, slot_dtype=slot_dtype,
                         cuda_graphs=cuda_graphs)

    @property
    def last_idx(self):
        return self.tk.last_idx

    def _active(self) -> bool:
        return (not self._selecting) and super()._active()

    # ---- load / unload
    def load_library(self, lib) -> None:
        super().load_library(lib)
        if getattr(lib, "sel_K", None) is None:
            raise ValueError("TopKLibraryInjector needs a TopKLibrary (residual library + sel_K attention keys)")
        first = self.itf.inject_layers[0]
        self.tk.set_keys(lib.sel_K, lib.mask[first])
        self.tk.last_idx = None

    def unload(self) -> None:
        super().unload()
        self.tk.clear()

    @property
    def full_read(self) -> bool:
        return self.tk.k >= self.tk.n_valid

    # ---- hooks
    def _attach(self) -> None:
        super()._attach()
        blocks = decoder_layers(self.model)

        def att_pre(mod, args, kwargs):
            if self._selecting:
                x = kwargs["hidden_states"] if "hidden_states" in kwargs else args[0]
                self.tk.pos = self.sel_pos
                with torch.no_grad():
                    self.tk.select_from_input(x)
                raise _StopSelect

        self._handles.append(self.tk.att.register_forward_pre_hook(att_pre, with_kwargs=True))

        def top_pre(mod, args, kwargs):  # every model(...) call: prefill, decode, training forwards
            if self._selecting or not self._active():
                return None
            x = kwargs.get("input_ids")
            if x is None:
                x = kwargs.get("inputs_embeds")
            if x is None and args:
                x = args[0]
            self._sel_this_forward = True
            if x is None or self.full_read:
                return None
            if x.shape[1] == 1 and self.tk.last_idx is not None:
                return None  # decode step: reuse the selected set
            kw = dict(kwargs)
            if "past_key_values" in kw:
                kw["past_key_values"] = None
            if "use_cache" in kw or hasattr(self.model, "generation_config"):
                kw["use_cache"] = False
            kw.pop("logits_to_keep", None)
            self._run_select(lambda: mod(*args, **kw))
            return None

        self._handles.append(self.model.register_forward_pre_hook(top_pre, with_kwargs=True))
        fake = not hasattr(self.model, "generate")

        def block0_pre(mod, args):  # models whose logits() bypasses model.__call__
            if self._selecting or not self._active():
                return None
            if not fake:
                self._sel_this_forward = False
                return None
            if self._sel_this_forward:
                self._sel_this_forward = False
                return None
            if self.full_read:
                return None
            x = args[0]
            if x.shape[1] == 1 and self.tk.last_idx is not None:
                return None
            self._run_select(lambda: self.model.forward(x))
            return None

        self._handles.append(blocks[0].register_forward_pre_hook(block0_pre))

    def _run_select(self, fn) -> None:
        self._selecting = True
        self.n_select_passes += 1
        try:
            with torch.no_grad():
                fn()
        except _StopSelect:
            pass
        finally:
            self._selecting = False
        if self.tk.last_idx is None:
            raise RuntimeError("D8 selection pass did not reach the selection layer")

    # ---- branch
    def _run_lib(self, h: torch.Tensor, li: int, inject: bool, sel: Optional[LayerSelector]):
        if self.lib is None or self.full_read:
            return super()._run_lib(h, li, inject, sel)
        if self.force_attn is not None or self.training_attn:
            raise NotImplementedError("force_attn / training_attn are not served by the xencb top-k read")
        if self.tk._idx32 is None:
            raise RuntimeError("TopKLibraryInjector: no selection for this forward (the selection pass did not run)")
        self._check_forward_only(h)
        if sel is not None and any(p.requires_grad for p in sel.parameters()):
            raise RuntimeError("the xencb Library read is forward-only; freeze the LayerSelector or use no_grad")
        lead, d_m = h.shape[:-1], h.shape[-1]
        h2 = h.reshape(-1, d_m)
        pages = self._pages(li, h)
        idx = self.tk._idx32
        B = h.shape[0] if h.dim() >= 3 else 1
        if idx.shape[0] != B:  # one selection serves every batch row
            idx = idx[:1]
        idx = _on(idx, h2)
        if self._fast_interface():
            q, g, log_gain, _ = self._query(h2, li)
        else:
            hn = ops.rms_norm(h2)
            q = self.itf.query(hn.view(*lead, -1)).reshape(-1, self.itf.d_s).float().contiguous()
        sel_col, log_alpha = None, 0.0
        if sel is not None:
            sel.weights_for(h, li)
            sel_col = sel._w[..., sel.pos[li]].reshape(-1).float().contiguous()
            log_alpha = _on(sel.log_alpha.detach().reshape(1), h2).float()
        r, attn = ops.topk_read(q, pages, idx, read_temp=self.read_temp, read_softmax=self.read_softmax,
                                want_attn=self.record_attn)
        if self.record_attn:
            # read attention at batch row 0, last position, on the [C, N] grid (zero off the selected set)
            C, N = pages.n_chunks, pages.page_rows
            T = h2.shape[0] // B
            full = torch.zeros(C * N, dtype=torch.float32, device=h2.device)
            full.index_put_((idx[0].long(),), attn[T - 1])
            self.last_attn[li] = full.view(C, N).cpu()
        self.last_route = None
        if not self._fast_interface():
            return self._duck_finish(h, hn, r, 1.0, li, inject, selector=sel)
        return self._finish(h, h2, r, g, 1.0, li, inject, sel_col=sel_col, log_alpha=log_alpha, log_scale=log_gain)


__all__ = ["attn_geometry", "reader_queries", "attn_layer_map", "sel_layer_for", "load_sel_kmap", "TopKLibrary",
           "attach_sel_keys", "TopKSelector", "TopKLibraryInjector"]
