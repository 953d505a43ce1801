"""Library: a stack of C chunk operators keyed by READER layer, and its device page layout.

Library mirrors xenc/library.py of the reference:
    K[li]    [C, N_max, d_s]  zero-padded chunk slots (tied: V is K unless the chunks are untied)
    mask[li] [C, N_max] bool  valid slots
    S[li]    [C, d_s]         L2(mean of the chunk's valid rows), the routing keys
built from rho-keyed chunks (cache dicts or KVSkill objects) with `reader_layers[i]` serving
`sorted(depths)[i]` (xenc/library.py:26-67), with .to / .subset / .from_doc_cache (:93-136).

The read kernels take a different, paged view (ops.Pages): one slot pool per layer plus a page table,
the valid-row counts and float32 summaries. Library.pages(li, device) builds it once per layer and device;
PagedLibrary holds one such view per layer for SEVERAL documents (one Library per batch row), the layout
batched decode reads.
"""

from __future__ import annotations

from typing import Optional

import torch

from .depth import key_for, rho_layer_map
from .ops import Pages


def _l2(x: torch.Tensor) -> torch.Tensor:
    return x / (x.norm(dim=-1, keepdim=True) + 1e-6)


def _rows_of(chunk, rho, which="K"):
    m = getattr(chunk, which, None) if not isinstance(chunk, dict) else chunk.get(which)
    if m is None:
        return None
    return m[key_for(m, rho)]


class Library:
    def __init__(self, chunks: list, reader_layers: list, depths, device="cpu", dtype=torch.float32,
                 meta: list | None = None, center: dict | None = None):
        if not chunks:
            raise ValueError("Library needs at least one chunk")
        depths = sorted(float(r) for r in depths)
        if len(reader_layers) != len(depths):
            raise ValueError(f"{len(reader_layers)} reader layers for {len(depths)} depths")
        self.depths = depths
        self.reader_layers = [int(li) for li in reader_layers]
        self.rho_of = dict(zip(self.reader_layers, depths))
        Ks = [c.K if not isinstance(c, dict) else c["K"] for c in chunks]
        Vs = [getattr(c, "V", None) if not isinstance(c, dict) else c.get("V") for c in chunks]
        untied = any(v is not None and v is not k for v, k in zip(Vs, Ks))
        if meta is None:
            meta = [dict(getattr(c, "meta", None) or {}) if not isinstance(c, dict)
                    else {k: v for k, v in c.items() if k not in ("K", "V")} for c in chunks]
        self.chunk_meta = meta
        self.K, self.mask, self.S = {}, {}, {}
        self.V = {} if untied else None
        self.center = center
        for li, rho in self.rho_of.items():
            rows = [k[key_for(k, rho)] for k in Ks]
            lens = [int(r.shape[0]) for r in rows]
            C, N, d = len(rows), max(lens), int(rows[0].shape[-1])
            K = torch.zeros(C, N, d, dtype=dtype, device=device)
            M = torch.zeros(C, N, dtype=torch.bool, device=device)
            for c, r in enumerate(rows):
                K[c, : lens[c]] = r.to(device=device, dtype=dtype)
                M[c, : lens[c]] = True
            if center is not None:
                try:
                    mu = center[key_for(center, rho)].to(device=device, dtype=dtype)
                except KeyError:
                    mu = None
                if mu is not None:
                    K = torch.where(M.unsqueeze(-1), _l2(K - mu), torch.zeros_like(K))
            self.K[li], self.mask[li] = K, M
            if untied:
                Vt = torch.zeros_like(K)
                for c, (v, k) in enumerate(zip(Vs, Ks)):
                    src = v if v is not None else k
                    Vt[c, : lens[c]] = src[key_for(src, rho)].to(device=device, dtype=dtype)
                self.V[li] = Vt
        self._summaries()
        self._page_cache: dict = {}

    def _summaries(self) -> None:
        self.S = {}
        for li, K in self.K.items():
            M = self.mask[li]
            cnt = M.sum(1, keepdim=True).clamp_min(1).to(K.dtype)
            self.S[li] = _l2((K * M.unsqueeze(-1).to(K.dtype)).sum(1) / cnt)

    # ------------------------------------------------------------------ properties
    @property
    def n_chunks(self) -> int:
        return next(iter(self.K.values())).shape[0]

    @property
    def d_s(self) -> int:
        return next(iter(self.K.values())).shape[-1]

    @property
    def layers(self) -> list:
        return sorted(self.K)

    def n_valid(self, li: int) -> torch.Tensor:
        return self.mask[li].sum(-1)

    # ------------------------------------------------------------------ ops
    def to(self, device=None, dtype=None) -> "Library":
        """In-place move / cast (mask stays bool); returns self."""
        for li in list(self.K):
            self.K[li] = self.K[li].to(device=device, dtype=dtype)
            self.S[li] = self.S[li].to(device=device, dtype=dtype)
            self.mask[li] = self.mask[li].to(device=device)
            if self.V is not None:
                self.V[li] = self.V[li].to(device=device, dtype=dtype)
        self._page_cache = {}
        return self

    def subset(self, idx) -> "Library":
        """Library of chunks `idx`, re-trimmed to its longest chunk (identical to building from those chunks)."""
        idx = [int(i) for i in (idx if hasattr(idx, "__iter__") else [idx])]
        if not idx:
            raise ValueError("empty subset")
        new = object.__new__(Library)
        new.depths, new.reader_layers, new.rho_of = self.depths, self.reader_layers, dict(self.rho_of)
        new.chunk_meta = [self.chunk_meta[i] for i in idx]
        new.center = self.center
        new.K, new.mask = {}, {}
        new.V = {} if self.V is not None else None
        sel = torch.tensor(idx, device=next(iter(self.K.values())).device)
        for li in self.K:
            M = self.mask[li].index_select(0, sel)
            n = int(M.sum(-1).max())
            new.mask[li] = M[:, :n].clone()
            new.K[li] = self.K[li].index_select(0, sel)[:, :n].clone()
            if new.V is not None:
                new.V[li] = self.V[li].index_select(0, sel)[:, :n].clone()
        new._summaries()
        new._page_cache = {}
        return new

    @staticmethod
    def from_doc_cache(cache: dict, reader_model, depths=None, device=None, dtype=torch.float32,
                       center: dict | None = None) -> "Library":
        depths = sorted(float(r) for r in (depths or cache["depths"]))
        rmap = rho_layer_map(reader_model, depths)
        if device is None:
            device = reader_model.device if hasattr(reader_model, "device") else "cpu"
        meta = [{"doc_id": cache.get("doc_id", ""), "start": int(c.get("start", 0)),
                 "n_tokens": int(c.get("n_tokens", 0)), "encoder": cache.get("encoder", "")}
                for c in cache["chunks"]]
        return Library(cache["chunks"], [rmap[r] for r in depths], depths, device, dtype, meta=meta, center=center)

    # ------------------------------------------------------------------ device view
    def pages(self, li: int, device, slot_dtype="auto", require_nonempty: bool = True) -> Pages:
        """The paged view of layer `li` on `device` (built once and cached).

        slot_dtype "auto" stores float32 rows as float16 slots, exactly for Libraries built from doc caches
        (float16 rows), rounded otherwise (centred Libraries: L2(K - mu) is not float16-exact) when the values fit
        float16's range; the summary keys S are kept from the float32 rows, so routing is unchanged, and the read
        of rounded rows stays within the path's 2e-3 output bound (each element moves by at most 2^-11 of itself).
        This keeps every float32 Library on the tensor-core read; slot_dtype=torch.float32 keeps float32 slots
        (the CUDA-core read). An empty chunk is rejected when `require_nonempty`: the reference's softmax read
        returns NaN for such a Library."""
        device = torch.device(device)
        key = (li, str(device), str(slot_dtype))
        hit = self._page_cache.get(key)
        if hit is not None:
            return hit
        K = self.K[li]
        nv = self.mask[li].sum(-1).to(torch.int32)
        if require_nonempty and bool((nv == 0).any()):
            bad = torch.nonzero(nv == 0).flatten().tolist()
            raise ValueError(f"Library layer {li}: chunks {bad} have no valid slot (the softmax read is NaN)")
        vslots = None
        if self.V is None:
            slots = _slot_storage(K.to(device), slot_dtype)
        else:
            slots, vslots = _untied_storage(K.to(device), self.V[li].to(device), slot_dtype)
        C = K.shape[0]
        view = Pages(slots=slots.contiguous(), page_of=torch.arange(C, dtype=torch.int32, device=device).view(1, C),
                     n_valid=nv.to(device).view(1, C),
                     S=self.S[li].to(device=device, dtype=torch.float32).view(1, C, -1).contiguous(),
                     vslots=None if vslots is None else vslots.contiguous())
        self._page_cache[key] = view
        return view


def _slot_storage(K: torch.Tensor, slot_dtype) -> torch.Tensor:
    if slot_dtype == "auto":
        if K.dtype == torch.float32:
            if bool(torch.isfinite(K).all()) and float(K.abs().max()) <= 65504.0:
                return K.to(torch.float16)
            return K
        if K.dtype in (torch.float16, torch.bfloat16):
            return K
        return K.to(torch.float32)
    return K.to(slot_dtype)


def _untied_storage(K: torch.Tensor, V: torch.Tensor, slot_dtype):
    """K and V pools of one dtype for an untied read, which runs on the tensor cores: float16 (or bfloat16 when
    asked for, or when K is bfloat16). "auto" rounds float32 rows to float16, which is exact for rows harvested
    into float16 doc caches."""
    if slot_dtype == "auto":
        dt = torch.bfloat16 if K.dtype == torch.bfloat16 else torch.float16
    else:
        dt = slot_dtype
    if dt not in (torch.float16, torch.bfloat16):
        raise NotImplementedError(f"untied Library values are read from float16 / bfloat16 slots, not {dt}")
    return K.to(dt), V.to(dt)


class PagedLibrary:
    """One Library per batch row, every layer held as one slot pool + page table on one device.

    pages[li] is an ops.Pages with n_lib Libraries; batch row b of a [B, T, d_m] hidden state reads
    Library b (rows_per_lib = T). Build with from_libraries(libs) or, for slots already on the device,
    from_pool(...) which computes the summary keys with the device kernel."""

    def __init__(self, pages: dict, depths: Optional[list] = None):
        if not pages:
            raise ValueError("PagedLibrary needs at least one layer")
        self._pages = dict(pages)
        first = next(iter(self._pages.values()))
        for li, p in self._pages.items():
            if p.n_lib != first.n_lib or p.d_s != first.d_s:
                raise ValueError("every layer of a PagedLibrary must hold the same Libraries")
        self.depths = depths

    @property
    def layers(self) -> list:
        return sorted(self._pages)

    @property
    def n_lib(self) -> int:
        return next(iter(self._pages.values())).n_lib

    @property
    def n_chunks(self) -> int:
        return next(iter(self._pages.values())).n_chunks

    @property
    def d_s(self) -> int:
        return next(iter(self._pages.values())).d_s

    @property
    def K(self) -> dict:
        """Layer -> slot pool (for the `li in lib.K` membership checks of the injectors)."""
        return {li: p.slots for li, p in self._pages.items()}

    @property
    def V(self) -> Optional[dict]:
        """Layer -> value pool when the Libraries are untied, else None (V = K)."""
        if all(p.vslots is None for p in self._pages.values()):
            return None
        return {li: p.vslots for li, p in self._pages.items()}

    def pages(self, li: int, device=None, slot_dtype="auto", require_nonempty: bool = True) -> Pages:
        p = self._pages[li]
        if device is not None and torch.device(device) != p.device:
            p = Pages(slots=p.slots.to(device), page_of=p.page_of.to(device), n_valid=p.n_valid.to(device),
                      S=p.S.to(device), n_chunks_of=None if p.n_chunks_of is None else p.n_chunks_of.to(device),
                      vslots=None if p.vslots is None else p.vslots.to(device))
            self._pages[li] = p
        return p

    @staticmethod
    def from_libraries(libs: list, device, slot_dtype=torch.float16) -> "PagedLibrary":
        """Stack Libraries with the same layers and d_s; library b serves batch row b. When any Library is
        untied, every layer gets a value pool too (a tied Library's values are its keys)."""
        if not libs:
            raise ValueError("from_libraries needs at least one Library")
        layers = libs[0].layers
        for lb in libs:
            if lb.layers != layers or lb.d_s != libs[0].d_s:
                raise ValueError("all Libraries must share layers and d_s")
        device = torch.device(device)
        pages = {}
        for li in layers:
            Cs = [lb.K[li].shape[0] for lb in libs]
            Nmax = max(lb.K[li].shape[1] for lb in libs)
            d = libs[0].d_s
            Cmax = max(Cs)
            dt = slot_dtype if slot_dtype != "auto" else torch.float16
            untied = any(lb.V is not None for lb in libs)
            if untied and dt not in (torch.float16, torch.bfloat16):
                raise NotImplementedError(f"untied Library values are read from float16 / bfloat16 slots, not {dt}")
            pool = torch.zeros(sum(Cs), Nmax, d, dtype=dt, device=device)
            vpool = torch.zeros_like(pool) if untied else None
            page_of = torch.zeros(len(libs), Cmax, dtype=torch.int32)
            n_valid = torch.zeros(len(libs), Cmax, dtype=torch.int32)
            S = torch.zeros(len(libs), Cmax, d, dtype=torch.float32, device=device)
            off = 0
            for b, lb in enumerate(libs):
                K = lb.K[li]
                C, Nb = K.shape[0], K.shape[1]
                pool[off:off + C, :Nb] = K.to(device=device, dtype=dt)
                if untied:
                    vpool[off:off + C, :Nb] = (lb.V[li] if lb.V is not None else K).to(device=device, dtype=dt)
                page_of[b, :C] = torch.arange(off, off + C, dtype=torch.int32)
                n_valid[b, :C] = lb.mask[li].sum(-1).to(torch.int32).cpu()
                S[b, :C] = lb.S[li].to(device=device, dtype=torch.float32)
                off += C
            n_chunks_of = torch.tensor(Cs, dtype=torch.int32, device=device)
            pages[li] = Pages(slots=pool, page_of=page_of.to(device), n_valid=n_valid.to(device), S=S,
                              n_chunks_of=None if len(set(Cs)) == 1 else n_chunks_of, vslots=vpool)
        return PagedLibrary(pages, depths=libs[0].depths)

    @staticmethod
    def from_doc_caches(caches: list, reader_model, depths=None, device=None, center: Optional[dict] = None,
                        slot_dtype="auto", page_rows: Optional[int] = None) -> "PagedLibrary":
        """Build on the device, one Library per doc cache (batch row b reads caches[b]), with what
        Library.from_doc_cache (xenc/library.py:125-136) and Library.__init__ / _summaries (:26-74) compute:
        per depth, every doc's chunk rows go to the device in one copy and one build launch pads them into
        pages, centres them when `center` is given and computes S from the float32 rows.

        slot_dtype "auto": float16 (the cache's rows are float16, so the copy of uncentred keys is exact; centred
        keys are rounded to float16 after the centring, with S from the float32 rows, so routing is unchanged and
        the read stays within the path's 2e-3 bound on the tensor-core kernel); torch.float32 keeps centred keys in
        float32 (the CUDA-core read)."""
        from .ops import library_build

        if not caches:
            raise ValueError("from_doc_caches needs at least one doc cache")
        depths = sorted(float(r) for r in (depths or caches[0]["depths"]))
        rmap = rho_layer_map(reader_model, depths)
        if device is None:
            device = reader_model.device if hasattr(reader_model, "device") else "cuda"
        device = torch.device(device)
        Cs = [len(c["chunks"]) for c in caches]
        if min(Cs) == 0:
            raise ValueError("Library needs at least one chunk")
        untied = any(ch.get("V") is not None for c in caches for ch in c["chunks"])
        n_lib, Cmax, total = len(caches), max(Cs), sum(Cs)
        lib_of = torch.repeat_interleave(torch.arange(n_lib), torch.tensor(Cs)).to(device)
        col_of = torch.cat([torch.arange(c) for c in Cs]).to(device)
        page_of = torch.zeros(n_lib, Cmax, dtype=torch.int32, device=device)
        page_of[lib_of, col_of] = torch.arange(total, dtype=torch.int32, device=device)
        pages = {}
        for rho in depths:
            li = rmap[rho]
            krows = [_rows_of(ch, rho, "K") for c in caches for ch in c["chunks"]]
            counts = [int(r.shape[0]) for r in krows]
            pr = int(page_rows or max(max(counts), 1))
            mu = None
            if center is not None:
                try:
                    mu = center[key_for(center, rho)].to(device=device, dtype=torch.float32)
                except KeyError:
                    mu = None
            if slot_dtype == "auto":
                dt = torch.float16
            else:
                dt = slot_dtype
            flat = torch.cat([r.reshape(-1, r.shape[-1]) for r in krows]).contiguous()
            if flat.dtype not in (torch.float16, torch.bfloat16, torch.float32):
                flat = flat.float()
            flat = flat.to(device)
            slots, nv, S = library_build(flat, counts, page_rows=pr, mu=mu, slot_dtype=dt)
            vslots = None
            if untied:
                if dt not in (torch.float16, torch.bfloat16):
                    raise NotImplementedError(f"untied Library values are read from float16 / bfloat16 slots, not {dt}")
                vrows = [(_rows_of(ch, rho, "V") if ch.get("V") is not None else _rows_of(ch, rho, "K"))
                         for c in caches for ch in c["chunks"]]
                if [int(r.shape[0]) for r in vrows] != counts:
                    raise ValueError("untied chunks need as many V rows as K rows")
                vflat = torch.cat([r.reshape(-1, r.shape[-1]) for r in vrows]).contiguous().to(device)
                vslots, _, _ = library_build(vflat, counts, page_rows=pr, slot_dtype=dt, want_summaries=False)
            n_valid = torch.zeros(n_lib, Cmax, dtype=torch.int32, device=device)
            n_valid[lib_of, col_of] = nv
            S2 = torch.zeros(n_lib, Cmax, S.shape[-1], dtype=torch.float32, device=device)
            S2[lib_of, col_of] = S
            pages[li] = Pages(slots=slots, page_of=page_of, n_valid=n_valid, S=S2,
                              n_chunks_of=None if len(set(Cs)) == 1 else torch.tensor(Cs, dtype=torch.int32,
                                                                                      device=device),
                              vslots=vslots)
        return PagedLibrary(pages, depths=depths)

    @staticmethod
    def from_pool(layer_slots: dict, page_of: torch.Tensor, n_valid: torch.Tensor,
                  n_chunks_of: Optional[torch.Tensor] = None, layer_vslots: Optional[dict] = None) -> "PagedLibrary":
        """Slots already resident on the device: {layer: pool [P, page_rows, d_s]}, a shared page table
        [n_lib, C] and valid-row counts [n_lib, C]; the summary keys are computed on the device.
        layer_vslots: {layer: value pool} of the same shapes for untied Libraries."""
        from .ops import summaries

        pages = {}
        for li, slots in layer_slots.items():
            po = page_of.to(device=slots.device, dtype=torch.int32).contiguous()
            nv = n_valid.to(device=slots.device, dtype=torch.int32).contiguous()
            pages[li] = Pages(slots=slots, page_of=po, n_valid=nv, S=summaries(slots, po, nv),
                              n_chunks_of=None if n_chunks_of is None else n_chunks_of.to(slots.device, torch.int32),
                              vslots=None if layer_vslots is None else layer_vslots[li])
        return PagedLibrary(pages)


__all__ = ["Library", "PagedLibrary"]
