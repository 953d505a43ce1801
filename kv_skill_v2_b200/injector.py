"""Reader-side injectors: the Library read behind the reference's LibraryInjector / XEncInjector API.

Mirrors xenc/injector.py of the reference:
* ExternalSkillInjector  -- the hook plumbing the reference inherits from the un-vendored deltaskill package:
  forward hooks on the reader's decoder blocks at itf.inject_layers, `enabled`, `mag_terms`, `gain_scale`,
  `calib`, `skill`, `detach()`, `_pos_mask(h)` (fields as xenc/injector.py:109-118,171-172,191-196 use them).
* XEncInjector           -- single-skill read with rho-keyed remapping and d_s / layer validation (:81-118).
* LibraryInjector        -- per-token top-k routing over chunk summaries, the masked within-chunk read and an
  optional LayerSelector (:121-273), plus bookkeeping: last_route, route_terms, mag_terms.

Compute path. For a ModelInterface or LinearInterface the whole branch runs in the xencb kernels: rms_norm +
query projection + L2 + gate (+ selector logits at the first candidate layer) in one projection, routing,
the split-K decode read, then the output projection with gain, gate, the selector's matched norm, the
position mask, the cast to h's dtype, the mag term and h + delta fused. A duck-typed interface (any object
with .query/.gate/.gain/.write, xenc/injector.py:54-77) keeps its own Python methods around the same
routing and read kernels. Tensors must be on a CUDA device; there is no CPU path.

Batched documents. load_library also takes a PagedLibrary (one Library per batch row); batch row b then
reads Library b. The reference holds a single Library per injector, which is the n_lib = 1 case.

Forward only: the kernels carry no autograd, so a call that would need gradients raises.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import ops
from .depth import KVSkill, decoder_layers, for_reader
from .interface import LinearInterface, ModelInterface
from .library import Library, PagedLibrary
from .selector import LayerSelector


def _on(t: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """`t` on `like.device`; the same object when already there (xenc/injector.py:40-42)."""
    return t if t.device == like.device else t.to(like.device)


def _model_device(model) -> torch.device:
    dev = getattr(model, "device", None)
    if isinstance(dev, torch.device):
        return dev
    return next(model.parameters()).device


def _f32_on(w: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    return w.detach().to(device=like.device, dtype=torch.float32).contiguous()


def _needs_grad(*objs) -> bool:
    if not torch.is_grad_enabled():
        return False
    for o in objs:
        if isinstance(o, torch.Tensor) and o.requires_grad:
            return True
        if isinstance(o, nn.Module) and any(p.requires_grad for p in o.parameters()):
            return True
    return False



# graphs of the fused hook path captured directly on a caller's input buffer, per (layer, shape, ...)
_PTR_GRAPHS = 4

class ExternalSkillInjector:
    """Forward-hook plumbing for a reader model (the deltaskill base class the reference subclasses)."""

    def __init__(self, model, interface, read_fp32: bool = True, read_softmax: bool = True, read_temp: float = 12.0):
        self.model, self.itf = model, interface
        self.read_fp32, self.read_softmax, self.read_temp = bool(read_fp32), bool(read_softmax), float(read_temp)
        self.enabled = True
        self._handles: list = []
        self.mag_terms: list = []
        self.gain_scale = 1.0
        self.calib: Optional[dict] = None
        self.skill: Optional[KVSkill] = None
        self.pos_mask: Optional[torch.Tensor] = None  # [B, T] multiplier of delta (None: all positions)
        # projection weights in the 3xF16 form (ops.weights_prep), keyed by storage, version and shape; each
        # entry keeps its source tensor alive so the key cannot be reused by another tensor
        self.gemm_f16x3 = True
        self._wprep: dict = {}
        self._attach()

    def _active(self) -> bool:
        return self.enabled and self.skill is not None

    def _pos_mask(self, h: torch.Tensor) -> Optional[torch.Tensor]:
        if self.pos_mask is None:
            return None
        return self.pos_mask.to(device=h.device, dtype=torch.float32).reshape(-1)

    def _attach(self) -> None:
        blocks = decoder_layers(self.model)
        for li in self.itf.inject_layers:
            def hook(mod, args, output, li=li):
                if not self._active():
                    return output
                is_tuple = isinstance(output, tuple)
                h = output[0] if is_tuple else output
                h_new, rel = self._inject(h, li)
                self.mag_terms.append(rel.mean())
                return (h_new,) + tuple(output[1:]) if is_tuple else h_new

            self._handles.append(blocks[li].register_forward_hook(hook))

    def detach(self) -> None:
        for hd in self._handles:
            hd.remove()
        self._handles.clear()

    def load(self, skill: KVSkill) -> None:
        self.skill = skill

    # subclasses provide _branch (delta in float32) and _inject (h + delta, rel)


class XEncInjector(ExternalSkillInjector):
    def load(self, skill: KVSkill) -> None:
        if skill.meta.get("keyed_by") == "rho":
            skill = for_reader(skill, self.model)
        if skill.d_s != self.itf.d_s:
            raise ValueError(f"skill d_s={skill.d_s} (encoder) != interface d_s={self.itf.d_s}")
        missing = set(self.itf.inject_layers) - set(skill.K)
        if missing:
            raise KeyError(f"skill has no operator for reader layers {sorted(missing)}")
        super().load(skill)

    # ------------------------------------------------------------------ single-skill pages
    def _skill_pages(self, li: int, like: torch.Tensor) -> ops.Pages:
        """The skill's layer as a one-chunk Library (moved once, cached on the skill)."""
        cache = self.skill.meta.setdefault("_xencb_pages", {})
        key = (li, str(like.device))
        if key in cache:
            return cache[key]
        K, V = self.skill.K[li], self.skill.V[li]
        untied = V is not K and not (V.shape == K.shape and torch.equal(V.to(K.device), K))
        Kd = K.to(like.device)
        n = int(Kd.shape[0])
        vslots = None
        if untied:
            # The untied read runs on the tensor cores: both pools in float16.
            slots, vslots = Kd.to(torch.float16), V.to(device=like.device, dtype=torch.float16).contiguous().view(1, n, -1)
        else:
            slots = Kd.to(torch.float16) if torch.equal(Kd.to(torch.float16).to(Kd.dtype), Kd) else Kd.float()
        pages = ops.Pages(slots=slots.contiguous().view(1, n, -1),
                          page_of=torch.zeros(1, 1, dtype=torch.int32, device=like.device),
                          n_valid=torch.full((1, 1), n, dtype=torch.int32, device=like.device),
                          S=torch.zeros(1, 1, Kd.shape[-1], dtype=torch.float32, device=like.device), vslots=vslots)
        cache[key] = pages
        return pages

    def _skill_read(self, q: torch.Tensor, li: int) -> torch.Tensor:
        pages = self._skill_pages(li, q)
        R = q.shape[0]
        idx = torch.zeros(R, 1, dtype=torch.int32, device=q.device)
        wk = torch.ones(R, 1, dtype=torch.float32, device=q.device)
        return ops.read_decode(q, pages, idx, wk, rows_per_lib=R, read_temp=self.read_temp,
                               read_softmax=self.read_softmax)

    # ------------------------------------------------------------------ shared projection machinery
    def _prep(self, W: torch.Tensor) -> Optional[torch.Tensor]:
        """W [out, in] float32 on the device in the 3xF16 form, or None (disabled, or in % 8 != 0)."""
        if not self.gemm_f16x3 or W.shape[-1] % 8 != 0 or not W.is_cuda:
            return None
        key = (W.data_ptr(), W._version, tuple(W.shape), str(W.device))
        hit = self._wprep.get(key)
        if hit is not None:
            return hit[1]
        if len(self._wprep) >= 64:
            self._wprep.clear()
        prep = ops.weights_prep(W)
        self._wprep[key] = (W, prep)
        return prep

    def _weights_key(self) -> tuple:
        """Storage and version of every interface parameter (a captured step is valid only for these)."""
        itf = self.itf
        if not isinstance(itf, nn.Module):
            return ()
        return tuple((p.data_ptr(), p._version) for p in itf.parameters())

    def _fast_interface(self) -> bool:
        return isinstance(self.itf, (ModelInterface, LinearInterface))

    def _query(self, h2: torch.Tensor, li: int, sel_fuse: Optional[LayerSelector] = None):
        """(q [R, d_s], gate [R] | None, log_gain | None, z | None) for rows h2 [R, d_m] (fast interfaces).

        The per-layer parameters (gate_b[pos], log_gain[pos]) stay on the device and are read by the kernels, so
        the hook path has no host reads and can be captured in a CUDA graph."""
        itf = self.itf
        sel_w = sel_b = None
        if sel_fuse is not None:
            sel_w = sel_fuse.u.weight.detach().float().to(h2.device)
            sel_b = sel_fuse.u.bias.detach().float().to(h2.device)
        if isinstance(itf, LinearInterface):
            W = _on(itf.w_in.detach(), h2).float()
            q, _, _, z = ops.project_in(h2, W, sel_w=sel_w, sel_b=sel_b, w_prep=self._prep(W))
            return q, None, None, z
        p = itf._pos[li]
        gate_w = _on(itf.gate_w.detach(), h2).float()
        gate_b = _on(itf.gate_b.detach()[p:p + 1], h2).float()
        gain = _on(itf.log_gain.detach()[p:p + 1], h2).float()
        lins = itf.query_weights()
        if len(lins) == 1:
            W, b = lins[0]
            Wf = _f32_on(W, h2)
            q, g, _, z = ops.project_in(h2, Wf, None if b is None else _on(b.detach(), h2).float(),
                                        gate_w=gate_w, gate_b=gate_b, sel_w=sel_w, sel_b=sel_b,
                                        w_prep=self._prep(Wf))
            return q, g, gain, z
        # low-rank A: rms_norm + first map (gate and selector logits on the normed input), then map + L2
        x = h2
        g = z = None
        for i, (W, b) in enumerate(lins):
            first, last = i == 0, i == len(lins) - 1
            Wf = _f32_on(W, h2)
            x, g_i, _, z_i = ops.project_in(x, Wf,
                                            None if b is None else _on(b.detach(), h2).float(), rms=first, l2=last,
                                            gate_w=gate_w if first else None, gate_b=gate_b,
                                            sel_w=sel_w if first else None, sel_b=sel_b if first else None,
                                            w_prep=self._prep(Wf))
            if first:
                g, z = g_i, z_i
        return x, g, gain, z

    def _query_route(self, h2: torch.Tensor, li: int, pages: ops.Pages, rpl: int, top_k: int, route_temp: float,
                     row_w: Optional[torch.Tensor]):
        """(q, gate | None, log_gain | None, idx, wk, w) from the fused input projection + routing of decode rows,
        or None when the interface's query map is not one linear layer (low-rank A: two projections)."""
        itf = self.itf
        if isinstance(itf, LinearInterface):
            W = _on(itf.w_in.detach(), h2).float()
            q, _, _, idx, wk, w, _ = ops.project_in_route(
                h2, W, S=pages.S, rows_per_lib=rpl, top_k=top_k, route_temp=route_temp,
                n_chunks_of=pages.n_chunks_of, row_w=row_w, w_prep=self._prep(W))
            return q, None, None, idx, wk, w
        lins = itf.query_weights()
        if len(lins) != 1:
            return None
        p = itf._pos[li]
        W, b = lins[0]
        Wf = _f32_on(W, h2)
        q, g, _, idx, wk, w, _ = ops.project_in_route(
            h2, Wf, None if b is None else _on(b.detach(), h2).float(), S=pages.S, rows_per_lib=rpl, top_k=top_k,
            route_temp=route_temp, n_chunks_of=pages.n_chunks_of, row_w=row_w,
            gate_w=_on(itf.gate_w.detach(), h2).float(), gate_b=_on(itf.gate_b.detach()[p:p + 1], h2).float(),
            w_prep=self._prep(Wf))
        return q, g, _on(itf.log_gain.detach()[p:p + 1], h2).float(), idx, wk, w

    def _write_weights(self, like: torch.Tensor):
        itf = self.itf
        if isinstance(itf, LinearInterface):
            return _on(itf.w_out.detach(), like).float(), None
        B = itf.B
        return _f32_on(B.weight, like), None if B.bias is None else _on(B.bias.detach(), like).float()

    def _calibrate(self, r: torch.Tensor, li: int):
        gcal = 1.0
        if self.calib is not None and li in self.calib:
            r = r * _on(torch.as_tensor(self.calib[li]["scale"], dtype=torch.float32), r)
            gcal = self.calib[li]["gain"]
            gcal = float(gcal) if not isinstance(gcal, torch.Tensor) or gcal.numel() == 1 else gcal
        return r, gcal

    def _check_forward_only(self, h: torch.Tensor) -> None:
        if _needs_grad(h, self.itf if isinstance(self.itf, nn.Module) else None):
            raise RuntimeError("the xencb Library read is forward-only (no autograd); run the reader under "
                               "torch.no_grad() / torch.inference_mode(), or freeze the interface")

    def _run(self, h: torch.Tensor, li: int, inject: bool):
        """Single-skill branch. inject=False -> delta (float32); inject=True -> (h + delta, rel)."""
        self._check_forward_only(h)
        lead, d_m = h.shape[:-1], h.shape[-1]
        h2 = h.reshape(-1, d_m)
        if self._fast_interface():
            q, g, log_gain, _ = self._query(h2, li)
            r = self._skill_read(q, li)
            r, gcal = self._calibrate(r, li)
            return self._finish(h, h2, r, g, gcal if not isinstance(gcal, torch.Tensor) else 1.0, li, inject,
                                extra=gcal if isinstance(gcal, torch.Tensor) else None, log_scale=log_gain)
        hn = ops.rms_norm(h2)
        q = self.itf.query(hn.view(*lead, -1)).reshape(-1, self.itf.d_s).float()
        r = self._skill_read(q, li)
        r, gcal = self._calibrate(r, li)
        return self._duck_finish(h, hn, r, gcal, li, inject)

    def _finish(self, h, h2, r, g, scale, li, inject, sel_col=None, log_alpha=0.0, extra=None, log_scale=None):
        lead = h.shape[:-1]
        W, b = self._write_weights(h2)
        wp = self._prep(W)
        pm = self._pos_mask(h) if inject else None
        if extra is not None:  # a tensor calibration gain: fold into the per-row gate
            g = (g if g is not None else torch.ones(r.shape[0], device=r.device)) * extra.reshape(-1).float()
        if inject:
            h_new = torch.empty_like(h2)
            _, h_new, rel = ops.project_out(r, W, h2, b_out=b, scale=float(self.gain_scale) * float(scale),
                                            log_scale=log_scale, gate=g, sel_w=sel_col, log_alpha=log_alpha,
                                            pos_mask=pm, want_delta=False,
                                            h_out=h_new, want_rel=True, w_prep=wp)
            return h_new.view(h.shape), rel
        delta, _, _ = ops.project_out(r, W, h2.float() if h2.dtype != torch.float32 else h2, b_out=b,
                                      scale=float(self.gain_scale) * float(scale), log_scale=log_scale, gate=g,
                                      sel_w=sel_col, log_alpha=log_alpha, want_delta=True, w_prep=wp)
        return delta.view(*lead, -1)

    def _duck_finish(self, h, hn, r, gcal, li, inject, selector=None):
        lead = h.shape[:-1]
        itf = self.itf
        hn3 = hn.view(*lead, -1)
        g = itf.gate(hn3, li)
        gain = _on(torch.as_tensor(itf.gain(li)), hn)
        delta = self.gain_scale * gain * gcal * g * itf.write(r.view(*lead, -1))
        delta = delta.float()
        if selector is not None:
            delta = selector.apply(delta, h, li)
        if not inject:
            return delta
        d = delta.to(h.dtype)
        pm = self._pos_mask(h)
        if pm is not None:
            d = d * pm.view(*lead, 1).to(d.dtype)
        rel = d.float().norm(dim=-1) / (h.float().norm(dim=-1) + 1e-6)
        return h + d, rel

    def _branch(self, h: torch.Tensor, li: int) -> torch.Tensor:
        return self._run(h, li, inject=False)

    def _inject(self, h: torch.Tensor, li: int):
        return self._run(h, li, inject=True)


class LibraryInjector(XEncInjector):
    def __init__(self, model, interface, read_softmax: bool = True, read_temp: float = 12.0, route_temp: float = 10.0,
                 top_k: int = 0, selector=None, read_fp32: bool = True, slot_dtype="auto", cuda_graphs: bool = True):
        self.lib = None
        # per-(layer, shape) CUDA graphs of the fused hook path (see _run_lib); cleared whenever the Library changes
        self.cuda_graphs = bool(cuda_graphs)
        self._graphs: dict = {}
        self.route_temp = float(route_temp)
        self.top_k = int(top_k)
        self.selector = selector
        self.slot_dtype = slot_dtype
        self.last_route: Optional[torch.Tensor] = None
        self.record_attn = False
        self.last_attn: dict = {}
        self.force_attn = None
        self.force_norm_match = False
        self.training_attn = False
        self.attn_pos: int = -1
        self.attn_terms: list = []
        self.route_terms: list = []
        super().__init__(model, interface, read_fp32=read_fp32, read_softmax=read_softmax, read_temp=read_temp)

    # ------------------------------------------------------------------ load / unload
    def load(self, skill: KVSkill) -> None:
        self.lib = None
        self._graphs.clear()
        super().load(skill)

    def load_library(self, lib) -> None:
        self._graphs.clear()
        if lib.d_s != self.itf.d_s:
            raise ValueError(f"library d_s={lib.d_s} (encoder) != interface d_s={self.itf.d_s}")
        missing = set(self.itf.inject_layers) - set(lib.K)
        if missing:
            raise KeyError(f"library has no operator for reader layers {sorted(missing)}")
        dev = _model_device(self.model)
        self.skill = None
        if isinstance(lib, Library):
            lib.to(dev)
            for li in self.itf.inject_layers:  # build the paged views now (one copy at load, as the reference)
                lib.pages(li, dev, self.slot_dtype, require_nonempty=self.read_softmax)
        elif isinstance(lib, PagedLibrary):
            if self.read_softmax:
                for li in self.itf.inject_layers:
                    p = lib.pages(li)
                    nv = p.n_valid
                    if p.n_chunks_of is not None:
                        live = torch.arange(p.n_chunks, device=nv.device).view(1, -1) < p.n_chunks_of.view(-1, 1)
                        nv = torch.where(live, nv, torch.ones_like(nv))
                    if bool((nv <= 0).any()):
                        raise ValueError(f"PagedLibrary layer {li}: a chunk has no valid slot (the softmax read is NaN)")
        else:
            raise TypeError(f"load_library expects a Library or PagedLibrary, got {type(lib).__name__}")
        self.lib = lib

    def unload(self) -> None:
        self._graphs.clear()
        self.skill = None
        self.lib = None
        self.mag_terms.clear()
        self.route_terms.clear()
        self.attn_terms.clear()
        self.last_route = None

    # ------------------------------------------------------------------ hooks
    def _active(self) -> bool:
        return self.enabled and (self.skill is not None or self.lib is not None)

    def _attach(self) -> None:
        blocks = decoder_layers(self.model)
        first = self.itf.inject_layers[0]

        def pre(mod, args):
            if self.selector is not None:
                self.selector.reset()

        self._handles.append(blocks[first].register_forward_pre_hook(pre))
        super()._attach()

    # ------------------------------------------------------------------ library views
    def _lib_layer(self, li: int, like: torch.Tensor):
        """(K, mask, S) of layer li on like.device (moved once, cached in the Library)."""
        lib = self.lib
        if not isinstance(lib, Library):
            raise TypeError("_lib_layer is defined for a single Library")
        if lib.K[li].device != like.device:
            lib.K[li] = lib.K[li].to(like.device)
            lib.mask[li] = lib.mask[li].to(like.device)
            lib.S[li] = lib.S[li].to(like.device)
        return lib.K[li], lib.mask[li], lib.S[li]

    def _pages(self, li: int, like: torch.Tensor) -> ops.Pages:
        if isinstance(self.lib, Library):
            return self.lib.pages(li, like.device, self.slot_dtype, require_nonempty=self.read_softmax)
        return self.lib.pages(li, like.device)

    def _rows_per_lib(self, h: torch.Tensor, pages: ops.Pages) -> int:
        R = h.numel() // h.shape[-1]
        if pages.n_lib == 1:
            return R
        if h.dim() < 2 or h.shape[0] != pages.n_lib:
            raise ValueError(f"a PagedLibrary of {pages.n_lib} documents needs h with batch size {pages.n_lib}, "
                             f"got {tuple(h.shape)}")
        return R // pages.n_lib

    # ------------------------------------------------------------------ routing
    def route(self, q: torch.Tensor, li: int) -> torch.Tensor:
        """Per-token routing weights over chunks [..., C]; sums to 1, exactly top_k nonzeros if set."""
        pages = self._pages(li, q)
        q2 = q.reshape(-1, q.shape[-1]).float()
        rpl = self._rows_per_lib(q, pages)
        _, _, w, _ = ops.route(q2, pages.S, rows_per_lib=rpl, top_k=self.top_k, route_temp=self.route_temp,
                               n_chunks_of=pages.n_chunks_of)
        return w.view(*q.shape[:-1], pages.n_chunks)

    # ------------------------------------------------------------------ branch
    def _selector_ours(self) -> Optional[LayerSelector]:
        return self.selector if isinstance(self.selector, LayerSelector) else None

    def _run(self, h: torch.Tensor, li: int, inject: bool):
        sel = self._selector_ours()
        if self.lib is None or (self.selector is not None and sel is None):
            # single-skill path, or a duck-typed selector object: delta first, then the selector's own apply
            if self.lib is None:
                if self.selector is None:
                    return super()._run(h, li, inject)
                delta = super()._run(h, li, inject=False)
            else:
                delta = self._run_lib(h, li, inject=False, sel=None)
            delta = self.selector.apply(delta, h, li)
            return self._torch_inject(h, delta) if inject else delta
        return self._run_lib(h, li, inject, sel)

    def _torch_inject(self, h: torch.Tensor, delta: torch.Tensor):
        """The hook arithmetic of xenc/injector.py:190-196 for a delta produced outside the fused path."""
        d = delta.to(h.dtype)
        pm = self._pos_mask(h)
        if pm is not None:
            d = d * pm.view(*h.shape[:-1], 1).to(d.dtype)
        rel = d.float().norm(dim=-1) / (h.float().norm(dim=-1) + 1e-6)
        return h + d, rel

    def _graphable(self, h: torch.Tensor, inject: bool, sel) -> bool:
        """The fused hook path can be replayed from a CUDA graph: injection, no selector (its weights change per
        forward), a fast interface, no calibration or position mask, no attention diagnostics, no grad, not inside
        a user's capture."""
        return (self.cuda_graphs and inject and sel is None and self._fast_interface() and h.is_cuda
                and self.calib is None and self.pos_mask is None and not self.record_attn
                and self.force_attn is None and not torch.is_grad_enabled()
                and not torch.cuda.is_current_stream_capturing())

    def _check_diagnostics(self) -> None:
        if self.training_attn and torch.is_grad_enabled():
            raise NotImplementedError("training_attn keeps the attention for a training loss (autograd); the xencb "
                                      "read is forward-only")

    def _read_with_diagnostics(self, h: torch.Tensor, li: int, q: torch.Tensor, pages: ops.Pages, idx, wk,
                               rpl: int, sparse: bool) -> torch.Tensor:
        """The read of _branch, with force_attn (the given [C, N] addressing replaces the computed one,
        xenc/injector.py:246-258) and record_attn (last_attn[li] = the last position's route-weighted slot
        attention of batch row 0, :259-260)."""
        force = self.force_attn
        fa = None
        if force is not None:
            fa = force.get(li) if isinstance(force, dict) else force
            if fa is None:
                raise ValueError(f"force_attn has no addressing for layer {li}")
            fa = _on(torch.as_tensor(fa), q).float()
            if tuple(fa.shape) != (pages.n_chunks, pages.page_rows):
                raise ValueError(f"force_attn {tuple(fa.shape)} != library [C,N] {(pages.n_chunks, pages.page_rows)}")
        r = None
        if fa is None or self.force_norm_match:
            r = ops.read_decode(q, pages, idx, wk, rows_per_lib=rpl, read_temp=self.read_temp,
                                read_softmax=self.read_softmax, sparse=sparse)
        scale = None
        if fa is not None:
            r, scale = ops.read_forced(fa, pages, q.shape[0], r0=r, norm_match=self.force_norm_match)
        if self.record_attn:
            row = (h.shape[-2] if h.dim() >= 3 else h.shape[0]) - 1  # batch row 0, last position
            if fa is not None:
                attn = fa * scale[row]
            else:
                attn = ops.read_attn(q, pages, idx, wk, row=row, rows_per_lib=rpl, read_temp=self.read_temp,
                                     read_softmax=self.read_softmax)
            self.last_attn[li] = attn.detach().float().cpu()
        return r

    def _run_lib(self, h: torch.Tensor, li: int, inject: bool, sel: Optional[LayerSelector]):
        self._check_diagnostics()
        if not self._graphable(h, inject, sel):
            return self._run_lib_eager(h, li, inject, sel)
        # CUDA-graph replay: the first call for a (layer, shape, dtype, Library view) runs eagerly (which also
        # validates and sizes the workspaces), then captures the same launches on static buffers; later calls
        # copy h in, replay, and return copies of the static outputs (so a caller may keep them).
        # A serving loop hands the hook the same few input buffers step after step: a graph captured on such a
        # buffer itself (up to _PTR_GRAPHS per layer and shape) replays with no copy-in. Further buffers share one
        # graph on a static input that h is copied into. A tensor later allocated at the same address, shape,
        # strides and dtype is read correctly by the same graph.
        pages = self._pages(li, h)
        base = (li, tuple(h.shape), tuple(h.stride()), h.dtype, h.device, id(pages), float(self.gain_scale),
                self.top_k, float(self.read_temp), float(self.route_temp), bool(self.read_softmax),
                self._weights_key(), bool(self.gemm_f16x3))
        ent = self._graphs.get((base, h.data_ptr()))
        if ent is None:
            ent = self._graphs.get((base, None))
            if ent is None:
                n_ptr = sum(1 for k in self._graphs if k[0] == base)
                on_buffer = n_ptr < _PTR_GRAPHS
                out = self._run_lib_eager(h, li, inject, sel)
                route_eager = self.last_route
                h_static = h.detach() if on_buffer else h.detach().clone()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    h_new_s, rel_s = self._run_lib_eager(h_static, li, inject, sel)
                # the entry keeps the prepared weights it captured alive
                self._graphs[(base, h.data_ptr() if on_buffer else None)] = (
                    graph, None if on_buffer else h_static, h_new_s, rel_s, self.last_route, pages,
                    list(self._wprep.values()))
                # the captured step has not run yet: this call's routing is the eager run's
                self.last_route = route_eager
                return out
        graph, h_static, h_new_s, rel_s, route_s, _, _ = ent
        if h_static is not None:
            h_static.copy_(h)
        graph.replay()
        self.last_route = route_s
        return h_new_s.clone(), rel_s.clone()

    def _run_lib_eager(self, h: torch.Tensor, li: int, inject: bool, sel: Optional[LayerSelector]):
        self._check_diagnostics()
        self._check_forward_only(h)
        if sel is not None and _needs_grad(sel):
            raise RuntimeError("the xencb Library read is forward-only; freeze the LayerSelector or use no_grad")
        lead, d_m = h.shape[:-1], h.shape[-1]
        h2 = h.reshape(-1, d_m)
        pages = self._pages(li, h)
        rpl = self._rows_per_lib(h, pages)

        fuse_sel = sel is not None and self._fast_interface() and li == sel.first_layer and not sel._explicit
        # the selector's weights for this layer come first: tokens it gives weight 0 here read nothing (the
        # reference reads every layer for every token and zeroes the delta afterwards, xenc/selector.py:106-110).
        # Unless the input projection computes them (fused logits), they are taken before it, so that the router
        # follows the projection directly in the stream and can start on its summary keys early.
        sel_col, log_alpha = None, 0.0

        def sel_column():
            return (sel._w[..., sel.pos[li]].reshape(-1).float().contiguous(),
                    _on(sel.log_alpha.detach().reshape(1), h2).float())

        if sel is not None and not fuse_sel:
            sel.weights_for(h, li)
            sel_col, log_alpha = sel_column()
        # decode rows: q and its routing in one pass after the projection GEMM
        routed = None
        if self._fast_interface() and not fuse_sel and rpl < 64:
            routed = self._query_route(h2, li, pages, rpl, self.top_k, self.route_temp, sel_col)
        if routed is not None:
            q, g, log_gain, idx, wk, w = routed
        else:
            if self._fast_interface():
                q, g, log_gain, z = self._query(h2, li, sel_fuse=sel if fuse_sel else None)
            else:
                hn = ops.rms_norm(h2)
                q = self.itf.query(hn.view(*lead, -1)).reshape(-1, self.itf.d_s).float().contiguous()
                z = None
            if fuse_sel:
                sel._w = sel._weights_from_logits(z.view(*lead, sel.n_cand))
                sel._explicit = False
                sel_col, log_alpha = sel_column()
            idx, wk, w, _ = ops.route(q, pages.S, rows_per_lib=rpl, top_k=self.top_k, route_temp=self.route_temp,
                                      n_chunks_of=pages.n_chunks_of, row_w=sel_col)
        # with a selector most rows read nothing at most depths: the sparse plan spreads the live rows' work
        if self.record_attn or self.force_attn is not None:
            r = self._read_with_diagnostics(h, li, q, pages, idx, wk, rpl, sparse=sel_col is not None)
        else:
            r = ops.read_decode(q, pages, idx, wk, rows_per_lib=rpl, read_temp=self.read_temp,
                                read_softmax=self.read_softmax, sparse=sel_col is not None)
        self.last_route = w.view(*lead, pages.n_chunks)
        if torch.is_grad_enabled():
            self.route_terms.append((li, self.last_route))

        if not self._fast_interface():
            return self._duck_finish(h, hn, r, 1.0, li, inject, selector=sel)
        return self._finish(h, h2, r, g, 1.0, li, inject, sel_col=sel_col, log_alpha=log_alpha, log_scale=log_gain)


__all__ = ["ExternalSkillInjector", "XEncInjector", "LibraryInjector", "itf_query", "itf_gate", "itf_gain",
           "itf_write"]


# duck-typed interface helpers (xenc/injector.py:54-77), for callers that use them directly
def itf_query(itf, hn: torch.Tensor) -> torch.Tensor:
    return itf.query(hn)


def itf_gate(itf, hn: torch.Tensor, li: int) -> torch.Tensor:
    return itf.gate(hn, li)


def itf_gain(itf, li: int, like: torch.Tensor) -> torch.Tensor:
    return _on(torch.as_tensor(itf.gain(li)), like)


def itf_write(itf, r: torch.Tensor) -> torch.Tensor:
    return itf.write(r)
