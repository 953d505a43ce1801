"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's own Library read.

Run where a checkout of the reference exists, naming its root in XENC_REF (there is no default):

    XENC_REF=<path to the reference checkout> python tests/golden/make_golden.py

It imports the reference's unchanged `xenc.library.Library`, `xenc.injector.LibraryInjector` and
`xenc.selector.LayerSelector`. Their dependency `deltaskill` is not vendored in the reference (it is a
sibling checkout, xenc/__init__.py:14-18), so a minimal stand-in is installed into `sys.modules` first:

* deltaskill.derive.rms_norm         x * rsqrt(mean(x^2) + 1e-6), no weight (ASSUMED: unpinned)
* deltaskill.derive.injection_layers [min(L-1, int(rho*L)) for rho in depths] (docs/XENC_SPEC.md:50)
* deltaskill.injector.ExternalSkillInjector  the fields the reference reads (xenc/injector.py:109-118,
                                     171-172,191-196): enabled, _handles, mag_terms, gain_scale=1, calib=None,
                                     skill=None; _attach() at construction; _pos_mask() -> None; detach().
* deltaskill.interface.ModelInterface A (Linear d_m->d_s, no bias), B (Linear d_s->d_m), gate_w [d_m],
                                     gate_b [L], log_gain [L], _pos -- the members xenc/injector.py:54-77
                                     reads (shapes ASSUMED).
* deltaskill.skill.KVSkill, deltaskill.backbone_utils.decoder_layers (and placeholders for the chat helpers
                                     that xenc.backbone imports; the read path never calls them).

Outputs are small .npz files; the tests (which never read the reference) compare the oracle and the CUDA
path against them. Inputs are generated with torch.Generator seeds so the cases are reproducible.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

HERE = Path(__file__).resolve().parent
REF = Path(os.environ["XENC_REF"]) if os.environ.get("XENC_REF") else None


# ------------------------------------------------------------------------------------ deltaskill stand-in
def _install_deltaskill_stub() -> None:
    pkg = types.ModuleType("deltaskill")
    pkg.__path__ = []  # mark as package

    derive = types.ModuleType("deltaskill.derive")

    def rms_norm(x, eps=1e-6):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)

    def injection_layers(model, depths):
        c = model.config
        c = c.get_text_config() if hasattr(c, "get_text_config") else c
        L = int(c.num_hidden_layers)
        return [min(L - 1, int(float(r) * L)) for r in depths]

    derive.rms_norm, derive.injection_layers = rms_norm, injection_layers

    bu = types.ModuleType("deltaskill.backbone_utils")
    bu.decoder_layers = lambda model: model.model.layers

    def _unused(*a, **k):  # chat / decoding helpers xenc.backbone imports; never called on the read path
        raise NotImplementedError("deltaskill stand-in: not part of the Library read")

    bu.chat_template_kwargs = bu.final_channel = bu.is_gpt_oss = bu.skip_special_on_decode = _unused

    skill = types.ModuleType("deltaskill.skill")

    class KVSkill:
        def __init__(self, K, V, d_s, text="", model_name="", meta=None):
            self.K, self.V, self.d_s, self.text, self.model_name = K, V, d_s, text, model_name
            self.meta = dict(meta or {})

    skill.KVSkill = KVSkill

    itf_mod = types.ModuleType("deltaskill.interface")

    class ModelInterface(nn.Module):
        def __init__(self, d_m, d_s, inject_layers, gate_bias_init=-2.0, gain_init=0.0, rank=0):
            super().__init__()
            self.d_m, self.d_s, self.inject_layers, self.rank = d_m, d_s, list(inject_layers), rank
            self._pos = {li: i for i, li in enumerate(self.inject_layers)}
            L = len(self.inject_layers)
            self.A = nn.Linear(d_m, d_s, bias=False)
            self.B = nn.Linear(d_s, d_m, bias=False)
            nn.init.zeros_(self.B.weight)
            self.gate_w = nn.Parameter(torch.zeros(d_m))
            self.gate_b = nn.Parameter(torch.full((L,), float(gate_bias_init)))
            self.log_gain = nn.Parameter(torch.full((L,), float(gain_init)))

    itf_mod.ModelInterface = ModelInterface

    inj = types.ModuleType("deltaskill.injector")

    class ExternalSkillInjector:
        def __init__(self, model, itf, read_fp32=True, read_softmax=True, read_temp=12.0):
            self.model, self.itf = model, itf
            self.read_fp32, self.read_softmax, self.read_temp = read_fp32, read_softmax, read_temp
            self.enabled, self._handles, self.mag_terms = True, [], []
            self.gain_scale, self.calib, self.skill = 1.0, None, None
            self._attach()

        def _pos_mask(self, h):
            return None

        def load(self, skill):
            self.skill = skill

        def detach(self):
            for hd in self._handles:
                hd.remove()
            self._handles.clear()

    inj.ExternalSkillInjector = ExternalSkillInjector

    for name, mod in (("deltaskill", pkg), ("deltaskill.derive", derive), ("deltaskill.backbone_utils", bu),
                      ("deltaskill.skill", skill), ("deltaskill.interface", itf_mod),
                      ("deltaskill.injector", inj)):
        sys.modules[name] = mod
    for sub in ("derive", "backbone_utils", "skill", "interface", "injector"):
        setattr(pkg, sub, sys.modules[f"deltaskill.{sub}"])


# ------------------------------------------------------------------------------------ fake reader
class _Cfg:
    def __init__(self, L, d):
        self.num_hidden_layers, self.hidden_size = L, d


class _Blocks(nn.Module):
    def __init__(self, d, L):
        super().__init__()
        self.layers = nn.ModuleList(nn.Linear(d, d) for _ in range(L))


class FakeReader(nn.Module):
    """A stack of Linear+tanh blocks exposing model.layers / config / device, like a decoder."""

    def __init__(self, d, L, seed):
        super().__init__()
        torch.manual_seed(seed)
        self.model = _Blocks(d, L)
        self.config = _Cfg(L, d)

    @property
    def device(self):
        return next(self.parameters()).device

    def forward(self, x):
        for blk in self.model.layers:
            x = torch.tanh(blk(x))
        return x


class Recorder:
    """Duck-typed interface (xenc/injector.py:54-77): q = L2(hn @ W_in); gate = gain = 1; write = r @ W_out.
    Records q and r of every call."""

    def __init__(self, W_in, W_out):
        self.W_in, self.W_out = W_in, W_out
        self.d_s = W_in.shape[1]
        self.inject_layers = []
        self.qs, self.rs = [], []

    def query(self, hn):
        q = hn @ self.W_in
        q = q / (q.norm(dim=-1, keepdim=True) + 1e-6)
        self.qs.append(q.detach().clone())
        return q

    def gate(self, hn, li):
        return torch.ones(*hn.shape[:-1], 1)

    def gain(self, li):
        return torch.tensor(1.0)

    def write(self, r):
        self.rs.append(r.detach().clone())
        return r @ self.W_out


def _unit_rows(n, d, g):
    x = torch.randn(n, d, generator=g)
    return (x / x.norm(dim=-1, keepdim=True)).half()  # doc caches store fp16 rows (xenc/depth_skill.py:263-266)


def _np(t):
    return t.detach().cpu().numpy()


def _pad(rows):
    C, N, d = len(rows), max(r.shape[0] for r in rows), rows[0].shape[-1]
    K = torch.zeros(C, N, d, dtype=torch.float16)
    for c, r in enumerate(rows):
        K[c, : r.shape[0]] = r
    return K


# ------------------------------------------------------------------------------------ cases
def case_read(name, rows, h, W_in, W_out, top_k, read_softmax, out, read_temp=12.0, route_temp=10.0,
              inputs_in=None, vrows=None, center=None):
    from xenc.injector import LibraryInjector
    from xenc.library import Library

    rho, L = 0.5, 8
    reader = FakeReader(8, L, 0)
    li = min(L - 1, int(rho * L))
    if vrows is None:
        chunks = [{"K": {rho: r}} for r in rows]
    else:  # untied values (harvest="attn"): the read weights V, the scores use K
        chunks = [{"K": {rho: r}, "V": {rho: v}} for r, v in zip(rows, vrows)]
    lib = Library(chunks, [li], [rho], center=None if center is None else {rho: center})
    itf = Recorder(W_in, W_out)
    itf.inject_layers = [li]
    inj = LibraryInjector(reader, itf, read_softmax=read_softmax, read_temp=read_temp, route_temp=route_temp,
                          top_k=top_k)
    inj.load_library(lib)
    with torch.no_grad():
        delta = inj._branch(h, li)
        w = inj.last_route
    rec = {"q": _np(itf.qs[-1]), "w": _np(w), "r": _np(itf.rs[-1]), "delta": _np(delta),
           "S": _np(lib.S[li]), "mask": _np(lib.mask[li]),
           "top_k": np.int32(top_k), "read_softmax": np.int32(read_softmax),
           "read_temp": np.float32(read_temp), "route_temp": np.float32(route_temp)}
    if inputs_in is None:
        rec.update({"K": _np(_pad(rows)), "n_valid": np.array([r.shape[0] for r in rows], np.int32),
                    "h": _np(h), "W_in": _np(W_in), "W_out": _np(W_out)})
    else:
        rec["inputs"] = np.array(inputs_in)
    if vrows is not None:
        rec["V"] = _np(_pad(vrows))
    if center is not None:
        rec["center"] = _np(center)
        rec["K_lib"] = _np(lib.K[li])  # the centered slots as the Library stores them
    out[name] = rec
    inj.detach()


def gen_cfg1(out):
    g = torch.Generator().manual_seed(0)
    C, N, d_s, d_m, T = 8, 512, 256, 512, 16
    rows = [_unit_rows(N if c < C - 1 else 300, d_s, g) for c in range(C)]
    h = torch.randn(1, T, d_m, generator=g)
    W_in = torch.randn(d_m, d_s, generator=g) * 0.02
    W_out = torch.randn(d_s, d_m, generator=g) * 0.02
    case_read("cfg1_softmax_top2", rows, h, W_in, W_out, 2, True, out)
    for nm, k, sm in (("cfg1_dense", 0, True), ("cfg1_linear_top2", 2, False), ("cfg1_topk_eq_C", C, True),
                      ("cfg1_linear_dense", 0, False)):
        case_read(nm, rows, h, W_in, W_out, k, sm, out, inputs_in="cfg1_softmax_top2")


def gen_small(out):
    g = torch.Generator().manual_seed(11)
    d_s, d_m = 24, 32
    rows = [_unit_rows(n, d_s, g) for n in (1, 17, 3, 9, 17)]
    h = torch.randn(2, 7, d_m, generator=g)
    W_in = torch.randn(d_m, d_s, generator=g) * 0.3
    W_out = torch.randn(d_s, d_m, generator=g) * 0.3
    case_read("small_ragged_top2", rows, h, W_in, W_out, 2, True, out)
    case_read("small_ragged_linear", rows, h, W_in, W_out, 3, False, out, inputs_in="small_ragged_top2")
    case_read("small_ragged_dense_t3", rows, h, W_in, W_out, 0, True, out, read_temp=3.0, route_temp=2.5,
              inputs_in="small_ragged_top2")
    g = torch.Generator().manual_seed(12)
    rows1 = [_unit_rows(11, 32, g)]
    h1 = torch.randn(1, 3, 40, generator=g)
    case_read("one_chunk", rows1, h1, torch.randn(40, 32, generator=g) * 0.3,
              torch.randn(32, 40, generator=g) * 0.3, 0, True, out)
    # long chunk rows that are not multiples of any tile, d_s = 520 (not a multiple of 256)
    g = torch.Generator().manual_seed(13)
    rows2 = [_unit_rows(n, 520, g) for n in (200, 333, 1, 97)]
    h2 = torch.randn(1, 5, 264, generator=g)
    case_read("odd_dims_top3", rows2, h2, torch.randn(264, 520, generator=g) * 0.05,
              torch.randn(520, 264, generator=g) * 0.05, 3, True, out)


def gen_untied(out):
    """Untied values (Library chunks with a separate V, xenc/library.py:46, 61-65; read xenc/injector.py:263-265)
    and a centered Library (xenc/library.py:56-58: K = L2(K - mu) on valid rows; V is not centered)."""
    g = torch.Generator().manual_seed(21)
    d_s, d_m = 64, 96
    ns = (100, 128, 37, 128, 1, 64)
    rows = [_unit_rows(n, d_s, g) for n in ns]
    vrows = [(torch.randn(n, d_s, generator=g) * 0.5).half() for n in ns]
    h = torch.randn(2, 5, d_m, generator=g)
    W_in = torch.randn(d_m, d_s, generator=g) * 0.1
    W_out = torch.randn(d_s, d_m, generator=g) * 0.1
    case_read("untied_top2", rows, h, W_in, W_out, 2, True, out, vrows=vrows)
    mu = torch.randn(d_s, generator=g) * 0.05
    case_read("untied_centered_linear", rows, h, W_in, W_out, 0, False, out, vrows=vrows, center=mu,
              inputs_in="untied_top2")


def gen_batch_docs(out):
    """Several documents, one query token each; every doc runs the reference on its own Library.
    Pins the batched (one Library per row) semantics to the single-Library reference."""
    g = torch.Generator().manual_seed(21)
    d_s, d_m, C, N = 64, 96, 6, 40
    W_in = torch.randn(d_m, d_s, generator=g) * 0.1
    W_out = torch.randn(d_s, d_m, generator=g) * 0.1
    Ks, nv, hs, qs, ws, rs, ds = [], [], [], [], [], [], []
    for b in range(4):
        n_last = int(torch.randint(1, N + 1, (1,), generator=g))
        rows = [_unit_rows(N if c < C - 1 else n_last, d_s, g) for c in range(C)]
        h = torch.randn(1, 1, d_m, generator=g)
        tmp = {}
        case_read("_doc", rows, h, W_in, W_out, 2, True, tmp)
        r = tmp["_doc"]
        K = torch.zeros(C, N, d_s, dtype=torch.float16)
        K[:, : r["K"].shape[1]] = torch.from_numpy(r["K"])
        Ks.append(_np(K)), nv.append(r["n_valid"]), hs.append(r["h"][0])
        qs.append(r["q"][0]), ws.append(r["w"][0]), rs.append(r["r"][0]), ds.append(r["delta"][0])
    out["batch_docs_top2"] = {"K": np.stack(Ks), "n_valid": np.stack(nv), "h": np.stack(hs), "q": np.stack(qs),
                              "w": np.stack(ws), "r": np.stack(rs), "delta": np.stack(ds), "W_in": _np(W_in),
                              "W_out": _np(W_out), "top_k": np.int32(2), "read_softmax": np.int32(1),
                              "read_temp": np.float32(12.0), "route_temp": np.float32(10.0)}


def gen_attn(out):
    """LibraryInjector's attention diagnostics (xenc/injector.py:246-260): record_attn (last_attn[li] = the
    last position's route-weighted slot attention of batch row 0, [C, N]) for a softmax top-k read and a linear
    dense read, and force_attn (a given [C, N] addressing in place of the computed one), with and without
    force_norm_match. Two batch rows, three positions, a ragged Library."""
    from xenc.injector import LibraryInjector
    from xenc.library import Library

    g = torch.Generator().manual_seed(41)
    d_s, d_m, C, N, rho, L = 48, 64, 5, 24, 0.5, 8
    counts = [24, 9, 24, 17, 3]
    rows = [_unit_rows(n, d_s, g) for n in counts]
    h = torch.randn(2, 3, d_m, generator=g)
    W_in = torch.randn(d_m, d_s, generator=g) * 0.2
    W_out = torch.randn(d_s, d_m, generator=g) * 0.2
    fa = torch.rand(C, N, generator=g) * (torch.arange(N).view(1, N) < torch.tensor(counts).view(C, 1))
    fa = fa / fa.sum()
    reader = FakeReader(8, L, 0)
    li = min(L - 1, int(rho * L))
    base = {"K": _np(_pad(rows)), "n_valid": np.array(counts, np.int32), "h": _np(h), "W_in": _np(W_in),
            "W_out": _np(W_out), "force": _np(fa), "layer": np.int32(li)}
    for name, top_k, sm, force, norm in (("attn_record_top2", 2, True, False, False),
                                         ("attn_record_linear", 0, False, False, False),
                                         ("attn_force", 2, True, True, False),
                                         ("attn_force_norm", 2, True, True, True)):
        lib = Library([{"K": {rho: r}} for r in rows], [li], [rho])
        itf = Recorder(W_in, W_out)
        itf.inject_layers = [li]
        inj = LibraryInjector(reader, itf, read_softmax=sm, read_temp=12.0, route_temp=10.0, top_k=top_k)
        inj.load_library(lib)
        inj.record_attn = True
        if force:
            inj.force_attn = {li: fa}
            inj.force_norm_match = norm
        with torch.no_grad():
            delta = inj._branch(h, li)
        rec = {"w": _np(inj.last_route), "r": _np(itf.rs[-1]), "delta": _np(delta), "last_attn": _np(inj.last_attn[li]),
               "top_k": np.int32(top_k), "read_softmax": np.int32(sm), "force_norm_match": np.int32(norm),
               "read_temp": np.float32(12.0), "route_temp": np.float32(10.0)}
        if name == "attn_record_top2":
            rec.update(base)
        else:
            rec["inputs"] = np.array("attn_record_top2")
        out[name] = rec
        inj.detach()


def gen_selector(out):
    from deltaskill.derive import rms_norm
    from xenc.selector import LayerSelector

    D, CAND = 40, [3, 5, 7, 9, 11, 13, 15, 17]
    g = torch.Generator().manual_seed(31)
    rec = {}
    for st in (0, 1):
        for k in (1, 2, 3):
            torch.manual_seed(100 + 10 * st + k)
            sel = LayerSelector(D, CAND, k=k, alpha_init=0.02, straight_through=bool(st))
            with torch.no_grad():
                sel.u.weight.copy_(torch.randn(sel.u.weight.shape, generator=g) * 0.3)
                sel.u.bias.copy_(torch.randn(sel.u.bias.shape, generator=g) * 0.3)
                sel.log_alpha.fill_(float(torch.randn(1, generator=g)) * 0.5 - 3.0)
            h = torch.randn(3, 7, D, generator=g) * 2.0
            deltas = torch.randn(len(CAND), 3, 7, D, generator=g)
            hs = torch.randn(len(CAND), 3, 7, D, generator=g) * 3.0
            hs[0] = h
            with torch.no_grad():
                sel.reset()
                outs = [sel.apply(deltas[i], hs[i], li) for i, li in enumerate(CAND)]
                w = sel.weights()
                z = sel.u(rms_norm(h.float()))
            key = f"st{st}_k{k}"
            rec.update({f"{key}_u_w": _np(sel.u.weight), f"{key}_u_b": _np(sel.u.bias),
                        f"{key}_log_alpha": np.float32(sel.log_alpha.item()), f"{key}_h": _np(hs),
                        f"{key}_delta": _np(deltas), f"{key}_z": _np(z), f"{key}_w": _np(w),
                        f"{key}_out": _np(torch.stack(outs))})
    rec["cand"] = np.array(CAND, np.int32)
    out["selector"] = rec


def gen_library(out):
    """Library construction: padding, mask, summaries, centering, subset (xenc/library.py)."""
    from xenc.library import Library

    g = torch.Generator().manual_seed(41)
    depths = [0.25, 0.5, 0.75, 1.0]
    layers = [2, 4, 6, 7]
    ns = (8, 5, 12, 1)
    chunks = [{"K": {r: _unit_rows(n, 24, g) for r in depths}} for n in ns]
    mu = {r: torch.randn(24, generator=g) * 0.2 for r in depths}
    lib = Library(chunks, layers, depths)
    libc = Library(chunks, layers, depths, center=mu)
    sub = lib.subset([1, 3])
    rec = {"layers": np.array(layers, np.int32), "depths": np.array(depths, np.float32),
           "n": np.array(ns, np.int32)}
    for i, li in enumerate(layers):
        rho = depths[i]
        rec[f"rows_{li}"] = _np(_pad([c["K"][rho] for c in chunks]))
        rec[f"mu_{li}"] = _np(mu[rho])
        rec[f"K_{li}"], rec[f"mask_{li}"], rec[f"S_{li}"] = _np(lib.K[li]), _np(lib.mask[li]), _np(lib.S[li])
        rec[f"Kc_{li}"], rec[f"Sc_{li}"] = _np(libc.K[li]), _np(libc.S[li])
        rec[f"Ksub_{li}"], rec[f"masksub_{li}"], rec[f"Ssub_{li}"] = (_np(sub.K[li]), _np(sub.mask[li]),
                                                                        _np(sub.S[li]))
    out["library"] = rec


def gen_hooked(out):
    """Full hook path on a fake reader with a ModelInterface (gate, gain, B) and a LayerSelector over 8
    candidate depths with top-4 routing: the model output and the per-layer mag terms."""
    from deltaskill.derive import injection_layers
    from deltaskill.interface import ModelInterface
    from xenc.injector import LibraryInjector
    from xenc.library import Library
    from xenc.selector import LayerSelector

    CAND = [0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9]
    d_m, d_s, L = 48, 32, 10
    reader = FakeReader(d_m, L, 5).eval()
    layers = injection_layers(reader, CAND)
    g = torch.Generator().manual_seed(51)
    chunks = [{"K": {r: _unit_rows(n, d_s, g) for r in CAND}} for n in (16, 9, 16, 4, 13)]
    lib = Library(chunks, layers, CAND)
    itf = ModelInterface(d_m, d_s, layers)
    with torch.no_grad():
        for p in itf.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.3)
    torch.manual_seed(52)
    sel = LayerSelector(d_m, layers, k=2, alpha_init=0.05)
    with torch.no_grad():
        sel.u.weight.copy_(torch.randn(sel.u.weight.shape, generator=g) * 0.3)
        sel.u.bias.copy_(torch.randn(sel.u.bias.shape, generator=g) * 0.3)
    x = torch.randn(2, 6, d_m, generator=g)
    with torch.no_grad():
        bare = reader(x)
    rec = {"x": _np(x), "bare": _np(bare), "layers": np.array(layers, np.int32),
           "cand": np.array(CAND, np.float32), "n": np.array((16, 9, 16, 4, 13), np.int32)}
    for i, blk in enumerate(reader.model.layers):
        rec[f"blk{i}_w"], rec[f"blk{i}_b"] = _np(blk.weight), _np(blk.bias)
    for i, li in enumerate(layers):
        rec[f"K_{li}"] = _np(lib.K[li])
    rec["A_w"], rec["B_w"] = _np(itf.A.weight), _np(itf.B.weight)
    rec["gate_w"], rec["gate_b"], rec["log_gain"] = _np(itf.gate_w), _np(itf.gate_b), _np(itf.log_gain)
    rec["u_w"], rec["u_b"], rec["log_alpha"] = _np(sel.u.weight), _np(sel.u.bias), np.float32(sel.log_alpha.item())
    for use_sel in (0, 1):
        inj = LibraryInjector(reader, itf, top_k=4, selector=sel if use_sel else None)
        inj.load_library(lib)
        with torch.no_grad():
            y = reader(x)
        rec[f"out_sel{use_sel}"] = _np(y)
        rec[f"mag_sel{use_sel}"] = np.array([float(m) for m in inj.mag_terms], np.float32)
        if use_sel:
            rec["sel_w"] = _np(sel.weights())
        inj.detach()
    out["hooked"] = rec


def gen_topk(out):
    """D8 top-k slot-selection read (xenc/topk_read.py): the reference's TopKLibraryInjector on a tiny attention
    reader (tests/_fixtures.TinyAttnReader) with a ModelInterface, three settings: query "last" + max pool +
    softmax read through both hook paths (model(x) and logits(x)) with record_attn; "all_mean" + mean pool + linear
    read at a training-style selection position; two batch rows with "all_max"."""
    sys.path.insert(0, str(HERE.parents[1]))
    from deltaskill.interface import ModelInterface
    from tests._fixtures import TinyAttnReader
    from xenc.library import Library
    from xenc.topk_read import TopKLibraryInjector, TopKSelector, attach_sel_keys

    D, L, NKV, HD, G = 32, 8, 2, 8, 2
    LAYERS, SEL, DS, DEP = [1, 3, 5, 7], 3, 24, [0.2, 0.4, 0.6, 0.8]

    def setup(seed, ns):
        g = torch.Generator().manual_seed(seed)
        m = TinyAttnReader(D, L, NKV, HD, G, seed=seed).eval().requires_grad_(False)
        chunks = [{"K": {r: _unit_rows(n, DS, g) for r in DEP}, "start": 16 * c, "n_tokens": n}
                  for c, n in enumerate(ns)]
        lib = Library(chunks, LAYERS, DEP)
        ac = {"chunks": [{"K": {0.25: torch.randn(n, NKV * HD, generator=g).half()}} for n in ns]}
        lib = attach_sel_keys(lib, ac, 0.25)
        itf = ModelInterface(D, DS, LAYERS)
        with torch.no_grad():
            for p_ in itf.parameters():
                p_.copy_(torch.randn(p_.shape, generator=g) * 0.3)
        rec = m.arrays()
        rec["n"] = np.array(ns, np.int32)
        for li in LAYERS:
            rec[f"K_{li}"] = _np(lib.K[li])
        rec["sel_K"] = _np(lib.sel_K)
        rec["A_w"], rec["B_w"] = _np(itf.A.weight), _np(itf.B.weight)
        rec["gate_w"], rec["gate_b"], rec["log_gain"] = _np(itf.gate_w), _np(itf.gate_b), _np(itf.log_gain)
        return g, m, lib, itf, rec

    # 1: query last, max pool, softmax read, k = 7 of 41 valid slots
    g, m, lib, itf, rec = setup(61, (16, 16, 9))
    x = torch.randn(1, 11, D, generator=g)
    inj = TopKLibraryInjector(m, itf, TopKSelector(m, SEL, k=7), read_temp=12.0)
    inj.load_library(lib)
    with torch.no_grad():
        y = m(x)
        rec["out_call"], rec["idx_call"], rec["scores_call"] = _np(y), _np(inj.last_idx), _np(inj.tk.last_scores)
        rec["mag_call"] = np.array([float(t) for t in inj.mag_terms], np.float32)
        inj.record_attn = True
        lg = m.logits(x)
    rec["x"], rec["logits"], rec["idx"] = _np(x), _np(lg), _np(inj.last_idx)
    for li in LAYERS:
        rec[f"attn_{li}"] = _np(inj.last_attn[li])
    rec.update({"k": np.int32(7), "query": np.array("last"), "pool": np.array("max"), "read_softmax": np.int32(1),
                "sel_pos": np.int32(-1), "passes": np.int32(inj.n_select_passes)})
    inj.detach()
    out["topk_last_softmax"] = rec

    # 2: query all_mean, mean pool, linear read, selection at the last prompt position (-4)
    g, m, lib, itf, rec = setup(62, (16, 12, 16))
    x = torch.randn(1, 10, D, generator=g)
    inj = TopKLibraryInjector(m, itf, TopKSelector(m, SEL, k=6, pool="mean", query="all_mean"), read_temp=12.0,
                              read_softmax=False)
    inj.load_library(lib)
    inj.sel_pos = -4
    with torch.no_grad():
        lg = m.logits(x)
    rec.update({"x": _np(x), "logits": _np(lg), "idx": _np(inj.last_idx), "scores": _np(inj.tk.last_scores),
                "k": np.int32(6), "query": np.array("all_mean"), "pool": np.array("mean"),
                "read_softmax": np.int32(0), "sel_pos": np.int32(-4)})
    inj.detach()
    out["topk_allmean_linear"] = rec

    # 3: two batch rows, query all_max: each row selects (and reads) its own slots
    g, m, lib, itf, rec = setup(63, (16, 16, 16, 5))
    x = torch.randn(2, 9, D, generator=g)
    inj = TopKLibraryInjector(m, itf, TopKSelector(m, SEL, k=5, query="all_max"), read_temp=12.0)
    inj.load_library(lib)
    with torch.no_grad():
        lg = m.logits(x)
    rec.update({"x": _np(x), "logits": _np(lg), "idx": _np(inj.last_idx), "scores": _np(inj.tk.last_scores),
                "k": np.int32(5), "query": np.array("all_max"), "pool": np.array("max"), "read_softmax": np.int32(1),
                "sel_pos": np.int32(-1)})
    inj.detach()
    out["topk_batch2_allmax"] = rec


def main() -> None:
    if REF is None:
        raise SystemExit("set XENC_REF to the root of a reference checkout (the directory holding xenc/)")
    if not (REF / "xenc" / "injector.py").exists():
        raise SystemExit(f"reference checkout not found at {REF}")
    sys.path.insert(0, str(REF))
    _install_deltaskill_stub()
    torch.set_num_threads(1)
    out: dict = {}
    gens = {"cfg1": gen_cfg1, "small": gen_small, "batch_docs": gen_batch_docs, "selector": gen_selector,
            "library": gen_library, "hooked": gen_hooked, "untied": gen_untied, "topk": gen_topk,
            "attn": gen_attn}
    wanted = sys.argv[1:] or list(gens)  # e.g. `python make_golden.py untied` regenerates one group
    for nm in wanted:
        gens[nm](out)
    for name, rec in out.items():
        if name.startswith("_"):
            continue
        np.savez_compressed(HERE / f"{name}.npz", **rec)
        print(f"wrote {name}.npz ({os.path.getsize(HERE / f'{name}.npz') / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
