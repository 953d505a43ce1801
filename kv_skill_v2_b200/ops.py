"""Tensor-level entry points of the Library read, one per C-ABI call (include/xencb.h).

Each function checks its tensors (CUDA device, dtype, contiguity), allocates outputs and the scratch
workspace through torch's caching allocator, and launches on the current torch stream of the tensors'
device. There is no CPU path: a CPU tensor raises RuntimeError.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _native as N

_DT = {torch.float32: N.F32, torch.float16: N.F16, torch.bfloat16: N.BF16}


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _cuda(what: str, *ts) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{what}: xencb kernels run on CUDA tensors only (got a {t.device} tensor); "
                               "the Library read has no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{what}: tensors on {dev} and {t.device}")
    return dev


def _f32(t: Optional[torch.Tensor], what: str) -> Optional[torch.Tensor]:
    if t is None:
        return None
    if t.dtype != torch.float32:
        raise ValueError(f"{what} must be float32, got {t.dtype}")
    return t.contiguous()


def _hdt(t: torch.Tensor, what: str) -> int:
    if t.dtype not in _DT:
        raise ValueError(f"{what}: dtype {t.dtype} not supported (float32 / float16 / bfloat16)")
    return _DT[t.dtype]


class _on_device:
    """Make `dev` the current CUDA device for the duration (the C side queries it)."""

    def __init__(self, dev: torch.device):
        self.dev = dev.index if dev.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def _workspace(nbytes: int, dev: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)


# ------------------------------------------------------------------------------------------------ rms / project
def rms_norm(h: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """float32 rms_norm of the last dim (deltaskill.derive.rms_norm as used at xenc/injector.py:235)."""
    dev = _cuda("rms_norm", h)
    h2 = h.reshape(-1, h.shape[-1]).contiguous()
    out = torch.empty(h2.shape, dtype=torch.float32, device=dev)
    with _on_device(dev):
        N.call("xencb_rms_norm", _ptr(h2), _hdt(h2, "h"), h2.shape[0], h2.shape[1], eps, _ptr(out), _stream(dev))
    return out.view(*h.shape[:-1], h.shape[-1])


def _dev_scalar(x, what: str):
    """(host value, device tensor | None): a one-element device tensor is passed by pointer (read by the kernel,
    so the call needs no host read and stays capturable in a CUDA graph); a number is passed by value."""
    if isinstance(x, torch.Tensor):
        if x.numel() != 1 or not x.is_cuda:
            raise ValueError(f"{what}: a tensor scalar must be one element on the CUDA device")
        return 0.0, x.detach().reshape(1).to(torch.float32).contiguous()
    return float(x), None


def weights_prep(w: torch.Tensor) -> torch.Tensor:
    """The 3xF16 form of a float32 weight [n, k] (k % 8 == 0) for project_in / project_out's w_prep: a 256-byte
    head, then the f16 pair hi, lo of w scaled by a power of two, in 128 x 64 tiles (4 bytes per weight, n rounded
    up to 128 and k to 64)."""
    dev = _cuda("weights_prep", w)
    w = _f32(w, "w")
    n, k = w.shape
    if k % 8:
        raise ValueError(f"weights_prep: k={k} must be a multiple of 8")
    with _on_device(dev):
        nbytes = N.lib().xencb_weights_prep_bytes(n, k)
        prep = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        N.call("xencb_weights_prep", _ptr(w), n, k, _ptr(prep), nbytes, _stream(dev))
    return prep


def project_in(h2: torch.Tensor, w_in: torch.Tensor, b_in=None, *, rms: bool = True, l2: bool = True,
               gate_w=None, gate_b=0.0, sel_w=None, sel_b=None, eps: float = 1e-6,
               w_prep: Optional[torch.Tensor] = None, prefer_prep: bool = False):
    """(q [R, d_s], gate [R] | None, rstd [R], z [R, n_cand] | None) for rows h2 [R, d_m].

    q = L2((rms_norm(h2) if rms else h2) @ w_in^T + b_in) (L2 only if l2); w_in is [d_s, d_m] (nn.Linear).
    gate_b: a number, or a one-element device tensor read by the kernel. w_prep: weights_prep(w_in), to run the
    GEMM as 3xF16 on the f16 tensor cores (same accuracy as 3xTF32, half its MMAs); prefer_prep=True passes only
    the prepared form (w_in then only gives the shape)."""
    dev = _cuda("project_in", h2, w_in, b_in, gate_w, sel_w, sel_b)
    h2 = h2.contiguous()
    w_in = _f32(w_in, "w_in")
    R, d_m = h2.shape
    d_s = w_in.shape[0]
    if w_in.shape[1] != d_m:
        raise ValueError(f"w_in is {tuple(w_in.shape)}, expected [d_s, {d_m}] (nn.Linear layout)")
    q = torch.empty(R, d_s, dtype=torch.float32, device=dev)
    gate = torch.empty(R, dtype=torch.float32, device=dev) if gate_w is not None else None
    rstd = torch.empty(R, dtype=torch.float32, device=dev)
    n_cand = 0 if sel_w is None else int(sel_w.shape[0])
    z = torch.empty(R, n_cand, dtype=torch.float32, device=dev) if sel_w is not None else None
    flags = (N.PIN_RMS if rms else 0) | (N.PIN_L2 if l2 else 0)
    # converted inputs are bound to locals so they outlive the launch
    b_in, gate_w = _f32(b_in, "b_in"), _f32(gate_w, "gate_w")
    sel_w, sel_b = _f32(sel_w, "sel_w"), _f32(sel_b, "sel_b")
    gb, gb_dev = _dev_scalar(gate_b, "gate_b")
    with _on_device(dev):
        ws_bytes = N.lib().xencb_project_in_workspace(R, d_m, d_s)
        ws = _workspace(ws_bytes, dev)
        w_arg = None if (prefer_prep and w_prep is not None) else w_in
        N.call("xencb_project_in", _ptr(h2), _hdt(h2, "h"), R, d_m, _ptr(w_arg), _ptr(w_prep), _ptr(b_in), d_s, flags,
               _ptr(gate_w), gb, _ptr(gb_dev), _ptr(sel_w), _ptr(sel_b), n_cand, eps, _ptr(q), _ptr(gate),
               _ptr(rstd), _ptr(z), _ptr(ws), ws.numel(), _stream(dev))
    return q, gate, rstd, z


def project_in_route(h2: torch.Tensor, w_in: torch.Tensor, b_in=None, *, S: torch.Tensor, rows_per_lib: int,
                     top_k: int, route_temp: float, n_chunks_of: Optional[torch.Tensor] = None,
                     row_w: Optional[torch.Tensor] = None, want_logits: bool = False, gate_w=None, gate_b=0.0,
                     eps: float = 1e-6, w_prep: Optional[torch.Tensor] = None):
    """project_in (rms + L2) and route for decode rows in one pass after the GEMM (xencb_project_in_route):
    (q, gate | None, rstd, idx, wk, w_dense, logits | None), the same values as project_in then route. Shapes
    the fused form does not take (rows_per_lib >= 64, very wide rows) run the two calls."""
    dev = _cuda("project_in_route", h2, w_in, b_in, gate_w, S, n_chunks_of, row_w)
    if int(rows_per_lib) >= 64:
        q, g, rstd, _ = project_in(h2, w_in, b_in, gate_w=gate_w, gate_b=gate_b, eps=eps, w_prep=w_prep)
        idx, wk, w, lg = route(q, S, rows_per_lib=rows_per_lib, top_k=top_k, route_temp=route_temp,
                               n_chunks_of=n_chunks_of, want_logits=want_logits, row_w=row_w)
        return q, g, rstd, idx, wk, w, lg
    h2 = h2.contiguous()
    w_in = _f32(w_in, "w_in")
    S = _f32(S, "S")
    R, d_m = h2.shape
    d_s = w_in.shape[0]
    if w_in.shape[1] != d_m:
        raise ValueError(f"w_in is {tuple(w_in.shape)}, expected [d_s, {d_m}] (nn.Linear layout)")
    n_lib, C, d2 = S.shape
    if d2 != d_s:
        raise ValueError(f"project_in_route: q has d_s={d_s}, S has {d2}")
    k = route_k(top_k, C)
    q = torch.empty(R, d_s, dtype=torch.float32, device=dev)
    gate = torch.empty(R, dtype=torch.float32, device=dev) if gate_w is not None else None
    rstd = torch.empty(R, dtype=torch.float32, device=dev)
    idx = torch.empty(R, k, dtype=torch.int32, device=dev)
    wk = torch.empty(R, k, dtype=torch.float32, device=dev)
    w = torch.empty(R, C, dtype=torch.float32, device=dev)
    lg = torch.empty(R, C, dtype=torch.float32, device=dev) if want_logits else None
    b_in, gate_w = _f32(b_in, "b_in"), _f32(gate_w, "gate_w")
    gb, gb_dev = _dev_scalar(gate_b, "gate_b")
    if n_chunks_of is not None:
        n_chunks_of = n_chunks_of.to(torch.int32).contiguous()
    if row_w is not None:
        row_w = _f32(row_w.reshape(-1), "row_w")
        if row_w.numel() != R:
            raise ValueError(f"project_in_route: row_w has {row_w.numel()} entries for {R} rows")
    with _on_device(dev):
        ws = _workspace(N.lib().xencb_project_in_workspace(R, d_m, d_s), dev)
        rc = N.lib().xencb_project_in_route(
            _ptr(h2), _hdt(h2, "h"), R, d_m, _ptr(w_in), _ptr(w_prep), _ptr(b_in), d_s, N.PIN_RMS | N.PIN_L2,
            _ptr(gate_w), gb, _ptr(gb_dev), None, None, 0, eps, _ptr(q), _ptr(gate), _ptr(rstd), None, _ptr(S), C,
            _ptr(n_chunks_of), int(rows_per_lib), n_lib, float(route_temp), int(top_k), _ptr(row_w), _ptr(idx),
            _ptr(wk), _ptr(w), _ptr(lg), _ptr(ws), ws.numel(), _stream(dev))
        if rc == N.ENOTSUP:  # nothing was launched: the two calls
            q, g2, rstd, _ = project_in(h2, w_in, b_in, gate_w=gate_w, gate_b=gate_b, eps=eps, w_prep=w_prep)
            idx, wk, w, lg = route(q, S, rows_per_lib=rows_per_lib, top_k=top_k, route_temp=route_temp,
                                   n_chunks_of=n_chunks_of, want_logits=want_logits, row_w=row_w)
            return q, g2, rstd, idx, wk, w, lg
        N.check(rc, "xencb_project_in_route")
    return q, gate, rstd, idx, wk, w, lg


def project_in_route_lse(h2: torch.Tensor, w_in: torch.Tensor, b_in=None, *, S: torch.Tensor, rows_per_lib: int,
                         route_temp: float, n_chunks_of: Optional[torch.Tensor] = None,
                         header_out: Optional[torch.Tensor] = None, eps: float = 1e-6,
                         w_prep: Optional[torch.Tensor] = None):
    """project_in (rms + L2) and the dense shard routing of route_lse in one pass after the GEMM
    (xencb_project_in_route_lse): (q, w [R, C] = e^(l - max), header [R, 4] = (max, sum, 0, 0)), the same values as
    project_in then route_lse. Shapes the fused form does not take run the two calls."""
    dev = _cuda("project_in_route_lse", h2, w_in, b_in, S, n_chunks_of)
    h2 = h2.contiguous()
    w_in = _f32(w_in, "w_in")
    S = _f32(S, "S")
    R, d_m = h2.shape
    d_s = w_in.shape[0]
    if w_in.shape[1] != d_m:
        raise ValueError(f"w_in is {tuple(w_in.shape)}, expected [d_s, {d_m}] (nn.Linear layout)")
    n_lib, C, d2 = S.shape
    if d2 != d_s:
        raise ValueError(f"project_in_route_lse: q has d_s={d_s}, S has {d2}")
    if header_out is None:
        header_out = torch.empty(R, 4, dtype=torch.float32, device=dev)
    elif header_out.dtype != torch.float32 or tuple(header_out.shape) != (R, 4) or not header_out.is_contiguous():
        raise ValueError("project_in_route_lse: header_out must be a contiguous float32 [R, 4] tensor")
    if n_chunks_of is not None:
        n_chunks_of = n_chunks_of.to(torch.int32).contiguous()
    two_calls = int(rows_per_lib) >= 64
    if not two_calls:
        q = torch.empty(R, d_s, dtype=torch.float32, device=dev)
        rstd = torch.empty(R, dtype=torch.float32, device=dev)
        w = torch.empty(R, C, dtype=torch.float32, device=dev)
        b_in = _f32(b_in, "b_in")
        with _on_device(dev):
            ws = _workspace(N.lib().xencb_project_in_workspace(R, d_m, d_s), dev)
            rc = N.lib().xencb_project_in_route_lse(
                _ptr(h2), _hdt(h2, "h"), R, d_m, _ptr(w_in), _ptr(w_prep), _ptr(b_in), d_s, N.PIN_RMS | N.PIN_L2,
                None, 0.0, None, eps, _ptr(q), None, _ptr(rstd), _ptr(S), C, _ptr(n_chunks_of), int(rows_per_lib),
                n_lib, float(route_temp), _ptr(w), _ptr(header_out), _ptr(ws), ws.numel(), _stream(dev))
            if rc != N.ENOTSUP:
                N.check(rc, "xencb_project_in_route_lse")
                return q, w, header_out
    q, _, _, _ = project_in(h2, w_in, b_in, eps=eps, w_prep=w_prep)
    w, _ = route_lse(q, S, rows_per_lib=rows_per_lib, route_temp=route_temp, n_chunks_of=n_chunks_of,
                     header_out=header_out)
    return q, w, header_out


def project_out(r: torch.Tensor, w_out: torch.Tensor, h2: torch.Tensor, *, b_out=None, scale: float = 1.0,
                log_scale: Optional[torch.Tensor] = None, gate=None, sel_w=None, log_alpha=0.0, pos_mask=None,
                want_delta: bool = True, h_out: Optional[torch.Tensor] = None, want_rel: bool = False,
                w_prep: Optional[torch.Tensor] = None, prefer_prep: bool = False):
    """(delta | None, h_out | None, rel | None).

    d = scale * exp(log_scale) * gate * (r @ w_out^T + b_out), w_out [d_m, d_s] (nn.Linear); optional
    LayerSelector matched norm with per-row weight sel_w and log_alpha (a number or a one-element device tensor;
    log_scale is a one-element device tensor or None);
    d *= pos_mask; delta = d in h2's dtype; h_out = h2 + delta; rel = ||delta|| / (||h2|| + 1e-6).
    w_prep: weights_prep(w_out) for the 3xF16 GEMM."""
    dev = _cuda("project_out", r, w_out, h2, b_out, gate, sel_w, pos_mask, h_out)
    r = _f32(r, "r")
    w_out = _f32(w_out, "w_out")
    h2 = h2.contiguous()
    R, d_s = r.shape
    d_m = w_out.shape[0]
    if w_out.shape[1] != d_s or h2.shape != (R, d_m):
        raise ValueError(f"project_out: r {tuple(r.shape)}, w_out {tuple(w_out.shape)}, h {tuple(h2.shape)}")
    delta = torch.empty_like(h2) if want_delta else None
    if h_out is not None and (h_out.shape != h2.shape or h_out.dtype != h2.dtype or not h_out.is_contiguous()):
        raise ValueError("project_out: h_out must match h (shape, dtype, contiguous)")
    rel = torch.empty(R, dtype=torch.float32, device=dev) if want_rel else None
    b_out, gate = _f32(b_out, "b_out"), _f32(gate, "gate")
    sel_w, pos_mask = _f32(sel_w, "sel_w"), _f32(pos_mask, "pos_mask")
    la, la_dev = _dev_scalar(log_alpha, "log_alpha")
    ls_dev = None if log_scale is None else _dev_scalar(log_scale, "log_scale")[1]
    with _on_device(dev):
        ws_bytes = N.lib().xencb_project_out_workspace(R, d_s, d_m)
        ws = _workspace(ws_bytes, dev)
        w_arg = None if (prefer_prep and w_prep is not None) else w_out
        N.call("xencb_project_out", _ptr(r), R, d_s, _ptr(w_arg), _ptr(w_prep), _ptr(b_out), d_m, float(scale),
               _ptr(ls_dev),
               _ptr(gate), _ptr(sel_w), la, _ptr(la_dev), _ptr(pos_mask), _ptr(h2), _hdt(h2, "h"), _ptr(delta),
               _ptr(h_out), _ptr(rel), _ptr(ws), ws.numel(), _stream(dev))
    return delta, h_out, rel


# ------------------------------------------------------------------------------------------------ routing
def route_k(top_k: int, n_chunks: int) -> int:
    return int(top_k) if 0 < int(top_k) < int(n_chunks) else int(n_chunks)


def route(q: torch.Tensor, S: torch.Tensor, *, rows_per_lib: int, top_k: int, route_temp: float,
          n_chunks_of: Optional[torch.Tensor] = None, want_logits: bool = False,
          row_w: Optional[torch.Tensor] = None):
    """(idx [R, k] int32, wk [R, k], w_dense [R, C], logits [R, C] | None); S is [n_lib, C, d_s] float32.
    row_w [R] (optional): rows with weight 0 get idx -1 / wk 0 (the read skips them); w_dense is unaffected."""
    dev = _cuda("route", q, S, n_chunks_of, row_w)
    q = _f32(q, "q")
    S = _f32(S, "S")
    R, d_s = q.shape
    n_lib, C, d2 = S.shape
    if d2 != d_s:
        raise ValueError(f"route: q has d_s={d_s}, S has {d2}")
    k = route_k(top_k, C)
    idx = torch.empty(R, k, dtype=torch.int32, device=dev)
    wk = torch.empty(R, k, dtype=torch.float32, device=dev)
    w = torch.empty(R, C, dtype=torch.float32, device=dev)
    lg = torch.empty(R, C, dtype=torch.float32, device=dev) if want_logits else None
    if n_chunks_of is not None:
        n_chunks_of = n_chunks_of.to(torch.int32).contiguous()
    if row_w is not None:
        row_w = _f32(row_w.reshape(-1), "row_w")
        if row_w.numel() != R:
            raise ValueError(f"route: row_w has {row_w.numel()} entries for {R} rows")
    with _on_device(dev):
        N.call("xencb_route", _ptr(q), R, d_s, _ptr(S), C, _ptr(n_chunks_of), int(rows_per_lib), n_lib,
               float(route_temp), int(top_k), _ptr(row_w), _ptr(idx), _ptr(wk), _ptr(w), _ptr(lg), _stream(dev))
    return idx, wk, w, lg


# ------------------------------------------------------------------------------------------------ read
def _vpool(pages) -> Optional[torch.Tensor]:
    v = pages.vslots
    if v is None:
        return None
    if v.shape != pages.slots.shape or v.dtype != pages.slots.dtype or v.device != pages.slots.device \
            or not v.is_contiguous():
        raise ValueError("Pages.vslots must match slots (shape, dtype, device) and be contiguous")
    return v


@dataclass
class Pages:
    """Device view of one depth of one or more Libraries, in the layout the read kernels take.

    slots    [P, page_rows, d_s] pool (float16 / bfloat16 / float32); page p = slots[p]
    page_of  [n_lib, C] int32 page of chunk c of Library l
    n_valid  [n_lib, C] int32 valid rows (the reference's mask, as a length)
    S        [n_lib, C, d_s] float32 summary keys
    n_chunks_of [n_lib] int32 chunks per Library (None: all have C)
    vslots   untied value pool (None: V = K, tied)"""

    slots: torch.Tensor
    page_of: torch.Tensor
    n_valid: torch.Tensor
    S: torch.Tensor
    n_chunks_of: Optional[torch.Tensor] = None
    vslots: Optional[torch.Tensor] = None  # untied values (harvest="attn"): same shape and dtype as slots

    @property
    def n_lib(self) -> int:
        return int(self.page_of.shape[0])

    @property
    def n_chunks(self) -> int:
        return int(self.page_of.shape[1])

    @property
    def d_s(self) -> int:
        return int(self.slots.shape[-1])

    @property
    def page_rows(self) -> int:
        return int(self.slots.shape[1])

    @property
    def device(self) -> torch.device:
        return self.slots.device


def read_decode(q: torch.Tensor, pages: Pages, idx: torch.Tensor, wk: torch.Tensor, *, rows_per_lib: int,
                read_temp: float = 12.0, read_softmax: bool = True, sparse: bool = False) -> torch.Tensor:
    """r [R, d_s] float32: the masked two-level read over each row's routed chunks. sparse=True plans for calls
    in which many rows read nothing (a selector's row mask): 128-row pieces, only the live ones listed on the
    device (xencb_read_decode_sparse); the same result within float32 rounding."""
    dev = _cuda("read_decode", q, pages.slots, pages.page_of, pages.n_valid, idx, wk)
    q = _f32(q, "q")
    wk = _f32(wk, "wk")
    R, d_s = q.shape
    slots = pages.slots
    if not slots.is_contiguous():
        raise ValueError("read_decode: the slot pool must be contiguous")
    if slots.shape[-1] != d_s:
        raise ValueError(f"read_decode: q has d_s={d_s}, slots have {slots.shape[-1]}")
    if idx.dtype != torch.int32 or idx.shape != wk.shape or idx.shape[0] != R:
        raise ValueError("read_decode: idx must be int32 [R, k] matching wk")
    k = int(idx.shape[1])
    idx = idx.contiguous()
    r = torch.empty(R, d_s, dtype=torch.float32, device=dev)
    dt = _hdt(slots, "slots")
    page_rows = pages.page_rows
    with _on_device(dev):
        name = "xencb_read_decode_sparse" if sparse else "xencb_read_decode"
        ws_bytes = getattr(N.lib(), name + "_workspace")(R, k, d_s, page_rows, dt)
        if ws_bytes == 0:
            N.check(N.EINVAL, "read_decode_workspace")
        ws = _workspace(ws_bytes, dev)
        N.call(name, _ptr(q), R, d_s, _ptr(slots), _ptr(_vpool(pages)), dt, slots.shape[0],
               page_rows * d_s, page_rows,
               _ptr(pages.page_of), _ptr(pages.n_valid), pages.n_chunks, int(rows_per_lib), pages.n_lib,
               _ptr(idx), _ptr(wk), k, float(read_temp), int(bool(read_softmax)), _ptr(r), _ptr(ws),
               ws.numel(), _stream(dev))
    return r


def read_attn(q: torch.Tensor, pages: Pages, idx: torch.Tensor, wk: torch.Tensor, *, row: int, rows_per_lib: int,
              read_temp: float = 12.0, read_softmax: bool = True) -> torch.Tensor:
    """[C, page_rows] float32: the route-weighted slot attention of query row `row` (record_attn,
    xenc/injector.py:259-260); zeros for chunks the row was not routed to and rows past n_valid."""
    dev = _cuda("read_attn", q, pages.slots, pages.page_of, pages.n_valid, idx, wk)
    q = _f32(q, "q")
    wk = _f32(wk, "wk")
    R, d_s = q.shape
    if not 0 <= int(row) < R:
        raise ValueError(f"read_attn: row {row} outside [0, {R})")
    if idx.dtype != torch.int32 or idx.shape != wk.shape or idx.shape[0] != R:
        raise ValueError("read_attn: idx must be int32 [R, k] matching wk")
    idx = idx.contiguous()
    out = torch.empty(pages.n_chunks, pages.page_rows, dtype=torch.float32, device=dev)
    slots = pages.slots
    with _on_device(dev):
        N.call("xencb_read_attn", _ptr(q), int(row), d_s, _ptr(slots), _hdt(slots, "slots"), slots.shape[0],
               pages.page_rows * d_s, pages.page_rows, _ptr(pages.page_of), _ptr(pages.n_valid), pages.n_chunks,
               int(rows_per_lib), pages.n_lib, _ptr(idx), _ptr(wk), int(idx.shape[1]), float(read_temp),
               int(bool(read_softmax)), _ptr(out), _stream(dev))
    return out


def read_forced(fa: torch.Tensor, pages: Pages, n_rows: int, *, r0: Optional[torch.Tensor] = None,
                norm_match: bool = False):
    """(r [n_rows, d_s], scale [n_rows]): the read with the given addressing fa [C, page_rows] in place of the
    computed one (force_attn, xenc/injector.py:246-258); with norm_match each row is scaled to ||r0[row]|| (r0 the
    ordinary read) over ||fa @ K||. One Library."""
    dev = _cuda("read_forced", fa, pages.slots, pages.page_of, pages.n_valid, r0)
    if pages.n_lib != 1:
        raise NotImplementedError("read_forced: force_attn addresses one Library")
    fa = _f32(fa, "force_attn")
    C, P = pages.n_chunks, pages.page_rows
    if tuple(fa.shape) != (C, P):
        raise ValueError(f"force_attn {tuple(fa.shape)} != library [C,N] {(C, P)}")
    d_s = pages.d_s
    r0 = _f32(r0, "r0")
    if norm_match and (r0 is None or tuple(r0.shape) != (int(n_rows), d_s)):
        raise ValueError(f"read_forced: norm_match needs r0 [{n_rows}, {d_s}]")
    r = torch.empty(int(n_rows), d_s, dtype=torch.float32, device=dev)
    scale = torch.empty(int(n_rows), dtype=torch.float32, device=dev)
    slots = pages.slots
    with _on_device(dev):
        ws = _workspace(N.lib().xencb_read_forced_workspace(C, d_s), dev)
        N.call("xencb_read_forced", _ptr(fa), d_s, _ptr(slots), _ptr(_vpool(pages)), _hdt(slots, "slots"),
               slots.shape[0], P * d_s, P, _ptr(pages.page_of), _ptr(pages.n_valid), C, _ptr(r0), int(n_rows),
               int(bool(norm_match)), _ptr(r), _ptr(scale), _ptr(ws), ws.numel(), _stream(dev))
    return r, scale


def read_multi(q: torch.Tensor, pages: Pages, w: torch.Tensor, *, rows_per_lib: int, read_temp: float = 12.0,
               read_softmax: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """r [R, d_s] float32 = sum_c w[row, c] * read(q[row], chunk c): the many-query read, in which up to 8 rows of
    a Library share each slot row fetched from HBM. w [R, C] float32 (0 = chunk not routed). Raises
    NotImplementedError for slot types / widths the kernel does not take (see read_weighted)."""
    dev = _cuda("read_multi", q, pages.slots, pages.page_of, pages.n_valid, w)
    q = _f32(q, "q")
    w = _f32(w, "w")
    R, d_s = q.shape
    slots = pages.slots
    if not slots.is_contiguous():
        raise ValueError("read_multi: the slot pool must be contiguous")
    if slots.shape[-1] != d_s:
        raise ValueError(f"read_multi: q has d_s={d_s}, slots have {slots.shape[-1]}")
    if tuple(w.shape) != (R, pages.n_chunks):
        raise ValueError(f"read_multi: w must be [{R}, {pages.n_chunks}], got {tuple(w.shape)}")
    if out is None:
        out = torch.empty(R, d_s, dtype=torch.float32, device=dev)
    elif out.dtype != torch.float32 or tuple(out.shape) != (R, d_s) or not out.is_contiguous():
        raise ValueError("read_multi: out must be a contiguous float32 [R, d_s] tensor")
    dt = _hdt(slots, "slots")
    nco = pages.n_chunks_of
    if nco is not None:
        nco = nco.to(torch.int32).contiguous()
    with _on_device(dev):
        ws_bytes = N.lib().xencb_read_multi_workspace(R, int(rows_per_lib), pages.n_chunks, d_s, pages.page_rows, dt)
        if ws_bytes == 0:  # the shapes were checked above: the kernel does not take this slot type / width
            N.check(N.ENOTSUP, "read_multi_workspace")
        ws = _workspace(ws_bytes, dev)
        N.call("xencb_read_multi", _ptr(q), R, d_s, _ptr(slots), _ptr(_vpool(pages)), dt, slots.shape[0],
               pages.page_rows * d_s,
               pages.page_rows, _ptr(pages.page_of), _ptr(pages.n_valid), pages.n_chunks, _ptr(nco),
               int(rows_per_lib), pages.n_lib, _ptr(w), float(read_temp), int(bool(read_softmax)), _ptr(out),
               _ptr(ws), ws.numel(), _stream(dev))
    return out


def read_prefill(q: torch.Tensor, pages: Pages, w: torch.Tensor, *, rows_per_lib: int, read_temp: float = 12.0,
                 read_softmax: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The dense read for many query tokens per Library on the tensor cores (two tcgen05 GEMMs): the same result
    as read_multi. Needs f16 slots, d_s % 64 == 0, page_rows <= 512 (NotImplementedError otherwise)."""
    dev = _cuda("read_prefill", q, pages.slots, pages.page_of, pages.n_valid, w)
    q = _f32(q, "q")
    w = _f32(w, "w")
    R, d_s = q.shape
    slots = pages.slots
    if slots.dtype != torch.float16 or d_s % 64 or pages.page_rows > 512:
        raise NotImplementedError("read_prefill: f16 slots, d_s % 64 == 0 and page_rows <= 512 are required")
    if not slots.is_contiguous() or slots.shape[-1] != d_s:
        raise ValueError(f"read_prefill: slots must be a contiguous [P, page_rows, {d_s}] pool")
    if tuple(w.shape) != (R, pages.n_chunks):
        raise ValueError(f"read_prefill: w must be [{R}, {pages.n_chunks}], got {tuple(w.shape)}")
    if out is None:
        out = torch.empty(R, d_s, dtype=torch.float32, device=dev)
    nco = pages.n_chunks_of
    if nco is not None:
        nco = nco.to(torch.int32).contiguous()
    with _on_device(dev):
        ws_bytes = N.lib().xencb_read_prefill_workspace(R, pages.n_chunks, d_s, pages.page_rows)
        ws = _workspace(ws_bytes, dev)
        N.call("xencb_read_prefill", _ptr(q), R, d_s, _ptr(slots), _ptr(_vpool(pages)), N.F16, slots.shape[0],
               pages.page_rows * d_s,
               pages.page_rows, _ptr(pages.page_of), _ptr(pages.n_valid), pages.n_chunks, _ptr(nco),
               int(rows_per_lib), pages.n_lib, _ptr(w), float(read_temp), int(bool(read_softmax)), _ptr(out),
               _ptr(ws), ws.numel(), _stream(dev))
    return out


def multi_supported(pages: Pages, n_rows: int, rows_per_lib: int) -> bool:
    """Whether read_multi takes this slot pool (f16 / bf16 slots, d_s % 16 == 0, the stages fit on chip)."""
    if pages.slots.dtype not in (torch.float16, torch.bfloat16) or pages.d_s % 16:
        return False
    with _on_device(pages.device):
        return N.lib().xencb_read_multi_workspace(int(n_rows), int(rows_per_lib), pages.n_chunks, pages.d_s,
                                                  pages.page_rows, _hdt(pages.slots, "slots")) > 0


def read_weighted(q: torch.Tensor, pages: Pages, w: torch.Tensor, *, rows_per_lib: int, read_temp: float = 12.0,
                  read_softmax: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """read_multi where the kernel takes the shape; otherwise the decode read over every chunk of each row
    (idx = 0..C-1, wk = w), which gives the same result with one chunk read per (row, chunk)."""
    multi_ok = multi_supported(pages, q.shape[0], rows_per_lib)
    if multi_ok:
        return read_multi(q, pages, w, rows_per_lib=rows_per_lib, read_temp=read_temp, read_softmax=read_softmax,
                          out=out)
    R = q.shape[0]
    idx = torch.arange(pages.n_chunks, dtype=torch.int32, device=q.device).expand(R, -1).contiguous()
    r = read_decode(q, pages, idx, w.contiguous(), rows_per_lib=rows_per_lib, read_temp=read_temp,
                    read_softmax=read_softmax)
    if out is not None:
        out.copy_(r)
        return out
    return r


def route_lse(q: torch.Tensor, S: torch.Tensor, *, rows_per_lib: int, route_temp: float,
              n_chunks_of: Optional[torch.Tensor] = None, header_out: Optional[torch.Tensor] = None):
    """Dense routing of a chunk shard: (w [R, C] = e^(l - max), header [R, 4] = (max, sum, 0, 0))."""
    dev = _cuda("route_lse", q, S, n_chunks_of)
    q = _f32(q, "q")
    S = _f32(S, "S")
    R, d_s = q.shape
    n_lib, C, d2 = S.shape
    if d2 != d_s:
        raise ValueError(f"route_lse: q has d_s={d_s}, S has {d2}")
    w = torch.empty(R, C, dtype=torch.float32, device=dev)
    if header_out is None:
        header_out = torch.empty(R, 4, dtype=torch.float32, device=dev)
    elif header_out.dtype != torch.float32 or tuple(header_out.shape) != (R, 4) or not header_out.is_contiguous():
        raise ValueError("route_lse: header_out must be a contiguous float32 [R, 4] tensor")
    if n_chunks_of is not None:
        n_chunks_of = n_chunks_of.to(torch.int32).contiguous()
    with _on_device(dev):
        N.call("xencb_route_lse", _ptr(q), R, d_s, _ptr(S), C, _ptr(n_chunks_of), int(rows_per_lib), n_lib,
               float(route_temp), _ptr(w), _ptr(header_out), _stream(dev))
    return w, header_out


def shard_block(n_rows: int, d_s: int, device, dtype=torch.float32) -> torch.Tensor:
    """One shard's partial as a flat float32 block: n_rows headers of 4 floats, then n_rows x d_s accumulators."""
    return torch.empty(n_rows * 4 + n_rows * d_s, dtype=dtype, device=device)


def shard_views(block: torch.Tensor, n_rows: int, d_s: int):
    """(header [n_rows, 4], acc [n_rows, d_s]) views of a shard block."""
    return block[:n_rows * 4].view(n_rows, 4), block[n_rows * 4:n_rows * 4 + n_rows * d_s].view(n_rows, d_s)


def shard_merge(parts: torch.Tensor, n_shards: int, n_rows: int, d_s: int,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """r [n_rows, d_s] from n_shards shard blocks laid end to end (what an all-gather of the blocks gives)."""
    dev = _cuda("shard_merge", parts)
    parts = _f32(parts, "parts")
    if parts.numel() != n_shards * (n_rows * 4 + n_rows * d_s):
        raise ValueError(f"shard_merge: parts has {parts.numel()} floats, expected {n_shards} blocks of "
                         f"{n_rows * 4 + n_rows * d_s}")
    if out is None:
        out = torch.empty(n_rows, d_s, dtype=torch.float32, device=dev)
    with _on_device(dev):
        N.call("xencb_shard_merge", _ptr(parts), int(n_shards), int(n_rows), int(d_s), _ptr(out), _stream(dev))
    return out


# ------------------------------------------------------------------------------------------------ selector
def selector_logits(h2: torch.Tensor, u_w: torch.Tensor, u_b=None, *, rms: bool, eps: float = 1e-6) -> torch.Tensor:
    dev = _cuda("selector_logits", h2, u_w, u_b)
    h2 = h2.contiguous()
    u_w, u_b = _f32(u_w, "u.weight"), _f32(u_b, "u.bias")
    z = torch.empty(h2.shape[0], u_w.shape[0], dtype=torch.float32, device=dev)
    with _on_device(dev):
        N.call("xencb_selector_logits", _ptr(h2), _hdt(h2, "h"), h2.shape[0], h2.shape[1], _ptr(u_w), _ptr(u_b),
               u_w.shape[0], int(bool(rms)), eps, _ptr(z), _stream(dev))
    return z


def selector_weights(z: torch.Tensor, k: int, straight_through: bool = False) -> torch.Tensor:
    dev = _cuda("selector_weights", z)
    z2 = _f32(z.reshape(-1, z.shape[-1]), "z")
    w = torch.empty_like(z2)
    with _on_device(dev):
        N.call("xencb_selector_weights", _ptr(z2), z2.shape[0], z2.shape[1], int(k), int(bool(straight_through)),
               _ptr(w), _stream(dev))
    return w.view(z.shape)


def selector_apply(delta: torch.Tensor, h: torch.Tensor, w: torch.Tensor, pos: int, log_alpha: float) -> torch.Tensor:
    """LayerSelector.apply's matched-norm rescale (xenc/selector.py:106-110); returns delta's dtype."""
    dev = _cuda("selector_apply", delta, h, w)
    d2 = delta.reshape(-1, delta.shape[-1]).contiguous()
    h2 = h.reshape(-1, h.shape[-1]).contiguous()
    w2 = _f32(w.reshape(-1, w.shape[-1]), "w")
    if h2.shape != d2.shape or w2.shape[0] != d2.shape[0]:
        raise ValueError(f"selector_apply: delta {tuple(delta.shape)}, h {tuple(h.shape)}, w {tuple(w.shape)}")
    out = torch.empty_like(d2)
    with _on_device(dev):
        N.call("xencb_selector_apply", _ptr(d2), _hdt(d2, "delta"), _ptr(h2), _hdt(h2, "h"), d2.shape[0],
               d2.shape[1], _ptr(w2), w2.shape[1], int(pos), float(log_alpha), _ptr(out), _stream(dev))
    return out.view(delta.shape)


# ------------------------------------------------------------------------------------------------ summaries
def summaries(slots: torch.Tensor, page_of: torch.Tensor, n_valid: torch.Tensor) -> torch.Tensor:
    """S [n_lib, C, d_s] float32 = L2(mean of the valid rows of each chunk's page)."""
    dev = _cuda("summaries", slots, page_of, n_valid)
    if not slots.is_contiguous():
        raise ValueError("summaries: the slot pool must be contiguous")
    n_lib, C = page_of.shape
    d_s = slots.shape[-1]
    S = torch.empty(n_lib, C, d_s, dtype=torch.float32, device=dev)
    page_of = page_of.to(torch.int32).contiguous()
    n_valid = n_valid.to(torch.int32).contiguous()
    with _on_device(dev):
        N.call("xencb_summaries", _ptr(slots), _hdt(slots, "slots"), slots.shape[0], slots.shape[1] * d_s,
               slots.shape[1],
               _ptr(page_of), _ptr(n_valid), n_lib, C, d_s, _ptr(S), _stream(dev))
    return S


def library_build(rows: torch.Tensor, counts, *, page_rows: Optional[int] = None, mu: Optional[torch.Tensor] = None,
                  slot_dtype=torch.float16, slots: Optional[torch.Tensor] = None,
                  page_of: Optional[torch.Tensor] = None, want_summaries: bool = True):
    """Build one depth of a Library on the device from its chunks' rows (xenc/library.py:47-74).

    rows [n_rows, d_s] (f16 / bf16 / f32, on the GPU): every chunk's rows concatenated in chunk order;
    counts: the row count of each chunk (host ints). mu [d_s]: centering, K = L2(K - mu) on the valid rows.
    Writes the chunks into `slots` [P, page_rows, d_s] at pages `page_of` [C] (default: a new pool, page c =
    chunk c) with zero rows after each chunk's count. Returns (slots, n_valid [C] int32, S [C, d_s] float32 or
    None); S is computed from the float32 rows before they are rounded to the slot type."""
    dev = _cuda("library_build", rows, mu, slots, page_of)
    counts = [int(n) for n in (counts.tolist() if torch.is_tensor(counts) else counts)]
    C = len(counts)
    if C == 0:
        raise ValueError("library_build: a Library needs at least one chunk")
    if any(n < 0 for n in counts):
        raise ValueError("library_build: chunk row counts must be >= 0")
    if rows.dim() != 2 or not rows.is_contiguous():
        raise ValueError("library_build: rows must be a contiguous [n_rows, d_s] tensor")
    n_rows, d_s = rows.shape
    if sum(counts) != n_rows:
        raise ValueError(f"library_build: counts sum to {sum(counts)}, rows has {n_rows}")
    page_rows = int(page_rows if page_rows is not None else max(max(counts), 1))
    if max(counts) > page_rows:
        raise ValueError(f"library_build: a chunk has {max(counts)} rows, pages hold {page_rows}")
    if slots is None:
        slots = torch.empty(C, page_rows, d_s, dtype=slot_dtype, device=dev)
    elif not slots.is_contiguous() or slots.dim() != 3 or tuple(slots.shape[1:]) != (page_rows, d_s):
        raise ValueError(f"library_build: slots must be a contiguous [P, {page_rows}, {d_s}] pool")
    if page_of is None:
        if slots.shape[0] < C:
            raise ValueError(f"library_build: {C} chunks need {C} pages, the pool has {slots.shape[0]}")
        page_of = torch.arange(C, dtype=torch.int32, device=dev)
    page_of = page_of.to(device=dev, dtype=torch.int32).contiguous().view(-1)
    if page_of.numel() != C:
        raise ValueError(f"library_build: page_of has {page_of.numel()} entries for {C} chunks")
    if mu is not None:
        mu = _f32(mu.reshape(-1), "mu")
        if mu.numel() != d_s:
            raise ValueError(f"library_build: mu has {mu.numel()} entries, d_s={d_s}")
    start = torch.zeros(C + 1, dtype=torch.int64)
    start[1:] = torch.tensor(counts, dtype=torch.int64).cumsum(0)
    start = start.to(dev, non_blocking=True)
    n_valid = torch.empty(C, dtype=torch.int32, device=dev)
    S = torch.empty(C, d_s, dtype=torch.float32, device=dev) if want_summaries else None
    with _on_device(dev):
        ws_bytes = N.lib().xencb_library_build_workspace(C, d_s, page_rows)
        if ws_bytes == 0:
            N.check(N.EINVAL, "library_build_workspace")
        ws = _workspace(ws_bytes, dev)
        N.call("xencb_library_build", _ptr(rows), _hdt(rows, "rows"), n_rows, _ptr(start), C, d_s, _ptr(mu),
               _ptr(slots), _hdt(slots, "slots"), slots.shape[0], page_rows * d_s, page_rows, _ptr(page_of),
               _ptr(n_valid), _ptr(S), _ptr(ws), ws.numel(), _stream(dev))
    return slots, n_valid, S


# ------------------------------------------------------------------------------------------------ D8 top-k read
_POOL = {"max": 0, "mean": 1}


def select_scores(q: torch.Tensor, keys: torch.Tensor, n_valid: torch.Tensor, *, page_rows: int,
                  rows_per_lib: int, n_chunks_of: Optional[torch.Tensor] = None, query_pool: str = "max",
                  head_pool: str = "max") -> torch.Tensor:
    """Selection scores [R, C * page_rows] (xenc/topk_read.py:215-239).

    q [R, T, n_q, hd] float32: the reader's queries at the selection layer (T = 1 for query "last");
    keys [n_lib, C * page_rows, n_kv, hd] (float32 / float16): the selection keys on the Library's slot grid;
    n_valid [n_lib, C]; query_pool pools positions ("max" / "mean"), head_pool pools heads ("max" / "mean")."""
    dev = _cuda("select_scores", q, keys, n_valid, n_chunks_of)
    q = _f32(q, "q")
    if q.dim() != 4:
        raise ValueError("select_scores: q must be [R, T, n_q, hd]")
    R, T, n_q, hd = q.shape
    if keys.dim() != 4 or keys.shape[-1] != hd:
        raise ValueError(f"select_scores: keys must be [n_lib, slots, n_kv, {hd}]")
    n_lib, S, n_kv, _ = keys.shape
    n_lib2, C = n_valid.shape
    if n_lib2 != n_lib or S != C * int(page_rows):
        raise ValueError(f"select_scores: keys hold {S} slots per Library, n_valid gives {C} x {page_rows}")
    keys = keys.contiguous()
    nv = n_valid.to(torch.int32).contiguous()
    nco = None if n_chunks_of is None else n_chunks_of.to(torch.int32).contiguous()
    out = torch.empty(R, S, dtype=torch.float32, device=dev)
    with _on_device(dev):
        N.call("xencb_select_scores", _ptr(q), R, T, n_q, n_kv, hd, _ptr(keys), _hdt(keys, "keys"), S * n_kv * hd,
               int(page_rows), C, _ptr(nv), _ptr(nco), int(rows_per_lib), n_lib, _POOL[query_pool],
               _POOL[head_pool], _ptr(out), _stream(dev))
    return out


def select_topk(scores: torch.Tensor, k: int):
    """(idx [R, k] int32, values [R, k] float32): the k largest scores per row, sorted descending (ties: lower
    slot first) -- sc.topk(k) of xenc/topk_read.py:254."""
    dev = _cuda("select_topk", scores)
    scores = _f32(scores, "scores")
    R, S = scores.shape
    idx = torch.empty(R, int(k), dtype=torch.int32, device=dev)
    val = torch.empty(R, int(k), dtype=torch.float32, device=dev)
    with _on_device(dev):
        N.call("xencb_select_topk", _ptr(scores), R, S, int(k), _ptr(idx), _ptr(val), _stream(dev))
    return idx, val


def topk_read(q: torch.Tensor, pages: Pages, idx: torch.Tensor, *, read_temp: float = 12.0,
              read_softmax: bool = True, want_attn: bool = False):
    """(r [R, d_s], attn [R, k] | None): the read restricted to the selected slots (xenc/topk_read.py:392-413).

    idx [n_sets, k] int32 flat slot indices (chunk * page_rows + row); rows are split evenly over the index
    sets in order, and set b reads Library b when pages holds several Libraries."""
    dev = _cuda("topk_read", q, pages.slots, pages.page_of, idx)
    q = _f32(q, "q")
    R, d_s = q.shape
    slots = pages.slots
    if not slots.is_contiguous() or slots.shape[-1] != d_s:
        raise ValueError(f"topk_read: slots must be a contiguous [P, page_rows, {d_s}] pool")
    if idx.dtype != torch.int32 or idx.dim() != 2:
        raise ValueError("topk_read: idx must be int32 [n_sets, k]")
    n_sets, k = idx.shape
    idx = idx.contiguous()
    r = torch.empty(R, d_s, dtype=torch.float32, device=dev)
    attn = torch.empty(R, k, dtype=torch.float32, device=dev) if want_attn else None
    with _on_device(dev):
        N.call("xencb_topk_read", _ptr(q), R, d_s, _ptr(slots), _ptr(_vpool(pages)), _hdt(slots, "slots"),
               slots.shape[0], pages.page_rows * d_s, pages.page_rows, _ptr(pages.page_of), pages.n_chunks,
               pages.n_lib, _ptr(idx), n_sets, k, float(read_temp), int(bool(read_softmax)), _ptr(r), _ptr(attn),
               _stream(dev))
    return r, attn


def read_kernel_events(before, after) -> None:
    """Instrumentation: the next read_decode on this thread records the torch.cuda.Events `before` / `after`
    (timing enabled) right around its main read kernel, leaving the merge out of the interval. One-shot."""
    for ev in (before, after):
        if ev is not None and not ev.cuda_event:
            ev.record()  # torch creates the CUDA event on its first record
    N.call("xencb_read_kernel_events", before.cuda_event if before is not None else None,
           after.cuda_event if after is not None else None)


def wait_selftest(dev: torch.device, limit_cycles: int = 2_000_000) -> int:
    """Run the bounded-wait self-test on `dev` (a wait that nothing satisfies must give up); returns the
    kernel's result (0 = gave up). The device status then carries XENCB_DEV_TIMEOUT."""
    dev = torch.device(dev)
    res = torch.full((1,), -1, dtype=torch.int32, device=dev)
    with _on_device(dev):
        N.call("xencb_wait_selftest", int(limit_cycles), _ptr(res), _stream(dev))
    return int(res.item())


def device_status(dev: torch.device, clear: bool = True) -> int:
    """Synchronise the current stream of `dev` and return the device status bits (XENCB_DEV_*)."""
    v = ctypes.c_uint(0)
    with _on_device(dev):
        N.call("xencb_device_status", _stream(dev), int(clear), ctypes.byref(v))
    return int(v.value)
