"""Parity at BASELINE.json's own shapes, through the product path the bench times.

* config 2 -- 64 documents x (64 chunks x 512 fp16 slots, the last chunk ragged), d_s 2048, d_m 4096, top-4: every
  document over four decode steps through LibraryInjector (graph-replayed hook), routing sets for all 256 tokens,
  the smallest top-k tie margin reported;
* config 3 -- 8 documents x 2048 tokens, 128 chunks x 512 slots, dense routing: bf16 hidden states through the
  input projection, dense routing, the tensor-core prefill read and the output projection, on 64 sampled tokens
  spread over all 8 documents;
* config 4 -- 32 documents x 8 candidate depths x (32 chunks x 512 slots), d_s 2048, d_m 5120, LayerSelector top-2
  depths, top-4 chunks per depth: the 8 hooked layers in order through LibraryInjector + LayerSelector.

Each is checked against the CPU oracle (oracle/xenc_oracle.py, the numpy restatement of xenc/injector.py:220-273
and xenc/selector.py:59-110): routing index sets identical per token, outputs within TOL relative to the largest
reference value. Each test prints one `PARITY {json}` line with the largest relative errors reached and the
smallest gap between the k-th and (k+1)-th routing logit (how close the routing came to a tie)."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import xenc_oracle as X
from tests._fixtures import TOL, rel_err, topk_sets

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _unit_pool(n_pages: int, N: int, d: int, g: torch.Generator, dev) -> torch.Tensor:
    """n_pages x N x d float16 rows, each a Gaussian row normalised to unit length (the configs' slots)."""
    pool = torch.empty(n_pages, N, d, dtype=torch.float16, device=dev)
    for c0 in range(0, n_pages, 64):
        x = torch.randn(min(64, n_pages - c0), N, d, generator=g, device=dev)
        pool[c0:c0 + x.shape[0]] = (x / x.norm(dim=-1, keepdim=True)).half()
    return pool


def _doc_slots(pool: torch.Tensor, nv_row: np.ndarray, C: int, b: int):
    """(K [C, N, d] float32 with rows past n_valid zeroed, mask [C, N]) of document b, on the host."""
    K = pool[b * C:(b + 1) * C].cpu().numpy().astype(np.float32)  # fp16 -> fp32 is exact
    M = np.arange(K.shape[1])[None, :] < nv_row[:, None]
    K[~M] = 0.0
    return K, M


def _tie_margin(logit: np.ndarray, k: int) -> float:
    """Smallest gap between the k-th and (k+1)-th largest logit over the rows."""
    s = -np.sort(-logit, axis=-1)
    return float((s[:, k - 1] - s[:, k]).min())


class _IdReader(torch.nn.Module):
    """A reader whose L blocks return their input: the hooks see the hidden state directly."""

    def __init__(self, L: int, dev):
        super().__init__()
        self.layers = torch.nn.ModuleList([torch.nn.Identity() for _ in range(L)])
        self._p = torch.nn.Parameter(torch.zeros(1, device=dev), requires_grad=False)

    def forward(self, x):
        for blk in self.layers:
            x = blk(x)
        return x


def test_config2_all_documents_four_steps(dev):
    from kv_skill_v2_b200 import LibraryInjector, LinearInterface, PagedLibrary, ops
    B, C, N, d_s, d_m, top_k, steps = 64, 64, 512, 2048, 4096, 4, 4
    g = torch.Generator(device=dev).manual_seed(2)
    slots = _unit_pool(B * C, N, d_s, g, dev)
    nv = torch.full((B, C), N, dtype=torch.int32, device=dev)
    nv[:, -1] = torch.randint(1, N + 1, (B,), generator=g, device=dev, dtype=torch.int32)
    for b in range(B):  # rows past n_valid are zero, as the Library pads them
        slots[b * C + C - 1, int(nv[b, -1]):] = 0
    po = torch.arange(B * C, dtype=torch.int32, device=dev).view(B, C)
    pages = ops.Pages(slots=slots, page_of=po, n_valid=nv, S=ops.summaries(slots, po, nv))
    W_in = torch.randn(d_m, d_s, generator=g, device=dev) * 0.02
    W_out = torch.randn(d_s, d_m, generator=g, device=dev) * 0.02
    itf = LinearInterface(W_in, W_out, [0]).to(dev).requires_grad_(False)
    inj = LibraryInjector(_IdReader(1, dev), itf, top_k=top_k)
    inj.load_library(PagedLibrary({0: pages}))
    hs = torch.randn(steps, B, 1, d_m, generator=g, device=dev)
    outs, routes = [], []
    buf = torch.empty(B, 1, d_m, device=dev)
    with torch.inference_mode():
        for t in range(steps):  # the first step runs eagerly and captures; later steps replay the graph
            buf.copy_(hs[t])
            outs.append(inj.model(buf).clone())
            routes.append(inj.last_route.reshape(B, C).clone())
    inj.detach()
    nv_h = nv.cpu().numpy()
    Wi, Wo = W_in.cpu().numpy(), W_out.cpu().numpy()
    H = hs.cpu().numpy().reshape(steps, B, d_m)
    err_d = err_S = 0.0
    margin = np.inf
    mismatches = []
    for b in range(B):
        K, M = _doc_slots(slots, nv_h[b], C, b)
        S_ref = X.summaries(K, M)
        err_S = max(err_S, rel_err(pages.S[b], S_ref))
        ref = X.branch(H[:, b], Wi, Wo, K, M, S_ref, top_k=top_k)
        margin = min(margin, _tie_margin(ref["logit"], top_k))
        got_sets = topk_sets(torch.stack([routes[t][b] for t in range(steps)]))
        for t, (gs, rs) in enumerate(zip(got_sets, topk_sets(ref["w"]))):
            if gs != rs:
                mismatches.append((b, t, sorted(gs), sorted(rs)))
        got_delta = torch.stack([outs[t][b, 0] for t in range(steps)]).cpu().numpy() - H[:, b]
        err_d = max(err_d, rel_err(got_delta, ref["delta"]))
    print("PARITY " + json.dumps({"config": 2, "tokens": B * steps, "routing_mismatches": len(mismatches),
                                  "min_topk_margin": margin, "max_rel_err_delta": err_d, "max_rel_err_S": err_S}))
    assert not mismatches, f"routing differs (doc, step, got, oracle): {mismatches[:4]}; min margin {margin:.3e}"
    assert err_S < 1e-5
    assert err_d < TOL
    assert ops.device_status(dev) == 0
    del slots, pages
    torch.cuda.empty_cache()


def test_config3_chain_from_bf16_hiddens(dev):
    from kv_skill_v2_b200 import ops
    B, T, C, N, d_s, d_m = 8, 2048, 128, 512, 2048, 4096
    g = torch.Generator(device=dev).manual_seed(3)
    slots = _unit_pool(B * C, N, d_s, g, dev)
    nv = torch.full((B, C), N, dtype=torch.int32, device=dev)
    nv[:, -1] = torch.randint(1, N + 1, (B,), generator=g, device=dev, dtype=torch.int32)
    for b in range(B):
        slots[b * C + C - 1, int(nv[b, -1]):] = 0
    po = torch.arange(B * C, dtype=torch.int32, device=dev).view(B, C)
    pages = ops.Pages(slots=slots, page_of=po, n_valid=nv, S=ops.summaries(slots, po, nv))
    W_in = torch.randn(d_s, d_m, generator=g, device=dev) * 0.02  # nn.Linear layout [out, in]
    W_out = torch.randn(d_m, d_s, generator=g, device=dev) * 0.02
    h = torch.randn(B * T, d_m, generator=g, device=dev).to(torch.bfloat16)
    P_in, P_out = ops.weights_prep(W_in), ops.weights_prep(W_out)
    with torch.inference_mode():  # the bench's step: 3xF16 projections, dense routing, tensor-core read
        q, _, _, _ = ops.project_in(h, W_in, w_prep=P_in)
        _, _, w, _ = ops.route(q, pages.S, rows_per_lib=T, top_k=0, route_temp=10.0)
        r = ops.read_prefill(q, pages, w, rows_per_lib=T, read_temp=12.0)
        h_out = torch.empty_like(h)
        ops.project_out(r, W_out, h, want_delta=False, h_out=h_out, w_prep=P_out)
        delta32, _, _ = ops.project_out(r, W_out, h.float(), want_delta=True, w_prep=P_out)
    torch.cuda.synchronize(dev)
    gs = torch.Generator().manual_seed(33)
    nv_h = nv.cpu().numpy()
    Wi, Wo = W_in.t().cpu().numpy(), W_out.t().cpu().numpy()
    errs = {"q": 0.0, "w": 0.0, "r": 0.0, "delta": 0.0, "h_out": 0.0}
    for b in range(B):
        tok = torch.randperm(T, generator=gs)[:8].sort().values + b * T
        td = tok.to(dev)
        hb = h[td].float().cpu().numpy()
        K, M = _doc_slots(slots, nv_h[b], C, b)
        ref = X.branch(hb, Wi, Wo, K, M, X.summaries(K, M), top_k=0)
        errs["q"] = max(errs["q"], rel_err(q[td], ref["q"]))
        errs["w"] = max(errs["w"], rel_err(w[td], ref["w"]))
        errs["r"] = max(errs["r"], rel_err(r[td], ref["r"]))
        errs["delta"] = max(errs["delta"], rel_err(delta32[td], ref["delta"]))
        # the bf16 output is h + delta rounded to bf16 (the hook's delta.to(h.dtype) and residual add,
        # xenc/injector.py:190-196): beyond one bf16 ulp of the exact sum, the error left is the delta's own
        want = torch.from_numpy(hb + ref["delta"])
        ulp = torch.ldexp(torch.ones_like(want), torch.frexp(want).exponent - 8).clamp_min(2.0 ** -126)
        excess = ((h_out[td].float().cpu() - want).abs() - ulp).clamp_min(0).max()
        errs["h_out"] = max(errs["h_out"], float(excess) / float(np.abs(ref["delta"]).max()))
    print("PARITY " + json.dumps({"config": 3, "tokens": 8 * B, **{f"max_rel_err_{k}": v for k, v in errs.items()}}))
    assert errs["q"] < 1e-5 and errs["w"] < 1e-4
    assert errs["r"] < TOL and errs["delta"] < TOL
    assert errs["h_out"] < TOL
    assert ops.device_status(dev) == 0
    del slots, pages
    torch.cuda.empty_cache()


def test_config4_selector_decode_full_shapes(dev):
    from kv_skill_v2_b200 import LayerSelector, LibraryInjector, LinearInterface, PagedLibrary, ops
    B, L, C, N, d_s, d_m, top_k, sel_k = 32, 8, 32, 512, 2048, 5120, 4, 2
    layers = list(range(L))
    g = torch.Generator(device=dev).manual_seed(4)
    po = torch.arange(B * C, dtype=torch.int32, device=dev).view(B, C)
    pools, nvs, pages = {}, {}, {}
    for li in layers:
        pool = _unit_pool(B * C, N, d_s, g, dev)
        nv = torch.full((B, C), N, dtype=torch.int32, device=dev)
        nv[:, -1] = torch.randint(1, N + 1, (B,), generator=g, device=dev, dtype=torch.int32)
        for b in range(B):
            pool[b * C + C - 1, int(nv[b, -1]):] = 0
        pools[li], nvs[li] = pool, nv
        pages[li] = ops.Pages(slots=pool, page_of=po, n_valid=nv, S=ops.summaries(pool, po, nv))
    W_in = torch.randn(d_m, d_s, generator=g, device=dev) * 0.02
    W_out = torch.randn(d_s, d_m, generator=g, device=dev) * 0.02
    itf = LinearInterface(W_in, W_out, layers).to(dev).requires_grad_(False)
    sel = LayerSelector(d_m, layers, k=sel_k).to(dev).requires_grad_(False)
    inj = LibraryInjector(_IdReader(L, dev), itf, top_k=top_k, selector=sel)
    inj.load_library(PagedLibrary(pages))
    h0 = torch.randn(B, 1, d_m, generator=g, device=dev)
    z = torch.randn(B, 1, L, generator=g, device=dev)
    hs, routes = [], []
    with torch.inference_mode():
        sel.set_logits(z)
        h = h0
        for li in layers:
            h, _ = inj._inject(h, li)
            hs.append(h.reshape(B, d_m).clone())
            routes.append(inj.last_route.reshape(B, C).clone())
        w_gpu = sel.weights().reshape(B, L).clone()
    inj.detach()
    # oracle: the reference reads every depth for every token and multiplies the unselected deltas by exact zeros
    # (xenc/selector.py:106-110); a zero-weight depth adds exactly 0 to h, so it is skipped here
    w_sel = X.selector_weights(z.cpu().numpy().reshape(B, L), sel_k)
    assert topk_sets(w_gpu) == topk_sets(w_sel)
    Wi, Wo = W_in.cpu().numpy(), W_out.cpu().numpy()
    hr = h0.cpu().numpy().reshape(B, d_m)
    margin = np.inf
    mismatches, err_h, err_step = [], 0.0, 0.0
    for p, li in enumerate(layers):
        hn = X.rms_norm(hr)
        q = X.query(hn, Wi)
        out = np.zeros((B, d_m), np.float32)
        nv_h = nvs[li].cpu().numpy()
        for b in range(B):
            K, M = _doc_slots(pools[li], nv_h[b], C, b)
            w, logit, _ = X.route(q[b:b + 1], X.summaries(K, M), 10.0, top_k)
            margin = min(margin, _tie_margin(logit, top_k))
            if topk_sets(routes[p][b:b + 1]) != topk_sets(w):
                mismatches.append((b, li))
            if w_sel[b, p] != 0:
                out[b] = (X.read(q[b:b + 1], K, M, w, 12.0, True) @ Wo)[0]
        delta = X.selector_apply(out, hr, w_sel[:, p], float(sel.log_alpha))
        got_delta = hs[p].cpu().numpy() - (h0.cpu().numpy().reshape(B, d_m) if p == 0 else hs[p - 1].cpu().numpy())
        live = w_sel[:, p] != 0
        assert not np.any(got_delta[~live]), f"layer {li}: a token the selector dropped changed h"
        if live.any():
            err_step = max(err_step, rel_err(got_delta[live], delta[live]))
        hr = (hr + delta).astype(np.float32)
    h_fin = hs[-1].cpu().numpy()
    h0n = h0.cpu().numpy().reshape(B, d_m)
    err_h = rel_err(h_fin - h0n, hr - h0n)
    print("PARITY " + json.dumps({"config": 4, "tokens": B, "depth_reads": int((w_sel != 0).sum()),
                                  "routing_checks": B * L, "routing_mismatches": len(mismatches),
                                  "min_topk_margin": margin, "max_rel_err_layer_delta": err_step,
                                  "max_rel_err_total_delta": err_h}))
    assert not mismatches, f"routing differs at (doc, layer) {mismatches[:6]}; min margin {margin:.3e}"
    assert err_step < TOL and err_h < TOL
    assert ops.device_status(dev) == 0
    del pools, pages
    torch.cuda.empty_cache()
