"""Multi-depth LayerSelector decode (BASELINE config 4 at reduced sizes): 8 candidate depths, each a paged
Library per document; per token the selector keeps its top-2 depths and only those depths are read.

The reference runs every depth's read for every token and zeroes the unselected deltas afterwards
(xenc/selector.py:95-110 applied at each hook, xenc/injector.py:271-272); the result is the same, which the
oracle comparison checks, while the route row mask makes the reads of the dropped (token, depth) pairs vanish."""

from __future__ import annotations

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


def test_route_row_mask_skips_rows_keeps_routing(dev):
    from kv_skill_v2_b200 import ops
    g = torch.Generator().manual_seed(4)
    S = torch.nn.functional.normalize(torch.randn(3, 10, 32, generator=g), dim=-1).to(dev)
    q = torch.nn.functional.normalize(torch.randn(6, 32, generator=g), dim=-1).to(dev)
    row_w = torch.tensor([0.7, 0.0, 0.3, 0.0, 1.0, 0.0], device=dev)
    for top_k in (0, 3):
        i0, k0, w0, _ = ops.route(q, S, rows_per_lib=2, top_k=top_k, route_temp=10.0)
        i1, k1, w1, _ = ops.route(q, S, rows_per_lib=2, top_k=top_k, route_temp=10.0, row_w=row_w)
        assert torch.equal(w0, w1), "w_dense must keep the routing of masked rows"
        keep = row_w != 0
        assert torch.equal(i0[keep], i1[keep]) and torch.equal(k0[keep], k1[keep])
        assert (i1[~keep] == -1).all() and (k1[~keep] == 0).all()


class _Identity(torch.nn.Module):
    def __init__(self, L, d_m, dev):
        super().__init__()
        self.layers = torch.nn.ModuleList([torch.nn.Identity() for _ in range(L)])
        self._p = torch.nn.Parameter(torch.zeros(1, device=dev), requires_grad=False)

    def forward(self, x):
        for blk in self.layers:
            x = blk(x)
        return x


def test_selector_decode_reads_only_selected_depths(dev):
    from kv_skill_v2_b200 import LayerSelector, LibraryInjector, LinearInterface, PagedLibrary, ops
    B, L, C, N, d_s, d_m, top_k = 3, 8, 8, 64, 256, 512, 4
    layers = list(range(L))
    g = torch.Generator().manual_seed(11)
    Ks = {}
    pages = {}
    nv = torch.full((B, C), N, dtype=torch.int32)
    nv[:, -1] = torch.tensor([1, 33, 64], dtype=torch.int32)
    for li in layers:
        K = torch.randn(B, C, N, d_s, generator=g)
        K = (K / K.norm(dim=-1, keepdim=True)).half()
        Ks[li] = K.float().numpy()
        slots = K.reshape(B * C, N, d_s).to(dev)
        po = torch.arange(B * C, dtype=torch.int32, device=dev).view(B, C)
        pages[li] = ops.Pages(slots=slots, page_of=po, n_valid=nv.to(dev), S=ops.summaries(slots, po, nv.to(dev)))
    plib = PagedLibrary(pages)
    W_in = torch.randn(d_m, d_s, generator=g) * 0.05
    W_out = torch.randn(d_s, d_m, generator=g) * 0.05
    itf = LinearInterface(W_in, W_out, layers).to(dev).requires_grad_(False)
    sel = LayerSelector(d_m, layers, k=2, alpha_init=0.05).to(dev).requires_grad_(False)
    reader = _Identity(L, d_m, dev)
    inj = LibraryInjector(reader, itf, top_k=top_k, selector=sel)
    inj.load_library(plib)
    h0 = torch.randn(B, 1, d_m, generator=g)
    z = torch.randn(B, 1, L, generator=g)

    with torch.no_grad():
        h = h0.to(dev)
        sel.set_logits(z.to(dev))
        routes = []
        for li in layers:
            h, _ = inj._inject(h, li)
            routes.append(inj.last_route.reshape(B, C).clone())
    # oracle: every depth read for every token, the selector's weights applied afterwards
    w_sel = X.selector_weights(z.numpy().reshape(B, L), 2)
    assert topk_sets(sel.weights().reshape(B, L)) == topk_sets(w_sel)
    hr = h0.numpy().reshape(B, d_m)
    M = np.arange(N)[None, :] < nv.numpy()[:, :, None]
    for p, li in enumerate(layers):
        hn = X.rms_norm(hr)
        q = X.query(hn, W_in.numpy())
        out = np.zeros((B, d_m), np.float32)
        for b in range(B):
            Sb = X.summaries(Ks[li][b], M[b])
            w, _, _ = X.route(q[b:b + 1], Sb, 10.0, top_k)
            assert topk_sets(routes[p][b:b + 1]) == topk_sets(w)
            r = X.read(q[b:b + 1], Ks[li][b], M[b], w, 12.0, True)
            out[b] = (r @ W_out.numpy())[0]
        delta = X.selector_apply(out, hr, w_sel[:, p], float(sel.log_alpha))
        hr = (hr + delta).astype(np.float32)
    got = h.reshape(B, d_m).cpu().numpy()
    assert rel_err(got - h0.numpy().reshape(B, d_m), hr - h0.numpy().reshape(B, d_m)) < TOL
    assert ops.device_status(dev) == 0
    inj.detach()
