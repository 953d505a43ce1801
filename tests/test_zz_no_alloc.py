"""The allocation-free read entry point, xencb_read_decode_noalloc.

It exists for callers that cannot allocate device memory (a host runtime that owns all device memory and
cannot hand out scratch, or a loop that must not allocate); it keeps its scratch in a fixed device array
inside libxencb.so. This file is named to be collected last, so a run that stops at the first failure has
already run every other test. Each test here calls the entry point through the C ABI (ctypes) and compares
it with xencb_read_decode (the workspace-taking entry point) on the same inputs."""

from __future__ import annotations

import ctypes

import pytest
import torch

from tests._fixtures import TOL, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _case(dev, seed, n_docs=8, C=16, N=256, d_s=512, top_k=3, dtype=torch.float16, short=False):
    from kv_skill_v2_b200 import ops
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(n_docs * C, N, d_s, generator=g, device=dev)
    slots = (x / x.norm(dim=-1, keepdim=True)).to(dtype).contiguous()
    nv = torch.full((n_docs, C), N, dtype=torch.int32, device=dev)
    if short:  # every chunk short: most row splits of a chunk hold no rows
        nv = torch.randint(1, max(2, N // 4), (n_docs, C), generator=g, device=dev, dtype=torch.int32)
    nv[:, -1] = torch.randint(1, N + 1, (n_docs,), generator=g, device=dev, dtype=torch.int32)
    page_of = torch.arange(n_docs * C, dtype=torch.int32, device=dev).view(n_docs, C)
    S = ops.summaries(slots, page_of, nv)
    pages = ops.Pages(slots=slots, page_of=page_of, n_valid=nv, S=S)
    q = torch.nn.functional.normalize(torch.randn(n_docs, d_s, generator=g, device=dev), dim=-1).contiguous()
    idx, wk, _, _ = ops.route(q, S, rows_per_lib=1, top_k=top_k, route_temp=10.0)
    return pages, q, idx, wk


def _noalloc(pages, q, idx, wk, r, read_temp=12.0, softmax=True) -> int:
    from kv_skill_v2_b200 import _native as N
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    R, d_s = q.shape
    dt = {torch.float16: N.F16, torch.bfloat16: N.BF16, torch.float32: N.F32}[pages.slots.dtype]
    return N.lib().xencb_read_decode_noalloc(
        p(q), R, d_s, p(pages.slots), dt, pages.slots.shape[0], pages.page_rows * d_s, pages.page_rows,
        p(pages.page_of), p(pages.n_valid), pages.n_chunks, 1, pages.n_lib, p(idx), p(wk), idx.shape[1],
        read_temp, int(softmax), p(r), ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream))


def test_noalloc_matches_workspace_read_two_calls_in_a_row(dev):
    from kv_skill_v2_b200 import ops
    for call, seed in enumerate((1, 2)):  # two calls in a row, different inputs: no state leaks between them
        pages, q, idx, wk = _case(dev, seed)
        want = ops.read_decode(q, pages, idx, wk, rows_per_lib=1)
        r = torch.full_like(q, float("nan"))
        assert _noalloc(pages, q, idx, wk, r) == 0
        torch.cuda.synchronize(dev)
        assert rel_err(r, want) < TOL, f"call {call}"
    assert ops.device_status(dev) == 0


def test_noalloc_rejects_oversized_calls(dev):
    from kv_skill_v2_b200 import _native as N
    R_big = 4096  # 4096 rows x 3 chunks x d_s floats of partials: far above the fixed array
    need = N.lib().xencb_read_decode_workspace(R_big, 3, 2048, 512, N.F16)
    assert need > N.NOALLOC_SCRATCH_BYTES
    qb = torch.zeros(R_big, 2048, device=dev)
    idxb = torch.zeros(R_big, 3, dtype=torch.int32, device=dev)
    wkb = torch.zeros(R_big, 3, device=dev)
    rb = torch.empty_like(qb)
    slots = torch.zeros(1, 512, 2048, dtype=torch.float16, device=dev)
    page_of = torch.zeros(1, 1, dtype=torch.int32, device=dev)
    nv = torch.ones(1, 1, dtype=torch.int32, device=dev)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = N.lib().xencb_read_decode_noalloc(p(qb), R_big, 2048, p(slots), N.F16, 1, 512 * 2048, 512, p(page_of), p(nv),
                                            1, R_big, 1, p(idxb), p(wkb), 3, 12.0, 1, p(rb),
                                            ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert rc == N.EINVAL
    assert b"fixed" in N.lib().xencb_last_error()


def test_noalloc_stale_scratch_from_a_larger_call(dev):
    """The fixed array keeps what the previous call left in it. A large call with every row split live fills it
    first; then smaller calls -- short chunks (most splits hold no rows) with the linear read, and bfloat16
    slots -- must not pick up any of those stale words: each matches xencb_read_decode on the same inputs."""
    from kv_skill_v2_b200 import _native as N
    from kv_skill_v2_b200 import ops
    ws = lambda n, k, d, rows, dt: N.lib().xencb_read_decode_workspace(n, k, d, rows, dt)
    n_big = 64
    while n_big > 8 and ws(n_big, 4, 512, 512, N.F16) > N.NOALLOC_SCRATCH_BYTES:
        n_big //= 2
    assert ws(n_big, 4, 512, 512, N.F16) <= N.NOALLOC_SCRATCH_BYTES
    pages, q, idx, wk = _case(dev, 7, n_docs=n_big, C=8, N=512, d_s=512, top_k=4)
    r = torch.full_like(q, float("nan"))
    assert _noalloc(pages, q, idx, wk, r) == 0
    torch.cuda.synchronize(dev)
    assert rel_err(r, ops.read_decode(q, pages, idx, wk, rows_per_lib=1)) < TOL, "large call"
    cases = [dict(seed=8, n_docs=6, C=12, N=512, d_s=512, top_k=3, short=True, softmax=False),
             dict(seed=9, n_docs=5, C=10, N=256, d_s=512, top_k=2, short=True, softmax=True),
             dict(seed=10, n_docs=7, C=9, N=384, d_s=256, top_k=3, dtype=torch.bfloat16, softmax=True),
             dict(seed=11, n_docs=7, C=9, N=384, d_s=256, top_k=3, dtype=torch.bfloat16, short=True, softmax=False)]
    for c in cases:
        softmax = c.pop("softmax")
        pages, q, idx, wk = _case(dev, **c)
        want = ops.read_decode(q, pages, idx, wk, rows_per_lib=1, read_softmax=softmax)
        r = torch.full_like(q, float("nan"))
        assert _noalloc(pages, q, idx, wk, r, softmax=softmax) == 0
        torch.cuda.synchronize(dev)
        assert torch.isfinite(r).all(), c
        assert rel_err(r, want) < TOL, c
    assert ops.device_status(dev) == 0
