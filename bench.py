#!/usr/bin/env python
"""Benchmark of the Library read at BASELINE config 2 (decode).

Workload (per GPU): 64 documents, each its own Library of C=64 chunks x 512 fp16 slots (d_s=2048; the last
chunk ragged, U{1..512} valid), reader width d_m=4096, one query token per document per step, top-4 chunk
routing, read_temp 12, route_temp 10. A step is one pass of the hot path for the 64 tokens: rms_norm +
query projection + L2, routing, the split-K masked read, output projection + residual + mag term.

* value: whole-job tokens/s with inputs resident in HBM (the step captured in a CUDA graph), timed per step
  with CUDA events on the launching stream, L2 flushed between steps outside the events (a 256 MiB write, then
  a read of the same buffer, so the flush's dirty lines are written back before the step, not during it);
  max over ranks. Multi-GPU runs are weak-scaled replicas (every rank its own 64 documents, no collective
  in the data path; one all-reduce of the elapsed time after timing).
* e2e: the same metric through the public API -- a reader model whose hooked block runs LibraryInjector --
  from pinned host hidden states, H2D copy and D2H copy of the result inside the timed region.
* roofline: the read kernel timed alone (CUDA events recorded by libxencb right around it, after an L2 flush);
  achieved = algorithmic bytes (valid slot rows of the routed chunks, read once, + q in) / time, against
  MEASURED_PEAKS.json hbm_gbs. The whole read op (kernel + merge, one graph replay) is reported beside it.
* cpu_baseline: the numpy oracle (a restatement of the reference's dense read) on host cores, on a bounded
  sample of the same workload.

--impl reference times that CPU implementation alone (rank 0; other ranks exit at once).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Library-read decode tokens/s per GPU; achieved HBM GB/s vs ~8 TB/s peak"
UNIT = "tokens/s"
CFG = dict(docs=64, C=64, N=512, d_s=2048, d_m=4096, top_k=4, T=1, read_temp=12.0, route_temp=10.0)
FALLBACK_HBM_GBS = 6650.0
FLUSH_BYTES = 256 << 20


def l2_flush(flush, i: int) -> None:
    """Evict L2 between timed steps: write a buffer of twice its size, then read the buffer back, so the dirty
    lines of the write go to HBM here, outside the timed region, instead of during the next step."""
    import torch
    flush.fill_(i & 0xFF)
    flush.view(torch.int32).sum()


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--docs", type=int, default=CFG["docs"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-only", action="store_true", help="only the read kernel loop (for profilers)")
    ap.add_argument("--no-sharded", action="store_true", help="skip the config-5 sharded read")
    ap.add_argument("--sharded-only", action="store_true",
                    help="only the config-5 sharded read; print its object as the line (for profilers)")
    ap.add_argument("--sharded-chunks", type=int, default=2048,
                    help="chunks of the config-5 Library (2048 = the config; smaller only for profiler captures)")
    ap.add_argument("--no-selector", action="store_true", help="skip the config-4 multi-depth selector decode")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 tensor-core prefill read")
    ap.add_argument("--prefill-only", action="store_true",
                    help="only the config-3 prefill; print its object as the line (for profilers)")
    ap.add_argument("--prefill-docs", type=int, default=8,
                    help="documents of the config-3 prefill (8 = the config; fewer only for profiler captures)")
    ap.add_argument("--no-library-build", action="store_true", help="skip the device Library build")
    ap.add_argument("--no-topk", action="store_true", help="skip the D8 top-k slot read")
    ap.add_argument("--topk-only", action="store_true", help="only the D8 top-k slot read")
    ap.add_argument("--library-build-only", action="store_true",
                    help="only the device Library build (config-2 shapes)")
    ap.add_argument("--library-build-docs", type=int, default=16,
                    help="documents per device Library build step (smaller for profiler captures)")
    ap.add_argument("--selector-only", action="store_true",
                    help="only the config-4 selector decode; print its object as the line (for profilers)")
    return ap.parse_args(argv)


def config_dict(docs: int) -> dict:
    return {"workload": "BASELINE config 2: decode, batch of independent documents, top-4 of 64 chunks",
            "docs_per_gpu": docs, "chunks": CFG["C"], "slots_per_chunk": CFG["N"], "d_s": CFG["d_s"],
            "d_m": CFG["d_m"], "top_k": CFG["top_k"], "query_tokens_per_doc": CFG["T"], "slot_dtype": "f16",
            "hidden_dtype": "f32", "weights_dtype": "f32", "read_temp": CFG["read_temp"],
            "route_temp": CFG["route_temp"], "last_chunk_valid": "U{1..512}",
            "l2": "flushed between timed steps (256 MiB write + read back); inputs per step > L2 as well",
            "parallelism": "replicas (weak scaling, one doc batch per GPU)"}


# ------------------------------------------------------------------------------------------------ reference arm
class CpuOracle:
    """The oracle's dense read (the reference's algorithm, xenc/injector.py:231-273) on config-2 shapes over
    `n_docs` documents; each call of one() reads one decode token of the next document."""

    def __init__(self, n_docs: int, seed: int = 0):
        import numpy as np

        from oracle import xenc_oracle as X

        self.np, self.X = np, X
        self.rng = np.random.default_rng(seed)
        C, N, d_s, d_m = CFG["C"], CFG["N"], CFG["d_s"], CFG["d_m"]
        self.W_in = self.rng.standard_normal((d_m, d_s), dtype=np.float32) * np.float32(0.02)
        self.W_out = self.rng.standard_normal((d_s, d_m), dtype=np.float32) * np.float32(0.02)
        self.docs = []
        for _ in range(n_docs):
            K = self.rng.standard_normal((C, N, d_s), dtype=np.float32)
            K /= np.linalg.norm(K, axis=-1, keepdims=True)
            K = K.astype(np.float16).astype(np.float32)
            M = np.ones((C, N), dtype=bool)
            M[-1, int(self.rng.integers(1, N + 1)):] = False
            self.docs.append((K, M, X.summaries(K, M)))
        self.n = 0
        self.cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()

    def one(self) -> float:
        K, M, S = self.docs[self.n % len(self.docs)]
        h = self.rng.standard_normal((1, CFG["d_m"]), dtype=self.np.float32)
        t0 = time.perf_counter()
        self.X.branch(h, self.W_in, self.W_out, K, M, S, top_k=CFG["top_k"])
        self.n += 1
        return time.perf_counter() - t0

    def sample(self, budget_s: float) -> dict:
        self.one()  # warm
        spent, n = 0.0, 0
        while spent < budget_s or n < len(self.docs):
            spent += self.one()
            n += 1
        return {"value": n / spent, "unit": UNIT, "cores": self.cores, "kind": "port",
                "sample": f"{n} decode tokens over {len(self.docs)} config-2 documents (dense read of all 64 "
                          f"chunks, as the reference computes it), numpy float32, {self.cores} BLAS threads, "
                          f"{spent:.1f} s"}


def run_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cpu = CpuOracle(n_docs=2)
    for _ in range(args.warmup):
        cpu.one()
    per_step = [cpu.one() for _ in range(args.steps)]
    value = len(per_step) / sum(per_step)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * statistics.mean(per_step), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": config_dict(CFG["docs"]),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu.cores, "kind": "port",
                             "sample": "each step: one config-2 decode token (dense read of all 64 chunks as the "
                                       "reference computes it) through the numpy oracle on host cores; "
                                       "2 documents cycled"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ our arm
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while running."""

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: str | None):
        self.bus_id = (bus_id or "").lower()
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-f", self.path], stdout=subprocess.DEVNULL,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return None
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            if self.bus_id and self.bus_id[-12:] not in f[1].lower():
                continue
            rows.append(f)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        for r in rows:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), r[6:10]):
                if v.lower() == "active":
                    reasons.add(name)
        busy = [s for s in sm if s > 0.5 * float(rows[0][3] or 1)] or sm
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": float(rows[0][3]),
                "reasons": sorted(reasons), "samples": len(rows)}


def hbm_peak() -> tuple:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def traffic_per_row() -> float | None:
    """DRAM bytes per routed slot row of the read kernel, from the committed ncu summary (if any)."""
    p = ROOT / "profiles" / "read_decode_cfg2_traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return float(d["dram_bytes"]) / float(d["slot_rows"])
    except (KeyError, ValueError, ZeroDivisionError):
        return None


def build_workload(torch, dev, docs: int, seed: int):
    from kv_skill_v2_b200 import ops

    C, N, d_s, d_m = CFG["C"], CFG["N"], CFG["d_s"], CFG["d_m"]
    g = torch.Generator(device=dev).manual_seed(1000 + seed)
    slots = torch.empty(docs * C, N, d_s, dtype=torch.float16, device=dev)
    for b in range(docs):  # one document at a time keeps the float32 temporaries small
        x = torch.randn(C, N, d_s, generator=g, device=dev)
        slots[b * C:(b + 1) * C] = (x / x.norm(dim=-1, keepdim=True)).half()
        del x
    nv = torch.full((docs, C), N, dtype=torch.int32, device=dev)
    nv[:, -1] = torch.randint(1, N + 1, (docs,), generator=g, device=dev, dtype=torch.int32)
    page_of = torch.arange(docs * C, dtype=torch.int32, device=dev).view(docs, C)
    S = ops.summaries(slots, page_of, nv)
    pages = ops.Pages(slots=slots, page_of=page_of, n_valid=nv, S=S)
    W_in = torch.randn(d_s, d_m, generator=g, device=dev) * 0.02   # nn.Linear layout [out, in]
    W_out = torch.randn(d_m, d_s, generator=g, device=dev) * 0.02
    return pages, W_in, W_out, g


CFG5 = dict(C=2048, N=512, d_s=2560, d_m=5120, T=8, read_temp=12.0, route_temp=10.0)


def run_sharded(torch, dist, dev, world: int, rank: int, steps: int, warmup: int, flush, stream,
                n_chunks: int = 2048) -> dict:
    """one Library of 2048 chunks x 512 fp16 slots (1,048,576 slots, d_s 2560), 8 query tokens,
    every chunk read (top_k 0); the chunks sharded evenly over the ranks, the partials exchanged once per step
    (pushed over NVLink peer memory, one GPU per rank) and merged. Strong scaling: the whole Library is the same at
    every N.

    A step: q = project_in(h) (replicated interface weights), the rank's partial (route_lse + read_multi over its
    chunks), the exchange of the partial blocks, shard merge, output projection + residual, captured as one CUDA
    graph with the exchange inside. Timed with CUDA events per step, max over ranks."""
    from kv_skill_v2_b200 import _native, ops
    from kv_skill_v2_b200.shard import ShardedRead, partition_chunks

    C, N, d_s, d_m, T = int(n_chunks), CFG5["N"], CFG5["d_s"], CFG5["d_m"], CFG5["T"]
    lo, hi = partition_chunks(C, world)[rank]
    Cl = hi - lo
    g = torch.Generator(device=dev).manual_seed(5000 + lo)
    slots = torch.empty(Cl, N, d_s, dtype=torch.float16, device=dev)
    for c0 in range(0, Cl, 64):
        x = torch.randn(min(64, Cl - c0), N, d_s, generator=g, device=dev)
        slots[c0:c0 + x.shape[0]] = (x / x.norm(dim=-1, keepdim=True)).half()
        del x
    page_of = torch.arange(Cl, dtype=torch.int32, device=dev).view(1, Cl)
    nv = torch.full((1, Cl), N, dtype=torch.int32, device=dev)
    pages = ops.Pages(slots=slots, page_of=page_of, n_valid=nv, S=ops.summaries(slots, page_of, nv))
    gw = torch.Generator(device=dev).manual_seed(55)  # the same interface and tokens on every rank
    W_in = torch.randn(d_s, d_m, generator=gw, device=dev) * 0.02
    W_out = torch.randn(d_m, d_s, generator=gw, device=dev) * 0.02
    hs = torch.randn(warmup + steps, T, d_m, generator=gw, device=dev)
    h = hs[0].clone()
    h_out = torch.empty_like(h)
    # N > 1: the blocks over NVLink peer memory when every rank has its own GPU (XENCB_SHARD_EXCHANGE=collective in
    # the environment: one NCCL all-gather instead)
    sr = ShardedRead(pages, T, rows_per_lib=T, exchange=os.environ.get("XENCB_SHARD_EXCHANGE", "auto"))
    P_in, P_out = ops.weights_prep(W_in), ops.weights_prep(W_out)  # 3xF16 form, prepared once
    if world > 1 and sr.exchange_kind == "peer":  # the peer exchange gives the all-gather's result, bit for bit
        sr_c = ShardedRead(pages, T, rows_per_lib=T, exchange="collective")
        q0, _, _, _ = ops.project_in(h, W_in, w_prep=P_in)
        ra = sr(q0).clone()
        assert torch.equal(ra, sr_c(q0)), "peer exchange differs from the all-gather"
        del sr_c

    def pre():  # the input projection fused with the shard's routing, then the read
        sr.partial_from_hidden(h, W_in, P_in)

    def post():
        r = sr.merge()
        ops.project_out(r, W_out, h, want_delta=False, h_out=h_out, w_prep=P_out)

    for _ in range(2):  # eager steps first: the communicator (or the peer mappings) exist before the capture
        pre(); sr.exchange(); post()
    torch.cuda.synchronize(dev)
    # the whole step, the all-gather included, is one CUDA graph
    g_step = torch.cuda.CUDAGraph()
    n0 = _native.launch_count()
    with torch.cuda.graph(g_step):
        pre()
        sr.exchange()
        post()
    kernels = _native.launch_count() - n0
    torch.cuda.synchronize(dev)

    def step(i):
        h.copy_(hs[i])
        g_step.replay()

    for i in range(warmup):
        l2_flush(flush, i)
        step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        l2_flush(flush, i)
        ev[i][0].record(stream)
        step(warmup + i)
        ev[i][1].record(stream)
    torch.cuda.synchronize(dev)
    t_ms = sum(a.elapsed_time(b) for a, b in ev)
    t_max = t_ms
    if world > 1:
        t = torch.tensor([t_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_max = float(t.item())
    # the read alone on this rank (route_lse + read_multi), for the roofline
    g_read = torch.cuda.CUDAGraph()
    q_s, _, _, _ = ops.project_in(h, W_in)
    with torch.cuda.graph(g_read):
        sr.partial(q_s)
    evr = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(max(steps, 20))]
    for i in range(3):
        l2_flush(flush, i)
        g_read.replay()
    for i in range(len(evr)):
        l2_flush(flush, i)
        evr[i][0].record(stream)
        g_read.replay()
        evr[i][1].record(stream)
    torch.cuda.synchronize(dev)
    t_read = statistics.mean(a.elapsed_time(b) for a, b in evr) / 1000.0

    # the other parts of the step, each replayed alone (every rank replays the same graphs in the same order):
    # the replicated input projection, the all-gather, merge + output projection; and, for the choice of keeping
    # the projections replicated, the input projection of one rank's share of W_in's rows (what a rank would run
    # with the projections sharded, before an extra all-gather of q)
    def timed(fn, n=20):
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph):
            fn()
        ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        gph.replay()
        for i in range(n):
            l2_flush(flush, i)
            ev2[i][0].record(stream)
            gph.replay()
            ev2[i][1].record(stream)
        torch.cuda.synchronize(dev)
        t = statistics.mean(a.elapsed_time(b) for a, b in ev2) * 1000.0
        del gph
        return t
    n_sh = max(64, (d_s // max(world, 1)) // 64 * 64)
    W_sh = W_in[:n_sh].contiguous()
    P_sh = ops.weights_prep(W_sh)
    comp = {"project_in": timed(lambda: ops.project_in(h, W_in, w_prep=P_in)),
            "route_lse_read_multi": t_read * 1e6,
            "exchange": timed(sr.exchange) if world > 1 else 0.0,
            "merge_project_out": timed(post),
            f"project_in_{n_sh}_of_{d_s}_rows": timed(lambda: ops.project_in(h, W_sh, w_prep=P_sh))}
    read_bytes = Cl * N * d_s * 2 + Cl * d_s * 4 + 2 * T * d_s * 4
    step_bytes = read_bytes + 2 * d_s * d_m * 4 + 2 * T * d_m * 4
    peak, peak_kind = hbm_peak()
    ms = t_max / steps
    del g_step, g_read
    kind = sr.exchange_kind
    sr.close()
    return {"workload": f"BASELINE config 5: one Library of {C} chunks x 512 fp16 slots ({C * N:,} slots), d_s 2560, "
                        "d_m 5120, 8 query tokens, dense read of every chunk; chunks sharded evenly over the GPUs, "
                        "partials (max, sum, acc) exchanged once per step and merged"
                        + ("" if C == CFG5["C"] else f" (REDUCED from {CFG5['C']} chunks for a profiler capture)"),
            "metric": "sharded Library-read tokens/s (whole job)", "value": T * steps / (t_max / 1000.0),
            "unit": "tokens/s", "n_gpus": world, "ms_per_step": ms, "scaling": "strong",
            "chunks_per_gpu": Cl, "kernels_per_step": kernels, "gpu_launches": kernels * steps,
            "components_us": comp, "exchange": kind,
            "step": "one CUDA graph per step: input projection (replicated) fused with the dense routing of the "
                    "rank's chunks, read_multi over them, the partial blocks pushed to every rank over NVLink peer memory (exchange 'peer'; "
                    "'collective': one NCCL all-gather), shard merge after the blocks' flags, output projection "
                    "(replicated)",
            "step_bytes_per_gpu": step_bytes, "step_hbm_gbs_per_gpu": step_bytes / (ms / 1000.0) / 1e9,
            "roofline": {"bound": "hbm", "kernel": "route_lse + read_multi_mma_kernel + read_multi_merge_kernel",
                         "achieved": read_bytes / t_read / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": read_bytes / t_read / 1e9 / peak, "algorithmic_bytes_per_launch": read_bytes,
                         "launch_us": t_read * 1e6, "peak_source": peak_kind},
            "l2": "flushed between steps (256 MiB write + read back); the slot shard alone is > L2 at every N <= 8"}


CFG4 = dict(docs=32, L=8, C=32, N=512, d_s=2048, d_m=5120, sel_k=2, top_k=4, read_temp=12.0, route_temp=10.0)


def run_selector(torch, dist, dev, world: int, rank: int, steps: int, warmup: int, flush, stream) -> dict:
    """32 documents per GPU, each with 8 candidate depths (a Library of 32 chunks x 512 fp16
    slots per depth, d_s 2048), d_m 5120, one query token per document; the LayerSelector keeps the top-2 depths
    per token from given logits z ~ N(0,1) and routing keeps the top-4 chunks within each selected depth.

    A step is the LibraryInjector's work at the 8 hooked layers for one token per document: selector weights,
    then per layer the fused input projection, routing with the selector's row mask (tokens that dropped this
    depth read nothing), the decode read and the output projection with the selector's matched-norm rescale and
    the residual. Weak scaling: every rank its own 32 documents."""
    from kv_skill_v2_b200 import LayerSelector, LibraryInjector, LinearInterface, PagedLibrary, _native, ops

    B, L, C, N, d_s, d_m = CFG4["docs"], CFG4["L"], CFG4["C"], CFG4["N"], CFG4["d_s"], CFG4["d_m"]
    g = torch.Generator(device=dev).manual_seed(4000 + rank)
    layers = list(range(L))
    po = torch.arange(B * C, dtype=torch.int32, device=dev).view(B, C)
    nv = torch.full((B, C), N, dtype=torch.int32, device=dev)
    slots = {}
    for li in layers:
        pool = torch.empty(B * C, N, d_s, dtype=torch.float16, device=dev)
        for c0 in range(0, B * C, 128):
            x = torch.randn(min(128, B * C - c0), N, d_s, generator=g, device=dev)
            pool[c0:c0 + x.shape[0]] = (x / x.norm(dim=-1, keepdim=True)).half()
            del x
        slots[li] = pool
    plib = PagedLibrary.from_pool(slots, po, nv)
    W_in = torch.randn(d_m, d_s, generator=g, device=dev) * 0.02
    W_out = torch.randn(d_s, d_m, generator=g, device=dev) * 0.02
    itf = LinearInterface(W_in, W_out, layers).to(dev).requires_grad_(False)
    sel = LayerSelector(d_m, layers, k=CFG4["sel_k"]).to(dev).requires_grad_(False)

    class Reader(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = torch.nn.ModuleList([torch.nn.Identity() for _ in range(L)])
            self._p = torch.nn.Parameter(torch.zeros(1, device=dev), requires_grad=False)

        def forward(self, x):
            for blk in self.layers:
                x = blk(x)
            return x

    reader = Reader()
    inj = LibraryInjector(reader, itf, top_k=CFG4["top_k"], read_temp=CFG4["read_temp"],
                          route_temp=CFG4["route_temp"], selector=sel)
    inj.load_library(plib)
    hs = torch.randn(warmup + steps, B, 1, d_m, generator=g, device=dev)
    zs = torch.randn(warmup + steps, B, 1, L, generator=g, device=dev)
    h_in, z_in = hs[0].clone(), zs[0].clone()
    h_out = torch.empty_like(h_in)

    def step():
        sel.set_logits(z_in)
        h = h_in
        for li in layers:
            h, _ = inj._inject(h, li)
        h_out.copy_(h)

    with torch.inference_mode():
        for _ in range(2):
            step()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        n0 = _native.launch_count()
        with torch.cuda.graph(graph):
            step()
        kernels = _native.launch_count() - n0
        torch.cuda.synchronize(dev)
        for i in range(warmup):
            h_in.copy_(hs[i]); z_in.copy_(zs[i])
            l2_flush(flush, i)
            graph.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            h_in.copy_(hs[warmup + i]); z_in.copy_(zs[warmup + i])
            l2_flush(flush, i)
            ev[i][0].record(stream)
            graph.replay()
            ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
        sel_rows = int((sel.weights() > 0).sum().item())  # (token, depth) reads of the last step
    t_ms = sum(a.elapsed_time(b) for a, b in ev)
    t_max = t_ms
    if world > 1:
        t = torch.tensor([t_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_max = float(t.item())
    ms = t_max / steps
    # algorithmic bytes of a step: the routed chunks of the selected depths (full chunks here), their summary
    # keys, the interface weights once, hidden in and out
    step_bytes = sel_rows * (CFG4["top_k"] * N * d_s * 2 + C * d_s * 4) + 2 * d_s * d_m * 4 + 2 * B * d_m * 4
    peak, peak_kind = hbm_peak()
    inj.detach()
    del graph
    return {"workload": "BASELINE config 4: 32 documents x 8 candidate depths (32 chunks x 512 fp16 slots each, "
                        "d_s 2048), d_m 5120, LayerSelector top-2 depths from given logits ~ N(0,1), top-4 chunks "
                        "per selected depth, 1 token per document per step",
            "metric": "multi-depth Library-read decode tokens/s (whole job)",
            "value": B * world * steps / (t_max / 1000.0), "unit": "tokens/s", "n_gpus": world, "ms_per_step": ms,
            "scaling": "weak", "kernels_per_step": kernels, "gpu_launches": kernels * steps,
            "depth_reads_per_step": sel_rows,
            "roofline": {"bound": "hbm", "kernel": "whole step (8 hooked layers)",
                         "achieved": step_bytes / (ms / 1000.0) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": step_bytes / (ms / 1000.0) / 1e9 / peak, "algorithmic_bytes_per_step": step_bytes,
                         "peak_source": peak_kind},
            "l2": "flushed between steps (256 MiB write + read back)"}


CFGB = dict(docs=16, C=64, N=512, d_s=2048)


def run_library_build(torch, dist, dev, world: int, rank: int, steps: int, warmup: int, stream,
                      cpu_seconds: float = 0.0, docs: int = 16) -> dict:
    """The device Library build (xenc/library.py:47-74) at config-2 shapes: one depth of 16 documents' Libraries
    (64 chunks x up to 512 fp16 rows, d_s 2048, the last chunk of each ragged), centred (K = L2(K - mu) on the
    valid rows) into float16 pages, with n_valid and S. A step is one build of all 16 Libraries (the build
    kernel + the summaries kernel). Inputs 2 GiB, outputs 2 GiB: larger than L2, so no flush is needed.
    Algorithmic bytes: valid rows read once, every page row written once, S and mu."""
    import numpy as np

    from kv_skill_v2_b200 import _native, ops

    B, C, N, d = int(docs), CFGB["C"], CFGB["N"], CFGB["d_s"]
    g = torch.Generator().manual_seed(5000 + rank)
    counts = [N] * (B * C)
    for b in range(B):
        counts[b * C + C - 1] = int(torch.randint(1, N + 1, (1,), generator=g))
    n_rows = sum(counts)
    gd = torch.Generator(device=dev).manual_seed(5000 + rank)
    rows = torch.empty(n_rows, d, dtype=torch.float16, device=dev)
    for r0 in range(0, n_rows, 65536):
        x = torch.randn(min(65536, n_rows - r0), d, generator=gd, device=dev)
        rows[r0:r0 + x.shape[0]] = (x / x.norm(dim=-1, keepdim=True)).half()
        del x
    mu = torch.randn(d, generator=gd, device=dev) * 0.01
    slots, nv, S = ops.library_build(rows, counts, page_rows=N, mu=mu, slot_dtype=torch.float16)
    # parity spot check against the oracle on three chunks (first, a ragged last one, one in the middle)
    from oracle import xenc_oracle as X
    starts = np.concatenate([[0], np.cumsum(counts)])
    for c in (0, C - 1, (B // 2) * C + 7):
        rr = rows[int(starts[c]):int(starts[c + 1])].float().cpu().numpy()
        K_ref, _, S_ref = X.build_library([rr], mu.cpu().numpy())
        assert np.abs(S[c].cpu().numpy() - S_ref[0]).max() <= 1e-6, "library_build: S differs from the oracle"
        got = slots[c, :counts[c]].float().cpu().numpy()
        assert np.abs(got - K_ref[0]).max() <= 1e-3 * np.abs(K_ref[0]).max(), "library_build: slots differ"
    start = torch.zeros(len(counts) + 1, dtype=torch.int64)
    start[1:] = torch.tensor(counts, dtype=torch.int64).cumsum(0)
    start = start.to(dev)
    page_of = torch.arange(B * C, dtype=torch.int32, device=dev)
    ws_bytes = _native.lib().xencb_library_build_workspace(B * C, d, N)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)

    def launch():
        _native.call("xencb_library_build", ops._ptr(rows), _native.F16, n_rows, ops._ptr(start), B * C, d,
                     ops._ptr(mu), ops._ptr(slots), _native.F16, B * C, N * d, N, ops._ptr(page_of), ops._ptr(nv),
                     ops._ptr(S), ops._ptr(ws), ws.numel(), ops._stream(dev))

    for _ in range(warmup):
        launch()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    n0 = _native.launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        ev[i][0].record(stream)
        launch()
        ev[i][1].record(stream)
    torch.cuda.synchronize(dev)
    kernels = _native.launch_count() - n0
    t_ms = sum(a.elapsed_time(b) for a, b in ev)
    if world > 1:
        t = torch.tensor([t_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_ms = float(t.item())
    ms = t_ms / steps
    step_bytes = n_rows * d * 2 + B * C * N * d * 2 + B * C * d * 4 + d * 4 + B * C * 4
    peak, peak_kind = hbm_peak()
    res = {"workload": f"device Library build at config-2 shapes: {B} documents x {C} chunks x <= {N} fp16 rows, "
                       f"d_s {d}, centred, into fp16 pages + n_valid + S (one depth)",
           "metric": "Libraries built per second (whole job)", "value": B * world / (ms / 1000.0),
           "unit": "Libraries/s", "ms_per_step": ms, "n_gpus": world, "scaling": "weak",
           "kernels_per_step": kernels // max(steps, 1), "gpu_launches": kernels,
           "roofline": {"bound": "hbm", "kernel": "library_build_kernel + library_summaries_kernel",
                        "achieved": step_bytes / (ms / 1000.0) / 1e9, "peak": peak, "unit": "GB/s",
                        "frac": step_bytes / (ms / 1000.0) / 1e9 / peak, "algorithmic_bytes_per_step": step_bytes,
                        "peak_source": peak_kind},
           "l2": f"inputs and outputs {B * C * N * d * 2 / 2**30:.1f} GiB each (larger than L2)"}
    if rank == 0 and world == 1 and cpu_seconds > 0:
        # the reference's build (padding, centring, summaries) restated in numpy, one Library at a time
        rr = rows[:sum(counts[:C])].float().cpu().numpy()
        chunks = np.split(rr, np.cumsum(counts[:C])[:-1])
        mu_h = mu.cpu().numpy()
        spent, n = 0.0, 0
        while spent < cpu_seconds and n < 50:
            t0 = time.perf_counter()
            X.build_library(chunks, mu_h)
            spent += time.perf_counter() - t0
            n += 1
        res["cpu_baseline"] = {"value": n / spent, "unit": "Libraries/s", "cores": 1, "kind": "port",
                               "sample": f"{n} builds of one {C}-chunk Library (oracle.build_library, numpy)"}
    del rows, slots, ws
    return res


CFGK = dict(docs=64, C=64, N=512, d_s=2048, n_q=32, n_kv=8, hd=128, k=64, sel_docs=16)


def run_topk(torch, dist, dev, world: int, rank: int, steps: int, warmup: int, flush, stream,
             cpu_seconds: float = 0.0) -> dict:
    """D8 top-k slot read (xenc/topk_read.py) at config-2 Library shapes: 64 documents of 64 chunks x 512 fp16
    slots (d_s 2048), k = 64 selected slots per document, one decode token per document.

    select: per document the selection scores of one query (32 query heads, 8 KV heads of 128: a Qwen3-8B-like
      geometry) against its 32,768 fp16 selection keys (64 MiB), pooled max over heads, then the top-64; run
      for 16 documents per step (1 GiB of keys: larger than L2). Algorithmic bytes: the keys once.
    read: per decode step the gathered read of 64 documents (64 slots each) -- scores, softmax over the 64, the
      weighted sum; algorithmic bytes: the 64 selected rows once per document (tied V = K), q and r.
      L2 flushed between steps."""
    import numpy as np

    from kv_skill_v2_b200 import _native, ops

    B, C, N, d = CFGK["docs"], CFGK["C"], CFGK["N"], CFGK["d_s"]
    n_q, n_kv, hd, k, SB = CFGK["n_q"], CFGK["n_kv"], CFGK["hd"], CFGK["k"], CFGK["sel_docs"]
    g = torch.Generator(device=dev).manual_seed(6000 + rank)
    S = C * N
    keys = (torch.randn(SB, S, n_kv, hd, generator=g, device=dev) * 0.1).half()
    nv = torch.full((SB, C), N, dtype=torch.int32, device=dev)
    nv[:, -1] = N // 3
    qs = torch.randn(SB, 1, n_q, hd, generator=g, device=dev)
    pool = torch.empty(B * C, N, d, dtype=torch.float16, device=dev)
    for c0 in range(0, B * C, 256):
        x = torch.randn(min(256, B * C - c0), N, d, generator=g, device=dev)
        pool[c0:c0 + x.shape[0]] = (x / x.norm(dim=-1, keepdim=True)).half()
        del x
    pages = ops.Pages(slots=pool, page_of=torch.arange(B * C, dtype=torch.int32, device=dev).view(B, C),
                      n_valid=torch.full((B, C), N, dtype=torch.int32, device=dev),
                      S=torch.zeros(1, 1, 1, device=dev))
    q = torch.nn.functional.normalize(torch.randn(B, d, generator=g, device=dev), dim=-1)
    idx = torch.stack([torch.randperm(S, device=dev)[:k] for _ in range(B)]).to(torch.int32)

    def select():
        sc = ops.select_scores(qs, keys, nv, page_rows=N, rows_per_lib=1)
        return ops.select_topk(sc, k)

    def read():
        return ops.topk_read(q, pages, idx)

    # parity spot checks against the oracle (one document each)
    from oracle import xenc_oracle as X
    sel_idx, _ = select()
    valid = (np.arange(N)[None, :] < nv[0].cpu().numpy()[:, None]).reshape(-1)
    ref_sc = X.topk_select_scores(qs[:1].permute(0, 2, 1, 3).cpu().numpy(), keys[0].float().cpu().numpy(), valid)
    assert set(sel_idx[0].cpu().tolist()) == set(X.topk_select(ref_sc, k)[0].tolist()), "select: sets differ"
    r, _ = read()
    Kf = pool[:C].float().reshape(C * N, d).cpu().numpy()
    ref_r, _ = X.topk_read(q[:1].cpu().numpy()[None], Kf, idx[:1].cpu().numpy())
    assert float(np.abs(r[0].cpu().numpy() - ref_r[0, 0]).max()) <= 2e-3 * float(np.abs(ref_r).max()), "read differs"

    def timed(fn, n_steps, flush_between):
        # each step is a CUDA graph replay (as in the other workloads), so the host's per-call work is not timed
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(dev)
        n0 = _native.launch_count()
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph):
            fn()
        per_step = _native.launch_count() - n0
        for _ in range(2):
            gph.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_steps)]
        for i in range(n_steps):
            if flush_between:
                l2_flush(flush, i)
            ev[i][0].record(stream)
            gph.replay()
            ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
        del gph
        t = sum(a.elapsed_time(b) for a, b in ev)
        if world > 1:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t / n_steps, per_step

    ms_sel, kern_sel = timed(select, max(3, steps // 20), False)
    ms_read, kern_read = timed(read, steps, True)
    peak, peak_kind = hbm_peak()
    sel_bytes = SB * S * n_kv * hd * 2 + SB * n_q * hd * 4 + SB * S * 4 * 2
    read_bytes = B * k * d * 2 + 2 * B * d * 4 + B * k * 4
    res = {"workload": f"D8 top-k slot read at config-2 Library shapes: {B} documents x {C} chunks x {N} fp16 slots, "
                       f"d_s {d}, k {k}; selection keys {n_kv} KV heads x {hd} (fp16), {n_q} query heads",
           "select": {"metric": "documents selected per second (whole job)", "value": SB * world / (ms_sel / 1e3),
                      "unit": "documents/s", "ms_per_step": ms_sel, "docs_per_step": SB, "kernels_per_step": kern_sel,
                      "roofline": {"bound": "hbm", "kernel": "select_scores_mma_kernel + select_topk_cluster_kernel",
                                   "achieved": sel_bytes / (ms_sel / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                                   "frac": sel_bytes / (ms_sel / 1e3) / 1e9 / peak,
                                   "algorithmic_bytes_per_step": sel_bytes, "peak_source": peak_kind},
                      "l2": "1 GiB of keys per step (larger than L2)"},
           "read": {"metric": "D8 decode-read tokens/s (whole job)", "value": B * world / (ms_read / 1e3),
                    "unit": "tokens/s", "ms_per_step": ms_read, "kernels_per_step": kern_read,
                    "roofline": {"bound": "hbm", "kernel": "topk_read_decode_kernel",
                                 "achieved": read_bytes / (ms_read / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                                 "frac": read_bytes / (ms_read / 1e3) / 1e9 / peak,
                                 "algorithmic_bytes_per_step": read_bytes, "peak_source": peak_kind},
                    "l2": "flushed between steps (256 MiB write + read back)"},
           "n_gpus": world, "scaling": "weak"}
    if rank == 0 and world == 1 and cpu_seconds > 0:
        kq = keys[0].float().cpu().numpy()
        q0 = qs[:1].permute(0, 2, 1, 3).cpu().numpy()
        spent, n = 0.0, 0
        while spent < cpu_seconds / 2 and n < 20:
            t0 = time.perf_counter()
            X.topk_select(X.topk_select_scores(q0, kq, valid), k)
            spent += time.perf_counter() - t0
            n += 1
        res["select"]["cpu_baseline"] = {"value": n / spent, "unit": "documents/s", "cores": 1, "kind": "port",
                                         "sample": f"{n} selections of one document (oracle, numpy)"}
        qn = q[:1].cpu().numpy()[None]
        ix = idx[:1].cpu().numpy()
        spent, n = 0.0, 0
        while spent < cpu_seconds / 2 and n < 2000:
            t0 = time.perf_counter()
            X.topk_read(qn, Kf, ix)
            spent += time.perf_counter() - t0
            n += 1
        res["read"]["cpu_baseline"] = {"value": n / spent, "unit": "tokens/s", "cores": 1, "kind": "port",
                                       "sample": f"{n} decode reads of one document (oracle.topk_read, numpy)"}
    del keys, pool
    return res


CFG3 = dict(docs=8, T=2048, C=128, N=512, d_s=2048, d_m=4096, read_temp=12.0, route_temp=10.0)


def tensor_peak() -> tuple:
    """(sustained dense bf16 TFLOP/s, source): the prefill GEMMs run inside a multi-millisecond step."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops_sustained"]), "measured sustained (MEASURED_PEAKS.json)"
        except (KeyError, ValueError):
            pass
    return 1400.0, "fallback 1.4 PFLOP/s sustained"


def run_prefill(torch, dist, dev, world: int, rank: int, steps: int, warmup: int, flush, stream,
                docs: int = 8) -> dict:
    """8 documents per GPU, each a Library of 128 chunks x 512 fp16 slots (65,536 slots,
    d_s 2048), T = 2048 query tokens per document with bf16 hidden states (d_m 4096), every chunk read (dense
    routing, full masked softmax per chunk). A step: input projection, dense routing, the tensor-core prefill
    read (scores GEMM with the chunk softmax folded into f16 weights, then the read GEMM), output projection +
    residual. Weak scaling: every rank its own documents."""
    from kv_skill_v2_b200 import _native, ops

    B, T, C, N, d_s, d_m = int(docs), CFG3["T"], CFG3["C"], CFG3["N"], CFG3["d_s"], CFG3["d_m"]
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    slots = torch.empty(B * C, N, d_s, dtype=torch.float16, device=dev)
    for c0 in range(0, B * C, 128):
        x = torch.randn(min(128, B * C - c0), N, d_s, generator=g, device=dev)
        slots[c0:c0 + x.shape[0]] = (x / x.norm(dim=-1, keepdim=True)).half()
        del x
    po = torch.arange(B * C, dtype=torch.int32, device=dev).view(B, C)
    nv = torch.full((B, C), N, dtype=torch.int32, device=dev)
    pages = ops.Pages(slots=slots, page_of=po, n_valid=nv, S=ops.summaries(slots, po, nv))
    W_in = torch.randn(d_s, d_m, generator=g, device=dev) * 0.02
    W_out = torch.randn(d_m, d_s, generator=g, device=dev) * 0.02
    R = B * T
    n_in = 2
    hs = (torch.randn(n_in, R, d_m, generator=g, device=dev)).to(torch.bfloat16)
    h = hs[0].clone()
    h_out = torch.empty_like(h)
    holder = {}
    P_in, P_out = ops.weights_prep(W_in), ops.weights_prep(W_out)  # 3xF16 form, prepared once

    def step():
        q, _, _, _ = ops.project_in(h, W_in, w_prep=P_in)
        _, _, w, _ = ops.route(q, pages.S, rows_per_lib=T, top_k=0, route_temp=CFG3["route_temp"])
        r = ops.read_prefill(q, pages, w, rows_per_lib=T, read_temp=CFG3["read_temp"])
        ops.project_out(r, W_out, h, want_delta=False, h_out=h_out, w_prep=P_out)
        holder["q"], holder["w"] = q, w

    with torch.inference_mode():
        step()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        n0 = _native.launch_count()
        with torch.cuda.graph(graph):
            step()
        kernels = _native.launch_count() - n0
        q_s, w_s = holder["q"], holder["w"]
        for i in range(warmup):
            h.copy_(hs[i % n_in])
            l2_flush(flush, i)
            graph.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            h.copy_(hs[i % n_in])
            l2_flush(flush, i)
            ev[i][0].record(stream)
            graph.replay()
            ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
        # the prefill read alone (both GEMMs), for the tensor roofline
        rg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(rg):
            ops.read_prefill(q_s, pages, w_s, rows_per_lib=T, read_temp=CFG3["read_temp"])
        n_rl = max(3, min(steps, 20))
        evr = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_rl)]
        rg.replay()
        for i in range(n_rl):
            l2_flush(flush, i)
            evr[i][0].record(stream)
            rg.replay()
            evr[i][1].record(stream)
        torch.cuda.synchronize(dev)
    t_ms = sum(a.elapsed_time(b) for a, b in ev)
    t_max = t_ms
    if world > 1:
        t = torch.tensor([t_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_max = float(t.item())
    ms = t_max / steps
    t_read = statistics.mean(a.elapsed_time(b) for a, b in evr) / 1000.0
    read_flop = 2 * 2.0 * R * (C * N) * d_s                      # scores + read GEMMs
    step_flop = read_flop + 2.0 * R * C * d_s + 2 * 2.0 * R * d_m * d_s  # + routing + both projections
    peak, peak_src = tensor_peak()
    del graph, rg
    return {"workload": f"BASELINE config 3: {B} documents x T=2048 tokens, 128 chunks x 512 fp16 slots each, d_s 2048, "
                        "d_m 4096, bf16 hiddens, every chunk read (dense routing, masked softmax per chunk)",
            "metric": "prefill Library-read tokens/s (whole job)", "value": R * world * steps / (t_max / 1000.0),
            "unit": "tokens/s", "n_gpus": world, "ms_per_step": ms, "scaling": "weak",
            "kernels_per_step": kernels, "gpu_launches": kernels * steps,
            "step_tflops": step_flop / (ms / 1000.0) / 1e12, "algorithmic_flop_per_step": step_flop,
            "roofline": {"bound": "tensor", "kernel": "prefill_scores_kernel + prefill_read_pair_kernel (+ q to f16)",
                         "achieved": read_flop / t_read / 1e12, "peak": peak, "unit": "TFLOP/s",
                         "frac": read_flop / t_read / 1e12 / peak, "algorithmic_flop_per_launch": read_flop,
                         "launch_ms": t_read * 1e3, "peak_source": peak_src},
            "l2": "flushed between steps (256 MiB write + read back); the slots (2 GiB) are > L2"}


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from kv_skill_v2_b200 import LibraryInjector, LinearInterface, PagedLibrary, _native, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the Library read has no CPU path)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    if args.sharded_only or args.selector_only or args.prefill_only or args.library_build_only or args.topk_only:
        flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        if args.topk_only:
            res = run_topk(torch, dist, dev, world, rank, args.steps, args.warmup, flush,
                           torch.cuda.current_stream(dev),
                           cpu_seconds=0.0 if args.no_cpu_baseline else args.cpu_seconds)
        elif args.library_build_only:
            res = run_library_build(torch, dist, dev, world, rank, args.steps, args.warmup,
                                    torch.cuda.current_stream(dev),
                                    cpu_seconds=0.0 if args.no_cpu_baseline else args.cpu_seconds,
                                    docs=args.library_build_docs)
        elif args.prefill_only:
            res = run_prefill(torch, dist, dev, world, rank, args.steps, args.warmup, flush,
                              torch.cuda.current_stream(dev), docs=args.prefill_docs)
        elif args.sharded_only:
            res = run_sharded(torch, dist, dev, world, rank, args.steps, args.warmup, flush,
                              torch.cuda.current_stream(dev), n_chunks=args.sharded_chunks)
        else:
            res = run_selector(torch, dist, dev, world, rank, args.steps, args.warmup, flush,
                               torch.cuda.current_stream(dev))
        res["device_status"] = ops.device_status(dev)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(res), flush=True)
        return

    docs, d_m = args.docs, CFG["d_m"]
    pages, W_in, W_out, g = build_workload(torch, dev, docs, rank)
    R = docs * CFG["T"]
    n_h = args.warmup + args.steps
    hs = torch.randn(n_h, R, d_m, generator=g, device=dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    # the interface weights in the 3xF16 form, prepared once as LibraryInjector does when it first uses them
    P_in, P_out = ops.weights_prep(W_in), ops.weights_prep(W_out)

    def step(h, h_out):
        q, _, _, idx, wk, _, _ = ops.project_in_route(h, W_in, S=pages.S, rows_per_lib=CFG["T"], top_k=CFG["top_k"],
                                                      route_temp=CFG["route_temp"], w_prep=P_in)
        r = ops.read_decode(q, pages, idx, wk, rows_per_lib=CFG["T"], read_temp=CFG["read_temp"])
        _, _, rel = ops.project_out(r, W_out, h, want_delta=False, h_out=h_out, want_rel=True, w_prep=P_out)
        return q, idx, wk, rel

    # ---- graph capture of one step on static buffers
    h_static = hs[0].clone()
    h_out = torch.empty_like(h_static)
    for _ in range(2):
        step(h_static, h_out)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    n0 = _native.launch_count()
    with torch.cuda.graph(graph):
        q_s, idx_s, wk_s, rel_s = step(h_static, h_out)
    torch.cuda.synchronize(dev)
    kernels_per_step = _native.launch_count() - n0  # libxencb kernels in the captured step; a replay re-issues them

    bus = None
    try:
        props = torch.cuda.get_device_properties(dev)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}"
    except AttributeError:
        pass
    sampler = ClockSampler(bus)
    with sampler:
        if args.kernel_only:
            # profiling mode: replays only; prints the slot rows each replay's read streamed, so that an ncu
            # capture of replay i can be set against its algorithmic bytes
            rows = []
            for i in range(args.warmup + args.steps):
                h_static.copy_(hs[i])
                graph.replay()
                rows.append(int(pages.n_valid.gather(1, idx_s.long().clamp_min(0)).sum().item()))
            torch.cuda.synchronize(dev)
            if rank == 0:
                print(json.dumps({"kernel_only": True, "docs": docs, "d_s": CFG["d_s"], "kernels_per_step": kernels_per_step,
                                  "slot_rows_per_replay": rows}), flush=True)
            return
        # ---- value: graph replays, events per step, L2 flush + next input between steps
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.warmup):
            h_static.copy_(hs[i])
            l2_flush(flush, i)
            graph.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        rows_read = 0
        for i in range(args.steps):
            h_static.copy_(hs[args.warmup + i])
            l2_flush(flush, i)
            ev[i][0].record(stream)
            graph.replay()
            ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t_ms = sum(a.elapsed_time(b) for a, b in ev)
        rows_read = int(pages.n_valid.gather(1, idx_s.long().clamp_min(0)).sum().item())  # routing of the last step
        t_max = t_ms
        if world > 1:
            t = torch.tensor([t_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_max = float(t.item())
        value = R * args.steps * world / (t_max / 1000.0)

        # ---- roofline: the read kernel alone (events recorded by libxencb right around it), q/idx/wk of the last
        # step, after an L2 flush; a sleep kernel keeps the stream busy while the host enqueues the call, so the
        # interval holds the kernel only. The whole read op (kernel + merge, one graph replay) is timed beside it.
        n_rl = max(args.steps, 50)
        evk = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_rl)]
        for i in range(3):
            l2_flush(flush, i)
            ops.read_decode(q_s, pages, idx_s, wk_s, rows_per_lib=CFG["T"])
        for i in range(n_rl):
            l2_flush(flush, i)
            torch.cuda._sleep(200000)
            ops.read_kernel_events(evk[i][0], evk[i][1])
            ops.read_decode(q_s, pages, idx_s, wk_s, rows_per_lib=CFG["T"])
        torch.cuda.synchronize(dev)
        t_read = statistics.mean(a.elapsed_time(b) for a, b in evk) / 1000.0
        rg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(rg):
            ops.read_decode(q_s, pages, idx_s, wk_s, rows_per_lib=CFG["T"])
        evr = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_rl)]
        for i in range(n_rl):
            l2_flush(flush, i)
            evr[i][0].record(stream)
            rg.replay()
            evr[i][1].record(stream)
        torch.cuda.synchronize(dev)
        t_read_op = statistics.mean(a.elapsed_time(b) for a, b in evr) / 1000.0
        read_bytes = rows_read * CFG["d_s"] * 2 + R * CFG["d_s"] * 4
        peak, peak_kind = hbm_peak()
        achieved = read_bytes / t_read / 1e9
        tpr = traffic_per_row()

        # ---- e2e: the public API (hooked reader + LibraryInjector), host buffers, copies inside the timed region
        class Reader(torch.nn.Module):
            def __init__(self):
                super().__init__()
                self.layers = torch.nn.ModuleList([torch.nn.Identity()])
                self._p = torch.nn.Parameter(torch.zeros(1, device=dev), requires_grad=False)

            def forward(self, x):
                for blk in self.layers:
                    x = blk(x)
                return x

        reader = Reader()
        itf = LinearInterface(W_in.t(), W_out.t(), [0]).to(dev).requires_grad_(False)
        inj = LibraryInjector(reader, itf, top_k=CFG["top_k"], read_temp=CFG["read_temp"], route_temp=CFG["route_temp"])
        inj.load_library(PagedLibrary({0: pages}))
        h_host = [hs[i].view(docs, CFG["T"], d_m).cpu().pin_memory() for i in range(min(n_h, 64))]
        out_host = [torch.empty(docs, CFG["T"], d_m, dtype=torch.float32).pin_memory() for _ in range(2)]
        # a serving loop: host->device copies of the next step's hidden states and device->host copies of the last
        # step's outputs run on a copy stream while the compute stream runs the hooked reader; two device input
        # buffers alternate. Timed as one device span from the first upload to the last download.
        cstream = torch.cuda.Stream(dev)
        h_dev = [torch.empty(docs, CFG["T"], d_m, dtype=torch.float32, device=dev) for _ in range(2)]
        h_ready = [torch.cuda.Event() for _ in range(2)]
        h_free = [torch.cuda.Event() for _ in range(2)]
        y_done = [torch.cuda.Event() for _ in range(2)]
        d2h_done = [torch.cuda.Event() for _ in range(2)]
        t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        waited = [0.0]

        def serve(n_steps, timed):
            ys = [None, None]
            with torch.cuda.stream(cstream):
                if timed:
                    t_start.record(cstream)
                h_dev[0].copy_(h_host[0], non_blocking=True)
                h_ready[0].record(cstream)
            for i in range(n_steps):
                b = i & 1
                if i + 1 < n_steps:  # upload the next step's input once its buffer is free
                    with torch.cuda.stream(cstream):
                        if i >= 1:
                            cstream.wait_event(h_free[1 - b])
                        h_dev[1 - b].copy_(h_host[(i + 1) % len(h_host)], non_blocking=True)
                        h_ready[1 - b].record(cstream)
                stream.wait_event(h_ready[b])
                if i >= 2:  # the host consumes step i-2's output before its buffer is reused: at most 2 steps in flight
                    tw = time.perf_counter()
                    d2h_done[b].synchronize()
                    waited[0] += time.perf_counter() - tw
                ys[b] = reader(h_dev[b])
                h_free[b].record(stream)
                y_done[b].record(stream)
                inj.mag_terms.clear()
                with torch.cuda.stream(cstream):  # download this step's output behind the next step's compute
                    cstream.wait_event(y_done[b])
                    out_host[b].copy_(ys[b], non_blocking=True)
                    d2h_done[b].record(cstream)
            if timed:
                t_end.record(cstream)

        with torch.inference_mode():
            serve(args.warmup, False)
            torch.cuda.synchronize(dev)
            t_host = time.perf_counter()
            waited[0] = 0.0
            serve(args.steps, True)
            t_host = time.perf_counter() - t_host
            torch.cuda.synchronize(dev)
        t_e2e = t_start.elapsed_time(t_end)
        if world > 1:
            t = torch.tensor([t_e2e], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_e2e = float(t.item())
        e2e = R * args.steps * world / (t_e2e / 1000.0)
        inj.detach()
        sharded = selector = prefill = lbuild = topk = None
        if not args.no_topk:
            topk = run_topk(torch, dist, dev, world, rank, args.steps, args.warmup, flush, stream)
        if not args.no_library_build:
            lbuild = run_library_build(torch, dist, dev, world, rank, max(3, args.steps // 20), args.warmup, stream)
        if not args.no_prefill:
            prefill = run_prefill(torch, dist, dev, world, rank, max(3, args.steps // 10), args.warmup, flush, stream)
        if not args.no_sharded:
            sharded = run_sharded(torch, dist, dev, world, rank, args.steps, args.warmup, flush, stream)
        if not args.no_selector:
            selector = run_selector(torch, dist, dev, world, rank, args.steps, args.warmup, flush, stream)
    status = ops.device_status(dev)
    clocks = sampler.summary()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = CpuOracle(n_docs=2).sample(args.cpu_seconds)

    if world > 1:
        del graph, rg
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded Gaussian unit slots, random weights)",
            "precision": "read: f16 slot, q and p operands with fp32 accumulate (q and the softmax weights p are "
                         "rounded to f16 before the tensor-core products); projections: fp32-faithful 3xF16 "
                         "(about 22-bit operands, fp32 accumulate); routing logits and softmax in fp32",
            "config": config_dict(docs),
            "roofline": {"bound": "hbm", "kernel": "read_decode_mma_kernel",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s", "algorithmic_bytes_per_launch": read_bytes,
                         "launch_us": t_read * 1e6,
                         "read_op_us": t_read_op * 1e6,
                         "read_op": "read_decode_mma_kernel + read_merge_kernel as one CUDA-graph replay, events "
                                    "around the replay",
                         "traffic": None if tpr is None else tpr * rows_read},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": R * d_m * 4, "d2h_bytes_per_step": R * d_m * 4,
                    "host_enqueue_us_per_step": 1e6 * t_host / args.steps,
                    "host_wait_us_per_step": 1e6 * waited[0] / args.steps,
                    "path": "LibraryInjector forward hook on a reader block (CUDA-graph replay of the fused hook path), "
                            "PagedLibrary of 64 documents; per step an H2D copy of h from pinned memory and a D2H "
                            "copy of the output, on a copy stream overlapping the neighbouring steps' compute "
                            "(double-buffered; the host reads step i-2's output before reusing its buffer); one "
                            "device-timed span over all steps; no L2 flush (each step "
                            "streams ~600 MB of slots and weights, above the 126 MB L2)"},
            "gpu_launches": kernels_per_step * args.steps,
            "sharded": sharded,
            "selector": selector,
            "prefill": prefill,
            "library_build": lbuild,
            "topk": topk,
            "clocks": clocks, "device_status": status}
    print(json.dumps(line), flush=True)


def main(argv=None) -> None:
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
