#!/usr/bin/env python
"""Benchmark of the Library read at BASELINE config 2 (decode).

Workload (per GPU): 64 documents, each its own Library of C=64 chunks x 512 fp16 slots (d_s=2048; the last
chunk ragged, U{1..512} valid), reader width d_m=4096, one query token per document per step, top-4 chunk
routing, read_temp 12, route_temp 10. A step is one pass of the hot path for the 64 tokens: rms_norm +
query projection + L2, routing, the split-K masked read, output projection + residual + mag term.

* value: whole-job tokens/s with inputs resident in HBM (the step captured in a CUDA graph), timed per step
  with CUDA events on the launching stream, L2 flushed (256 MiB write) between steps outside the events;
  max over ranks. Multi-GPU runs are weak-scaled replicas (every rank its own 64 documents, no collective
  in the data path; one all-reduce of the elapsed time after timing).
* e2e: the same metric through the public API -- a reader model whose hooked block runs LibraryInjector --
  from pinned host hidden states, H2D copy and D2H copy of the result inside the timed region.
* roofline: the read (read_decode_kernel + its merge) timed alone; achieved = algorithmic bytes (valid slot
  rows of the routed chunks, read once, + q in + r out) / time, against MEASURED_PEAKS.json hbm_gbs.
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
    return ap.parse_args(argv)


def config_dict(docs: int) -> dict:
    return {"workload": "BASELINE config 2: decode, batch of independent documents, top-4 of 64 chunks",
            "docs_per_gpu": docs, "chunks": CFG["C"], "slots_per_chunk": CFG["N"], "d_s": CFG["d_s"],
            "d_m": CFG["d_m"], "top_k": CFG["top_k"], "query_tokens_per_doc": CFG["T"], "slot_dtype": "f16",
            "hidden_dtype": "f32", "weights_dtype": "f32", "read_temp": CFG["read_temp"],
            "route_temp": CFG["route_temp"], "last_chunk_valid": "U{1..512}",
            "l2": "flushed between timed steps (256 MiB write); inputs per step > L2 as well",
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


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from kv_skill_v2_b200 import LibraryInjector, LinearInterface, PagedLibrary, ops

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

    docs, d_m = args.docs, CFG["d_m"]
    pages, W_in, W_out, g = build_workload(torch, dev, docs, rank)
    R = docs * CFG["T"]
    n_h = args.warmup + args.steps
    hs = torch.randn(n_h, R, d_m, generator=g, device=dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(h, h_out):
        q, _, _, _ = ops.project_in(h, W_in)
        idx, wk, _, _ = ops.route(q, pages.S, rows_per_lib=CFG["T"], top_k=CFG["top_k"], route_temp=CFG["route_temp"])
        r = ops.read_decode(q, pages, idx, wk, rows_per_lib=CFG["T"], read_temp=CFG["read_temp"])
        _, _, rel = ops.project_out(r, W_out, h, want_delta=False, h_out=h_out, want_rel=True)
        return q, idx, wk, rel

    kernels_per_step = 8  # gemm+finish (in), logits+topk, read+merge, gemm+finish (out)

    # ---- graph capture of one step on static buffers
    h_static = hs[0].clone()
    h_out = torch.empty_like(h_static)
    for _ in range(2):
        step(h_static, h_out)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        q_s, idx_s, wk_s, rel_s = step(h_static, h_out)
    torch.cuda.synchronize(dev)

    bus = None
    try:
        props = torch.cuda.get_device_properties(dev)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}"
    except AttributeError:
        pass
    sampler = ClockSampler(bus)
    with sampler:
        if args.kernel_only:
            for i in range(args.warmup + args.steps):
                h_static.copy_(hs[i])
                graph.replay()
            torch.cuda.synchronize(dev)
            return
        # ---- value: graph replays, events per step, L2 flush + next input between steps
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.warmup):
            h_static.copy_(hs[i])
            flush.fill_(i & 0xFF)
            graph.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        rows_read = 0
        for i in range(args.steps):
            h_static.copy_(hs[args.warmup + i])
            flush.fill_(i & 0xFF)
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

        # ---- roofline: the read alone (read_decode_kernel + merge), q/idx/wk of the last step
        rg = torch.cuda.CUDAGraph()
        ops.read_decode(q_s, pages, idx_s, wk_s, rows_per_lib=CFG["T"])
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(rg):
            ops.read_decode(q_s, pages, idx_s, wk_s, rows_per_lib=CFG["T"])
        n_rl = max(args.steps, 50)
        evr = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_rl)]
        for i in range(3):
            flush.fill_(i)
            rg.replay()
        for i in range(n_rl):
            flush.fill_(i & 0xFF)
            evr[i][0].record(stream)
            rg.replay()
            evr[i][1].record(stream)
        torch.cuda.synchronize(dev)
        t_read = statistics.mean(a.elapsed_time(b) for a, b in evr) / 1000.0
        read_bytes = rows_read * CFG["d_s"] * 2 + 2 * R * CFG["d_s"] * 4
        peak, peak_kind = hbm_peak()
        achieved = read_bytes / t_read / 1e9
        tpr = traffic_per_row()

        # ---- e2e: the public API (hooked reader + LibraryInjector), host buffers, copies inside the events
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
        out_host = torch.empty(docs, CFG["T"], d_m, dtype=torch.float32).pin_memory()
        eve = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        with torch.inference_mode():
            for i in range(args.warmup):
                reader(h_host[i % len(h_host)].to(dev, non_blocking=True))
                inj.mag_terms.clear()
            torch.cuda.synchronize(dev)
            for i in range(args.steps):
                flush.fill_(i & 0xFF)
                eve[i][0].record(stream)
                hd = h_host[i % len(h_host)].to(dev, non_blocking=True)
                y = reader(hd)
                out_host.copy_(y, non_blocking=True)
                eve[i][1].record(stream)
                inj.mag_terms.clear()
            torch.cuda.synchronize(dev)
        t_e2e = sum(a.elapsed_time(b) for a, b in eve)
        if world > 1:
            t = torch.tensor([t_e2e], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_e2e = float(t.item())
        e2e = R * args.steps * world / (t_e2e / 1000.0)
        inj.detach()
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
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Gaussian unit slots, random weights)",
            "config": config_dict(docs),
            "roofline": {"bound": "hbm", "kernel": "read_decode_kernel + read_merge_kernel",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s", "algorithmic_bytes_per_launch": read_bytes,
                         "launch_us": t_read * 1e6,
                         "traffic": None if tpr is None else tpr * rows_read},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": R * d_m * 4, "d2h_bytes_per_step": R * d_m * 4,
                    "path": "LibraryInjector forward hook on a reader block, PagedLibrary of 64 documents"},
            "gpu_launches": kernels_per_step * args.steps,
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
