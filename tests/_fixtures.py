"""Shared helpers for the tests: golden-case loading, error metrics, a tiny fake reader."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = 2e-3  # max|out - ref| <= TOL * max|ref| (the path's stated output tolerance)


def load_case(name: str) -> dict:
    """A golden case with its inputs (cases that share inputs name the case holding them)."""
    rec = dict(np.load(GOLDEN / f"{name}.npz"))
    if "inputs" in rec:
        base = dict(np.load(GOLDEN / f"{str(rec.pop('inputs'))}.npz"))
        for k in ("K", "n_valid", "h", "W_in", "W_out"):
            rec[k] = base[k]
    return rec


def rel_err(a, b) -> float:
    a = a.detach().cpu().double().numpy() if isinstance(a, torch.Tensor) else np.asarray(a, np.float64)
    b = b.detach().cpu().double().numpy() if isinstance(b, torch.Tensor) else np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def topk_sets(w) -> list:
    w = w.detach().cpu().numpy() if isinstance(w, torch.Tensor) else np.asarray(w)
    return [frozenset(np.flatnonzero(row > 0).tolist()) for row in w.reshape(-1, w.shape[-1])]


class _Cfg:
    def __init__(self, L, d):
        self.num_hidden_layers, self.hidden_size = L, d


class _Blocks(nn.Module):
    def __init__(self, d, L):
        super().__init__()
        self.layers = nn.ModuleList(nn.Linear(d, d) for _ in range(L))


class TinyReader(nn.Module):
    """A stack of Linear + tanh blocks with model.layers / config / device, like a decoder."""

    def __init__(self, d: int, L: int, seed: int = 0):
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


def unit_rows(n: int, d: int, g: torch.Generator) -> torch.Tensor:
    x = torch.randn(n, d, generator=g)
    return (x / x.norm(dim=-1, keepdim=True)).half().float()
