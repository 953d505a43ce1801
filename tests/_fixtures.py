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


class _TinyAttention(nn.Module):
    """An attention stand-in with the members the D8 selector reads: q_proj (n_kv * groups heads), k_proj, v_proj,
    o_proj, head_dim, num_key_value_groups. It mixes values causally (running mean over positions)."""

    def __init__(self, d: int, n_kv: int, head_dim: int, groups: int):
        super().__init__()
        self.head_dim, self.num_key_value_groups = head_dim, groups
        self.q_proj = nn.Linear(d, n_kv * groups * head_dim)
        self.k_proj = nn.Linear(d, n_kv * head_dim)
        self.v_proj = nn.Linear(d, n_kv * head_dim)
        self.o_proj = nn.Linear(n_kv * head_dim, d)

    def forward(self, x):
        v = self.v_proj(x)
        T = v.shape[1]
        run = v.cumsum(1) / torch.arange(1, T + 1, device=v.device, dtype=v.dtype).view(1, T, 1)
        return self.o_proj(run)


class _TinyAttnBlock(nn.Module):
    def __init__(self, d: int, n_kv: int, head_dim: int, groups: int):
        super().__init__()
        self.mlp = nn.Linear(d, d)
        self.self_attn = _TinyAttention(d, n_kv, head_dim, groups)

    def forward(self, x):
        return torch.tanh(self.mlp(x) + 0.5 * self.self_attn(x))


class TinyAttnReader(nn.Module):
    """A decoder stand-in whose blocks carry attention modules (model.layers[i].self_attn), forward(x [B,T,d]) ->
    hidden state, logits(x) through an lm_head (bypassing __call__, as the reference's fake models do)."""

    def __init__(self, d: int = 32, L: int = 8, n_kv: int = 2, head_dim: int = 8, groups: int = 2, vocab: int = 50,
                 seed: int = 0):
        super().__init__()
        torch.manual_seed(seed)
        self.model = nn.Module()
        self.model.layers = nn.ModuleList(_TinyAttnBlock(d, n_kv, head_dim, groups) for _ in range(L))
        self.config = _Cfg(L, d)
        self.lm_head = nn.Linear(d, vocab)

    @property
    def device(self):
        return next(self.parameters()).device

    def forward(self, x):
        for blk in self.model.layers:
            x = blk(x)
        return x

    def logits(self, x):
        return self.lm_head(self.forward(x))

    def arrays(self) -> dict:
        return {f"m_{k}": v.detach().cpu().numpy() for k, v in self.state_dict().items()}

    def load_arrays(self, rec: dict) -> "TinyAttnReader":
        sd = {k[2:]: torch.from_numpy(np.asarray(v)) for k, v in rec.items() if k.startswith("m_")}
        self.load_state_dict(sd)
        return self
