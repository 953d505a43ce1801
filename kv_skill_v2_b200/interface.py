"""Reader <-> encoder interface: build / save / load, EncoderLens, param groups, counts.

Mirrors xenc/interface.py of the reference (make_interface :22-28, EncoderLens :31-43, interface_param_groups
:46-66, save_interface :74-86 with format "xenc.interface.v1", load_interface :89-106, count_params
:109-119). The interface class itself comes from the un-vendored deltaskill package in the reference; the
members the Library read uses (xenc/injector.py:54-77: A, B, gate_w, gate_b, log_gain, _pos) are restated
here as ModelInterface. Their exact parameterisation inside deltaskill (biases, init) is not in the
reference tree, so it is an assumption: A and B are bias-free Linear maps (or a rank-r pair for A), B is
zero-initialised so the branch is a no-op at init.

The Library read never calls the interface's Python methods for these two classes: LibraryInjector reads
their weights and runs the fused projection kernels. query/gate/gain/write exist for duck-typed callers.
"""

from __future__ import annotations

import os

import torch
import torch.nn as nn

FORMAT = "xenc.interface.v1"


class ModelInterface(nn.Module):
    def __init__(self, d_m: int, d_s: int, inject_layers: list, gate_bias_init: float = -2.0,
                 gain_init: float = 0.0, rank: int = 0):
        super().__init__()
        self.d_m, self.d_s = int(d_m), int(d_s)
        self.inject_layers = [int(li) for li in inject_layers]
        self.rank = int(rank or 0)
        self._pos = {li: i for i, li in enumerate(self.inject_layers)}
        if self.rank > 0:
            self.A = nn.Sequential(nn.Linear(self.d_m, self.rank, bias=False), nn.Linear(self.rank, self.d_s, bias=False))
        else:
            self.A = nn.Linear(self.d_m, self.d_s, bias=False)
        self.B = nn.Linear(self.d_s, self.d_m, bias=False)
        nn.init.zeros_(self.B.weight)
        n = len(self.inject_layers)
        self.gate_w = nn.Parameter(torch.zeros(self.d_m))
        self.gate_b = nn.Parameter(torch.full((n,), float(gate_bias_init)))
        self.log_gain = nn.Parameter(torch.full((n,), float(gain_init)))

    # duck-typed API (xenc/injector.py:54-77)
    def query(self, hn: torch.Tensor) -> torch.Tensor:
        q = self.A(hn)
        return q / (q.norm(dim=-1, keepdim=True) + 1e-6)

    def gate(self, hn: torch.Tensor, li: int) -> torch.Tensor:
        return torch.sigmoid(hn @ self.gate_w + self.gate_b[self._pos[li]]).unsqueeze(-1)

    def gain(self, li: int) -> torch.Tensor:
        return self.log_gain[self._pos[li]].exp()

    def write(self, r: torch.Tensor) -> torch.Tensor:
        return self.B(r)

    # weights in the layout the kernels take
    def query_weights(self) -> list:
        """[(weight [out, in] float32, bias or None), ...] of A's Linear maps in order."""
        mods = list(self.A) if isinstance(self.A, nn.Sequential) else [self.A]
        return [(m.weight, m.bias) for m in mods]


class LinearInterface(nn.Module):
    """q = L2(hn @ W_in); gate = gain = 1; write(r) = r @ W_out -- the interface of BASELINE config 1
    (W_in [d_m, d_s], W_out [d_s, d_m])."""

    def __init__(self, W_in: torch.Tensor, W_out: torch.Tensor, inject_layers: list | None = None):
        super().__init__()
        if W_in.shape[1] != W_out.shape[0] or W_in.shape[0] != W_out.shape[1]:
            raise ValueError(f"W_in {tuple(W_in.shape)} and W_out {tuple(W_out.shape)} do not pair up")
        self.d_m, self.d_s = int(W_in.shape[0]), int(W_in.shape[1])
        self.inject_layers = [int(li) for li in (inject_layers or [])]
        # stored as nn.Linear weights ([out, in]), the layout the projection kernels take
        self.w_in = nn.Parameter(W_in.detach().t().contiguous().float())
        self.w_out = nn.Parameter(W_out.detach().t().contiguous().float())

    def query(self, hn):
        q = hn @ self.w_in.t()
        return q / (q.norm(dim=-1, keepdim=True) + 1e-6)

    def gate(self, hn, li):
        return torch.ones(*hn.shape[:-1], 1, dtype=hn.dtype, device=hn.device)

    def gain(self, li):
        return torch.ones((), device=self.w_in.device)

    def write(self, r):
        return r @ self.w_out.t()


def make_interface(d_reader: int, d_encoder: int, reader_layers: list, rank: int = 0, gate_bias_init: float = -2.0,
                   gain_init: float = 0.0) -> ModelInterface:
    layers = [int(li) for li in reader_layers]
    if len(set(layers)) != len(layers):
        raise ValueError(f"duplicate reader layers: {layers}")
    return ModelInterface(int(d_reader), int(d_encoder), layers, gate_bias_init=gate_bias_init, gain_init=gain_init,
                          rank=int(rank or 0))


class EncoderLens(nn.Module):
    """Per-encoder map d_enc -> d_core on the last dim (orthogonal init, no bias)."""

    def __init__(self, d_enc: int, d_core: int):
        super().__init__()
        self.d_enc, self.d_core = int(d_enc), int(d_core)
        self.proj = nn.Linear(self.d_enc, self.d_core, bias=False)
        nn.init.orthogonal_(self.proj.weight)

    def forward(self, K: torch.Tensor) -> torch.Tensor:
        if K.shape[-1] != self.d_enc:
            raise ValueError(f"EncoderLens expects last dim {self.d_enc}, got {K.shape[-1]}")
        return self.proj(K.to(self.proj.weight.dtype))


def interface_param_groups(itf: nn.Module, lr: float, selector=None, selector_lr: float | None = None,
                           lr_A: float | None = None) -> list:
    trainable = [p for p in itf.parameters() if p.requires_grad]
    if lr_A is not None and hasattr(itf, "A"):
        a_ids = {id(p) for p in itf.A.parameters()}
        groups = [{"params": [p for p in trainable if id(p) not in a_ids], "lr": lr, "name": "interface"},
                  {"params": [p for p in itf.A.parameters() if p.requires_grad], "lr": float(lr_A),
                   "name": "interface_A"}]
        groups = [g for g in groups if g["params"]]
    else:
        groups = [{"params": trainable, "lr": lr, "name": "interface"}]
    if selector is not None:
        seen = {id(p) for g in groups for p in g["params"]}
        extra = [p for p in selector.parameters() if p.requires_grad and id(p) not in seen]
        if extra:
            groups.append({"params": extra, "lr": lr if selector_lr is None else selector_lr, "name": "selector"})
    return groups


def _config(itf: ModelInterface) -> dict:
    return {"d_m": itf.d_m, "d_s": itf.d_s, "inject_layers": list(itf.inject_layers), "rank": int(itf.rank or 0)}


def save_interface(itf: ModelInterface, path: str, selector=None, extra: dict | None = None) -> None:
    """Atomic save (write to a temporary file, then rename)."""
    blob = {"format": FORMAT, "config": _config(itf),
            "state_dict": {k: v.detach().cpu() for k, v in itf.state_dict().items()},
            "selector": None, "extra": extra}
    if selector is not None:
        blob["selector"] = {"config": selector.config(),
                            "state_dict": {k: v.detach().cpu() for k, v in selector.state_dict().items()}}
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    tmp = path + ".tmp"
    torch.save(blob, tmp)
    os.replace(tmp, path)


def load_interface(path: str, d_reader: int, d_encoder: int, reader_layers: list, map_location="cpu"):
    """-> (itf, selector or None, extra); ValueError when the saved (d_m, d_s, layers) differ."""
    from .selector import LayerSelector

    blob = torch.load(path, map_location=map_location, weights_only=False)
    cfg = blob["config"]
    want = (int(d_reader), int(d_encoder), [int(li) for li in reader_layers])
    got = (cfg["d_m"], cfg["d_s"], list(cfg["inject_layers"]))
    if want != got:
        raise ValueError(f"interface at {path} has (d_m, d_s, layers)={got}, expected {want}")
    itf = make_interface(d_reader, d_encoder, reader_layers, rank=cfg.get("rank", 0))
    itf.load_state_dict(blob["state_dict"], strict=True)
    sel = None
    if blob.get("selector") is not None:
        sc = blob["selector"]["config"]
        sel = LayerSelector(sc["d_m"], sc["cand_layers"], k=sc["k"], straight_through=sc.get("straight_through", False))
        sel.load_state_dict(blob["selector"]["state_dict"], strict=True)
    return itf, sel, blob.get("extra")


def count_params(itf: nn.Module, selector=None) -> dict:
    n = sum(p.numel() for p in itf.parameters())
    out = {"interface": n}
    for name in ("A", "B"):
        m = getattr(itf, name, None)
        if isinstance(m, nn.Module):
            out[name] = sum(p.numel() for p in m.parameters())
    out["gate_gain"] = n - out.get("A", 0) - out.get("B", 0)
    out["selector"] = sum(p.numel() for p in selector.parameters()) if selector is not None else 0
    out["total"] = n + out["selector"]
    return out
