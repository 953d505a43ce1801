"""LayerSelector: sparse top-k gate over candidate reader layers (mirrors xenc/selector.py).

Per forward: at the first candidate layer the selector reads rms_norm(h) once and stores per-token weights
w [B, T, n_cand] (top-k of z = u(hn), softmax over the kept, zeros elsewhere; straight-through forward is
1/k on the kept). Each candidate layer's delta is rescaled to a matched norm,
||out|| / ||h|| == w_l * exp(log_alpha) (xenc/selector.py:95-110).

The arithmetic runs in the xencb kernels (selector_logits, selector_weights, selector_apply). Inside
LibraryInjector the logits are fused into the input projection and the rescale into the output
projection; the methods here serve direct calls. Forward only: the kernels carry no autograd.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import ops

_EPS = 1e-6


class LayerSelector(nn.Module):
    def __init__(self, d_m: int, cand_layers: list, k: int = 2, alpha_init: float = 0.02,
                 straight_through: bool = False):
        super().__init__()
        cand_layers = [int(li) for li in cand_layers]
        if len(set(cand_layers)) != len(cand_layers):
            raise ValueError(f"duplicate candidate layers: {cand_layers}")
        if not 1 <= k <= len(cand_layers):
            raise ValueError(f"k={k} must be in [1, {len(cand_layers)}]")
        if len(cand_layers) > 32:
            raise ValueError(f"at most 32 candidate layers are supported, got {len(cand_layers)}")
        if alpha_init <= 0:
            raise ValueError("alpha_init must be > 0")
        self.d_m, self.k = int(d_m), int(k)
        self.cand_layers = sorted(cand_layers)
        self.n_cand = len(self.cand_layers)
        self.pos = {li: i for i, li in enumerate(self.cand_layers)}
        self.first_layer = self.cand_layers[0]
        self.straight_through = bool(straight_through)
        self.u = nn.Linear(self.d_m, self.n_cand, bias=True)
        self.log_alpha = nn.Parameter(torch.tensor(math.log(alpha_init)))
        self._w: torch.Tensor | None = None
        self._explicit = False

    # ------------------------------------------------------------------ weights
    def _weights_from_logits(self, z: torch.Tensor) -> torch.Tensor:
        return ops.selector_weights(z.float(), self.k, self.straight_through)

    def _logits(self, h: torch.Tensor, rms: bool) -> torch.Tensor:
        h2 = h.reshape(-1, h.shape[-1])
        z = ops.selector_logits(h2, self.u.weight.detach().float().to(h.device),
                                self.u.bias.detach().float().to(h.device), rms=rms)
        return z.view(*h.shape[:-1], self.n_cand)

    def compute(self, hn0: torch.Tensor) -> None:
        """hn0: [B, T, d_m] RMS-normed residual at the first candidate layer -> stores w [B, T, n_cand]."""
        self._check_no_grad()
        self._w = self._weights_from_logits(self._logits(hn0, rms=False))
        self._explicit = True

    def set_logits(self, z: torch.Tensor) -> None:
        """Store the weights of given logits z [..., n_cand] (used by the fused input projection)."""
        self._w = self._weights_from_logits(z)
        self._explicit = True

    def reset(self) -> None:
        self._w = None
        self._explicit = False

    def weights(self) -> torch.Tensor | None:
        return self._w

    @torch.no_grad()
    def entropy(self) -> torch.Tensor | None:
        if self._w is None:
            return None
        w = self._w.detach().float().clamp_min(0)
        return -(w * torch.log(w.clamp_min(1e-12))).sum(-1).mean()

    def alpha(self) -> torch.Tensor:
        return self.log_alpha.exp()

    # ------------------------------------------------------------------ apply
    def weights_for(self, h: torch.Tensor, li: int) -> torch.Tensor:
        """The per-token weight column of candidate layer li, computing the weights at the first layer
        (or when missing / stale) exactly as apply() does. Returns float32 [..] with h's leading shape."""
        p = self.pos[li]  # KeyError for a non-candidate layer is intended
        if li == self.first_layer:
            if not self._explicit or self._w is None:
                self._w = self._weights_from_logits(self._logits(h, rms=True))
            self._explicit = False
        elif self._w is None or self._w.shape[:-1] != h.shape[:-1]:
            self._w = self._weights_from_logits(self._logits(h, rms=True))
            self._explicit = False
        return self._w[..., p]

    def apply(self, delta: torch.Tensor, h: torch.Tensor, li: int) -> torch.Tensor:
        """Matched-norm rescale of `delta`, weighted by w[..., pos[li]]; returns delta's dtype."""
        self._check_no_grad()
        p = self.pos[li]
        self.weights_for(h, li)
        return ops.selector_apply(delta, h, self._w.reshape(-1, self.n_cand), p, float(self.log_alpha.detach()))

    def _check_no_grad(self) -> None:
        if torch.is_grad_enabled() and any(q.requires_grad for q in self.parameters()):
            raise RuntimeError("LayerSelector: the xencb kernels are forward-only; run under torch.no_grad() "
                               "or torch.inference_mode(), or freeze the selector")

    def extra_repr(self) -> str:
        return (f"d_m={self.d_m}, cand_layers={self.cand_layers}, k={self.k}, "
                f"straight_through={self.straight_through}")

    def config(self) -> dict:
        return {"d_m": self.d_m, "cand_layers": list(self.cand_layers), "k": self.k,
                "straight_through": self.straight_through}


__all__ = ["LayerSelector"]
