"""Depth bookkeeping shared by Library and the injectors.

* injection_layers(model, depths): reader layer of depth rho = min(L - 1, int(rho * L))
  (the deltaskill.derive.injection_layers contract stated at docs/XENC_SPEC.md:50 of the reference).
* rho_layer_map: {rho: layer}, raising DepthCollisionError when two depths land on one layer
  (xenc/depth_skill.py:63-74).
* key_for: float-tolerant lookup of a rho key (xenc/depth_skill.py:77-84).
* KVSkill: the (K, V, d_s, text, model_name, meta) record the injectors load; for_reader remaps a
  rho-keyed skill onto reader layers (xenc/depth_skill.py:273-282).
"""

from __future__ import annotations

from typing import Iterable

DEPTHS = [0.25, 0.5, 0.75, 1.0]
CAND = [0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9]


class DepthCollisionError(ValueError, AssertionError):
    """Two depths map to the same physical layer."""


def num_layers(model_or_L) -> int:
    if isinstance(model_or_L, int):
        return model_or_L
    cfg = model_or_L.config
    cfg = cfg.get_text_config() if hasattr(cfg, "get_text_config") else cfg
    return int(cfg.num_hidden_layers)


def injection_layers(model_or_L, depths: Iterable[float]) -> list:
    L = num_layers(model_or_L)
    return [min(L - 1, int(float(r) * L)) for r in depths]


def rho_layer_map(model_or_L, depths: Iterable[float] = DEPTHS) -> dict:
    depths = sorted(float(r) for r in depths)
    out = {r: injection_layers(model_or_L, [r])[0] for r in depths}
    if len(set(out.values())) != len(depths):
        raise DepthCollisionError(f"depth collision on L={num_layers(model_or_L)}: {depths} -> {list(out.values())}")
    return out


def key_for(d: dict, rho: float):
    if rho in d:
        return rho
    for k in d:
        if abs(float(k) - float(rho)) < 1e-6:
            return k
    raise KeyError(f"no operator for depth rho={rho}; have {sorted(d)}")


class KVSkill:
    """One document operator: K / V dicts keyed by reader layer (or by depth when meta['keyed_by'] == 'rho')."""

    def __init__(self, K: dict, V: dict, d_s: int, text: str = "", model_name: str = "", meta: dict | None = None):
        self.K, self.V, self.d_s = K, V, int(d_s)
        self.text, self.model_name = text, model_name
        self.meta = dict(meta or {})


def for_reader(skill_rho: KVSkill, reader_model, depths=None) -> KVSkill:
    """rho-keyed -> reader-layer-keyed view (same tensors, no copy)."""
    depths = sorted(float(r) for r in (depths or skill_rho.meta["depths"]))
    rmap = rho_layer_map(reader_model, depths)
    K = {li: skill_rho.K[key_for(skill_rho.K, r)] for r, li in rmap.items()}
    V = {li: skill_rho.V[key_for(skill_rho.V, r)] for r, li in rmap.items()}
    meta = {**skill_rho.meta, "keyed_by": "layer", "rho_of": {li: r for r, li in rmap.items()}}
    return KVSkill(K=K, V=V, d_s=skill_rho.d_s, text=skill_rho.text, model_name=skill_rho.model_name, meta=meta)


def decoder_layers(model):
    """The decoder block list of an HF-style model (model.model.layers) or a bare stack (model.layers)."""
    for path in (("model", "layers"), ("model", "language_model", "layers"), ("layers",)):
        obj = model
        try:
            for name in path:
                obj = getattr(obj, name)
            return obj
        except AttributeError:
            continue
    raise AttributeError("cannot find the decoder layers (expected model.model.layers or model.layers)")
