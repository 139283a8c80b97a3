"""Layer policy manifest: per-layer routing between the exact split path and the exact
GPU fallback.

Schema of the reference's manifest (docs/layer_policy_manifest.example.json):
``policy_version`` (1), ``model_family``, ``quantization``, ``residual_target``,
``default_mode`` ("exact" or "approximate"), ``approximate_layers`` {layer: parameters
of an approximate base}, ``exact_layers_until_calibrated`` [layers], ``notes``.

The approximate bases the reference researches (Chebyshev/low-rank, with holdout
proxies) are not part of the exact path this library implements, and the manifest's
own rule is that "fallback retains the exact FFN path". So a layer routes as:

* ``exact``       - host base + GPU residual (the split), no fallback tiles;
* ``approximate`` - no exact host base is produced for it: every tile of the layer is
  flagged for the GPU's exact unsplit path (the layer must be loaded with its fallback
  data, ``LayerSpec(..., keep_fallback=True)``).

``fallback_tiles(layer, n_tiles)`` gives the mask ``ffnrm_ffn_forward`` takes; deadline
misses of the base workers (``worker.assemble_base``) are OR-ed in by the caller.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

MODES = ("exact", "approximate")


@dataclass
class LayerPolicy:
    default_mode: str = "exact"
    approximate: dict = field(default_factory=dict)   # layer -> parameters
    exact: frozenset = frozenset()
    meta: dict = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: dict) -> "LayerPolicy":
        if int(d.get("policy_version", 1)) != 1:
            raise ValueError(f"unsupported policy_version {d.get('policy_version')}")
        mode = d.get("default_mode", "exact")
        if mode not in MODES:
            raise ValueError(f"default_mode must be one of {MODES}, not {mode!r}")
        approx = {}
        for k, v in d.get("approximate_layers", {}).items():
            layer = int(k)
            if layer < 0 or not isinstance(v, dict):
                raise ValueError(f"bad approximate layer entry {k!r}")
            approx[layer] = v
        exact = frozenset(int(x) for x in d.get("exact_layers_until_calibrated", []))
        both = exact & set(approx)
        if both:
            raise ValueError(f"layers listed as both exact and approximate: {sorted(both)}")
        meta = {k: d[k] for k in ("model_family", "quantization", "residual_target", "notes") if k in d}
        return cls(mode, approx, exact, meta)

    @classmethod
    def load(cls, path: Path) -> "LayerPolicy":
        return cls.from_dict(json.loads(Path(path).read_text(encoding="utf-8")))

    def mode(self, layer: int) -> str:
        if layer in self.exact:
            return "exact"
        if layer in self.approximate:
            return "approximate"
        return self.default_mode

    def needs_fallback_data(self, layer: int) -> bool:
        return self.mode(layer) == "approximate"

    def fallback_tiles(self, layer: int, n_tiles: int) -> np.ndarray | None:
        """None for a split layer; all tiles flagged for a layer routed to the exact
        GPU path."""
        if self.mode(layer) == "exact":
            return None
        return np.ones(n_tiles, dtype=np.uint8)
