"""Seeded synthetic inputs for the five benchmark configurations of this path.

The reference measures on one real Qwen3.5-2B GGUF layer, which is not available
here; these generators stand in with the distributions the configurations
specify: Q4 codes uniform in [0, 15] in 32-groups along d_model, fp16-exact
alpha = |N(0, 0.02)| / 8 and beta = -(same law) ("fp16 mins"), activations
N(0, 1) (optionally with a seeded fraction of channels scaled x20 as outliers)
quantised per token and group, and fp16 N(0, 0.02) down weights [d_model, d_ff].
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .formats import quantize_groupwise_q8


@dataclass(frozen=True)
class FfnConfig:
    key: str
    workload: str
    d_model: int
    d_ff: int
    layers: int
    residual_bits: int
    tokens: tuple[int, ...]
    base_tile_rows: int = 256
    outlier_fraction: float = 0.0
    base_modes: tuple[str, ...] = ("host",)
    extra: dict = field(default_factory=dict)


CONFIGS = {
    "c1": FfnConfig("c1", "single SwiGLU FFN layer d_model=2048 d_ff=5632, decode T=1, r=2",
                    2048, 5632, 1, 2, (1,)),
    "c2": FfnConfig("c2", "Llama-7B-shape FFN stack: 32 layers d_model=4096 d_ff=11008, decode T=1/8/64, r=2, "
                    "base sums streamed from pinned host memory", 4096, 11008, 32, 2, (1, 8, 64)),
    "c3": FfnConfig("c3", "27B-class FFN stack: 46 layers d_model=4608 d_ff=36864, decode T=16, r=1, 1% outlier "
                    "channels x20", 4608, 36864, 46, 1, (16,), outlier_fraction=0.01, base_modes=("host", "hbm")),
    "c4": FfnConfig("c4", "70B-class FFN stack: 80 layers d_model=8192 d_ff=28672, prefill T=2048 + decode T=32, r=2",
                    8192, 28672, 80, 2, (2048, 32), base_modes=("hbm",)),
    "c5": FfnConfig("c5", "residual tile sweep: one layer d_model=4096 d_ff=14336, tile rows 64-1024, r=1/2/3, "
                    "T=1-128, 0-5% fallback tiles", 4096, 14336, 1, 2, (1, 8, 32, 128),
                    extra={"tile_rows": (64, 128, 256, 512, 1024), "residual_bits": (1, 2, 3),
                           "fallback_fraction": (0.0, 0.01, 0.05)}),
}


@dataclass
class LayerData:
    gate_codes: np.ndarray   # [F, D] uint8 0..15
    up_codes: np.ndarray
    gate_alpha: np.ndarray   # [F, G] f32 (fp16-exact)
    up_alpha: np.ndarray
    gate_beta: np.ndarray
    up_beta: np.ndarray
    down: np.ndarray         # [D, F] fp16


def _scales(rng: np.random.Generator, shape) -> np.ndarray:
    return (np.abs(rng.standard_normal(shape, dtype=np.float32)) * np.float32(0.02 / 8)).astype(
        np.float16).astype(np.float32)


def make_layer(seed: int, d_ff: int, d_model: int, rows: slice | None = None) -> LayerData:
    """One layer's weights. ``rows`` selects a d_ff shard: the full layer is drawn from
    the layer's seed and the shard's rows (and down columns) are kept, so shards
    agree with the unsharded layer."""
    rng = np.random.default_rng(seed)
    G = d_model // 32
    gate = rng.integers(0, 16, (d_ff, d_model), dtype=np.uint8)
    up = rng.integers(0, 16, (d_ff, d_model), dtype=np.uint8)
    ga, ua = _scales(rng, (d_ff, G)), _scales(rng, (d_ff, G))
    gb, ub = -_scales(rng, (d_ff, G)), -_scales(rng, (d_ff, G))
    down = (rng.standard_normal((d_model, d_ff), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    if rows is not None:
        gate, up, ga, ua, gb, ub = (a[rows] for a in (gate, up, ga, ua, gb, ub))
        down = np.ascontiguousarray(down[:, rows])
    return LayerData(np.ascontiguousarray(gate), np.ascontiguousarray(up), ga, ua, gb, ub, down)


def make_activations(seed: int, tokens: int, d_model: int, outlier_fraction: float = 0.0):
    """x ~ N(0,1) [T, D] (outlier channels x20) -> (x, z int8 [T, D], s f32 [T, G])."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((tokens, d_model), dtype=np.float32)
    if outlier_fraction > 0:
        ch = rng.choice(d_model, max(1, int(round(outlier_fraction * d_model))), replace=False)
        x[:, ch] *= np.float32(20.0)
    z, s = quantize_groupwise_q8(x)
    return x, z, s


def flagged_tiles(seed: int, n_tiles: int, fraction: float) -> np.ndarray:
    """Seeded fallback-tile mask with round(fraction * n_tiles) flagged tiles."""
    mask = np.zeros(n_tiles, dtype=np.uint8)
    k = int(round(fraction * n_tiles))
    if k:
        mask[np.random.default_rng(seed).choice(n_tiles, k, replace=False)] = 1
    return mask


def make_layer_device(seed: int, d_ff: int, d_model: int, rows: slice | None = None, device="cuda",
                      on_device: bool = False) -> LayerData:
    """Same distributions as :func:`make_layer`, drawn with torch's seeded CUDA
    generator (fast for full-size stacks); returns host numpy arrays, or the torch
    tensors on the device with ``on_device``. Every rank draws the full layer and keeps
    its shard, so shards of one seed agree."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    G = d_model // 32

    def scales():
        v = torch.randn(d_ff, G, generator=gen, device=device).abs_() * (0.02 / 8)
        return v.half().float()

    gate = torch.randint(0, 16, (d_ff, d_model), generator=gen, device=device, dtype=torch.uint8)
    up = torch.randint(0, 16, (d_ff, d_model), generator=gen, device=device, dtype=torch.uint8)
    ga, ua, gb, ub = scales(), scales(), -scales(), -scales()
    down = (torch.randn(d_model, d_ff, generator=gen, device=device) * 0.02).half()
    rows = rows or slice(0, d_ff)
    if on_device:
        cut = lambda t: t[rows].contiguous()
        return LayerData(cut(gate), cut(up), cut(ga), cut(ua), cut(gb), cut(ub), down[:, rows].contiguous())
    host = lambda t: t[rows].contiguous().cpu().numpy()
    return LayerData(host(gate), host(up), host(ga), host(ua), host(gb), host(ub),
                     down[:, rows].contiguous().cpu().numpy())
