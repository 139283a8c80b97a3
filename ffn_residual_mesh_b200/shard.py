"""d_ff sharding across GPUs: one process per GPU, row-parallel down projection,
one allreduce of the fp32 partial output per layer.

The reference has no multi-GPU code; this is the tensor-parallel split the path
admits: gate/up output rows (d_ff) are independent, so rank k holds the contiguous
rows ``shard_rows(F, N, k)`` of gate/up codes, alpha, its slice of the base sums,
and the matching columns of the down weight. Its down projection yields a partial
``y_k [T, D]``; ``sum_k y_k`` (NCCL allreduce over NVLink) is the layer output.
"""
from __future__ import annotations

import numpy as np

from .engine import ResidualMesh, cast_f16


def shard_rows(d_ff: int, world: int, rank: int, align: int = 8) -> slice:
    """Contiguous, ``align``-aligned row range of ``rank`` (the last rank takes the rest)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    per = (d_ff // world) // align * align
    if per == 0:
        raise ValueError(f"d_ff={d_ff} too small for {world} shards of {align}-row alignment")
    begin = rank * per
    end = d_ff if rank == world - 1 else begin + per
    return slice(begin, end)


class ShardedFfnStack:
    """A ``ResidualMesh`` over this rank's d_ff shard plus the per-layer allreduce."""

    def __init__(self, d_model, d_ff, residual_bits, n_layers, max_tokens, base_tile_rows=256,
                 rank=0, world=1, device=0, group=None):
        self.rank, self.world, self.group = rank, world, group
        self.rows = shard_rows(d_ff, world, rank)
        self.d_model, self.d_ff_total = d_model, d_ff
        self.mesh = ResidualMesh(d_model, self.rows.stop - self.rows.start, residual_bits, n_layers, max_tokens,
                                 base_tile_rows, device)
        self._y32 = None

    @property
    def d_ff(self) -> int:
        return self.mesh.d_ff

    def _partial(self, tokens, device):
        import torch
        if self._y32 is None or self._y32.shape[0] < tokens:
            self._y32 = torch.empty(self.mesh.max_tokens, self.d_model, device=device)
        return self._y32[:tokens]

    def forward(self, layer, z, s, gate_base, up_base, y16, fallback_tiles=None, stream=None):
        """Device buffers; gate_base/up_base are this rank's [T, F_shard] slices."""
        if self.world == 1:
            self.mesh.forward(layer, z, s, gate_base, up_base, fallback_tiles=fallback_tiles, y16=y16, stream=stream)
            return
        import torch.distributed as dist
        y32 = self._partial(z.shape[0], z.device)
        self.mesh.forward(layer, z, s, gate_base, up_base, fallback_tiles=fallback_tiles, y32=y32, stream=stream)
        dist.all_reduce(y32, group=self.group)
        cast_f16(y32, y16, stream=stream)

    def forward_host(self, layer, z, s, gate_base, up_base, y16, staging=None, fallback_tiles=None):
        """Host (pinned) buffers in and out. One GPU: the C-ABI host-streamed call.
        Several: H2D of the shard's inputs, forward, allreduce, D2H of y."""
        if self.world == 1:
            self.mesh.forward_host(layer, z, s, gate_base, up_base, y16, fallback_tiles=fallback_tiles)
            return
        import torch
        st = staging
        T = z.shape[0]
        zd, sd, gd, ud, yd = st["z"][:T], st["s"][:T], st["gb"][:T], st["ub"][:T], st["y16"][:T]
        zd.copy_(z, non_blocking=True)
        sd.copy_(s, non_blocking=True)
        gd.copy_(gate_base, non_blocking=True)
        ud.copy_(up_base, non_blocking=True)
        self.forward(layer, zd, sd, gd, ud, yd)
        y16.copy_(yd, non_blocking=True)

    def staging(self, device):
        """Device staging buffers for forward_host with world > 1."""
        import torch
        T, D, F, G = self.mesh.max_tokens, self.d_model, self.d_ff, self.d_model // 32
        return {"z": torch.empty(T, D, dtype=torch.int8, device=device),
                "s": torch.empty(T, G, device=device),
                "gb": torch.empty(T, F, device=device), "ub": torch.empty(T, F, device=device),
                "y16": torch.empty(T, D, dtype=torch.float16, device=device)}

    def close(self):
        self.mesh.close()


def reduce_partials(partials: list[np.ndarray]) -> np.ndarray:
    """Host-side sum of per-shard partial outputs (the allreduce's result)."""
    out = np.zeros_like(partials[0], dtype=np.float64)
    for p in partials:
        out += p
    return out
