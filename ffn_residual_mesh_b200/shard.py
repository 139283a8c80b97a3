"""d_ff sharding across GPUs: one process per GPU, row-parallel down projection,
one reduction of the fp32 partial output per layer.

The reference has no multi-GPU code; this is the tensor-parallel split the path
admits: gate/up output rows (d_ff) are independent, so rank k holds the contiguous
rows ``shard_rows(F, N, k)`` of gate/up codes, alpha, its slice of the base sums,
and the matching columns of the down weight. Its down projection yields a partial
``y_k [T, D]``; ``sum_k y_k`` is the layer output. The sum runs as one kernel per
layer over NVLink (``ffnrm_peer_allreduce``: push partials into peer memory, per-chunk
flags, sum in rank order, fp16 out); ``FFNRM_PEER_REDUCE=0`` selects an NCCL allreduce
plus a cast instead.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import _native as N
from .engine import ResidualMesh, _addr, _stream, cast_f16


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


class PeerReduce:
    """This rank's end of the NVLink layer-output reduction. Construction is collective:
    every rank of ``group`` creates its receive region and the ranks exchange CUDA IPC
    handles through the process group."""

    def __init__(self, world, rank, device, max_elems, group=None):
        import torch.distributed as dist
        self._h = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * N.IPC_HANDLE_BYTES)()
        N.check(N.lib().ffnrm_peer_create(ctypes.byref(self._h), device, world, rank, max_elems, handle))
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        table = (ctypes.c_uint8 * (N.IPC_HANDLE_BYTES * world)).from_buffer_copy(b"".join(handles))
        N.check(N.lib().ffnrm_peer_connect(self._h, table))

    def allreduce(self, partial, y16=None, y32=None, stream=None) -> None:
        """y = sum over ranks of ``partial`` (f32), written as fp16 ``y16`` and/or f32 ``y32``."""
        n = int(np.prod(partial.shape))
        N.check(N.lib().ffnrm_peer_allreduce(self._h, _addr(partial), n, _addr(y16) if y16 is not None else None,
                                             _addr(y32) if y32 is not None else None, _stream(stream)))

    def check(self, stream=None) -> None:
        N.check(N.lib().ffnrm_peer_check(self._h, _stream(stream)))

    def close(self) -> None:
        if self._h:
            N.lib().ffnrm_peer_destroy(self._h)
            self._h = ctypes.c_void_p()


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
        self.peer = None
        if world > 1 and os.environ.get("FFNRM_PEER_REDUCE", "1") != "0":
            self.peer = PeerReduce(world, rank, device, max_tokens * d_model, group=group)
        # FFNRM_PEER_FUSED=1: down projection and reduce-scatter in one kernel (ffnrm_ffn_forward_reduced)
        self.fused = os.environ.get("FFNRM_PEER_FUSED", "0") != "0"

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
        if self.peer is not None and self.fused:
            # down projection and reduce-scatter in one kernel, then the sum and all-gather
            T = self.mesh._check_act(z, s)
            self.mesh._check_tf("gate_base", gate_base, T)
            self.mesh._check_tf("up_base", up_base, T)
            N.check(N.lib().ffnrm_ffn_forward_reduced(self.mesh.handle, self.peer._h, layer, _addr(z), _addr(s), T,
                                                      _addr(gate_base), _addr(up_base), _addr(fallback_tiles),
                                                      _addr(y16), _stream(stream)))
            return
        import torch.distributed as dist
        y32 = self._partial(z.shape[0], z.device)
        self.mesh.forward(layer, z, s, gate_base, up_base, fallback_tiles=fallback_tiles, y32=y32, stream=stream)
        if self.peer is not None:
            self.peer.allreduce(y32, y16=y16, stream=stream)
            return
        dist.all_reduce(y32, group=self.group)
        cast_f16(y32, y16, stream=stream)

    def forward_host(self, layer, z, s, gate_base, up_base, y16, staging=None, fallback_tiles=None, y_to_host=True):
        """Host (pinned) buffers in and out. One GPU: the C-ABI host-streamed call. Several:
        the shard's host-streamed call into its device partial (base upload on the copy
        stream, overlapping the previous layer), the reduction, one D2H of y."""
        if self.world == 1:
            self.mesh.forward_host(layer, z, s, gate_base, up_base, y16, fallback_tiles=fallback_tiles)
            return
        T = z.shape[0]
        st = staging if staging is not None else self.staging(None)
        y32, yd = self._partial(T, st["y16"].device), st["y16"][:T]
        self.mesh.forward_host_partial(layer, z, s, gate_base, up_base, y32, fallback_tiles=fallback_tiles)
        if self.peer is not None:
            self.peer.allreduce(y32, y16=yd)
        else:
            import torch.distributed as dist
            dist.all_reduce(y32, group=self.group)
            cast_f16(y32, yd)
        if y_to_host:  # every rank holds the same y; a caller may read it back on one rank only
            y16.copy_(yd, non_blocking=True)

    def staging(self, device):
        """Device staging of y for forward_host with world > 1."""
        import torch
        device = torch.device("cuda", self.mesh.device) if device is None else device
        return {"y16": torch.empty(self.mesh.max_tokens, self.d_model, dtype=torch.float16, device=device)}

    def close(self):
        if self.peer is not None:
            # every rank has finished its reductions before any region is unmapped
            import torch
            import torch.distributed as dist
            torch.cuda.synchronize()
            self.peer.check()
            dist.barrier(group=self.group)
            self.peer.close()
            self.peer = None
        self.mesh.close()


def reduce_partials(partials: list[np.ndarray]) -> np.ndarray:
    """Host-side sum of per-shard partial outputs (the allreduce's result)."""
    out = np.zeros_like(partials[0], dtype=np.float64)
    for p in partials:
        out += p
    return out
