"""d_ff sharding host logic on CPU: two gloo ranks each evaluate their row shard with
the oracle; the allreduce of the partial outputs equals the unsharded layer output."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch.multiprocessing as mp

from ffn_residual_mesh_b200.shard import reduce_partials, shard_rows


@pytest.mark.parametrize("F,world", [(11008, 2), (11008, 8), (28672, 8), (130, 2), (37, 1)])
def test_shard_rows_partition(F, world):
    parts = [shard_rows(F, world, k) for k in range(world)]
    assert parts[0].start == 0 and parts[-1].stop == F
    for a, b in zip(parts, parts[1:]):
        assert a.stop == b.start
    for p in parts[:-1]:
        assert (p.stop - p.start) % 8 == 0
    with pytest.raises(ValueError):
        shard_rows(F, world, world)


def _rank(rank, world, port, out):
    import torch
    import torch.distributed as dist

    from ffn_residual_mesh_b200 import synth
    from oracle import ffnrm_oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    D, F, T, r = 256, 96, 3, 2
    rows = shard_rows(F, world, rank)
    L = synth.make_layer(5, F, D, rows=rows)
    _, z, s = synth.make_activations(6, T, D)
    ref = O.ffn_forward(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.gate_beta, L.up_beta, L.down, z, s, r)
    y = torch.from_numpy(ref["y"].copy())
    dist.all_reduce(y)
    if rank == 0:
        out.put(y.numpy())
    dist.destroy_process_group()


def test_two_rank_allreduce_matches_unsharded():
    from ffn_residual_mesh_b200 import synth
    from oracle import ffnrm_oracle as O
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(k, 2, port, q)) for k in range(2)]
    for p in procs:
        p.start()
    y = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    D, F, T = 256, 96, 3
    L = synth.make_layer(5, F, D)
    _, z, s = synth.make_activations(6, T, D)
    full = O.ffn_forward(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.gate_beta, L.up_beta, L.down, z, s, 2)
    np.testing.assert_allclose(y, full["y"], rtol=1e-9, atol=1e-12)
    parts = [O.ffn_forward(*(getattr(synth.make_layer(5, F, D, rows=shard_rows(F, 2, k)), a) for a in
                             ("gate_codes", "up_codes", "gate_alpha", "up_alpha", "gate_beta", "up_beta", "down")),
                           z, s, 2)["y"] for k in range(2)]
    np.testing.assert_allclose(reduce_partials(parts), full["y"], rtol=1e-9, atol=1e-12)
