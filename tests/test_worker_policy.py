"""Base-worker wire protocol (src/phone_ffn_loopback.py:29-197) and the layer policy
manifest (docs/layer_policy_manifest.example.json) on the CPU: frame round trip and
integrity checks, concurrent row-shard dispatch, the deadline rule (late or corrupted
tiles become exact-fallback tiles), assembly of returned base tiles into the base
buffer with the fallback mask, and per-layer routing."""
from __future__ import annotations

import struct
import time

import numpy as np
import pytest

from conftest import GOLDEN


def req(tile, row_start=0, row_count=4):
    from ffn_residual_mesh_b200.worker import REQUEST, Frame
    return Frame(REQUEST, 7, 2, 3, tile, row_start, row_count, b"descriptor")


def test_frame_round_trip_and_checksum():
    from ffn_residual_mesh_b200.worker import HEADER, Frame, ProtocolError
    f = req(4)
    wire = f.encode()
    assert wire[:4] == b"PFFN" and len(wire) == HEADER.size + len(b"descriptor") == 48
    assert Frame.decode(wire) == f
    bad = bytearray(wire)
    bad[-1] ^= 1
    with pytest.raises(ProtocolError):
        Frame.decode(bytes(bad))
    with pytest.raises(ProtocolError):
        Frame.decode(wire[:10])
    with pytest.raises(ProtocolError):
        Frame.decode(b"XFFN" + wire[4:])
    with pytest.raises(ProtocolError):
        Frame.decode(wire + b"x")  # length mismatch
    assert issubclass(ProtocolError, ValueError)


def test_wire_layout_is_network_order():
    from ffn_residual_mesh_b200.worker import RESPONSE, Frame
    import zlib
    f = Frame(RESPONSE, 1, 2, 3, 4, 5, 6, b"abc")
    magic, ver, kind, *ints = struct.unpack("!4sBB8I", f.encode()[:38])
    assert (magic, ver, kind) == (b"PFFN", 1, RESPONSE)
    assert ints == [1, 2, 3, 4, 5, 6, 3, zlib.crc32(b"abc")]


def test_workers_answer_ordered_and_concurrently():
    from ffn_residual_mesh_b200.worker import BaseCluster, BaseWorker
    workers = [BaseWorker(0, 0, 4, lambda f: b"base-a", delay_ms=20),
               BaseWorker(1, 4, 4, lambda f: b"base-b", delay_ms=20)]
    t0 = time.monotonic()
    res = BaseCluster(workers).dispatch([req(2, 4), req(1, 0)], deadline_ms=500)
    assert time.monotonic() - t0 < 0.2
    assert [r.tile_id for r in res.responses] == [1, 2]
    assert [r.payload for r in res.responses] == [b"base-a", b"base-b"]
    assert res.fallback_tiles == () and res.deadline_misses == 0 and res.protocol_errors == 0


def test_deadline_miss_and_errors_fall_back():
    from ffn_residual_mesh_b200.worker import BaseCluster, BaseWorker
    late = BaseWorker(0, 0, 4, lambda f: b"late", delay_ms=300)
    t0 = time.monotonic()
    res = BaseCluster([late]).dispatch([req(1)], deadline_ms=5)
    assert time.monotonic() - t0 < 0.2  # the step does not wait for the straggler
    assert res.responses == () and res.fallback_tiles == (1,) and res.deadline_misses == 1

    def boom(f):
        raise RuntimeError("worker crashed")
    res = BaseCluster([BaseWorker(0, 0, 8, boom)]).dispatch([req(0, 0), req(3, 4)], deadline_ms=500)
    assert res.fallback_tiles == (0, 3) and res.protocol_errors == 2
    # a tile no worker owns goes straight to the fallback
    res = BaseCluster([BaseWorker(0, 0, 4, lambda f: b"x")]).dispatch([req(5, 8)], deadline_ms=100)
    assert res.fallback_tiles == (5,) and res.protocol_errors == 0
    with pytest.raises(ValueError):
        BaseCluster([late]).dispatch([req(1)], deadline_ms=0)


def test_assemble_base_tiles_and_fallback_mask():
    from ffn_residual_mesh_b200.worker import (BaseCluster, BaseWorker, ProtocolError, assemble_base, base_payload,
                                               tile_requests)
    T, F, tile = 3, 20, 8
    rng = np.random.default_rng(0)
    base = rng.normal(size=(T, F)).astype(np.float32)
    compute = lambda f: base_payload(base[:, f.row_start:f.row_start + f.row_count])
    workers = [BaseWorker(0, 0, 16, compute), BaseWorker(1, 16, 4, compute, delay_ms=300)]
    reqs = tile_requests(F, tile)
    assert [(r.row_start, r.row_count) for r in reqs] == [(0, 8), (8, 8), (16, 4)]
    res = BaseCluster(workers).dispatch(reqs, deadline_ms=100)
    out = np.zeros((T, F), np.float32)
    mask = assemble_base(res, out, tile)
    assert mask.tolist() == [0, 0, 1]
    np.testing.assert_array_equal(out[:, :16], base[:, :16])
    assert not out[:, 16:].any()
    from ffn_residual_mesh_b200.worker import RESPONSE, DispatchResult, Frame
    bad = DispatchResult((Frame(RESPONSE, 0, 0, 0, 0, 0, 8, b"\0" * 8),), (), 0, 0)
    with pytest.raises(ProtocolError):
        assemble_base(bad, out, tile)


def test_layer_policy_routing():
    from ffn_residual_mesh_b200.policy import LayerPolicy
    p = LayerPolicy.load(GOLDEN / "layer_policy.json")
    assert [p.mode(l) for l in range(7)] == ["exact", "exact", "approximate", "exact", "exact", "approximate", "exact"]
    assert p.fallback_tiles(0, 4) is None
    assert p.fallback_tiles(2, 4).tolist() == [1, 1, 1, 1]
    assert p.needs_fallback_data(5) and not p.needs_fallback_data(6)
    assert p.meta["quantization"] == "Q4_K_M"
    approx_default = LayerPolicy.from_dict({"default_mode": "approximate", "exact_layers_until_calibrated": [1]})
    assert approx_default.mode(0) == "approximate" and approx_default.mode(1) == "exact"
    for bad in ({"policy_version": 2}, {"default_mode": "fast"},
                {"approximate_layers": {"1": {}}, "exact_layers_until_calibrated": [1]}):
        with pytest.raises(ValueError):
            LayerPolicy.from_dict(bad)
