"""Host base producer of libffnrm.so (CPU, no GPU): exact table dots and base sums from
the reference's radix table artifact, checked against the reference-generated values
(tests/golden/c1_decode_t1_r2.npz: radix_p_hi and radix_base from the reference's
evaluate_radix_table / projection_from_group_dots, block 4; the exporter-written
artifact_table_b2, block 2) and the oracle for batches and block size 8; per-tile
readiness flags and the deadline rule of src/phone_ffn_loopback.py:155-197 (a producer
that misses its deadline hands its tiles to the GPU's exact fallback path)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import ffnrm_oracle as O


def producer(threads=4):
    from ffn_residual_mesh_b200 import build
    from ffn_residual_mesh_b200.artifacts import BaseProducer
    build.build(runners=False)
    return BaseProducer(threads)


def base_ref(p_hi, z, s, alpha, beta, mult=4):
    """s * (alpha * mult * P_hi + beta * zsum) summed over groups in float64."""
    zs = z.reshape(-1, 32).astype(np.float64).sum(1)
    return (s[None, :] * (alpha * mult * p_hi + beta * zs[None, :])).sum(1)


def test_dots_and_base_match_reference_block4():
    from ffn_residual_mesh_b200.artifacts import radix_table, table_dots
    c = np.load(GOLDEN / "c1_decode_t1_r2.npz")
    F, D = int(c["F"]), int(c["D"])
    q_hi = (c["codes"] >> 2).reshape(F, D // 32, 32)
    table, high = O.compile_radix_table(q_hi, block_size=4)
    t, keep = radix_table(table, high, c["alpha"], c["beta"], 4)
    np.testing.assert_array_equal(table_dots(t, c["z"][0]), c["radix_p_hi"])
    p = producer()
    base, late = p.from_table(t, c["z"], c["s"], multiplier=4, tile_rows=32)
    assert late is None
    want = np.asarray(c["radix_base"], np.float64).reshape(-1)
    scale = np.abs(want).max()
    assert np.abs(base[0] - want).max() <= 2e-5 * scale
    p.close()


def test_exporter_artifact_block2_and_batches():
    from ffn_residual_mesh_b200.artifacts import radix_table, read_table_artifact, table_dots
    A = read_table_artifact(GOLDEN / "artifact_table_b2", 2)
    src = np.load(GOLDEN / "artifact_source.npz")
    rng = np.random.default_rng(5)
    z = rng.integers(-128, 128, (5, A.hidden), dtype=np.int8)
    z[0] = A.z
    s = rng.uniform(0.001, 0.05, (5, A.hidden // 32)).astype(np.float32)
    p = producer(3)
    for proj in ("gate", "up"):
        t, keep = radix_table(A.table[proj], A.high_sum[proj], A.alpha[proj], A.beta[proj], 2)
        q_hi = (src[f"{proj}_codes"] >> 2).reshape(A.rows, A.hidden // 32, 32)
        base, _ = p.from_table(t, z, s, tile_rows=40)
        for k in range(5):
            p_hi = O.group_dots(q_hi, z[k:k + 1])[0]
            np.testing.assert_array_equal(table_dots(t, z[k]), p_hi)
            want = base_ref(p_hi, z[k], s[k], A.alpha[proj].astype(np.float64), A.beta[proj].astype(np.float64))
            assert np.abs(base[k] - want).max() <= 2e-5 * np.abs(want).max()
    p.close()


def test_block8_and_thread_count_invariance():
    from ffn_residual_mesh_b200.artifacts import radix_table, table_dots
    rng = np.random.default_rng(9)
    F, D = 40, 64
    q_hi = rng.integers(0, 4, (F, D // 32, 32), dtype=np.uint8)
    alpha = rng.uniform(0, 0.01, (F, D // 32)).astype(np.float32)
    beta = -rng.uniform(0, 0.01, (F, D // 32)).astype(np.float32)
    table, high = O.compile_radix_table(q_hi, block_size=8)
    t, keep = radix_table(table, high, alpha, beta, 8)
    z = rng.integers(-128, 128, (3, D), dtype=np.int8)
    s = rng.uniform(0.001, 0.05, (3, D // 32)).astype(np.float32)
    for k in range(3):
        np.testing.assert_array_equal(table_dots(t, z[k]), O.evaluate_radix_table(
            table, high, O.encode_signed_base4_states(z[k], 8), blocks_per_group=4))
    one, _ = producer(1).from_table(t, z, s, tile_rows=8)
    many, _ = producer(6).from_table(t, z, s, tile_rows=8)
    np.testing.assert_array_equal(one, many)  # each row is summed by one thread in group order


def test_tile_ready_flags_and_deadline():
    from ffn_residual_mesh_b200.artifacts import radix_table, read_table_artifact
    A = read_table_artifact(GOLDEN / "artifact_table_b2", 2)
    t, keep = radix_table(A.table["gate"], A.high_sum["gate"], A.alpha["gate"], A.beta["gate"], 2)
    p = producer(2)
    ntile = -(-A.rows // 32)
    ready = np.zeros((2, ntile), dtype=np.uint32)
    z = np.stack([A.z, A.z])
    s = np.stack([A.s, A.s])
    base, late = p.from_table(t, z, s, tile_rows=32, tile_ready=ready, deadline_s=3600.0)
    assert (ready == 1).all()
    assert late is not None and not late.any()
    np.testing.assert_array_equal(base[0], base[1])
    # a producer that cannot meet its deadline: every tile is flagged for the GPU fallback
    base2, late2 = p.from_table(t, z, s, tile_rows=32, deadline_s=1e-9)
    assert late2.shape == (ntile,) and late2.all()
    np.testing.assert_array_equal(base2, base)


def test_argument_errors():
    from ffn_residual_mesh_b200.artifacts import RadixTable, radix_table
    with pytest.raises(ValueError):
        producer(0)
    p = producer(1)
    bad = RadixTable(10, 48, 4, 0, 0, 0, 0)
    with pytest.raises(ValueError):
        p.from_table(bad, np.zeros((1, 48), np.int8), np.zeros((1, 1), np.float32))
    with pytest.raises(ValueError):
        radix_table(np.zeros((2, 16, 4), np.uint8), np.zeros((4, 2), np.int16), np.zeros((4, 2)), np.zeros((4, 2)), 4)
