"""Pin the CPU oracle before trusting it (no GPU needed).

1. The reference unit tests' known-answer vectors
   (tests/test_exact_radix_main_table.py:21-89, tests/test_export_cuda_residual_artifact.py:14-34).
2. The golden fixtures produced by the reference's own Python functions
   (tests/golden/make_golden.py).
3. The reference's AVX2 CPU evaluator compiled from its source into oracle/_ref
   (direct_q4 / fused_base verified integer dots), when that build is present.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import ffnrm_oracle as O
from oracle import refcpu

CASES = sorted(p.stem for p in GOLDEN.glob("c*.npz"))


def test_kat_two_bit_packing():
    k = np.load(GOLDEN / "kat.npz")
    assert O.pack_2bit_rows(k["pack_codes"]).tolist() == [[228, 27]]
    np.testing.assert_array_equal(O.pack_2bit_rows(k["pack_codes"]), k["pack_bytes"])
    np.testing.assert_array_equal(k["pack_bytes_v2"], k["pack_bytes"])
    np.testing.assert_array_equal(O.unpack_2bit_rows(k["pack_bytes"], 8), k["pack_codes"])


def test_kat_groupwise_q8():
    k = np.load(GOLDEN / "kat.npz")
    z, s = O.quantize_groupwise_q8(k["quant_x"], group_size=4)
    np.testing.assert_allclose(s, [[1 / 127, 2 / 127]], rtol=1e-6)
    np.testing.assert_array_equal(z[0, :4], [-127, -64, 0, 127])
    np.testing.assert_array_equal(z[0, 4:], [-127, 0, 64, 127])
    np.testing.assert_array_equal(z, k["quant_z"])
    np.testing.assert_array_equal(s, k["quant_s"])


def test_kat_radix_table_signed_extremes():
    k = np.load(GOLDEN / "kat.npz")
    table, hs = O.compile_radix_table(k["radix_q_hi"], 4)
    for tok, expect in zip(k["radix_z"], k["radix_dots"]):
        got = O.evaluate_radix_table(table, hs, O.encode_signed_base4_states(tok.reshape(-1), 4), 2)
        np.testing.assert_array_equal(got, expect)
        np.testing.assert_array_equal(got, np.einsum("rgi,gi->rg", k["radix_q_hi"].astype(np.int32), tok.astype(np.int32)))


def test_radix_block_two_exact():
    rng = np.random.default_rng(8)
    q_hi = rng.integers(0, 4, size=(3, 2, 8), dtype=np.uint8)
    z = rng.integers(-128, 128, size=(16,), dtype=np.int16).astype(np.int8)
    table, hs = O.compile_radix_table(q_hi, block_size=2)
    got = O.evaluate_radix_table(table, hs, O.encode_signed_base4_states(z, 2), blocks_per_group=4)
    np.testing.assert_array_equal(got, np.einsum("rgi,gi->rg", q_hi.astype(np.int32), z.reshape(2, 8).astype(np.int32)))


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_fixtures(name):
    c = dict(np.load(GOLDEN / f"{name}.npz"))
    r = int(c["r"])
    z, s = O.quantize_groupwise_q8(c["x"])
    np.testing.assert_array_equal(z, c["z"])
    np.testing.assert_array_equal(s, c["s"])
    q_hi, q_lo = O.split_codes(c["codes"], r)
    np.testing.assert_array_equal(O.group_dots(q_lo, z), c["p_lo"])
    np.testing.assert_array_equal(O.group_dots(q_hi, z), c["p_hi"])
    np.testing.assert_array_equal(O.group_dots(c["codes"], z), c["p_full"])
    host = O.host_base(c["codes"], c["alpha"], c["beta"], z, s, r)
    res = O.residual(c["codes"], c["alpha"], z, s, r)
    np.testing.assert_allclose(host, c["host"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(res, c["res"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(O.full_projection(c["codes"], c["alpha"], c["beta"], z, s), c["full"], rtol=1e-4, atol=1e-5)
    out = O.ffn_forward(c["codes"], c["codes_up"], c["alpha"], c["alpha_up"], c["beta"], c["beta_up"], c["down"],
                        z, s, r, fallback_tiles=np.isin(np.arange(-(-int(c["F"]) // int(c["tile_rows"]))), c["flagged"]),
                        tile_rows=int(c["tile_rows"]))
    np.testing.assert_allclose(out["g"], c["g"], rtol=1e-4, atol=1e-5)
    assert np.linalg.norm(out["y"] - c["y"]) / np.linalg.norm(c["y"]) < 1e-5
    if r == 2:
        np.testing.assert_array_equal(O.pack_2bit_rows(q_lo), c["qlo2_rowpacked"])
        if "radix_p_hi" in c:
            np.testing.assert_array_equal(c["radix_p_hi"], c["p_hi"][0])
            np.testing.assert_allclose(c["radix_base"], host[0], rtol=1e-4, atol=1e-5)
    assert O.pack_bitplanes(q_lo, r) == c["lo_bitplanes"].tobytes()
    assert O.pack_bitplanes(q_hi, 4 - r) == c["hi_bitplanes"].tobytes()
    np.testing.assert_array_equal(O.unpack_bitplanes(c["lo_bitplanes"].tobytes(), q_lo.size, r), q_lo.ravel())


@pytest.mark.skipif(not refcpu.available(), reason="oracle/_ref not built (make -C oracle)")
@pytest.mark.parametrize("name", ["c2_decode_t8_r2", "c3_decode_t16_r1_outliers"])
def test_oracle_matches_reference_avx2_build(name):
    c = dict(np.load(GOLDEN / f"{name}.npz"))
    m = refcpu.RefFfn(c["codes"], c["codes_up"], c["alpha"], c["alpha_up"], c["beta"], c["beta_up"], c["down"],
                      threads=4)
    g, u, dots = m.gate_up(c["z"], c["s"], with_dots=True)
    np.testing.assert_array_equal(dots[0], c["p_full"])
    np.testing.assert_array_equal(dots[1], O.group_dots(c["codes_up"], c["z"]))
    full = O.full_projection(c["codes"], c["alpha"], c["beta"], c["z"], c["s"])
    np.testing.assert_allclose(g, full, rtol=1e-4, atol=1e-5)
    y = m.forward(c["z"], c["s"])
    ref = O.ffn_forward(c["codes"], c["codes_up"], c["alpha"], c["alpha_up"], c["beta"], c["beta_up"], c["down"],
                        c["z"], c["s"], int(c["r"]))
    assert np.linalg.norm(y - ref["y"]) / np.linalg.norm(ref["y"]) < 1e-5
    m.close()


@pytest.mark.skipif(not refcpu.available(), reason="oracle/_ref not built (make -C oracle)")
def test_oracle_matches_reference_fused_base_radix_table():
    c = dict(np.load(GOLDEN / "c1_decode_t1_r2.npz"))
    q_hi = (c["codes"] >> 2).reshape(int(c["F"]), -1, 32)
    table, hs = O.compile_radix_table(q_hi, 4)
    base, p_hi = refcpu.fused_base(table, hs, c["alpha"], c["beta"], c["z"][0], c["s"][0], 4, threads=3)
    np.testing.assert_array_equal(p_hi, c["p_hi"][0])
    np.testing.assert_allclose(base, O.host_base(c["codes"], c["alpha"], c["beta"], c["z"], c["s"], 2)[0],
                               rtol=1e-4, atol=1e-5)
