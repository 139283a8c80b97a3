"""The product's host-side formats and generators against the oracle / fixtures (CPU)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN
from ffn_residual_mesh_b200 import formats, synth
from oracle import ffnrm_oracle as O


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_quantize_bit_exact_vs_oracle(seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((7, 512)).astype(np.float32)
    x[:, rng.choice(512, 5)] *= 20
    x[2, :32] = 0.0          # all-zero group -> 1e-12 clamp
    x[3, 40] = 1e30          # huge value
    z, s = formats.quantize_groupwise_q8(x)
    zo, so = O.quantize_groupwise_q8(x)
    np.testing.assert_array_equal(z, zo)
    np.testing.assert_array_equal(s, so)


def test_quantize_matches_reference_fixtures():
    for p in GOLDEN.glob("c*.npz"):
        c = np.load(p)
        z, s = formats.quantize_groupwise_q8(c["x"])
        np.testing.assert_array_equal(z, c["z"])
        np.testing.assert_array_equal(s, c["s"])


def test_quantize_rejects_ragged_groups():
    with pytest.raises(ValueError):
        formats.quantize_groupwise_q8(np.zeros((1, 33), np.float32))


def test_packing_vs_reference_bytes():
    k = np.load(GOLDEN / "kat.npz")
    np.testing.assert_array_equal(formats.pack_qlo2_rows(k["pack_codes"]), k["pack_bytes"])
    np.testing.assert_array_equal(formats.unpack_qlo2_rows(k["pack_bytes"], 8), k["pack_codes"])
    for p in GOLDEN.glob("c*.npz"):
        c = np.load(p)
        r = int(c["r"])
        hi, lo = formats.split_codes(c["codes"], r)
        assert formats.pack_bitplanes(lo, r) == c["lo_bitplanes"].tobytes()
        assert formats.pack_bitplanes(hi, 4 - r) == c["hi_bitplanes"].tobytes()
        np.testing.assert_array_equal(formats.unpack_bitplanes(c["hi_bitplanes"].tobytes(), hi.size, 4 - r), hi.ravel())
        if r == 2:
            np.testing.assert_array_equal(formats.pack_qlo2_rows(lo), c["qlo2_rowpacked"])
    with pytest.raises(ValueError):
        formats.pack_qlo2_rows(np.array([[4, 0, 0, 0]], np.uint8))
    with pytest.raises(ValueError):
        formats.unpack_bitplanes(b"\x00" * 3, 32, 1)


def test_synthetic_distributions():
    L = synth.make_layer(3, 64, 512)
    assert L.gate_codes.dtype == np.uint8 and L.gate_codes.max() <= 15
    assert np.array_equal(L.gate_alpha, L.gate_alpha.astype(np.float16).astype(np.float32))
    assert (L.gate_alpha >= 0).all() and (L.gate_beta <= 0).all()
    assert L.down.dtype == np.float16 and L.down.shape == (512, 64)
    # a shard equals the matching rows / columns of the full layer
    S = synth.make_layer(3, 64, 512, rows=slice(16, 48))
    np.testing.assert_array_equal(S.gate_codes, L.gate_codes[16:48])
    np.testing.assert_array_equal(S.down, L.down[:, 16:48])
    x, z, s = synth.make_activations(5, 4, 512, outlier_fraction=0.01)
    assert z.dtype == np.int8 and s.shape == (4, 16)
    assert (np.abs(x).max(axis=0) > 10).sum() >= 1
    m = synth.flagged_tiles(1, 40, 0.05)
    assert m.sum() == 2
