"""GGUF Q4_K ingest against the reference's own outputs and the gguf package.

* ``tests/golden/q4k_layer.gguf`` holds a synthetic layer written with the ``gguf``
  package; ``artifact_q4k_r2/`` is what the reference's
  scripts/compile_q4k_host_base_gpu_residual.py made of it (load_q4k_codes of
  scripts/scan_q4k_hierarchical_code_split.py:23-48 underneath) and ``q4k_down.json``
  the sha256 of scripts/export_down_fp16.py's fp16 down. Both are reproduced byte for
  byte by ``ffn_residual_mesh_b200.q4k``.
* Every block type the reader decodes is checked bit for bit against
  ``gguf.quants.dequantize`` on seeded blocks (skipped where ``gguf`` is absent).
* A GPU case loads the GGUF layer through the C ABI (f32 alphas: Q4_K's d·sc is not
  fp16-exact) and checks the forward against the oracle.
"""
from __future__ import annotations

import hashlib
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from ffn_residual_mesh_b200 import q4k

GOLD = Path(__file__).resolve().parent / "golden"
MODEL = GOLD / "q4k_layer.gguf"


def test_reader_metadata_and_tensors():
    g = q4k.GgufFile(MODEL)
    assert g.version == 3
    assert g.metadata["ffnrm.test.u32"] == 7
    assert g.metadata["ffnrm.test.array"] == [1, 2, 3]
    assert g.metadata["ffnrm.test.string"] == "synthetic"
    assert g.metadata["ffnrm.test.f32"] == 0.5
    t = g.info("blk.0.ffn_gate.weight")
    assert (t.type, t.rows, t.row_values, t.n_bytes) == (q4k.Q4_K, 256, 256, 256 * 144)
    assert g.info("blk.0.ffn_down.weight").type == q4k.Q6_K


def test_compiled_artifact_is_byte_identical_to_reference(tmp_path):
    ref = json.loads((GOLD / "artifact_q4k_r2" / "manifest.json").read_text())
    m = q4k.compile_artifact(MODEL, 0, 2, tmp_path)
    for p in ("gate", "up"):
        a, b = ref["projections"][p], m["projections"][p]
        for key in ("host_high_bitplanes", "gpu_residual_bitplanes"):
            assert a[key] == b[key], (p, key)
        for key in ("alpha", "beta"):
            assert a[key] == b[key]
            assert (tmp_path / b[key]["file"]).read_bytes() == (GOLD / "artifact_q4k_r2" / a[key]["file"]).read_bytes()
        for key in ("shape", "q4k_source_bytes", "host_artifact_bytes", "gpu_residual_package_bytes"):
            assert a[key] == b[key]
    assert ref["pair_totals"] == m["pair_totals"]
    for key in ("magic", "version", "layer", "residual_bits", "host_high_bits", "access_contract"):
        assert ref[key] == m[key]


def test_layer_codes_match_reference_artifact():
    layer = q4k.load_layer(MODEL, 0)
    got = q4k.read_artifact(GOLD / "artifact_q4k_r2")
    for p, (codes, alpha, beta) in (("gate", (layer.gate_codes, layer.gate_alpha, layer.gate_beta)),
                                    ("up", (layer.up_codes, layer.up_alpha, layer.up_beta))):
        rc, ra, rb = got[p]
        np.testing.assert_array_equal(codes, rc)
        np.testing.assert_array_equal(alpha, ra)
        np.testing.assert_array_equal(beta, rb)
        assert codes.max() <= 15


def test_down_matches_reference_export():
    ref = json.loads((GOLD / "q4k_down.json").read_text())
    down = q4k.load_down_fp16(q4k.GgufFile(MODEL), 0)
    assert list(down.shape) == ref["shape"] and down.dtype == np.float16
    assert hashlib.sha256(np.ascontiguousarray(down).tobytes()).hexdigest() == ref["sha256"]


def test_artifact_reader_rejects_corruption(tmp_path):
    q4k.compile_artifact(MODEL, 0, 1, tmp_path)
    q4k.read_artifact(tmp_path)
    f = tmp_path / "up.gpu_residual.bitplanes"
    b = bytearray(f.read_bytes())
    b[5] ^= 1
    f.write_bytes(bytes(b))
    with pytest.raises(ValueError, match="sha256"):
        q4k.read_artifact(tmp_path)


def test_reader_rejects_bad_files(tmp_path):
    raw = MODEL.read_bytes()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + raw[4:])
    with pytest.raises(q4k.GgufError, match="not a GGUF"):
        q4k.GgufFile(bad)
    bad.write_bytes(raw[:4] + struct.pack("<I", 9) + raw[8:])
    with pytest.raises(q4k.GgufError, match="version"):
        q4k.GgufFile(bad)
    bad.write_bytes(raw[:200])
    with pytest.raises(q4k.GgufError, match="truncated"):
        q4k.GgufFile(bad)
    bad.write_bytes(raw[:-1000])
    with pytest.raises(q4k.GgufError, match="past the end"):
        q4k.GgufFile(bad)
    g = q4k.GgufFile(MODEL)
    with pytest.raises(q4k.GgufError, match="no tensor"):
        g.info("blk.7.ffn_gate.weight")
    with pytest.raises(q4k.GgufError, match="expected Q4_K"):
        q4k.load_q4k_projection(g, 0, "down")


def _write_blocks(path, tensors):
    gguf = pytest.importorskip("gguf")
    w = gguf.GGUFWriter(str(path), "llama")
    for name, data, qtype in tensors:
        if qtype is None:
            w.add_tensor(name, data)
        else:
            w.add_tensor(name, data, raw_dtype=getattr(gguf.GGMLQuantizationType, qtype))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def _blocks(rng, rows, nblk, nbytes, f16_at):
    b = rng.integers(0, 256, size=(rows, nblk, nbytes), dtype=np.uint8)
    for off in f16_at:
        v = (rng.standard_normal((rows, nblk)) * 0.01).astype(np.float16)
        b[:, :, off:off + 2] = v.view(np.uint8).reshape(rows, nblk, 2)
    return b.reshape(rows, -1)


def test_dequantize_matches_gguf_package(tmp_path):
    gguf = pytest.importorskip("gguf")
    from gguf.quants import dequantize
    rng = np.random.default_rng(5)
    path = tmp_path / "types.gguf"
    _write_blocks(path, [
        ("q4k", _blocks(rng, 48, 3, 144, [0, 2]), "Q4_K"),
        ("q6k", _blocks(rng, 40, 2, 210, [208]), "Q6_K"),
        ("q80", _blocks(rng, 24, 8, 34, [0]), "Q8_0"),
        ("f16", rng.standard_normal((8, 64)).astype(np.float16), None),
        ("f32", rng.standard_normal((8, 64)).astype(np.float32), None),
    ])
    reader = gguf.GGUFReader(str(path))
    mine = q4k.GgufFile(path)
    for t in reader.tensors:
        ref = dequantize(t.data, t.tensor_type).astype(np.float32)
        got = mine.dequantize(t.name)
        np.testing.assert_array_equal(ref.reshape(got.shape), got, err_msg=t.name)


@pytest.mark.gpu
def test_gguf_layer_forward_matches_oracle():
    import torch

    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import ResidualMesh
    from oracle import ffnrm_oracle as O
    layer = q4k.load_layer(MODEL, 0)
    F, D = layer.gate_codes.shape
    dev = torch.device("cuda:0")
    for r, T in ((2, 8), (1, 40), (3, 3)):
        ctx = ResidualMesh(D, F, r, 1, T, base_tile_rows=64, device=0)
        try:
            ctx.load_layer(0, layer.spec())
            _, z, s = synth.make_activations(31 + T, T, D)
            gb = O.host_base(layer.gate_codes, layer.gate_alpha, layer.gate_beta, z, s, r)
            ub = O.host_base(layer.up_codes, layer.up_alpha, layer.up_beta, z, s, r)
            y16 = torch.empty(T, D, dtype=torch.float16, device=dev)
            t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
            ctx.forward(0, t(z), t(s), t(gb.astype(np.float32)), t(ub.astype(np.float32)), y16=y16)
            torch.cuda.synchronize()
            ref = O.ffn_forward(layer.gate_codes, layer.up_codes, layer.gate_alpha, layer.up_alpha, layer.gate_beta,
                                layer.up_beta, layer.down, z, s, r, gate_base=gb, up_base=ub)["y"]
            y = y16.float().cpu().numpy().astype(np.float64)
            assert np.abs(y - ref).max() < 1e-2, (r, T)
            assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-3, (r, T)
        finally:
            ctx.close()
