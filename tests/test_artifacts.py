"""The on-disk artifact contract (CPU): the package reads the directories the reference's
own exporters wrote (tests/golden/artifact_*, made by tests/golden/make_golden.py through
scripts/export_cuda_residual_artifact_v2.py and scripts/export_radix_table_artifact.py),
writes byte-identical ones, and rejects corrupted or mis-sized files; the drop-in runner
executables keep the reference runners' usage / error exit codes
(src/exact_residual_cuda_runner.cu:460-464,591-594) without touching a GPU."""
from __future__ import annotations

import json
import shutil
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import ffnrm_oracle as O

RES = GOLDEN / "artifact_residual_v2"
TAB = GOLDEN / "artifact_table_b2"


def source():
    return np.load(GOLDEN / "artifact_source.npz")


def test_reads_reference_residual_artifact():
    from ffn_residual_mesh_b200.artifacts import read_residual_artifact
    from ffn_residual_mesh_b200.formats import pack_qlo2_rows, quantize_groupwise_q8
    A = read_residual_artifact(RES)
    src = source()
    assert (A.rows, A.hidden, A.layer) == (96, 512, 23)
    for p in ("gate", "up"):
        np.testing.assert_array_equal(A.codes[p], pack_qlo2_rows(src[f"{p}_codes"] & 3))
        np.testing.assert_array_equal(A.alpha[p], src[f"{p}_alpha"])
    z, s = quantize_groupwise_q8(src["x"].reshape(1, -1))
    np.testing.assert_array_equal(A.z, z[0])
    np.testing.assert_array_equal(A.s, s[0])


def test_writer_matches_reference_exporter(tmp_path):
    from ffn_residual_mesh_b200.artifacts import write_residual_artifact
    src = source()
    ref = json.loads((RES / "manifest.json").read_text())
    q4 = {p: ref["projections"][p]["source_q4_bytes"] for p in ("gate", "up")}
    m = write_residual_artifact(tmp_path, {p: src[f"{p}_codes"] & 3 for p in ("gate", "up")},
                                {p: src[f"{p}_alpha"] for p in ("gate", "up")}, src["x"], layer=23,
                                source_q4_bytes=q4)
    for f in RES.glob("*.bin"):
        assert (tmp_path / f.name).read_bytes() == f.read_bytes(), f.name
    m["activation"].pop("source")
    ref["activation"].pop("source")
    assert m == ref


def test_table_artifact_round_trip(tmp_path):
    from ffn_residual_mesh_b200.artifacts import read_table_artifact, write_table_artifact
    T = read_table_artifact(TAB, block_size=2)
    src = source()
    ref = json.loads((TAB / "manifest.json").read_text())
    assert (T.rows, T.hidden, T.block_size) == (96, 512, 2)
    np.testing.assert_array_equal(T.states, O.encode_signed_base4_states(T.z, 2))
    tables, highs = {}, {}
    for p in ("gate", "up"):
        q_hi = (src[f"{p}_codes"] >> 2).reshape(96, 16, 32)
        tables[p], highs[p] = O.compile_radix_table(q_hi, block_size=2)
        np.testing.assert_array_equal(T.table[p], tables[p])
        np.testing.assert_array_equal(T.high_sum[p], highs[p])
    q4 = {p: ref["projections"][p]["q4_source_bytes"] for p in ("gate", "up")}
    m = write_table_artifact(tmp_path, tables, highs, T.alpha, T.beta, T.z, T.s, T.states, 2, source_q4_bytes=q4)
    for f in TAB.glob("*.bin"):
        assert (tmp_path / f.name).read_bytes() == f.read_bytes(), f.name
    assert m == ref
    with pytest.raises(ValueError):
        read_table_artifact(TAB, block_size=4)


def corrupt_copy(tmp_path, name, mutate):
    d = tmp_path / "art"
    shutil.copytree(RES, d)
    f = d / name
    data = bytearray(f.read_bytes())
    f.write_bytes(bytes(mutate(data)))
    return d


def flip(data):
    data[100] ^= 1
    return data


def test_checksum_and_size_mismatch_raise(tmp_path):
    from ffn_residual_mesh_b200.artifacts import read_residual_artifact
    with pytest.raises(ValueError, match="sha256"):
        read_residual_artifact(corrupt_copy(tmp_path, "gate.qlo2.rowpacked.bin", flip))
    shutil.rmtree(tmp_path / "art")
    with pytest.raises(ValueError, match="size"):
        read_residual_artifact(corrupt_copy(tmp_path, "up.alpha.f32.bin", lambda d: d[:-4]))


@pytest.fixture(scope="module")
def runners():
    from ffn_residual_mesh_b200 import build
    build.build()
    return {n: str(build.BIN_DIR / n) for n in build.RUNNERS}


def run(cmd):
    return subprocess.run(cmd, capture_output=True, text=True, timeout=60)


def test_runner_usage_exits_2(runners):
    for name, argv in (("exact_residual_cuda_runner", []), ("exact_main_residual_cuda_runner", ["a", "b"]),
                       ("exact_cpu_base_gpu_full_ffn_runner", ["a"] * 9)):
        r = run([runners[name], *argv])
        assert r.returncode == 2 and r.stderr.startswith("usage: " + name), (name, r.stderr)


def test_runner_errors_exit_1(runners, tmp_path):
    r = run([runners["exact_residual_cuda_runner"], str(tmp_path / "missing"), str(tmp_path / "o.json")])
    assert r.returncode == 1 and r.stderr.startswith("error: cannot open")
    bad = corrupt_copy(tmp_path, "gate.qlo2.rowpacked.bin", flip)
    r = run([runners["exact_residual_cuda_runner"], str(bad), str(tmp_path / "o.json"), "32", "1"])
    assert r.returncode == 1 and "sha256 mismatch" in r.stderr, r.stderr
    r = run([runners["exact_residual_cuda_runner"], str(RES), str(tmp_path / "o.json"), "50", "1"])
    assert r.returncode == 1 and "incompatible with tile" in r.stderr
    r = run([runners["exact_main_residual_cuda_runner"], str(TAB), str(RES), str(tmp_path / "o.json"), "4", "32", "1", "2"])
    assert r.returncode == 1 and "does not match the table artifact" in r.stderr, r.stderr
    r = run([runners["exact_cpu_base_gpu_full_ffn_runner"], str(TAB), str(RES), str(tmp_path / "down.bin"),
             str(tmp_path / "o.json"), "2", "32", "1", "2"])
    assert r.returncode == 1 and r.stderr.startswith("error: cannot open"), r.stderr
    assert not (tmp_path / "o.json").exists()
