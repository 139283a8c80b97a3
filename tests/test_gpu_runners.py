"""The drop-in runner executables on artifacts written by the reference's own exporters.

``tests/golden/artifact_residual_v2`` (scripts/export_cuda_residual_artifact_v2.py) and
``tests/golden/artifact_table_b2`` (scripts/export_radix_table_artifact.py, block 2) come from
the reference code (tests/golden/make_golden.py); the down projection is the same synthetic
layer's, written in the raw fp16 layout of scripts/export_down_fp16.py. Each runner is called
with the reference's argv, must exit 0 and print ``wrote <path>``, and its JSON must carry
every key the reference runner writes (the key lists below restate those output blocks) with
the validation figures inside the path's tolerance.
"""
from __future__ import annotations

import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
RES, TAB = GOLD / "artifact_residual_v2", GOLD / "artifact_table_b2"

# src/exact_residual_cuda_runner.cu:533-583
RESIDUAL_TOP = {"experiment", "layer", "gpu", "shape", "projections", "pair"}
RESIDUAL_PROJ = {"tile_payload_bytes", "full_payload_bytes", "validation_max_abs", "validation_rel_l2",
                 "copy_only_gpu_ms", "copy_only_host_ms", "kernel_only_gpu_ms", "serial_copy_compute_gpu_ms",
                 "serial_copy_compute_host_ms", "double_buffer_overlap_gpu_ms", "double_buffer_overlap_host_ms",
                 "overlap_speedup_vs_serial", "hidden_copy_ms", "visible_copy_wait_ms"}
# src/exact_main_residual_cuda_runner.cu:418-438
MAIN_PROJ = {"cpu_main_ms", "gpu_serial_copy_compute_ms", "gpu_overlap_ms", "residual_validation_max_abs",
             "residual_validation_rel_l2", "serial_cpu_plus_gpu_ms", "cpu_gpu_concurrent_wall_ms",
             "serial_to_concurrent_speedup"}
# src/exact_cpu_base_gpu_full_ffn_runner.cu:418-438
FULL_TOP = {"experiment", "gpu", "shape", "cpu_base_gate_up_ms", "gpu_serial_copy_compute_ms", "serial_cpu_plus_gpu_ms",
            "gpu_double_buffer_overlap_ms", "gpu_overlap_speedup_vs_gpu_serial", "cpu_gpu_critical_lower_bound_ms",
            "serial_to_cpu_gpu_lower_bound_speedup", "h2d", "correctness"}


@pytest.fixture(scope="module")
def bins():
    from ffn_residual_mesh_b200 import build
    build.build()
    return {n: str(build.BIN_DIR / n) for n in build.RUNNERS}


def _run(cmd, out: Path) -> dict:
    r = subprocess.run([str(c) for c in cmd], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip().endswith(f"wrote {out}"), r.stdout
    return json.loads(out.read_text())


def test_exact_residual_runner(bins, tmp_path):
    out = tmp_path / "residual.json"
    j = _run([bins["exact_residual_cuda_runner"], RES, out, 32, 2], out)
    assert RESIDUAL_TOP <= set(j)
    assert j["experiment"] == "cuda_exact_qlo2_residual_runner_v1"
    assert j["shape"] == {"rows": 96, "hidden": 512, "groups": 16, "tile_rows": 32, "tile_count": 3}
    for p in ("gate", "up"):
        row = j["projections"][p]
        assert RESIDUAL_PROJ <= set(row), RESIDUAL_PROJ - set(row)
        assert row["validation_rel_l2"] < 1e-5 and row["validation_max_abs"] < 1e-4, row
        # one 32-row tile of the row-packed payload: 2-bit codes (D/4) + f32 alphas (4·G) per row
        assert row["tile_payload_bytes"] == 32 * (512 // 4 + 4 * 16)
    assert {"full_payload_bytes", "serial_gpu_ms", "overlap_gpu_ms", "overlap_speedup_vs_serial"} <= set(j["pair"])


def test_exact_main_residual_runner(bins, tmp_path):
    out = tmp_path / "main.json"
    j = _run([bins["exact_main_residual_cuda_runner"], TAB, RES, out, 2, 32, 2, 4], out)
    assert {"experiment", "gpu", "shape", "projections", "pair"} <= set(j)
    assert j["experiment"] == "cuda_cpu_main_plus_exact_residual_v1"
    assert j["shape"]["rows"] == 96 and j["shape"]["hidden"] == 512 and j["shape"]["tile_rows"] == 32
    for p in ("gate", "up"):
        row = j["projections"][p]
        assert MAIN_PROJ <= set(row), MAIN_PROJ - set(row)
        assert row["residual_validation_rel_l2"] < 1e-5, row
    assert {"serial_cpu_plus_gpu_ms", "concurrent_wall_ms", "speedup"} <= set(j["pair"])


def test_exact_cpu_base_gpu_full_ffn_runner(bins, tmp_path):
    from ffn_residual_mesh_b200.artifacts import write_down_fp16
    src = np.load(GOLD / "artifact_source.npz")
    down = tmp_path / "down.f16"
    write_down_fp16(down, src["down"])
    out = tmp_path / "full.json"
    j = _run([bins["exact_cpu_base_gpu_full_ffn_runner"], TAB, RES, down, out, 2, 32, 2, 4], out)
    assert FULL_TOP <= set(j), FULL_TOP - set(j)
    assert j["experiment"] == "cpu_base_gpu_residual_swiglu_down_v1"
    assert j["shape"]["tile_count"] == 3
    assert j["h2d"]["resident_down_bytes"] == src["down"].size * 2
    assert {"residual_gate_up_bytes", "base_gate_up_bytes"} <= set(j["h2d"])
    c = j["correctness"]
    assert "status" in c
    assert c["y_rel_l2"] < 1e-3 and c["y_max_abs"] < 1e-2, c
