"""The reference's on-disk artifact contract, read and written unchanged.

* Residual directory, format ``FFN_EXACT_QLO2_ROWPACKED_V2``
  (scripts/export_cuda_residual_artifact_v2.py:56-125): ``{gate,up}.qlo2.rowpacked.bin``
  u8 [F, D/4], ``{gate,up}.alpha.f32.bin`` f32 [F, G], ``activation.z.i8.bin`` [D],
  ``activation.scale.f32.bin`` [G] and ``manifest.json`` with the shapes, file names and
  sha256 of the code and alpha files.
* Radix table directory, format ``FFN_RADIX_TABLE_ARTIFACT_V1``
  (scripts/export_radix_table_artifact.py:17-80): ``{p}.table.u8.bin``
  [D/bs, 4^bs, F], ``{p}.high_sum.i16.bin`` [F, G], ``{p}.alpha.f32.bin``,
  ``{p}.beta.f32.bin``, ``states.u16.bin`` [4, D/bs], the activation files, manifest.
* Down projection: raw fp16 [D, F] (scripts/export_down_fp16.py:19-21).

Readers check every file size against the manifest and verify the listed checksums
(``ValueError`` on any mismatch, like the reference's Python adapter,
scripts/native_radix_cpu.py:74-79). Writers produce the same files and manifest keys as
the reference's exporters, from arrays instead of a GGUF model (the GGUF decode is the
cold-start step the reference keeps out of the runtime contract).

``BaseProducer`` drives the host base producer of ``libffnrm.so`` on a table artifact.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import _native as N
from .formats import pack_qlo2_rows, quantize_groupwise_q8

RESIDUAL_FORMAT = "FFN_EXACT_QLO2_ROWPACKED_V2"
TABLE_FORMAT = "FFN_RADIX_TABLE_ARTIFACT_V1"
PROJECTIONS = ("gate", "up")


def sha256_hex(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def _read(path: Path, dtype, count: int, what: str) -> np.ndarray:
    raw = Path(path).read_bytes()
    want = count * np.dtype(dtype).itemsize
    if len(raw) != want:
        raise ValueError(f"{what} size does not match manifest ({len(raw)} bytes, expected {want})")
    return np.frombuffer(raw, dtype=dtype).copy()


# ---------------------------------------------------------------------------
# residual artifact
# ---------------------------------------------------------------------------
@dataclass
class ResidualArtifact:
    manifest: dict
    layer: int
    rows: int
    hidden: int
    codes: dict          # projection -> u8 [rows, hidden/4] row-packed low codes
    alpha: dict          # projection -> f32 [rows, hidden/32]
    z: np.ndarray        # int8 [hidden]
    s: np.ndarray        # f32 [hidden/32]


def write_residual_artifact(out: Path, low_codes: dict, alpha: dict, x: np.ndarray, layer: int = 23,
                            source: str = "synthetic", source_q4_bytes: dict | None = None) -> dict:
    """Write a residual directory from 2-bit low codes [F, D] and alphas [F, G] per
    projection and one f32 activation row ``x`` [D] (quantised per 32-group as the
    exporter does). Returns the manifest."""
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    projections = {}
    for p in PROJECTIONS:
        codes = np.asarray(low_codes[p], dtype=np.uint8)
        a = np.ascontiguousarray(np.asarray(alpha[p], dtype="<f4"))
        packed = np.ascontiguousarray(pack_qlo2_rows(codes))
        cb, ab = packed.tobytes(), a.tobytes()
        (out / f"{p}.qlo2.rowpacked.bin").write_bytes(cb)
        (out / f"{p}.alpha.f32.bin").write_bytes(ab)
        m = {"projection": p, "layer": layer, "rows": int(codes.shape[0]), "hidden": int(codes.shape[1]),
             "residual_bits": 2, "lossless": True, "runtime_weight_reads": 0,
             "runtime_contract": "packed exact residual and alpha only; raw GGUF is cold-start-only",
             "packed_code_bytes": len(cb), "alpha_bytes": len(ab), "payload_bytes": len(cb) + len(ab)}
        m.update({"source_q4_bytes": int((source_q4_bytes or {}).get(p, 0)),
                  "packed_code_file": f"{p}.qlo2.rowpacked.bin", "packed_code_sha256": sha256_hex(cb),
                  "alpha_file": f"{p}.alpha.f32.bin", "alpha_sha256": sha256_hex(ab),
                  "alpha_shape": list(a.shape), "packed_row_bytes": int(packed.shape[1])})
        projections[p] = m
    hidden = int(projections["gate"]["hidden"])
    xv = np.asarray(x, dtype=np.float32).reshape(-1)
    if xv.size != hidden:
        raise ValueError(f"expected {hidden} float32 activation values, found {xv.size}")
    z, s = quantize_groupwise_q8(xv.reshape(1, hidden))
    zb, sb = np.ascontiguousarray(z[0]).tobytes(), np.ascontiguousarray(s[0].astype("<f4")).tobytes()
    (out / "activation.z.i8.bin").write_bytes(zb)
    (out / "activation.scale.f32.bin").write_bytes(sb)
    manifest = {"format": RESIDUAL_FORMAT, "layer": layer, "lossless": True, "runtime_weight_reads": 0,
                "activation": {"source": source, "z_file": "activation.z.i8.bin", "z_bytes": len(zb),
                               "scale_file": "activation.scale.f32.bin", "scale_bytes": len(sb), "group_size": 32},
                "projections": projections}
    (out / "manifest.json").write_text(json.dumps(manifest, ensure_ascii=False, indent=2), encoding="utf-8")
    return manifest


def read_residual_artifact(path: Path, verify: bool = True) -> ResidualArtifact:
    path = Path(path)
    m = json.loads((path / "manifest.json").read_text(encoding="utf-8"))
    codes, alpha = {}, {}
    shape = None
    for p in PROJECTIONS:
        pm = m["projections"][p]
        rows, hidden = int(pm["rows"]), int(pm["hidden"])
        if rows <= 0 or hidden <= 0 or hidden % 32:
            raise ValueError("artifact shape is incompatible with the QLO2 layout")
        if int(pm.get("residual_bits", 2)) != 2:
            raise ValueError("QLO2 row-packed artifacts hold 2-bit residuals")
        cb = (path / pm.get("packed_code_file", f"{p}.qlo2.rowpacked.bin")).read_bytes()
        ab = (path / pm.get("alpha_file", f"{p}.alpha.f32.bin")).read_bytes()
        if len(cb) != rows * hidden // 4:
            raise ValueError(f"{p} packed code size does not match manifest")
        if len(ab) != rows * (hidden // 32) * 4:
            raise ValueError(f"{p} alpha size does not match manifest")
        if verify:
            for key, data, what in (("packed_code_sha256", cb, "packed codes"), ("alpha_sha256", ab, "alpha")):
                if key in pm and sha256_hex(data) != pm[key]:
                    raise ValueError(f"{p} {what} sha256 mismatch")
        codes[p] = np.frombuffer(cb, dtype=np.uint8).reshape(rows, hidden // 4).copy()
        alpha[p] = np.frombuffer(ab, dtype="<f4").reshape(rows, hidden // 32).copy()
        if shape is not None and shape != (rows, hidden):
            raise ValueError("gate and up shapes differ")
        shape = (rows, hidden)
    act = m.get("activation", {})
    rows, hidden = shape
    z = _read(path / act.get("z_file", "activation.z.i8.bin"), np.int8, hidden, "activation z")
    s = _read(path / act.get("scale_file", "activation.scale.f32.bin"), "<f4", hidden // 32, "activation scale")
    return ResidualArtifact(m, int(m.get("layer", -1)), rows, hidden, codes, alpha, z, s)


# ---------------------------------------------------------------------------
# radix table artifact
# ---------------------------------------------------------------------------
@dataclass
class TableArtifact:
    manifest: dict
    block_size: int
    rows: int
    hidden: int
    table: dict       # projection -> u8 [blocks, 4^bs, rows]
    high_sum: dict    # projection -> i16 [rows, G]
    alpha: dict       # projection -> f32 [rows, G]
    beta: dict
    states: np.ndarray  # u16 [4, blocks]
    z: np.ndarray
    s: np.ndarray


def write_table_artifact(out: Path, tables: dict, high_sums: dict, alpha: dict, beta: dict, z: np.ndarray,
                         s: np.ndarray, states: np.ndarray, block_size: int, layer: int = 23,
                         source_q4_bytes: dict | None = None) -> dict:
    """Write a radix table directory from compiled tables (the exporter's file layout and
    manifest keys). ``tables[p]`` u8 [blocks, 4^bs, F]; ``high_sums[p]`` [F, G]."""
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    np.asarray(states, dtype="<u2").tofile(out / "states.u16.bin")
    np.asarray(s, dtype="<f4").reshape(-1).tofile(out / "activation.scale.f32.bin")
    np.asarray(z, dtype=np.int8).reshape(-1).tofile(out / "activation.z.i8.bin")
    projections = {}
    for p in PROJECTIONS:
        t = np.ascontiguousarray(tables[p], dtype=np.uint8)
        hs = np.ascontiguousarray(high_sums[p], dtype="<i2")
        a = np.ascontiguousarray(alpha[p], dtype="<f4")
        b = np.ascontiguousarray(beta[p], dtype="<f4")
        t.tofile(out / f"{p}.table.u8.bin")
        hs.tofile(out / f"{p}.high_sum.i16.bin")
        a.tofile(out / f"{p}.alpha.f32.bin")
        b.tofile(out / f"{p}.beta.f32.bin")
        rows, groups = hs.shape
        projections[p] = {"rows": int(rows), "hidden": int(groups * 32), "groups": int(groups),
                          "block_size": block_size, "blocks": int(t.shape[0]), "state_count": int(t.shape[1]),
                          # the exporter reports the in-memory size of its int64 high_sum (8 B per
                          # entry) although the file holds int16; the key keeps that meaning
                          "table_bytes": int(t.nbytes), "high_sum_bytes": int(hs.size * 8), "alpha_bytes": int(a.nbytes),
                          "beta_bytes": int(b.nbytes), "q4_source_bytes": int((source_q4_bytes or {}).get(p, 0)),
                          "files": {"table": f"{p}.table.u8.bin", "high_sum": f"{p}.high_sum.i16.bin",
                                    "alpha": f"{p}.alpha.f32.bin", "beta": f"{p}.beta.f32.bin"}}
    zz = np.asarray(z).reshape(-1)
    manifest = {"format": TABLE_FORMAT, "layer": layer, "block_size": block_size,
                "activation": {"hidden": int(zz.size), "groups": int(zz.size // 32), "group_size": 32,
                               "files": {"z": "activation.z.i8.bin", "scale": "activation.scale.f32.bin",
                                         "states": "states.u16.bin"}},
                "projections": projections,
                "runtime_contract": "CPU reads finite radix table entries; GPU reads packed exact residual tiles; "
                                    "raw GGUF is cold-start-only"}
    (out / "manifest.json").write_text(json.dumps(manifest, ensure_ascii=False, indent=2), encoding="utf-8")
    return manifest


def read_table_artifact(path: Path, block_size: int | None = None) -> TableArtifact:
    path = Path(path)
    m = json.loads((path / "manifest.json").read_text(encoding="utf-8"))
    bs = int(m.get("block_size", block_size or 4))
    if block_size is not None and bs != block_size:
        raise ValueError(f"block size {block_size} does not match the table artifact's {bs}")
    if bs not in (2, 4, 8):
        raise ValueError("block size must be 2, 4, or 8")
    out = {k: {} for k in ("table", "high_sum", "alpha", "beta")}
    shape = None
    for p in PROJECTIONS:
        pm = m["projections"][p]
        rows, hidden = int(pm["rows"]), int(pm["hidden"])
        groups, blocks, states = hidden // 32, hidden // bs, 4 ** bs
        files = pm.get("files", {})
        out["table"][p] = _read(path / files.get("table", f"{p}.table.u8.bin"), np.uint8, blocks * states * rows,
                                f"{p} table").reshape(blocks, states, rows)
        out["high_sum"][p] = _read(path / files.get("high_sum", f"{p}.high_sum.i16.bin"), "<i2", rows * groups,
                                   f"{p} high_sum").reshape(rows, groups)
        out["alpha"][p] = _read(path / files.get("alpha", f"{p}.alpha.f32.bin"), "<f4", rows * groups,
                                f"{p} alpha").reshape(rows, groups)
        out["beta"][p] = _read(path / files.get("beta", f"{p}.beta.f32.bin"), "<f4", rows * groups,
                               f"{p} beta").reshape(rows, groups)
        if shape is not None and shape != (rows, hidden):
            raise ValueError("gate and up shapes differ")
        shape = (rows, hidden)
    rows, hidden = shape
    f = m.get("activation", {}).get("files", {})
    z = _read(path / f.get("z", "activation.z.i8.bin"), np.int8, hidden, "activation z")
    s = _read(path / f.get("scale", "activation.scale.f32.bin"), "<f4", hidden // 32, "activation scale")
    st = _read(path / f.get("states", "states.u16.bin"), "<u2", 4 * (hidden // bs), "states").reshape(4, hidden // bs)
    return TableArtifact(m, bs, rows, hidden, out["table"], out["high_sum"], out["alpha"], out["beta"], st, z, s)


def write_down_fp16(path: Path, down: np.ndarray) -> None:
    np.ascontiguousarray(down, dtype="<f2").tofile(path)


def read_down_fp16(path: Path, hidden: int, rows: int) -> np.ndarray:
    return _read(Path(path), "<f2", hidden * rows, "down fp16").reshape(hidden, rows)


# ---------------------------------------------------------------------------
# host base producer
# ---------------------------------------------------------------------------
class RadixTable(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int32), ("hidden", ctypes.c_int32), ("block_size", ctypes.c_int32),
                ("table", ctypes.c_void_p), ("high_sum", ctypes.c_void_p), ("alpha", ctypes.c_void_p),
                ("beta", ctypes.c_void_p)]


def radix_table(table: np.ndarray, high_sum: np.ndarray, alpha: np.ndarray, beta: np.ndarray,
                block_size: int) -> tuple[RadixTable, tuple]:
    """The C view of one projection's table (arrays kept alive by the returned tuple)."""
    keep = (np.ascontiguousarray(table, dtype=np.uint8), np.ascontiguousarray(high_sum, dtype=np.int16),
            np.ascontiguousarray(alpha, dtype=np.float32), np.ascontiguousarray(beta, dtype=np.float32))
    rows, groups = keep[1].shape
    if keep[0].shape != (groups * 32 // block_size, 4 ** block_size, rows):
        raise ValueError("table shape does not match high_sum and block_size")
    t = RadixTable(rows, groups * 32, block_size, *(a.ctypes.data for a in keep))
    return t, keep


class BaseProducer:
    """Exact base sums on the host's cores (``ffnrm_base_from_table``)."""

    _h = None

    def __init__(self, threads: int):
        h = ctypes.c_void_p()
        N.check(N.lib().ffnrm_base_producer_create(ctypes.byref(h), int(threads)))
        self._h = h
        self.threads = int(threads)

    def close(self):
        if self._h is not None:
            N.lib().ffnrm_base_producer_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def from_table(self, table: RadixTable, z: np.ndarray, s: np.ndarray, multiplier: int = 4, tile_rows: int = 256,
                   out: np.ndarray | None = None, tile_ready: np.ndarray | None = None,
                   deadline_s: float | None = None) -> tuple[np.ndarray, np.ndarray | None]:
        z = np.ascontiguousarray(np.atleast_2d(z), dtype=np.int8)
        s = np.ascontiguousarray(np.atleast_2d(s), dtype=np.float32)
        T = z.shape[0]
        if z.shape[1] != table.hidden or s.shape != (T, table.hidden // 32):
            raise ValueError("activation shape does not match the table")
        if out is None:
            out = np.empty((T, table.rows), dtype=np.float32)
        if out.dtype != np.float32 or out.shape != (T, table.rows) or not out.flags["C_CONTIGUOUS"]:
            raise ValueError("out must be a contiguous f32 [tokens, rows] array")
        ntile = -(-table.rows // tile_rows)
        late = np.zeros(ntile, dtype=np.uint8) if deadline_s else None
        N.check(N.lib().ffnrm_base_from_table(
            self._h, ctypes.byref(table), z.ctypes.data, s.ctypes.data, T, int(multiplier), out.ctypes.data,
            int(tile_rows), tile_ready.ctypes.data if tile_ready is not None else None,
            int(deadline_s * 1e9) if deadline_s else 0, late.ctypes.data if late is not None else None))
        return out, late


def table_dots(table: RadixTable, z: np.ndarray) -> np.ndarray:
    """Exact P_hi [rows, G] of one token from the table (``ffnrm_table_dots``)."""
    z = np.ascontiguousarray(z, dtype=np.int8).reshape(-1)
    out = np.empty((table.rows, table.hidden // 32), dtype=np.int32)
    N.check(N.lib().ffnrm_table_dots(ctypes.byref(table), z.ctypes.data, out.ctypes.data))
    return out
