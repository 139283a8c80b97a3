"""GGUF ingest: Q4_K gate/up projections to split-path layers and artifacts.

The reference reads real model weights with the third-party ``gguf`` package
(``GGUFReader`` + ``gguf.quants``, version 0.19.0 in this image, no pin in the
reference): ``load_q4k_codes`` (scripts/scan_q4k_hierarchical_code_split.py:23-48)
turns a Q4_K FFN projection into 4-bit codes with per-32-group ``alpha = d·sc`` and
``beta = -dmin·m``; ``compile_projection`` (scripts/compile_q4k_host_base_gpu_residual.py:55-96)
writes the host-high / GPU-residual bit-plane artifact; ``export_down_fp16.py`` writes
the dequantised down projection as row-major fp16 ``[hidden, ffn]``.

This module reads the GGUF container itself (no third-party dependency at run time)
from the published format: little-endian header ``"GGUF"``, version (2 or 3), tensor
and metadata counts; typed metadata key/values; tensor infos (name, dims innermost
first, ggml type, offset); tensor data from the first ``general.alignment`` boundary
after the infos. Block layouts follow the published ggml quantisation formats:

* Q4_K, 256 values in 144 bytes: fp16 ``d``, fp16 ``dmin``, 12 bytes of eight
  6-bit (scale, min) pairs, 128 bytes of nibbles. Value ``64c + l`` (l < 32) is the low
  nibble of byte ``32c + l`` in sub-block ``2c``; value ``64c + 32 + l`` its high nibble
  in sub-block ``2c + 1``; ``y = d·sc·q - dmin·m``.
* Q6_K, 256 values in 210 bytes: 128 bytes low nibbles, 64 bytes of 2-bit highs,
  16 int8 scales, fp16 ``d``; ``y = d·sc·(q - 32)``.
* Q8_0, 32 values in 34 bytes: fp16 ``d``, 32 int8; ``y = d·q``.
* F32, F16, BF16 as stored.

The codes keep the reference's block ordering, so a Q4_K row of ``hidden`` values
is exactly ``hidden / 32`` code groups with one (alpha, beta) each: the split path's
layer format with no re-quantisation.
"""
from __future__ import annotations

import hashlib
import json
import platform
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .formats import pack_bitplanes, unpack_bitplanes

GGUF_MAGIC = b"GGUF"
QK_K = 256
Q4_K_BLOCK = 144
Q6_K_BLOCK = 210
Q8_0_BLOCK = 34
GROUP = 32

# ggml tensor types this reader decodes
F32, F16, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 8, 12, 14, 30
TYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", BF16: "BF16"}
# (values per block, bytes per block)
BLOCKS = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, Q8_0_BLOCK), Q4_K: (QK_K, Q4_K_BLOCK),
          Q6_K: (QK_K, Q6_K_BLOCK)}

ARTIFACT_MAGIC = "FFN_HOST_BASE_GPU_RESIDUAL_V1"

# metadata value types: fixed-size scalars (struct code) and the variable ones
_SCALARS = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
_STRING, _ARRAY = 8, 9


class GgufError(ValueError):
    """The file is not a GGUF container this reader understands, or a tensor is
    missing or of an unsupported type."""


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dims: tuple          # innermost first, as stored (ne[0] = values per row)
    type: int
    offset: int          # absolute file offset of the data

    @property
    def rows(self) -> int:
        return int(np.prod(self.dims[1:], dtype=np.int64)) if len(self.dims) > 1 else 1

    @property
    def row_values(self) -> int:
        return int(self.dims[0])

    @property
    def n_bytes(self) -> int:
        per, nb = BLOCKS[self.type]
        return self.rows * (self.row_values // per) * nb


class _Cursor:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, fmt: str):
        size = struct.calcsize("<" + fmt)
        if self.pos + size > len(self.buf):
            raise GgufError("truncated GGUF header")
        v = struct.unpack_from("<" + fmt, self.buf, self.pos)
        self.pos += size
        return v[0] if len(v) == 1 else v

    def string(self) -> str:
        n = self.take("Q")
        if self.pos + n > len(self.buf):
            raise GgufError("truncated GGUF string")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8")
        self.pos += n
        return s

    def value(self, vtype: int):
        if vtype in _SCALARS:
            return self.take(_SCALARS[vtype])
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            etype, n = self.take("I"), self.take("Q")
            if etype in _SCALARS:
                code = _SCALARS[etype]
                size = struct.calcsize("<" + code)
                if self.pos + size * n > len(self.buf):
                    raise GgufError("truncated GGUF array")
                arr = list(struct.unpack_from(f"<{n}{code}", self.buf, self.pos))
                self.pos += size * n
                return arr
            return [self.value(etype) for _ in range(n)]
        raise GgufError(f"unknown GGUF metadata type {vtype}")


class GgufFile:
    """A GGUF file opened read-only through a memory map: ``metadata`` (key -> value),
    ``tensors`` (name -> TensorInfo), ``raw(name)`` the tensor's bytes as
    ``uint8 [rows, row_bytes]``."""

    def __init__(self, path: Path):
        self.path = Path(path)
        self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        c = _Cursor(memoryview(self._map))
        if bytes(c.take("4s")) != GGUF_MAGIC:
            raise GgufError(f"{self.path}: not a GGUF file")
        self.version = c.take("I")
        if self.version not in (2, 3):
            raise GgufError(f"{self.path}: unsupported GGUF version {self.version}")
        n_tensors, n_kv = c.take("Q"), c.take("Q")
        self.metadata = {}
        for _ in range(n_kv):
            key = c.string()
            self.metadata[key] = c.value(c.take("I"))
        infos = []
        for _ in range(n_tensors):
            name = c.string()
            nd = c.take("I")
            dims = tuple(c.take("Q") for _ in range(nd))
            infos.append((name, dims, c.take("I"), c.take("Q")))
        align = int(self.metadata.get("general.alignment", 32))
        if align <= 0 or align & (align - 1):
            raise GgufError(f"{self.path}: bad general.alignment {align}")
        data = -(-c.pos // align) * align
        self.tensors = {}
        for name, dims, ttype, off in infos:
            t = TensorInfo(name, dims, ttype, data + off)
            if ttype in BLOCKS:
                per, _ = BLOCKS[ttype]
                if t.row_values % per:
                    raise GgufError(f"{name}: row of {t.row_values} values is not whole {TYPE_NAMES[ttype]} blocks")
                if t.offset + t.n_bytes > self._map.size:
                    raise GgufError(f"{name}: data runs past the end of the file")
            self.tensors[name] = t

    def info(self, name: str) -> TensorInfo:
        t = self.tensors.get(name)
        if t is None:
            raise GgufError(f"{self.path}: no tensor {name!r}")
        if t.type not in BLOCKS:
            raise GgufError(f"{name}: unsupported ggml type {t.type}")
        return t

    def raw(self, name: str) -> np.ndarray:
        t = self.info(name)
        return self._map[t.offset:t.offset + t.n_bytes].reshape(t.rows, -1)

    def dequantize(self, name: str) -> np.ndarray:
        """The tensor as f32 [rows, row_values]."""
        t = self.info(name)
        return dequantize(self.raw(name), t.type, t.row_values)


def _f16(raw: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(raw).view(np.float16).astype(np.float32)


def q4k_scale_min(scales: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Eight 6-bit (scale, min) pairs from the 12 packed bytes of each Q4_K block:
    pairs 0-3 are the low six bits of bytes 0-3 / 4-7; pairs 4-7 take their low four
    bits from bytes 8-11 (scale: low nibble, min: high nibble) and their top two bits
    from the top bits of bytes 0-3 / 4-7."""
    q = scales.astype(np.uint8)
    sc = np.empty(q.shape[:-1] + (8,), dtype=np.uint8)
    mn = np.empty_like(sc)
    sc[..., :4] = q[..., 0:4] & 63
    mn[..., :4] = q[..., 4:8] & 63
    sc[..., 4:] = (q[..., 8:12] & 0x0F) | ((q[..., 0:4] >> 6) << 4)
    mn[..., 4:] = (q[..., 8:12] >> 4) | ((q[..., 4:8] >> 6) << 4)
    return sc, mn


def q4k_decode(raw: np.ndarray, row_values: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Q4_K rows -> (codes u8 [rows, row_values] in 0..15, alpha f32 [rows, row_values/32],
    beta f32 [rows, row_values/32]), so that value = alpha·code + beta per 32-group.
    The reference's load_q4k_codes, scripts/scan_q4k_hierarchical_code_split.py:23-48."""
    rows = raw.shape[0]
    nb = row_values // QK_K
    b = np.asarray(raw, dtype=np.uint8).reshape(rows, nb, Q4_K_BLOCK)
    d = _f16(b[:, :, 0:2]).reshape(rows, nb, 1)
    dmin = _f16(b[:, :, 2:4]).reshape(rows, nb, 1)
    sc, mn = q4k_scale_min(b[:, :, 4:16])
    alpha = (d * sc.astype(np.float32)).reshape(rows, nb * 8)
    beta = (-dmin * mn.astype(np.float32)).reshape(rows, nb * 8)
    qs = b[:, :, 16:].reshape(rows, nb, 4, 32)
    codes = np.stack([qs & 0x0F, qs >> 4], axis=3).reshape(rows, row_values)
    return np.ascontiguousarray(codes), np.ascontiguousarray(alpha), np.ascontiguousarray(beta)


def _q6k(raw: np.ndarray, row_values: int) -> np.ndarray:
    rows, nb = raw.shape[0], row_values // QK_K
    b = np.asarray(raw, dtype=np.uint8).reshape(rows * nb, Q6_K_BLOCK)
    ql, qh = b[:, 0:128].reshape(-1, 2, 64), b[:, 128:192].reshape(-1, 2, 32)
    sc = b[:, 192:208].view(np.int8).astype(np.float32).reshape(-1, 2, 8)
    d = _f16(b[:, 208:210]).reshape(-1, 1, 1)
    # per 128-value half: four 32-value quarters from (low nibble of ql[0:32], bits 0-1 of qh),
    # (low of ql[32:64], bits 2-3), (high of ql[0:32], bits 4-5), (high of ql[32:64], bits 6-7)
    lo = np.concatenate([ql[:, :, 0:32] & 15, ql[:, :, 32:64] & 15, ql[:, :, 0:32] >> 4, ql[:, :, 32:64] >> 4], axis=2)
    hi = np.concatenate([(qh >> 0) & 3, (qh >> 2) & 3, (qh >> 4) & 3, (qh >> 6) & 3], axis=2)
    q = (lo | (hi << 4)).astype(np.float32) - 32.0          # [blocks, 2, 128]
    scale = np.repeat(sc, 16, axis=2)                          # one scale per 16 values
    return (d * scale * q).reshape(rows, row_values)


def dequantize(raw: np.ndarray, ttype: int, row_values: int) -> np.ndarray:
    """ggml block data [rows, row_bytes] -> f32 [rows, row_values]."""
    rows = raw.shape[0]
    if ttype == F32:
        return np.ascontiguousarray(raw).view("<f4").reshape(rows, row_values).copy()
    if ttype == F16:
        return _f16(raw).reshape(rows, row_values)
    if ttype == BF16:
        u = np.ascontiguousarray(raw).view("<u2").astype(np.uint32) << 16
        return u.view(np.float32).reshape(rows, row_values)
    if ttype == Q8_0:
        b = np.asarray(raw, dtype=np.uint8).reshape(-1, Q8_0_BLOCK)
        return (_f16(b[:, 0:2]) * b[:, 2:].view(np.int8).astype(np.float32)).reshape(rows, row_values)
    if ttype == Q4_K:
        codes, alpha, beta = q4k_decode(raw, row_values)
        g = codes.reshape(rows, -1, GROUP).astype(np.float32)
        return (alpha[:, :, None] * g + beta[:, :, None]).reshape(rows, row_values)
    if ttype == Q6_K:
        return _q6k(raw, row_values)
    raise GgufError(f"unsupported ggml type {ttype}")


@dataclass
class Q4kLayer:
    """One FFN layer from a GGUF file, in the split path's layer format."""
    gate_codes: np.ndarray   # u8 [F, D], 0..15
    up_codes: np.ndarray
    gate_alpha: np.ndarray   # f32 [F, D/32]
    up_alpha: np.ndarray
    gate_beta: np.ndarray
    up_beta: np.ndarray
    down: np.ndarray | None  # fp16 [D, F]
    q4k_bytes: int           # Q4_K bytes of gate + up in the file

    def spec(self):
        """The ``LayerSpec`` for ``ResidualMesh.load_layer`` (betas kept for fallback)."""
        from .engine import LayerSpec
        return LayerSpec(self.gate_codes, self.up_codes, self.gate_alpha, self.up_alpha, self.down,
                         self.gate_beta, self.up_beta)


def projection_name(layer: int, projection: str) -> str:
    return f"blk.{layer}.ffn_{projection}.weight"


def load_q4k_projection(g: GgufFile, layer: int, projection: str):
    """(codes, alpha, beta, q4k bytes) of ``blk.{layer}.ffn_{projection}.weight``, which
    must be Q4_K (the reference raises on any other type)."""
    name = projection_name(layer, projection)
    t = g.info(name)
    if t.type != Q4_K:
        raise GgufError(f"expected Q4_K tensor type {Q4_K}, got {t.type} for {name}")
    codes, alpha, beta = q4k_decode(g.raw(name), t.row_values)
    return codes, alpha, beta, t.n_bytes


def load_down_fp16(g: GgufFile, layer: int) -> np.ndarray:
    """``blk.{layer}.ffn_down.weight`` dequantised to fp16 [hidden, ffn] (row-major, as
    scripts/export_down_fp16.py writes it)."""
    return g.dequantize(projection_name(layer, "down")).astype(np.float16)


def load_layer(path: Path, layer: int, with_down: bool = True) -> Q4kLayer:
    g = GgufFile(path)
    gc, ga, gb, gn = load_q4k_projection(g, layer, "gate")
    uc, ua, ub, un = load_q4k_projection(g, layer, "up")
    if gc.shape != uc.shape:
        raise GgufError(f"layer {layer}: gate {gc.shape} and up {uc.shape} differ")
    down = None
    if with_down:
        down = load_down_fp16(g, layer)
        if down.shape != (gc.shape[1], gc.shape[0]):
            raise GgufError(f"layer {layer}: down {down.shape} does not match [hidden, ffn] "
                            f"{(gc.shape[1], gc.shape[0])}")
    return Q4kLayer(gc, uc, ga, ua, gb, ub, down, gn + un)


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _write_array(path: Path, array: np.ndarray, dtype: str) -> dict:
    v = np.ascontiguousarray(array.astype(dtype, copy=False))
    path.write_bytes(v.tobytes())
    return {"file": path.name, "shape": list(v.shape), "dtype": dtype, "bytes": path.stat().st_size}


def compile_projection(g: GgufFile, layer: int, projection: str, residual_bits: int, out: Path) -> dict:
    """One projection's host-high / GPU-residual bit planes plus alpha and beta, checked
    by decoding the written streams (scripts/compile_q4k_host_base_gpu_residual.py:55-96).
    Codes, alpha and beta are written in the Q4_K block shape [rows, blocks, 256 | 8]."""
    codes, alpha, beta, q4_bytes = load_q4k_projection(g, layer, projection)
    rows, width = codes.shape
    blocks = width // QK_K
    codes = codes.reshape(rows, blocks, QK_K)
    low = codes & ((1 << residual_bits) - 1)
    high = codes >> residual_bits
    high_path = out / f"{projection}.host_high.bitplanes"
    low_path = out / f"{projection}.gpu_residual.bitplanes"
    high_path.write_bytes(pack_bitplanes(high, 4 - residual_bits))
    low_path.write_bytes(pack_bitplanes(low, residual_bits))
    a_info = _write_array(out / f"{projection}.alpha.f32", alpha.reshape(rows, blocks, 8), "<f4")
    b_info = _write_array(out / f"{projection}.beta.f32", beta.reshape(rows, blocks, 8), "<f4")
    n = codes.size
    back = (unpack_bitplanes(high_path.read_bytes(), n, 4 - residual_bits) << residual_bits) | \
        unpack_bitplanes(low_path.read_bytes(), n, residual_bits)
    if not np.array_equal(back.reshape(codes.shape), codes):
        raise RuntimeError(f"artifact code reconstruction failed for {projection}")
    hb, lb = high_path.stat().st_size, low_path.stat().st_size
    return {
        "projection": projection,
        "shape": [rows, blocks, QK_K],
        "q4k_source_bytes": int(q4_bytes),
        "host_high_bits": 4 - residual_bits,
        "gpu_residual_bits": residual_bits,
        "host_high_bitplanes": {"file": high_path.name, "bytes": hb, "sha256": _sha256(high_path)},
        "gpu_residual_bitplanes": {"file": low_path.name, "bytes": lb, "sha256": _sha256(low_path)},
        "alpha": a_info,
        "beta": b_info,
        "host_artifact_bytes": hb + b_info["bytes"] + a_info["bytes"],
        "gpu_residual_package_bytes": lb + a_info["bytes"],
    }


def compile_artifact(model: Path, layer: int, residual_bits: int, out: Path) -> dict:
    """The host-base / GPU-residual artifact directory of one layer (gate and up) with its
    manifest (scripts/compile_q4k_host_base_gpu_residual.py:107-160); returns the manifest."""
    if not 1 <= residual_bits <= 3:
        raise ValueError("residual bits must be 1, 2, or 3")
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    g = GgufFile(model)
    rows = [compile_projection(g, layer, p, residual_bits, out) for p in ("gate", "up")]
    manifest = {
        "magic": ARTIFACT_MAGIC,
        "version": 1,
        "model": str(model),
        "layer": layer,
        "residual_bits": residual_bits,
        "host_high_bits": 4 - residual_bits,
        "compile_phase": "raw Q4_K is scanned once here; runtime must use this manifest and payloads only",
        "runtime_formula": "host_base = alpha * 2^r * dot(x, q_hi) + beta * sum(x); "
                           "gpu_residual = alpha * dot(x, q_lo); merged = host_base + gpu_residual",
        "platform": platform.platform(),
        "projections": {r["projection"]: r for r in rows},
        "pair_totals": {k: sum(r[k] for r in rows)
                        for k in ("host_artifact_bytes", "gpu_residual_package_bytes", "q4k_source_bytes")},
        "access_contract": {
            "cold_start_raw_weight_scan": True,
            "runtime_raw_weight_scan": False,
            "runtime_reads": ["manifest.json", "host_high.bitplanes", "gpu_residual.bitplanes", "alpha", "beta"],
            "fallback": "raw GGUF may be opened only by an explicitly counted exact fallback path",
        },
    }
    (out / "manifest.json").write_text(json.dumps(manifest, ensure_ascii=False, indent=2), encoding="utf-8")
    return manifest


def read_artifact(path: Path, verify: bool = True) -> dict:
    """Read a compiled host-base / GPU-residual directory back into per-projection
    ``(codes u8 [rows, hidden], alpha, beta f32 [rows, hidden/32])`` with the
    manifest's sha256 checked; ``codes = high << r | low``."""
    path = Path(path)
    m = json.loads((path / "manifest.json").read_text(encoding="utf-8"))
    if m.get("magic") != ARTIFACT_MAGIC or int(m.get("version", 0)) != 1:
        raise ValueError(f"{path}: not a {ARTIFACT_MAGIC} artifact")
    r = int(m["residual_bits"])
    out = {}
    for name, p in m["projections"].items():
        rows, blocks, width = (int(v) for v in p["shape"])
        n = rows * blocks * width
        planes = {}
        for key, bits in (("host_high_bitplanes", 4 - r), ("gpu_residual_bitplanes", r)):
            f = path / p[key]["file"]
            if verify and _sha256(f) != p[key]["sha256"]:
                raise ValueError(f"{f}: sha256 does not match the manifest")
            planes[key] = unpack_bitplanes(f.read_bytes(), n, bits)
        codes = (planes["host_high_bitplanes"] << r) | planes["gpu_residual_bitplanes"]
        ab = []
        for key in ("alpha", "beta"):
            a = np.fromfile(path / p[key]["file"], dtype="<f4")
            if a.size != rows * blocks * 8:
                raise ValueError(f"{name}.{key}: {a.size} values, expected {rows * blocks * 8}")
            ab.append(a.reshape(rows, blocks * 8))
        out[name] = (codes.reshape(rows, blocks * width), ab[0], ab[1])
    return out
