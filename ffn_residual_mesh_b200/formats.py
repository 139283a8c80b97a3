"""Host-side data formats of the path: activation quantisation and code packing.

These are the product's own implementations of the reference's host contract
(the tests check them against the oracle and the reference-generated fixtures):

* ``quantize_groupwise_q8``  — scripts/benchmark_exact_radix_split_pipeline.py:39-47
* ``pack_qlo2_rows`` / ``unpack_qlo2_rows`` — the FFN_EXACT_QLO2_ROWPACKED_V2 codes
  (scripts/export_cuda_residual_artifact_v2.py:13-24)
* ``pack_bitplanes`` / ``unpack_bitplanes`` — the FFN_HOST_BASE_GPU_RESIDUAL_V1 planes
  (scripts/compile_q4k_host_base_gpu_residual.py:17-38)
* ``split_codes`` — ``q = 2**r * q_hi + q_lo``
"""
from __future__ import annotations

import numpy as np

GROUP = 32


def quantize_groupwise_q8(x: np.ndarray, group_size: int = GROUP) -> tuple[np.ndarray, np.ndarray]:
    """int8 codes and f32 scales per token and group of ``group_size`` channels.

    ``s = max(max|x| / 127, 1e-12)`` computed in float32 and ``z = clip(rint(x / s))``
    with IEEE division and round-half-even, matching the reference bit for bit.
    """
    x = np.asarray(x, dtype=np.float32)
    if x.ndim != 2 or x.shape[1] % group_size:
        raise ValueError("x must have shape [tokens, hidden] with complete groups")
    grouped = x.reshape(x.shape[0], x.shape[1] // group_size, group_size)
    amax = np.abs(grouped).max(axis=2)
    scale = np.maximum(amax / np.float32(127.0), np.float32(1e-12)).astype(np.float32)
    q = np.rint(grouped / scale[..., None])
    z = np.clip(q, -128, 127).astype(np.int8).reshape(x.shape)
    return z, scale


def split_codes(codes: np.ndarray, residual_bits: int) -> tuple[np.ndarray, np.ndarray]:
    if not 1 <= residual_bits <= 4:
        raise ValueError("residual_bits must be in [1, 4]")
    q = np.asarray(codes, dtype=np.uint8)
    return q >> residual_bits, q & np.uint8((1 << residual_bits) - 1)


def pack_qlo2_rows(codes: np.ndarray) -> np.ndarray:
    """[rows, width] codes in [0, 3] -> [rows, width/4] bytes, code 4j+i at bits 2i of byte j."""
    c = np.asarray(codes, dtype=np.uint8)
    if c.ndim != 2 or c.shape[1] % 4:
        raise ValueError("2-bit rows must have a width divisible by four")
    if c.size and c.max() > 3:
        raise ValueError("2-bit codes must be in [0, 3]")
    quads = c.reshape(c.shape[0], -1, 4).astype(np.uint8)
    return (quads[..., 0] | (quads[..., 1] << 2) | (quads[..., 2] << 4) | (quads[..., 3] << 6)).astype(np.uint8)


def unpack_qlo2_rows(packed: np.ndarray, width: int) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint8)
    if p.ndim != 2 or p.shape[1] * 4 != width:
        raise ValueError("packed row width does not match requested output width")
    shifts = np.array([0, 2, 4, 6], dtype=np.uint8)
    return ((p[..., None] >> shifts) & 3).reshape(p.shape[0], width).astype(np.uint8)


def pack_bitplanes(values: np.ndarray, bits: int) -> bytes:
    """``bits`` little-endian planes over the flattened stream, plane 0 first."""
    if not 1 <= bits <= 4:
        raise ValueError("bits must be in [1, 4]")
    flat = np.asarray(values, dtype=np.uint8).ravel()
    return b"".join(np.packbits((flat >> b) & 1, bitorder="little").tobytes() for b in range(bits))


def unpack_bitplanes(raw: bytes, count: int, bits: int) -> np.ndarray:
    plane = (count + 7) // 8
    if len(raw) != plane * bits:
        raise ValueError("bitplane payload length does not match manifest")
    buf = np.frombuffer(raw, dtype=np.uint8)
    out = np.zeros(count, dtype=np.uint8)
    for b in range(bits):
        out |= np.unpackbits(buf[b * plane:(b + 1) * plane], bitorder="little")[:count] << b
    return out
