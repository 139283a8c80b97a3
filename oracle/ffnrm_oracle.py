"""CPU oracle for the exact integer-domain gated-FFN base/residual split.

TEST INFRASTRUCTURE ONLY. This module is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The product path (``ffn_residual_mesh_b200``) never imports or calls it and fails
loudly when its CUDA library is missing.

Every function restates one piece of the reference implementation in plain
numpy, citing the reference file and line range it follows (paths are relative
to the reference project root). Parity is pinned three ways:

* the known-answer vectors of the reference's own unit tests
  (``tests/test_exact_radix_main_table.py:76-89``,
  ``tests/test_export_cuda_residual_artifact.py:14-34``);
* golden fixtures in ``tests/golden/`` produced by importing the reference's
  Python functions (``tests/golden/make_golden.py``);
* the reference's AVX2 CPU evaluator (``src/radix_cpu_kernels.h``) compiled from
  its own source into ``oracle/_ref/`` (``oracle/Makefile``).

Notation: T tokens, D = d_model (reference "hidden"), F = d_ff (reference
"rows"), G = D/32 groups, r = residual bits, ``q = 2**r * q_hi + q_lo``.
"""
from __future__ import annotations

import numpy as np

GROUP = 32


# ---------------------------------------------------------------------------
# Activation quantisation
# ---------------------------------------------------------------------------
def quantize_groupwise_q8(x: np.ndarray, group_size: int = GROUP) -> tuple[np.ndarray, np.ndarray]:
    """Per-token, per-group symmetric int8 quantisation.

    Follows ``scripts/benchmark_exact_radix_split_pipeline.py:39-47``:
    ``s = max(max|x|/127, 1e-12)`` in float32, ``z = clip(rint(x/s), -128, 127)``.
    """
    v = np.asarray(x, dtype=np.float32)
    if v.ndim != 2 or v.shape[1] % group_size:
        raise ValueError("x must have shape [tokens, hidden] with complete groups")
    g = v.reshape(v.shape[0], -1, group_size)
    s = np.max(np.abs(g), axis=2) / np.float32(127.0)
    s = np.maximum(s, np.float32(1e-12)).astype(np.float32)
    z = np.clip(np.rint(g / s[:, :, None]), -128, 127).astype(np.int8)
    return z.reshape(v.shape), s


# ---------------------------------------------------------------------------
# Code packing formats (the on-disk artifact contract)
# ---------------------------------------------------------------------------
def pack_2bit_rows(codes: np.ndarray) -> np.ndarray:
    """Row-packed 2-bit codes: byte j of a row holds codes 4j..4j+3 at bit pairs 0,2,4,6.

    Follows ``scripts/benchmark_exact_radix_split_pipeline.py:15-26`` and
    ``scripts/export_cuda_residual_artifact_v2.py:13-24`` (format
    ``FFN_EXACT_QLO2_ROWPACKED_V2``).
    """
    c = np.asarray(codes, dtype=np.uint8)
    if c.ndim != 2 or c.shape[1] % 4:
        raise ValueError("2-bit rows must have a width divisible by four")
    if np.any(c > 3):
        raise ValueError("2-bit codes must be in [0, 3]")
    out = np.zeros((c.shape[0], c.shape[1] // 4), dtype=np.uint8)
    for pos in range(4):
        out |= (c[:, pos::4] << (2 * pos)).astype(np.uint8)
    return out


def unpack_2bit_rows(packed: np.ndarray, width: int) -> np.ndarray:
    """Inverse of :func:`pack_2bit_rows` (``benchmark_exact_radix_split_pipeline.py:29-36``)."""
    p = np.asarray(packed, dtype=np.uint8)
    if p.ndim != 2 or width != p.shape[1] * 4:
        raise ValueError("packed row width does not match requested output width")
    out = np.empty((p.shape[0], width), dtype=np.uint8)
    for pos in range(4):
        out[:, pos::4] = (p >> (2 * pos)) & 3
    return out


def pack_bitplanes(values: np.ndarray, bits: int) -> bytes:
    """Independent little-endian bit planes over the flattened value stream.

    Follows ``scripts/compile_q4k_host_base_gpu_residual.py:17-26``: plane b holds
    bit b of every value, 8 values per byte, value 8j+i at bit i of byte j.
    """
    if bits < 1 or bits > 4:
        raise ValueError("bits must be in [1, 4]")
    flat = np.asarray(values, dtype=np.uint8).reshape(-1)
    return b"".join(np.packbits((flat >> b) & 1, bitorder="little").tobytes() for b in range(bits))


def unpack_bitplanes(raw: bytes, count: int, bits: int) -> np.ndarray:
    """Inverse of :func:`pack_bitplanes` (``compile_q4k_host_base_gpu_residual.py:29-38``)."""
    plane_bytes = (count + 7) // 8
    if len(raw) != plane_bytes * bits:
        raise ValueError("bitplane payload length does not match manifest")
    out = np.zeros(count, dtype=np.uint8)
    for b in range(bits):
        plane = np.frombuffer(raw, dtype=np.uint8, count=plane_bytes, offset=b * plane_bytes)
        out |= np.unpackbits(plane, bitorder="little")[:count].astype(np.uint8) << b
    return out


def split_codes(codes: np.ndarray, residual_bits: int) -> tuple[np.ndarray, np.ndarray]:
    """Exact split ``q = 2**r * q_hi + q_lo``.

    Follows ``scripts/scan_q4k_host_base_gpu_residual.py:45-47`` (floor-div / mod)
    and ``scripts/compile_q4k_host_base_gpu_residual.py:60-62`` (shift / mask).
    """
    if residual_bits < 1 or residual_bits > 4:
        raise ValueError("residual_bits must be in [1, 4]")
    q = np.asarray(codes, dtype=np.uint8)
    return (q >> residual_bits).astype(np.uint8), (q & ((1 << residual_bits) - 1)).astype(np.uint8)


# ---------------------------------------------------------------------------
# Radix table (the host CPU base evaluator's data structure)
# ---------------------------------------------------------------------------
def compile_radix_table(q_hi: np.ndarray, block_size: int = 4) -> tuple[np.ndarray, np.ndarray]:
    """Exact base-4 partial-sum table ``table[b, state, row]`` and ``high_sum[row, g]``.

    Follows ``scripts/benchmark_exact_radix_split_pipeline.py:50-64``.
    """
    q = np.asarray(q_hi, dtype=np.uint8)
    if q.ndim != 3:
        raise ValueError("q_hi must have shape [rows, groups, group_size]")
    rows, groups, gs = q.shape
    if block_size not in (2, 4, 8) or gs % block_size:
        raise ValueError("block_size must be one of 2, 4, or 8 and divide group_size")
    blocks = q.reshape(rows, groups * gs // block_size, block_size).transpose(1, 0, 2).astype(np.int32)
    states = np.arange(4 ** block_size, dtype=np.int64)
    digits = np.stack([(states >> (2 * p)) & 3 for p in range(block_size)], axis=1).astype(np.int32)
    table = np.einsum("brc,sc->bsr", blocks, digits).astype(np.uint8)
    return table, q.astype(np.int32).sum(axis=2)


def encode_signed_base4_states(z: np.ndarray, block_size: int = 4) -> np.ndarray:
    """``z+128`` as four base-4 digit streams, one state index per block.

    Follows ``scripts/benchmark_exact_radix_split_pipeline.py:67-79``.
    """
    v = np.asarray(z, dtype=np.int8).reshape(-1)
    if block_size not in (2, 4, 8) or v.size % block_size:
        raise ValueError("block_size must be one of 2, 4, or 8 and divide the input width")
    u = (v.astype(np.int32) + 128).reshape(-1, block_size)
    weights = (4 ** np.arange(block_size, dtype=np.int64))[None, :]
    return np.stack([np.sum(((u >> (2 * d)) & 3) * weights, axis=1) for d in range(4)]).astype(np.int64)


def evaluate_radix_table(table: np.ndarray, high_sum: np.ndarray, states: np.ndarray,
                         blocks_per_group: int) -> np.ndarray:
    """Exact signed group dots ``P_hi[row, g]`` from the table (one token).

    Follows ``scripts/benchmark_exact_radix_split_pipeline.py:82-109``.
    """
    lut = np.asarray(table, dtype=np.uint8)
    st = np.asarray(states, dtype=np.int64)
    rows, groups = high_sum.shape
    if st.shape[0] != 4 or lut.shape[0] != st.shape[1] or lut.shape[0] != groups * blocks_per_group:
        raise ValueError("state streams do not match the compiled table")
    idx = np.arange(lut.shape[0])
    dot = np.zeros((groups, rows), dtype=np.int64)
    for d in range(4):
        sel = lut[idx, st[d]].astype(np.int64).reshape(groups, blocks_per_group, rows).sum(axis=1)
        dot += sel << (2 * d)
    dot -= 128 * np.asarray(high_sum, dtype=np.int64).T
    return dot.T.astype(np.int32)


# ---------------------------------------------------------------------------
# Integer group dots and scaled projections
# ---------------------------------------------------------------------------
def group_dots(codes: np.ndarray, z: np.ndarray) -> np.ndarray:
    """Exact int32 group dots ``P[t, row, g] = sum_i codes[row, g, i] * z[t, g, i]``.

    Batched form of ``direct_group_dots``
    (``scripts/benchmark_exact_radix_split_pipeline.py:162-164``), which handles one
    token; the batch loop is the restatement ``host_gpu_replay`` performs with
    einsum (``scripts/scan_q4k_host_base_gpu_residual.py:48-49``).
    ``codes`` is [F, D] or [F, G, 32] uint8; ``z`` is [T, D] or [D] int8.
    """
    c = np.asarray(codes, dtype=np.uint8)
    F = c.shape[0]
    c = c.reshape(F, -1, GROUP)
    G = c.shape[1]
    zz = np.asarray(z, dtype=np.int8).reshape(-1, G, GROUP)
    # one [F, 32] x [32, T] product per group, in float64: exact, |P| <= 32*15*128 < 2**53
    cg = np.ascontiguousarray(c.transpose(1, 0, 2)).astype(np.float64)   # [G, F, 32]
    zg = np.ascontiguousarray(zz.transpose(1, 2, 0)).astype(np.float64)  # [G, 32, T]
    prod = np.matmul(cg, zg)                                             # [G, F, T]
    return np.rint(prod).astype(np.int32).transpose(2, 1, 0).copy()      # [T, F, G]


def group_sums(z: np.ndarray) -> np.ndarray:
    """``zsum[t, g] = sum_i z[t, g, i]`` (``radix_cpu_kernels.h:84-88``)."""
    zz = np.asarray(z, dtype=np.int8)
    return zz.reshape(zz.shape[0] if zz.ndim == 2 else 1, -1, GROUP).astype(np.int32).sum(axis=2)


def scaled_projection(dots: np.ndarray, z: np.ndarray, s: np.ndarray, alpha: np.ndarray,
                      beta: np.ndarray | None, code_multiplier: int = 1) -> np.ndarray:
    """``out[t, row] = sum_g s[t,g] * (alpha[row,g]*mult*P[t,row,g] + beta[row,g]*zsum[t,g])``.

    Batched restatement of ``projection_from_group_dots``
    (``scripts/benchmark_exact_radix_split_pipeline.py:112-129``) and of the
    per-row loop of ``cpu_eval`` (``src/exact_cpu_base_gpu_full_ffn_runner.cu:154-165``).
    Evaluated in float64; ``beta=None`` drops the min term (the GPU residual).
    """
    P = np.asarray(dots, dtype=np.float64)
    ss = np.asarray(s, dtype=np.float64).reshape(P.shape[0], 1, -1)
    term = np.asarray(alpha, dtype=np.float64)[None] * (code_multiplier * P)
    if beta is not None:
        zs = group_sums(z).astype(np.float64).reshape(P.shape[0], 1, -1)
        term = term + np.asarray(beta, dtype=np.float64)[None] * zs
    return np.sum(ss * term, axis=2)


def host_base(codes: np.ndarray, alpha, beta, z, s, residual_bits: int) -> np.ndarray:
    """Host base partial sums ``alpha*2**r*dot(q_hi) + beta*sum(z)``, scaled by s.

    Follows ``host_gpu_replay`` (``scripts/scan_q4k_host_base_gpu_residual.py:22-53``,
    line 51) and ``cpu_eval`` (``src/exact_cpu_base_gpu_full_ffn_runner.cu:160-162``,
    where the multiplier is the literal 4 of r=2).
    """
    q_hi, _ = split_codes(codes, residual_bits)
    return scaled_projection(group_dots(q_hi, z), z, s, alpha, beta, 1 << residual_bits)


def residual(codes: np.ndarray, alpha, z, s, residual_bits: int) -> np.ndarray:
    """GPU residual ``sum_g s*alpha*dot(q_lo)``.

    Follows ``host_gpu_replay`` line 52 (``scan_q4k_host_base_gpu_residual.py:52``)
    and the reference ``residual_kernel`` (``src/exact_residual_cuda_runner.cu:122-159``),
    which evaluates the same sum per element in fp32.
    """
    _, q_lo = split_codes(codes, residual_bits)
    return scaled_projection(group_dots(q_lo, z), z, s, alpha, None, 1)


def full_projection(codes: np.ndarray, alpha, beta, z, s) -> np.ndarray:
    """Unsplit Q4 projection (the exact fallback / ``direct_q4`` path).

    Follows ``projection_from_group_dots(direct_group_dots(codes, z), ..., 1)`` as
    used for validation in ``scripts/benchmark_cpu_base_gpu_full_ffn.py:363-368`` and
    ``direct_q4`` (``src/radix_cpu_kernels.h:228-248``).
    """
    return scaled_projection(group_dots(codes, z), z, s, alpha, beta, 1)


def dequant_projection(codes: np.ndarray, alpha, beta, z, s, code_multiplier: int = 1) -> np.ndarray:
    """``out[t, row] = sum_k mult*codes[row,k]*alpha[row,k/32]*z[t,k]*s[t,k/32]`` (+ the beta term).

    The per-element form of the same sum, as the reference's ``residual_kernel``
    evaluates it (``q * alpha * z * scale`` per code,
    ``src/exact_residual_cuda_runner.cu:141-143``), here as one float64 GEMM so that
    full-size layers check in seconds. Every product ``alpha*q*s*z`` is exact in
    float64 (at most 45 significant bits); only the float64 summation rounds.
    ``beta`` adds ``sum_g s[t,g]*beta[row,g]*zsum[t,g]`` (``projection_from_group_dots``,
    ``scripts/benchmark_exact_radix_split_pipeline.py:112-129``).
    """
    c = np.asarray(codes, dtype=np.uint8)
    F, D = c.shape[0], c.size // c.shape[0]
    G = D // GROUP
    w = (c.reshape(F, G, GROUP).astype(np.float64) * np.asarray(alpha, np.float64)[:, :, None] *
         code_multiplier).reshape(F, D)
    zz = np.asarray(z, dtype=np.int8).reshape(-1, G, GROUP)
    ss = np.asarray(s, dtype=np.float64).reshape(zz.shape[0], G)
    x = (zz.astype(np.float64) * ss[:, :, None]).reshape(zz.shape[0], D)
    out = x @ w.T
    if beta is not None:
        out += (ss * group_sums(z).astype(np.float64)) @ np.asarray(beta, np.float64).T
    return out


def residual_fast(codes, alpha, z, s, residual_bits: int) -> np.ndarray:
    """:func:`residual` through :func:`dequant_projection` (same sum, float64 GEMM)."""
    _, q_lo = split_codes(codes, residual_bits)
    return dequant_projection(q_lo, alpha, None, z, s)


def host_base_fast(codes, alpha, beta, z, s, residual_bits: int) -> np.ndarray:
    """:func:`host_base` through :func:`dequant_projection` (same sum, float64 GEMM)."""
    q_hi, _ = split_codes(codes, residual_bits)
    return dequant_projection(q_hi, alpha, beta, z, s, 1 << residual_bits)


def full_projection_fast(codes, alpha, beta, z, s) -> np.ndarray:
    """:func:`full_projection` through :func:`dequant_projection`."""
    return dequant_projection(codes, alpha, beta, z, s)


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """``h = g / (1 + exp(-g)) * u`` (``benchmark_cpu_base_gpu_full_ffn.py:369``;
    ``exact_cpu_base_gpu_full_ffn_runner.cu:225-227``)."""
    g = np.asarray(g, dtype=np.float64)
    return g / (1.0 + np.exp(-g)) * np.asarray(u, dtype=np.float64)


def down_projection(h: np.ndarray, down_f16: np.ndarray) -> np.ndarray:
    """``y = h @ down.T`` with fp16 weights ``down[D, F]`` (``benchmark_cpu_base_gpu_full_ffn.py:370``)."""
    return np.asarray(h, dtype=np.float64) @ np.asarray(down_f16, dtype=np.float16).astype(np.float64).T


def tile_rows_mask(fallback_tiles: np.ndarray | None, F: int, tile_rows: int) -> np.ndarray:
    """Rows covered by flagged tiles (``src/phone_ffn_loopback.py:155-197``:
    a tile whose base missed its deadline is recomputed on the exact path)."""
    rows = np.zeros(F, dtype=bool)
    if fallback_tiles is None:
        return rows
    for tile in np.flatnonzero(np.asarray(fallback_tiles)):
        rows[tile * tile_rows:(tile + 1) * tile_rows] = True
    return rows


def ffn_forward(gate_codes, up_codes, gate_alpha, up_alpha, gate_beta, up_beta, down_f16,
                z, s, residual_bits: int, gate_base=None, up_base=None,
                fallback_tiles=None, tile_rows: int = 256, fast: bool = False) -> dict:
    """The full split path: merge base+residual before SwiGLU, then fp16 down.

    ``g = g_base + g_res``, ``u = u_base + u_res``, ``h = SiLU(g)*u``, ``y = h @ down.T``
    (``src/exact_cpu_base_gpu_full_ffn_runner.cu:217-240``;
    ``scripts/benchmark_cpu_base_gpu_full_ffn.py:360-371``). Rows in flagged tiles
    take the unsplit projection instead of base+residual. When no base is given
    the host base is computed here. Returns float64 intermediates. ``fast`` evaluates
    the same sums through :func:`dequant_projection` (large shapes).
    """
    hb, rs, fp = (host_base_fast, residual_fast, full_projection_fast) if fast else (host_base, residual,
                                                                                     full_projection)
    if gate_base is None:
        gate_base = hb(gate_codes, gate_alpha, gate_beta, z, s, residual_bits)
    if up_base is None:
        up_base = hb(up_codes, up_alpha, up_beta, z, s, residual_bits)
    g_res = rs(gate_codes, gate_alpha, z, s, residual_bits)
    u_res = rs(up_codes, up_alpha, z, s, residual_bits)
    g = np.asarray(gate_base, dtype=np.float64) + g_res
    u = np.asarray(up_base, dtype=np.float64) + u_res
    F = g.shape[1]
    flagged = tile_rows_mask(fallback_tiles, F, tile_rows)
    if flagged.any():
        g[:, flagged] = fp(gate_codes[flagged], gate_alpha[flagged], gate_beta[flagged], z, s)
        u[:, flagged] = fp(up_codes[flagged], up_alpha[flagged], up_beta[flagged], z, s)
    h = swiglu(g, u)
    return {"gate_res": g_res, "up_res": u_res, "g": g, "u": u, "h": h, "y": down_projection(h, down_f16)}
