"""Generate the golden fixtures in this directory from the reference's own code.

Run in a container that has the reference checkout (it is not needed at test time):

    python tests/golden/make_golden.py --reference <reference checkout> [--only NAME ...]

Every value stored as an expected output is computed by a function imported from
the reference's ``scripts/`` directory, never by this repository's oracle:

* ``quantize_groupwise_q8``, ``pack_2bit_rows``, ``direct_group_dots``,
  ``compile_radix_table``, ``encode_signed_base4_states``, ``evaluate_radix_table``,
  ``projection_from_group_dots``  (scripts/benchmark_exact_radix_split_pipeline.py)
* ``pack_row_codes`` (scripts/export_cuda_residual_artifact_v2.py)
* ``pack_bitplanes`` (scripts/compile_q4k_host_base_gpu_residual.py)
* ``load_q4k_codes`` via compile_q4k_host_base_gpu_residual.py main() and
  export_down_fp16.py main() on a GGUF file written with the ``gguf`` package
* ``host_gpu_replay`` (scripts/scan_q4k_host_base_gpu_residual.py) for batched
  host-base / residual / merged projections at r = 1, 2, 3
* the SwiGLU + down formula of scripts/benchmark_cpu_base_gpu_full_ffn.py:369-370.

Inputs follow the synthetic distributions of the five benchmark configurations,
shrunk to sizes a CPU test handles in well under a second: Q4 codes uniform in
[0, 15], fp16-exact alpha = |N(0,0.02)|/8 and beta = -(same law), activations
N(0,1) (optionally with 1% outlier channels x20) quantised per token and group,
fp16 down weights N(0,0.02).
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# name: (F rows, D hidden, T tokens, r residual bits, outlier fraction, seed, tile_rows, flagged tiles)
CASES = {
    "c1_decode_t1_r2": (96, 512, 1, 2, 0.0, 101, 32, ()),
    "c2_decode_t8_r2": (160, 512, 8, 2, 0.0, 202, 64, ()),
    "c3_decode_t16_r1_outliers": (64, 768, 16, 1, 0.01, 303, 32, ()),
    "c4_decode_t32_r2": (128, 512, 32, 2, 0.0, 404, 64, ()),
    "c5_t5_r3_fallback": (200, 256, 5, 3, 0.0, 505, 64, (1, 3)),
    "c5_t3_r2_fallback": (130, 256, 3, 2, 0.0, 506, 32, (0, 4)),
    # full 70B-class d_model, rows cut to 64, one flagged tile
    "c4_d8192_t16_r2_fallback": (64, 8192, 16, 2, 0.0, 408, 32, (1,)),
}


def synth(F, D, T, outliers, seed):
    rng = np.random.default_rng(seed)
    G = D // 32
    codes = rng.integers(0, 16, (F, D), dtype=np.uint8)
    alpha = (np.abs(rng.normal(0, 0.02, (F, G))) / 8).astype(np.float16).astype(np.float32)
    beta = -(np.abs(rng.normal(0, 0.02, (F, G))) / 8).astype(np.float16).astype(np.float32)
    x = rng.normal(size=(T, D)).astype(np.float32)
    if outliers:
        ch = rng.choice(D, max(1, int(round(outliers * D))), replace=False)
        x[:, ch] *= 20.0
    down = rng.normal(0, 0.02, (D, F)).astype(np.float16)
    return codes, alpha, beta, x, down


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True, help="the reference checkout (its scripts/ are imported)")
    ap.add_argument("--only", nargs="*", default=None, help="generate only these cases (and skip the KAT file)")
    args = ap.parse_args()
    sys.path.insert(0, str(args.reference / "scripts"))
    import torch
    from benchmark_exact_radix_split_pipeline import (compile_radix_table, direct_group_dots,
                                                      encode_signed_base4_states, evaluate_radix_table,
                                                      pack_2bit_rows, projection_from_group_dots,
                                                      quantize_groupwise_q8)
    from compile_q4k_host_base_gpu_residual import pack_bitplanes
    from export_cuda_residual_artifact_v2 import pack_row_codes
    from scan_q4k_host_base_gpu_residual import host_gpu_replay

    # Known-answer vectors taken from the reference's unit tests.
    if args.only is None:
        write_kats(quantize_groupwise_q8, pack_2bit_rows, pack_row_codes, compile_radix_table,
                   evaluate_radix_table, encode_signed_base4_states)

    if args.only is None or "artifacts" in args.only:
        make_artifacts()
    if args.only is None or "gguf" in args.only:
        make_gguf()

    for name, (F, D, T, r, outliers, seed, tile_rows, flagged) in CASES.items():
        if args.only is not None and name not in args.only:
            continue
        make_case(name, F, D, T, r, outliers, seed, tile_rows, flagged, torch, compile_radix_table, direct_group_dots,
                  encode_signed_base4_states, evaluate_radix_table, pack_bitplanes, pack_row_codes, host_gpu_replay,
                  projection_from_group_dots, quantize_groupwise_q8)


def make_gguf():
    """``q4k_layer.gguf``: one synthetic FFN layer (d_model 256, d_ff 256) in a GGUF file
    written by the ``gguf`` package (the reference's own GGUF dependency): gate and up
    Q4_K blocks and a Q6_K down, every byte seeded-random except the fp16 block scales
    (|normal| sized so that dequantised weights are about 0.02), plus metadata of several value types. From it, the reference's
    own code writes the expected outputs:

    * ``artifact_q4k_r2/``: scripts/compile_q4k_host_base_gpu_residual.py main() at r = 2
      (bit planes, alpha, beta and manifest, which records sha256 of each stream);
    * ``q4k_down.json``: shape and sha256 of the fp16 bytes that scripts/export_down_fp16.py
      main() writes for the down projection."""
    import hashlib
    import json
    import tempfile

    import compile_q4k_host_base_gpu_residual as comp
    import export_down_fp16 as exdown
    from gguf import GGMLQuantizationType as Q
    from gguf import GGUFWriter
    rng = np.random.default_rng(909)
    F, D = 256, 256

    def blocks(rows, nblk, nbytes, f16_at, scale):
        # block scales of the size real weights have (|w| ~ 0.02 after dequantisation)
        b = rng.integers(0, 256, size=(rows, nblk, nbytes), dtype=np.uint8)
        for off in f16_at:
            v = (np.abs(rng.standard_normal((rows, nblk))) * scale).astype(np.float16)
            b[:, :, off:off + 2] = v.view(np.uint8).reshape(rows, nblk, 2)
        return b.reshape(rows, -1)

    path = HERE / "q4k_layer.gguf"
    w = GGUFWriter(str(path), "llama")
    w.add_uint32("ffnrm.test.u32", 7)
    w.add_array("ffnrm.test.array", [1, 2, 3])
    w.add_string("ffnrm.test.string", "synthetic")
    w.add_float32("ffnrm.test.f32", 0.5)
    w.add_tensor("blk.0.ffn_gate.weight", blocks(F, D // 256, 144, [0, 2], 5e-5), raw_dtype=Q.Q4_K)
    w.add_tensor("blk.0.ffn_up.weight", blocks(F, D // 256, 144, [0, 2], 5e-5), raw_dtype=Q.Q4_K)
    w.add_tensor("blk.0.ffn_down.weight", blocks(D, F // 256, 210, [208], 1e-5), raw_dtype=Q.Q6_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    argv, cwd = sys.argv, os.getcwd()
    with tempfile.TemporaryDirectory() as tmp:
        os.chdir(HERE)  # the manifest records the model path: keep it relative
        try:
            sys.argv = ["compile", path.name, "--layer", "0", "--residual-bits", "2",
                        "--out", str(HERE / "artifact_q4k_r2")]
            comp.main()
            down = Path(tmp) / "down.f16"
            sys.argv = ["export", path.name, "--layer", "0", "--out", str(down)]
            exdown.main()
            raw = down.read_bytes()
        finally:
            sys.argv = argv
            os.chdir(cwd)
    man = HERE / "artifact_q4k_r2" / "manifest.json"
    m = json.loads(man.read_text())
    m["platform"] = "recorded"  # host-specific text, not part of the contract
    man.write_text(json.dumps(m, ensure_ascii=False, indent=2), encoding="utf-8")
    (HERE / "q4k_down.json").write_text(json.dumps(
        {"shape": [D, F], "dtype": "float16", "bytes": len(raw), "sha256": hashlib.sha256(raw).hexdigest()},
        indent=2) + "\n")
    print("gguf ok")


def make_artifacts():
    """Artifact directories written by the reference's own exporters
    (scripts/export_cuda_residual_artifact_v2.py:56-125 and
    scripts/export_radix_table_artifact.py:17-80), run unmodified through their main()
    with the GGUF loader replaced by the synthetic c1-shaped layer (96 rows, d_model
    512; gate from seed 101, up from seed 108): ``artifact_residual_v2/`` and
    ``artifact_table_b2/`` (block size 2)."""
    import tempfile
    import export_cuda_residual_artifact_v2 as exp_res
    import export_radix_table_artifact as exp_tab
    F, D, seed = 96, 512, 101
    layers = {"gate": synth(F, D, 1, 0.0, seed), "up": synth(F, D, 1, 0.0, seed + 7)}

    def fake_loader(model, layer, projection):
        codes, alpha, beta, _, _ = layers[projection]
        return codes.reshape(F, D // 32, 32), alpha, beta, int(codes.size // 2 + alpha.size * 2)

    x = layers["gate"][3][0]
    with tempfile.TemporaryDirectory() as tmp:
        xin = Path(tmp) / "x.f32"
        x.astype("<f4").tofile(xin)
        exp_res.load_q4_projection = fake_loader
        exp_tab.load_q4_projection = fake_loader
        argv, cwd = sys.argv, os.getcwd()
        os.chdir(tmp)  # the manifests record the input path: keep it relative
        try:
            sys.argv = ["export", "synthetic.gguf", "--layer", "23", "--input", xin.name,
                        "--out", str(HERE / "artifact_residual_v2")]
            exp_res.main()
            sys.argv = ["export", "synthetic.gguf", xin.name, "--layer", "23", "--block-size", "2",
                        "--out", str(HERE / "artifact_table_b2")]
            exp_tab.main()
        finally:
            sys.argv = argv
            os.chdir(cwd)
    np.savez_compressed(HERE / "artifact_source.npz", F=F, D=D, x=x,
                        **{f"{p}_{k}": v for p, (c, a, b, _, down) in layers.items()
                           for k, v in (("codes", c), ("alpha", a), ("beta", b))},
                        down=layers["gate"][4])
    print("artifacts ok")


def write_kats(quantize_groupwise_q8, pack_2bit_rows, pack_row_codes, compile_radix_table, evaluate_radix_table,
               encode_signed_base4_states):
    kat_x = np.array([[-1.0, -0.5, 0.0, 1.0, -2.0, 0.0, 1.0, 2.0]], dtype=np.float32)
    kat_z, kat_s = quantize_groupwise_q8(kat_x, group_size=4)
    kat_codes = np.array([[0, 1, 2, 3, 3, 2, 1, 0]], dtype=np.uint8)
    q_hi_kat = (np.arange(2 * 2 * 8, dtype=np.uint8).reshape(2, 2, 8) * 3 + 1) & 3
    z_kat = np.array([[[-128, -65, -1, 0, 1, 63, 64, 127], [127, 64, 63, 1, 0, -1, -65, -128]],
                      [[-17, 5, 12, 31, -44, 88, -99, 106], [13, -26, 39, -52, 65, -78, 91, -104]]], dtype=np.int8)
    table_kat, hs_kat = compile_radix_table(q_hi_kat, block_size=4)
    radix_dots = np.stack([evaluate_radix_table(table_kat, hs_kat, encode_signed_base4_states(t.reshape(-1), 4), 2)
                           for t in z_kat])
    np.savez_compressed(HERE / "kat.npz", quant_x=kat_x, quant_z=kat_z, quant_s=kat_s,
                        pack_codes=kat_codes, pack_bytes=pack_2bit_rows(kat_codes),
                        pack_bytes_v2=pack_row_codes(kat_codes, bits=2),
                        radix_q_hi=q_hi_kat, radix_z=z_kat, radix_dots=radix_dots)


def make_case(name, F, D, T, r, outliers, seed, tile_rows, flagged, torch, compile_radix_table, direct_group_dots,
              encode_signed_base4_states, evaluate_radix_table, pack_bitplanes, pack_row_codes, host_gpu_replay,
              projection_from_group_dots, quantize_groupwise_q8):
    codes, alpha, beta, x, down = synth(F, D, T, outliers, seed)
    z, s = quantize_groupwise_q8(x, group_size=32)
    G = D // 32
    q_hi, q_lo = codes >> r, codes & ((1 << r) - 1)
    grouped = lambda c: c.reshape(F, G, 32)
    p_lo = np.stack([direct_group_dots(grouped(q_lo), z[t]) for t in range(T)]).astype(np.int32)
    p_hi = np.stack([direct_group_dots(grouped(q_hi), z[t]) for t in range(T)]).astype(np.int32)
    p_full = np.stack([direct_group_dots(grouped(codes), z[t]) for t in range(T)]).astype(np.int32)
    # Batched split through the reference's host/GPU replay on dequantised activations.
    xq = torch.from_numpy((z.reshape(T, G, 32).astype(np.float32) * s[:, :, None]).reshape(T, D))
    blocks = D // 256
    host, res, merged = host_gpu_replay(xq, codes.reshape(F, blocks, 256),
                                        alpha.reshape(F, blocks, 8), beta.reshape(F, blocks, 8), r)
    full = np.stack([projection_from_group_dots(direct_group_dots(grouped(codes), z[t]), z[t:t + 1],
                                                s[t:t + 1], alpha, beta, 1) for t in range(T)])
    # Second projection (up) from the same law with a shifted seed.
    codes_u, alpha_u, beta_u, _, _ = synth(F, D, T, 0.0, seed + 7)
    host_u, res_u, merged_u = host_gpu_replay(xq, codes_u.reshape(F, blocks, 256),
                                              alpha_u.reshape(F, blocks, 8), beta_u.reshape(F, blocks, 8), r)
    full_u = np.stack([projection_from_group_dots(direct_group_dots(grouped(codes_u), z[t]), z[t:t + 1],
                                                  s[t:t + 1], alpha_u, beta_u, 1) for t in range(T)])
    g = merged.double().numpy()
    u = merged_u.double().numpy()
    rows = np.zeros(F, dtype=bool)
    for tile in flagged:
        rows[tile * tile_rows:(tile + 1) * tile_rows] = True
    g[:, rows] = full[:, rows]
    u[:, rows] = full_u[:, rows]
    hidden = g / (1.0 + np.exp(-g)) * u  # benchmark_cpu_base_gpu_full_ffn.py:369
    y = hidden @ down.astype(np.float64).T  # :370
    extra = {}
    if r == 2:
        extra["qlo2_rowpacked"] = pack_row_codes(q_lo, bits=2)
        extra["qlo2_rowpacked_up"] = pack_row_codes(codes_u & 3, bits=2)
        if T == 1:
            table, high_sum = compile_radix_table(grouped(q_hi), block_size=4)
            states = encode_signed_base4_states(z[0], block_size=4)
            radix_hi = evaluate_radix_table(table, high_sum, states, blocks_per_group=8)
            extra["radix_p_hi"] = radix_hi
            extra["radix_base"] = projection_from_group_dots(radix_hi, z, s, alpha, beta, code_multiplier=4)
    extra["lo_bitplanes"] = np.frombuffer(pack_bitplanes(q_lo, r), dtype=np.uint8)
    extra["hi_bitplanes"] = np.frombuffer(pack_bitplanes(q_hi, 4 - r), dtype=np.uint8)
    np.savez_compressed(
        HERE / f"{name}.npz", F=F, D=D, T=T, r=r, tile_rows=tile_rows, flagged=np.array(flagged, dtype=np.int32),
        codes=codes, alpha=alpha, beta=beta, codes_up=codes_u, alpha_up=alpha_u, beta_up=beta_u,
        x=x, z=z, s=s, down=down, p_lo=p_lo, p_hi=p_hi, p_full=p_full,
        host=host.numpy(), res=res.numpy(), merged=merged.numpy(), full=full,
        host_up=host_u.numpy(), res_up=res_u.numpy(), merged_up=merged_u.numpy(), full_up=full_u,
        g=g, u=u, h=hidden, y=y, **extra)
    print(name, "ok")


if __name__ == "__main__":
    main()
