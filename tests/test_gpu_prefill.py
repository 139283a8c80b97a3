"""GPU parity of the prefill residual (tokens on the tensor-core M axis, 64 rows of both
projections on N, 2-bit records widened to fp16 in shared memory), through the C ABI.

The kernel takes batches of at least ``FFNRM_PREFILL_TOKENS`` tokens without fallback
tiles; each test sets that threshold (below the batch where a smaller batch keeps the
oracle quick). The dots are exact integers computed in fp16 x fp16 -> fp32 (activations
and low codes exact in fp16), checked bit for bit. Cases: residual bits 1/2/3 (plane and pair records), ragged d_ff (a
missing second 64-row tile, rows past d_ff inside a tile), ragged token counts, f32
alphas (not fp16-exact), residual mode (g/u out) and forward mode (h -> down), two token
tiles with the integer dots checked bit-exact against the oracle's ``group_dots``
(scripts/benchmark_exact_radix_split_pipeline.py:162-164).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ffnrm_oracle as O

pytestmark = pytest.mark.gpu

Y_MAX_ABS, Y_REL_L2 = 1e-2, 1e-3


def close_rows(actual, expected, rtol=2e-5):
    scale = np.maximum(np.abs(expected).max(axis=-1, keepdims=True), 1e-30)
    err = np.abs(np.asarray(actual, np.float64) - expected)
    assert (err <= rtol * scale).all(), f"max err/scale {float((err / scale).max()):.3e} > {rtol}"


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def run(cuda, monkeypatch, D, F, T, r, seed, f32_alpha=False, threshold=None):
    import torch
    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh
    if threshold is not None:
        monkeypatch.setenv("FFNRM_PREFILL_TOKENS", str(threshold))
    L = synth.make_layer(3000 + seed, F, D)
    if f32_alpha:
        # scales that fp16 cannot hold exactly: the layer keeps f32 alphas on the device
        rng = np.random.default_rng(seed)
        L.gate_alpha = (L.gate_alpha * (1 + rng.uniform(1e-4, 2e-4, L.gate_alpha.shape))).astype(np.float32)
        L.up_alpha = (L.up_alpha * (1 + rng.uniform(1e-4, 2e-4, L.up_alpha.shape))).astype(np.float32)
    _, z, s = synth.make_activations(4000 + seed, T, D)
    ctx = ResidualMesh(D, F, r, 1, T)
    ctx.load_layer(0, LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down, L.gate_beta, L.up_beta))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    zd, sd = dev(z), dev(s)
    g = torch.empty(T, F, device=cuda)
    u = torch.empty_like(g)
    dots = torch.full((2, T, F, D // 32), -7, dtype=torch.int32, device=cuda)
    ctx.residual(0, zd, sd, g, u, dots)
    g2 = torch.empty_like(g)
    u2 = torch.empty_like(g)
    ctx.residual(0, zd, sd, g2, u2)  # the same kernel without the dot output
    gb = O.host_base_fast(L.gate_codes, L.gate_alpha, L.gate_beta, z, s, r)
    ub = O.host_base_fast(L.up_codes, L.up_alpha, L.up_beta, z, s, r)
    y32 = torch.empty(T, D, device=cuda)
    ctx.forward(0, zd, sd, dev(gb.astype(np.float32)), dev(ub.astype(np.float32)), y32=y32)
    torch.cuda.synchronize()
    ctx.check_device_error()
    out = {k: v.cpu().numpy() for k, v in (("g", g), ("u", u), ("g2", g2), ("u2", u2), ("dots", dots), ("y", y32))}
    ref = O.ffn_forward(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.gate_beta, L.up_beta, L.down, z, s, r,
                        gate_base=gb, up_base=ub, fast=True)
    ctx.close()
    return L, z, out, ref


CASES = [
    # name, d_model, d_ff, tokens, residual bits, f32 alpha, threshold
    ("r2_two_token_tiles", 2048, 256, 256, 2, False, 256),
    ("r1_planes", 1024, 256, 200, 1, False, 128),
    ("r3_pair_and_plane", 1024, 256, 200, 3, False, 128),
    ("ragged_dff_half_tile", 1024, 130, 160, 2, False, 128),
    ("ragged_dff_inside_tile", 1024, 200, 300, 2, False, 128),
    ("f32_alpha", 1024, 192, 140, 2, True, 128),
]


@pytest.mark.parametrize("name,D,F,T,r,f32_alpha,threshold", CASES, ids=[c[0] for c in CASES])
def test_prefill_parity(name, D, F, T, r, f32_alpha, threshold, cuda, monkeypatch):
    L, z, out, ref = run(cuda, monkeypatch, D, F, T, r, seed=len(name), f32_alpha=f32_alpha, threshold=threshold)
    mask = (1 << r) - 1
    np.testing.assert_array_equal(out["dots"][0], O.group_dots(L.gate_codes & mask, z))
    np.testing.assert_array_equal(out["dots"][1], O.group_dots(L.up_codes & mask, z))
    close_rows(out["g"], ref["gate_res"])
    close_rows(out["u"], ref["up_res"])
    np.testing.assert_array_equal(out["g2"], out["g"])
    np.testing.assert_array_equal(out["u2"], out["u"])
    err = np.abs(out["y"] - ref["y"])
    assert err.max() <= Y_MAX_ABS
    assert rel_l2(out["y"], ref["y"]) < 1e-5


def test_prefill_matches_token_tile_kernels(cuda, monkeypatch):
    """The same 300-token batch through the prefill kernel and through the row-on-M
    kernels (prefill disabled): bit-identical dots, residuals within fp32 rounding."""
    import torch
    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh
    D, F, T = 2048, 320, 300
    L = synth.make_layer(77, F, D)
    _, z, s = synth.make_activations(78, T, D)
    res = {}
    for thr in ("256", "0"):
        monkeypatch.setenv("FFNRM_PREFILL_TOKENS", thr)
        ctx = ResidualMesh(D, F, 2, 1, T)
        ctx.load_layer(0, LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down))
        zd, sd = torch.from_numpy(z).to(cuda), torch.from_numpy(s).to(cuda)
        g = torch.empty(T, F, device=cuda)
        u = torch.empty_like(g)
        dots = torch.zeros((2, T, F, D // 32), dtype=torch.int32, device=cuda)
        ctx.residual(0, zd, sd, g, u, dots)
        torch.cuda.synchronize()
        ctx.check_device_error()
        res[thr] = (dots.cpu().numpy(), g.cpu().numpy().astype(np.float64))
        ctx.close()
    np.testing.assert_array_equal(res["256"][0], res["0"][0])
    close_rows(res["256"][1], res["0"][1])
