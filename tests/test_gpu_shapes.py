"""GPU parity at the shapes the five configurations run (d_model 4096 / 4608 / 8192,
decode T = 8..128, prefill T = 2048, fallback tiles at T = 128), through the C ABI.

Rows (d_ff) are cut to a few row tiles so the CPU oracle stays quick; the kernels tile
over d_ff, so every code path a full layer takes (token tiles, K tiles, scale windows)
runs here. Bars as in test_gpu_parity: integer group
dots bit-exact, residual projections within fp32 rounding of float64 (2e-5 of the row
scale), y within max-abs 1e-2 and relative L2 1e-3 (h reaches the down projection as
fp16 hi + lo, so y in fact stays within 1e-5 relative).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ffnrm_oracle as O

pytestmark = pytest.mark.gpu

Y_MAX_ABS, Y_REL_L2 = 1e-2, 1e-3


def assert_y(y, ref, fp16_output=False):
    """The north-star bar on y: max-abs 1e-2 and relative L2 1e-3. An fp16 output is
    further allowed its own rounding (half an fp16 ulp of the value, 0.016 for |y| in
    [32, 64)), which no fp16 result can avoid."""
    err = np.abs(np.asarray(y, np.float64) - ref)
    allow = Y_MAX_ABS + (0.5 * np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64) if fp16_output else 0.0)
    assert (err <= allow).all(), f"max-abs excess {float((err - allow).max()):.3e}"
    assert rel_l2(y, ref) < Y_REL_L2


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def close_rows(actual, expected, rtol=2e-5):
    scale = np.maximum(np.abs(expected).max(axis=-1, keepdims=True), 1e-30)
    err = np.abs(np.asarray(actual, np.float64) - expected)
    assert (err <= rtol * scale).all(), f"max err/scale {float((err / scale).max()):.3e} > {rtol}"


def dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def flagged_mask(F, tile_rows, fraction, seed):
    n = -(-F // tile_rows)
    k = max(1, int(round(fraction * n))) if fraction > 0 else 0
    mask = np.zeros(n, np.uint8)
    if k:
        mask[np.random.default_rng(seed).choice(n, k, replace=False)] = 1
    return mask


def run_layer(cuda, D, F, T, r, outliers=0.0, tile_rows=256, fraction=0.0, dots=True, seed=0, max_tokens=None):
    import torch
    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh
    L = synth.make_layer(1000 + seed, F, D)
    _, z, s = synth.make_activations(2000 + seed, T, D, outlier_fraction=outliers)
    tiles = flagged_mask(F, tile_rows, fraction, seed) if fraction else None
    ctx = ResidualMesh(D, F, r, 1, max_tokens or T, base_tile_rows=tile_rows)
    ctx.load_layer(0, LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down, L.gate_beta, L.up_beta,
                                keep_fallback=tiles is not None))
    zd, sd = dev(z, cuda), dev(s, cuda)
    g = torch.empty(T, F, device=cuda)
    u = torch.empty_like(g)
    dd = torch.full((2, T, F, D // 32), -7, dtype=torch.int32, device=cuda) if dots else None
    ctx.residual(0, zd, sd, g, u, dd)
    gb = O.host_base_fast(L.gate_codes, L.gate_alpha, L.gate_beta, z, s, r)
    ub = O.host_base_fast(L.up_codes, L.up_alpha, L.up_beta, z, s, r)
    y32 = torch.empty(T, D, device=cuda)
    y16 = torch.empty(T, D, dtype=torch.float16, device=cuda)
    ctx.forward(0, zd, sd, dev(gb.astype(np.float32), cuda), dev(ub.astype(np.float32), cuda),
                fallback_tiles=dev(tiles, cuda) if tiles is not None else None, y32=y32, y16=y16)
    torch.cuda.synchronize()
    ctx.check_device_error()
    out = {"g": g.cpu().numpy(), "u": u.cpu().numpy(), "y32": y32.cpu().numpy(), "y16": y16.float().cpu().numpy(),
           "dots": dd.cpu().numpy() if dots else None}
    ref = O.ffn_forward(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.gate_beta, L.up_beta, L.down, z, s, r,
                        gate_base=gb, up_base=ub, fallback_tiles=tiles, tile_rows=tile_rows, fast=True)
    ctx.close()
    return L, z, s, out, ref


SHAPES = [
    # name, d_model, d_ff rows, tokens, residual bits, outlier fraction
    ("c2_t8", 4096, 1024, 8, 2, 0.0),
    ("c2_t64", 4096, 1024, 64, 2, 0.0),
    ("c3_t16_r1_outliers", 4608, 512, 16, 1, 0.01),
    ("c4_decode_t32", 8192, 512, 32, 2, 0.0),
    ("c5_t128_r3", 4096, 512, 128, 3, 0.0),
    ("c5_t100_r1", 4096, 320, 100, 1, 0.0),
]


@pytest.mark.parametrize("name,D,F,T,r,outliers", SHAPES, ids=[s[0] for s in SHAPES])
def test_config_shape_parity(name, D, F, T, r, outliers, cuda):
    L, z, s, out, ref = run_layer(cuda, D, F, T, r, outliers=outliers, seed=len(name) + T)
    mask = (1 << r) - 1
    np.testing.assert_array_equal(out["dots"][0], O.group_dots(L.gate_codes & mask, z))
    np.testing.assert_array_equal(out["dots"][1], O.group_dots(L.up_codes & mask, z))
    close_rows(out["g"], ref["gate_res"])
    close_rows(out["u"], ref["up_res"])
    assert_y(out["y32"], ref["y"])
    assert_y(out["y16"], ref["y"], fp16_output=True)
    assert rel_l2(out["y32"], ref["y"]) < 1e-5


def test_prefill_t2048_d8192(cuda):
    """Config 4 prefill: 2048 tokens at d_model 8192 (16 token tiles of 128, 64 K tiles,
    8 scale windows)."""
    L, z, s, out, ref = run_layer(cuda, 8192, 512, 2048, 2, dots=False, seed=4)
    close_rows(out["g"], ref["gate_res"])
    close_rows(out["u"], ref["up_res"])
    assert_y(out["y32"], ref["y"])
    assert_y(out["y16"], ref["y"], fp16_output=True)
    assert rel_l2(out["y32"], ref["y"]) < 1e-5


def test_prefill_dots_d8192_t256(cuda):
    """Integer group dots bit-exact over two prefill token tiles at d_model 8192."""
    L, z, s, out, ref = run_layer(cuda, 8192, 192, 256, 2, seed=5)
    np.testing.assert_array_equal(out["dots"][0], O.group_dots(L.gate_codes & 3, z))
    np.testing.assert_array_equal(out["dots"][1], O.group_dots(L.up_codes & 3, z))
    assert rel_l2(out["y32"], ref["y"]) < Y_REL_L2


@pytest.mark.parametrize("r", [1, 2, 3])
@pytest.mark.parametrize("tile_rows", [64, 1024])
def test_fallback_tiles_t128(r, tile_rows, cuda):
    """Config 5: 128 tokens with 5 % of the tiles flagged: flagged rows take the unsplit
    projection (and ignore the base), the others base + residual."""
    L, z, s, out, ref = run_layer(cuda, 4096, 2048, 128, r, tile_rows=tile_rows, fraction=0.05, dots=False,
                                  seed=10 * r + tile_rows % 7)
    assert_y(out["y32"], ref["y"])
    assert_y(out["y16"], ref["y"], fp16_output=True)
    assert rel_l2(out["y32"], ref["y"]) < 1e-5


@pytest.mark.parametrize("T", [3, 8, 40, 128])
def test_fallback_rows_unsplit_on_tensor_cores(T, cuda):
    """Every tile flagged: the residual call returns the exact unsplit projections."""
    import torch
    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh
    D, F, r = 1024, 200, 2
    L = synth.make_layer(70 + T, F, D)
    _, z, s = synth.make_activations(71 + T, T, D)
    ctx = ResidualMesh(D, F, r, 1, T, base_tile_rows=64)
    ctx.load_layer(0, LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down, L.gate_beta, L.up_beta,
                                keep_fallback=True))
    g = torch.empty(T, F, device=cuda)
    u = torch.empty_like(g)
    ctx.residual(0, dev(z, cuda), dev(s, cuda), g, u, fallback_tiles=dev(np.ones(4, np.uint8), cuda))
    torch.cuda.synchronize()
    ctx.check_device_error()
    close_rows(g.cpu().numpy(), O.full_projection_fast(L.gate_codes, L.gate_alpha, L.gate_beta, z, s))
    close_rows(u.cpu().numpy(), O.full_projection_fast(L.up_codes, L.up_alpha, L.up_beta, z, s))
    ctx.close()


@pytest.mark.parametrize("kernel", ["bytes", "mma"])
def test_packed_records_match_other_residual_kernels(kernel, cuda, monkeypatch):
    """The packed-record tcgen05 kernel, the byte-code tcgen05 kernel and the mma.sync
    tiles give the same integer dots on the same layer (c2 shape, 64 tokens)."""
    import torch
    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh
    D, F, T, r = 4096, 256, 64, 2
    L = synth.make_layer(90, F, D)
    _, z, s = synth.make_activations(91, T, D)
    res = {}
    for k in ("packed", kernel):
        monkeypatch.setenv("FFNRM_RESIDUAL_KERNEL", k)
        ctx = ResidualMesh(D, F, r, 1, T)
        ctx.load_layer(0, LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down))
        g = torch.empty(T, F, device=cuda)
        u = torch.empty_like(g)
        dots = torch.empty((2, T, F, D // 32), dtype=torch.int32, device=cuda)
        ctx.residual(0, dev(z, cuda), dev(s, cuda), g, u, dots)
        torch.cuda.synchronize()
        ctx.check_device_error()
        res[k] = (dots.cpu().numpy(), g.cpu().numpy())
        ctx.close()
    np.testing.assert_array_equal(res["packed"][0], res[kernel][0])
    close_rows(res["packed"][1], res[kernel][1].astype(np.float64))
