"""GPU parity: the CUDA path through the C ABI against the reference-generated
golden fixtures and the CPU oracle.

Bars: integer group dots bit-exact; residual / merged projections within fp32
rounding of a float64 reference (rtol 1e-5 of the row scale); the post-down
output within max-abs 1e-2 and relative L2 1e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import ffnrm_oracle as O

pytestmark = pytest.mark.gpu

CASES = ["c1_decode_t1_r2", "c2_decode_t8_r2", "c3_decode_t16_r1_outliers", "c4_decode_t32_r2",
         "c4_d8192_t16_r2_fallback", "c5_t5_r3_fallback", "c5_t3_r2_fallback"]
Y_MAX_ABS, Y_REL_L2 = 1e-2, 1e-3


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def close_rows(actual, expected, rtol=1e-5):
    """fp32 accumulation vs float64: error bounded relative to the row's magnitude scale."""
    scale = np.maximum(np.abs(expected).max(axis=-1, keepdims=True), 1e-30)
    err = np.abs(np.asarray(actual, np.float64) - expected)
    bound = np.broadcast_to(rtol * scale, err.shape)
    assert (err <= bound).all(), f"max err/scale {float((err / scale).max()):.3e} > {rtol}"


def make_ctx(c, tokens=None, keep_fallback=True):
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh
    F, D, T, r = int(c["F"]), int(c["D"]), int(c["T"]), int(c["r"])
    ctx = ResidualMesh(D, F, r, 1, tokens or T, base_tile_rows=int(c["tile_rows"]))
    ctx.load_layer(0, LayerSpec(c["codes"], c["codes_up"], c["alpha"], c["alpha_up"], c["down"],
                                c["beta"], c["beta_up"], keep_fallback=keep_fallback))
    return ctx


def dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("name", CASES)
def test_residual_group_dots_bit_exact(name, cuda):
    import torch
    c = load(name)
    F, D, T = int(c["F"]), int(c["D"]), int(c["T"])
    ctx = make_ctx(c)
    g = torch.empty(T, F, device=cuda)
    u = torch.empty_like(g)
    dots = torch.full((2, T, F, D // 32), -7, dtype=torch.int32, device=cuda)
    ctx.residual(0, dev(c["z"], cuda), dev(c["s"], cuda), g, u, dots)
    torch.cuda.synchronize()
    d = dots.cpu().numpy()
    np.testing.assert_array_equal(d[0], c["p_lo"])
    r = int(c["r"])
    np.testing.assert_array_equal(d[1], O.group_dots(c["codes_up"] & ((1 << r) - 1), c["z"]))
    # merged integer accumulator 2^r*P_hi + P_lo equals the unsplit dot
    np.testing.assert_array_equal((c["p_hi"].astype(np.int64) << r) + d[0], c["p_full"])
    close_rows(g.cpu().numpy(), c["res"].astype(np.float64), rtol=2e-5)
    close_rows(u.cpu().numpy(), c["res_up"].astype(np.float64), rtol=2e-5)
    ctx.close()


@pytest.mark.parametrize("name", CASES)
def test_ffn_forward_device_base(name, cuda):
    import torch
    c = load(name)
    F, D, T = int(c["F"]), int(c["D"]), int(c["T"])
    ctx = make_ctx(c)
    n_tiles = -(-F // int(c["tile_rows"]))
    tiles = np.zeros(n_tiles, np.uint8)
    tiles[c["flagged"]] = 1
    y32 = torch.empty(T, D, device=cuda)
    y16 = torch.empty(T, D, dtype=torch.float16, device=cuda)
    ctx.forward(0, dev(c["z"], cuda), dev(c["s"], cuda), dev(c["host"].astype(np.float32), cuda),
                dev(c["host_up"].astype(np.float32), cuda), fallback_tiles=dev(tiles, cuda) if tiles.any() else None,
                y32=y32, y16=y16)
    torch.cuda.synchronize()
    for y in (y32.cpu().numpy(), y16.float().cpu().numpy()):
        assert np.abs(y - c["y"]).max() < Y_MAX_ABS
        assert rel_l2(y, c["y"]) < Y_REL_L2
    assert rel_l2(y32.cpu().numpy(), c["y"]) < 1e-5
    ctx.close()


@pytest.mark.parametrize("name", ["c2_decode_t8_r2", "c5_t5_r3_fallback"])
def test_ffn_forward_host_streamed(name, cuda):
    c = load(name)
    F, D, T = int(c["F"]), int(c["D"]), int(c["T"])
    ctx = make_ctx(c)
    tiles = np.zeros(-(-F // int(c["tile_rows"])), np.uint8)
    tiles[c["flagged"]] = 1
    import torch
    y16 = np.zeros((T, D), np.float16)
    gb = np.ascontiguousarray(c["host"], np.float32)
    ub = np.ascontiguousarray(c["host_up"], np.float32)
    for _ in range(3):  # both double-buffer slots, then the first again
        y16[:] = 0
        ctx.forward_host(0, np.ascontiguousarray(c["z"]), np.ascontiguousarray(c["s"]), gb, ub, y16.view(np.uint16),
                         fallback_tiles=tiles if tiles.any() else None)
        torch.cuda.synchronize()
        assert np.abs(y16.astype(np.float64) - c["y"]).max() < Y_MAX_ABS
        assert rel_l2(y16, c["y"]) < Y_REL_L2
    ctx.close()


def test_fallback_rows_are_unsplit_projection(cuda):
    """All tiles flagged: the residual call returns the exact unsplit projection."""
    import torch
    c = load("c5_t5_r3_fallback")
    F, D, T = int(c["F"]), int(c["D"]), int(c["T"])
    ctx = make_ctx(c)
    tiles = np.ones(-(-F // int(c["tile_rows"])), np.uint8)
    g = torch.empty(T, F, device=cuda)
    u = torch.empty_like(g)
    ctx.residual(0, dev(c["z"], cuda), dev(c["s"], cuda), g, u, fallback_tiles=dev(tiles, cuda))
    torch.cuda.synchronize()
    close_rows(g.cpu().numpy(), c["full"], rtol=2e-5)
    close_rows(u.cpu().numpy(), c["full_up"], rtol=2e-5)
    ctx.close()


@pytest.mark.parametrize("fmt", ["qlo2", "bitplanes"])
def test_artifact_code_formats(fmt, cuda):
    """Codes given in the reference's on-disk layouts give the same dots and output."""
    import torch
    from ffn_residual_mesh_b200 import _native as N
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh
    name = "c2_decode_t8_r2" if fmt == "qlo2" else "c5_t5_r3_fallback"
    c = load(name)
    F, D, T, r = int(c["F"]), int(c["D"]), int(c["T"]), int(c["r"])
    if fmt == "qlo2":
        spec = LayerSpec(c["qlo2_rowpacked"], c["qlo2_rowpacked_up"], c["alpha"], c["alpha_up"], c["down"],
                         codes_format=N.CODES_QLO2_ROWPACKED)
    else:
        up_lo = np.frombuffer(O.pack_bitplanes(c["codes_up"] & ((1 << r) - 1), r), np.uint8)
        up_hi = np.frombuffer(O.pack_bitplanes(c["codes_up"] >> r, 4 - r), np.uint8)
        spec = LayerSpec(c["lo_bitplanes"], up_lo, c["alpha"], c["alpha_up"], c["down"], c["beta"], c["beta_up"],
                         codes_format=N.CODES_BITPLANES, gate_high=c["hi_bitplanes"], up_high=up_hi)
    ctx = ResidualMesh(D, F, r, 1, T, base_tile_rows=int(c["tile_rows"]))
    ctx.load_layer(0, spec)
    g = torch.empty(T, F, device=cuda)
    u = torch.empty_like(g)
    dots = torch.empty((2, T, F, D // 32), dtype=torch.int32, device=cuda)
    ctx.residual(0, dev(c["z"], cuda), dev(c["s"], cuda), g, u, dots)
    y16 = torch.empty(T, D, dtype=torch.float16, device=cuda)
    tiles = np.zeros(-(-F // int(c["tile_rows"])), np.uint8)
    tiles[c["flagged"]] = 1
    ctx.forward(0, dev(c["z"], cuda), dev(c["s"], cuda), dev(c["host"].astype(np.float32), cuda),
                dev(c["host_up"].astype(np.float32), cuda),
                fallback_tiles=dev(tiles, cuda) if tiles.any() else None, y16=y16)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dots.cpu().numpy()[0], c["p_lo"])
    assert rel_l2(y16.float().cpu().numpy(), c["y"]) < Y_REL_L2
    ctx.close()


@pytest.mark.parametrize("T", [1, 2, 3, 4, 5, 9, 17])
def test_token_chunking_ragged(T, cuda):
    """Token counts that are not multiples of the kernel's token chunk."""
    import torch
    c = load("c4_decode_t32_r2")
    F, D = int(c["F"]), int(c["D"])
    ctx = make_ctx(c, tokens=32)
    z, s = c["z"][:T], c["s"][:T]
    g = torch.empty(T, F, device=cuda)
    u = torch.empty_like(g)
    dots = torch.empty((2, T, F, D // 32), dtype=torch.int32, device=cuda)
    ctx.residual(0, dev(z, cuda), dev(s, cuda), g, u, dots)
    y32 = torch.empty(T, D, device=cuda)
    ctx.forward(0, dev(z, cuda), dev(s, cuda), dev(c["host"][:T].astype(np.float32), cuda),
                dev(c["host_up"][:T].astype(np.float32), cuda), y32=y32)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dots.cpu().numpy()[0], c["p_lo"][:T])
    assert rel_l2(y32.cpu().numpy(), c["y"][:T]) < 1e-5
    ctx.close()


def test_errors_are_reported(cuda):
    import torch
    from ffn_residual_mesh_b200.engine import ResidualMesh
    c = load("c1_decode_t1_r2")
    with pytest.raises(ValueError):
        ResidualMesh(100, 64, 2, 1, 1)          # d_model not a multiple of 256
    with pytest.raises(ValueError):
        ResidualMesh(256, 64, 4, 1, 1)          # residual bits out of range
    ctx = make_ctx(c, keep_fallback=False)
    F, D = int(c["F"]), int(c["D"])
    z = dev(c["z"], cuda)
    s = dev(c["s"], cuda)
    g = torch.empty(1, F, device=cuda)
    with pytest.raises(ValueError):
        ctx.residual(0, z, s, g, g[:, :-1])
    with pytest.raises(RuntimeError, match="not loaded"):
        ResidualMesh(D, F, 2, 2, 1).residual(1, z, s, g, torch.empty_like(g))
    with pytest.raises(RuntimeError, match="fallback"):
        ctx.residual(0, z, s, g, torch.empty_like(g), fallback_tiles=dev(np.ones(3, np.uint8), cuda))
    ctx.close()


def test_full_layer_shape_property(cuda):
    """Full config-1 layer shape (d_model 2048, d_ff 5632): integer dots of a row
    sample equal the oracle, and y equals the oracle chain at full size."""
    import torch
    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh
    D, F, T, r = 2048, 5632, 3, 2
    L = synth.make_layer(11, F, D)
    _, z, s = synth.make_activations(12, T, D)
    ctx = ResidualMesh(D, F, r, 1, T)
    ctx.load_layer(0, LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down, L.gate_beta, L.up_beta))
    g = torch.empty(T, F, device=cuda)
    u = torch.empty_like(g)
    dots = torch.empty((2, T, F, D // 32), dtype=torch.int32, device=cuda)
    ctx.residual(0, dev(z, cuda), dev(s, cuda), g, u, dots)
    gb = O.host_base(L.gate_codes, L.gate_alpha, L.gate_beta, z, s, r)
    ub = O.host_base(L.up_codes, L.up_alpha, L.up_beta, z, s, r)
    y32 = torch.empty(T, D, device=cuda)
    ctx.forward(0, dev(z, cuda), dev(s, cuda), dev(gb.astype(np.float32), cuda), dev(ub.astype(np.float32), cuda),
                y32=y32)
    torch.cuda.synchronize()
    rows = np.random.default_rng(0).choice(F, 256, replace=False)
    np.testing.assert_array_equal(dots.cpu().numpy()[0][:, rows], O.group_dots(L.gate_codes[rows] & 3, z))
    ref = O.ffn_forward(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.gate_beta, L.up_beta, L.down, z, s, r,
                        gate_base=gb, up_base=ub)
    assert rel_l2(y32.cpu().numpy(), ref["y"]) < 1e-5
    ctx.close()


@pytest.mark.parametrize("T,F,r", [(70, 1000, 2), (40, 333, 1), (33, 200, 3)])
def test_multi_chunk_batches_ragged_rows(T, F, r, cuda):
    """Batches spanning several token tiles of both tensor-core kernels, with a
    d_ff that is not a multiple of the 32-row blocks."""
    import torch
    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh
    D = 1024
    L = synth.make_layer(21 + r, F, D)
    _, z, s = synth.make_activations(22 + T, T, D)
    ctx = ResidualMesh(D, F, r, 1, T, base_tile_rows=64)
    ctx.load_layer(0, LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down, L.gate_beta, L.up_beta,
                                keep_fallback=True))
    g = torch.empty(T, F, device=cuda)
    u = torch.empty_like(g)
    dots = torch.empty((2, T, F, D // 32), dtype=torch.int32, device=cuda)
    ctx.residual(0, dev(z, cuda), dev(s, cuda), g, u, dots)
    gb = O.host_base(L.gate_codes, L.gate_alpha, L.gate_beta, z, s, r)
    ub = O.host_base(L.up_codes, L.up_alpha, L.up_beta, z, s, r)
    tiles = np.zeros(-(-F // 64), np.uint8)
    tiles[1] = 1
    y32 = torch.empty(T, D, device=cuda)
    ctx.forward(0, dev(z, cuda), dev(s, cuda), dev(gb.astype(np.float32), cuda), dev(ub.astype(np.float32), cuda),
                fallback_tiles=dev(tiles, cuda), y32=y32)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dots.cpu().numpy()[0], O.group_dots(L.gate_codes & ((1 << r) - 1), z))
    np.testing.assert_array_equal(dots.cpu().numpy()[1], O.group_dots(L.up_codes & ((1 << r) - 1), z))
    close_rows(g.cpu().numpy(), O.residual(L.gate_codes, L.gate_alpha, z, s, r), rtol=2e-5)
    ref = O.ffn_forward(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.gate_beta, L.up_beta, L.down, z, s, r,
                        gate_base=gb, up_base=ub, fallback_tiles=tiles, tile_rows=64)
    assert rel_l2(y32.cpu().numpy(), ref["y"]) < 1e-5
    assert np.abs(y32.cpu().numpy() - ref["y"]).max() < Y_MAX_ABS
    ctx.close()


def test_empty_batch_is_a_no_op(cuda):
    import torch
    c = load("c1_decode_t1_r2")
    F, D = int(c["F"]), int(c["D"])
    ctx = make_ctx(c)
    z = torch.empty(0, D, dtype=torch.int8, device=cuda)
    s = torch.empty(0, D // 32, device=cuda)
    e = torch.empty(0, F, device=cuda)
    ctx.residual(0, z, s, e, e)
    ctx.forward(0, z, s, e, e, y32=torch.empty(0, D, device=cuda))
    torch.cuda.synchronize()
    ctx.close()


def test_graph_capture_of_host_streamed_calls(cuda):
    """A captured sequence of host-streamed forwards (copy-stream fork/join inside the
    capture) replays to the same output; host buffers refilled in place are picked up."""
    import torch
    from ffn_residual_mesh_b200.graphs import StepGraph
    c = load("c2_decode_t8_r2")
    F, D, T = int(c["F"]), int(c["D"]), int(c["T"])
    ctx = make_ctx(c)
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
    z, s = pin(c["z"]), pin(c["s"])
    gb, ub = pin(c["host"].astype(np.float32)), pin(c["host_up"].astype(np.float32))
    ys = [torch.zeros(T, D, dtype=torch.float16).pin_memory() for _ in range(3)]

    def step():
        for y in ys:
            ctx.forward_host(0, z, s, gb, ub, y)

    g = StepGraph(step)
    for y in ys:
        y.zero_()
    g.replay()
    torch.cuda.synchronize()
    for y in ys:
        assert rel_l2(y.float().numpy(), c["y"]) < Y_REL_L2
    gb.zero_()   # a changed host input is read by the next replay
    ub.zero_()
    g.replay()
    torch.cuda.synchronize()
    ref0 = O.ffn_forward(c["codes"], c["codes_up"], c["alpha"], c["alpha_up"], c["beta"], c["beta_up"], c["down"],
                         c["z"], c["s"], int(c["r"]), gate_base=np.zeros((T, F)), up_base=np.zeros((T, F)))["y"]
    assert rel_l2(ys[0].float().numpy(), ref0) < Y_REL_L2
    ctx.check_device_error()
    g.close()
    ctx.close()


def test_eager_call_after_capture(cuda):
    """Eager host-streamed calls keep working after a captured sequence."""
    import torch
    from ffn_residual_mesh_b200.graphs import StepGraph
    c = load("c2_decode_t8_r2")
    T, D = int(c["T"]), int(c["D"])
    ctx = make_ctx(c)
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
    z, s = pin(c["z"]), pin(c["s"])
    gb, ub = pin(c["host"].astype(np.float32)), pin(c["host_up"].astype(np.float32))
    y = torch.zeros(T, D, dtype=torch.float16).pin_memory()
    g = StepGraph(lambda: ctx.forward_host(0, z, s, gb, ub, y))
    g.replay()
    for _ in range(3):
        y.zero_()
        ctx.forward_host(0, z, s, gb, ub, y)
        torch.cuda.synchronize()
        assert rel_l2(y.float().numpy(), c["y"]) < Y_REL_L2
    g.replay()
    torch.cuda.synchronize()
    g.close()
    ctx.close()


@pytest.mark.parametrize("T,F,r,half_alpha", [(5, 200, 2, True), (16, 64, 1, True), (17, 1000, 3, False),
                                              (64, 1000, 2, True), (100, 130, 2, False), (33, 333, 1, False)])
def test_tensor_core_residual_tiles(T, F, r, half_alpha, cuda, monkeypatch):
    """Batches of 3+ tokens run on the tcgen05 kind::i8 tiles over the packed records
    (64 gate + 64 up rows x 16..128 tokens): group dots bit-exact against the oracle
    and against the mma.sync tiles, residuals and the forward output within tolerance,
    for r = 1/2/3, fp16-exact and f32 alpha, ragged d_ff and partial token tiles."""
    import torch
    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh
    D = 1024
    L = synth.make_layer(40 + T, F, D)
    if not half_alpha:  # not representable in fp16: the kernels read f32 scales
        L.gate_alpha[:] = L.gate_alpha * np.float32(1 + 2 ** -20)
        L.up_alpha[:] = L.up_alpha * np.float32(1 + 2 ** -20)
    _, z, s = synth.make_activations(41 + T, T, D)
    gb = O.host_base(L.gate_codes, L.gate_alpha, L.gate_beta, z, s, r)
    ub = O.host_base(L.up_codes, L.up_alpha, L.up_beta, z, s, r)
    spec = LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down, L.gate_beta, L.up_beta)
    results = {}
    for legacy in ("packed", "mma"):
        monkeypatch.setenv("FFNRM_RESIDUAL_KERNEL", legacy)
        ctx = ResidualMesh(D, F, r, 1, T)
        ctx.load_layer(0, spec)
        g = torch.empty(T, F, device=cuda)
        u = torch.empty_like(g)
        dots = torch.full((2, T, F, D // 32), -7, dtype=torch.int32, device=cuda)
        ctx.residual(0, dev(z, cuda), dev(s, cuda), g, u, dots)
        y32 = torch.empty(T, D, device=cuda)
        ctx.forward(0, dev(z, cuda), dev(s, cuda), dev(gb.astype(np.float32), cuda), dev(ub.astype(np.float32), cuda),
                    y32=y32)
        torch.cuda.synchronize()
        ctx.check_device_error()
        results[legacy] = (dots.cpu().numpy(), g.cpu().numpy(), u.cpu().numpy(), y32.cpu().numpy())
        ctx.close()
    dots, g, u, y = results["packed"]
    mask = (1 << r) - 1
    np.testing.assert_array_equal(dots[0], O.group_dots(L.gate_codes & mask, z))
    np.testing.assert_array_equal(dots[1], O.group_dots(L.up_codes & mask, z))
    np.testing.assert_array_equal(dots, results["mma"][0])
    close_rows(g, O.residual(L.gate_codes, L.gate_alpha, z, s, r), rtol=2e-5)
    close_rows(u, O.residual(L.up_codes, L.up_alpha, z, s, r), rtol=2e-5)
    ref = O.ffn_forward(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.gate_beta, L.up_beta, L.down, z, s, r,
                        gate_base=gb, up_base=ub)
    assert rel_l2(y, ref["y"]) < 1e-5
    assert np.abs(y - ref["y"]).max() < Y_MAX_ABS
    assert rel_l2(y, results["mma"][3]) < 1e-5
