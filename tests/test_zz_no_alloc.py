"""The allocation-free down projection against the context-based forward (GPU).

`ffnrm_down_project_noalloc` serves callers that cannot allocate device memory: code
running while a CUDA graph is captured, or behind an allocator that forbids cudaMalloc on
the serving path. It reduces its split-K partial sums inside a thread-block cluster, so its
only scratch is one status word in a file-scope device variable of the library. These
tests call it through the C ABI, twice in a row, and check its output against the existing
entry point `ffnrm_ffn_forward` on the same layer and inputs, within the tolerances of the
other parity tests - with a status word of the caller, and with status = NULL read back
through `ffnrm_noalloc_status`. One test captures the call into a CUDA graph in global
capture mode, where any allocation would fail the capture, and replays it. The file is
collected last so a first failure here leaves every other test already run; it also passes
alone in a fresh process (`pytest tests/test_zz_no_alloc.py -m gpu`).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import ffnrm_oracle as O

pytestmark = pytest.mark.gpu

Y_MAX_ABS, Y_REL_L2 = 1e-2, 1e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def setup_layer(T, cuda):
    """One layer: the reference output of the context path and the padded device inputs
    (down, h as fp16 hi + lo) of the allocation-free call."""
    import torch

    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh

    D, F, r = 1024, 1000, 2
    L = synth.make_layer(31, F, D)
    _, z, s = synth.make_activations(32 + T, T, D)
    gb = O.host_base(L.gate_codes, L.gate_alpha, L.gate_beta, z, s, r)
    ub = O.host_base(L.up_codes, L.up_alpha, L.up_beta, z, s, r)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    ctx = ResidualMesh(D, F, r, 1, T)
    ctx.load_layer(0, LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down, L.gate_beta, L.up_beta))
    y_ref = torch.empty(T, D, device=cuda)
    ctx.forward(0, dev(z), dev(s), dev(gb.astype(np.float32)), dev(ub.astype(np.float32)), y32=y_ref)
    torch.cuda.synchronize()
    ctx.close()
    ref = O.ffn_forward(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.gate_beta, L.up_beta, L.down, z, s, r,
                        gate_base=gb, up_base=ub)
    h = ref["h"].astype(np.float32)
    h_hi = h.astype(np.float16)
    h_lo = (h - h_hi.astype(np.float32)).astype(np.float16)
    ld = (F + 7) // 8 * 8
    pad = lambda a: np.pad(a, ((0, 0), (0, ld - a.shape[1])))
    return D, F, ld, y_ref.cpu().numpy(), dev(pad(L.down)), dev(pad(h_hi)), dev(pad(h_lo))


def call(lib, D, F, ld, T, down, hi, lo, y32, y16, status):
    import torch
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.ffnrm_down_project_noalloc(down.data_ptr(), ld, hi.data_ptr(), lo.data_ptr(), ld, D, F, T,
                                          y32.data_ptr(), y16.data_ptr(),
                                          status.data_ptr() if status is not None else None, stream)


def check(got32, got16, want):
    assert np.isfinite(got32).all()
    assert rel_l2(got32, want) < 1e-5
    assert np.abs(got32 - want).max() < Y_MAX_ABS
    assert rel_l2(got16, want) < Y_REL_L2


@pytest.mark.parametrize("own_status", [True, False], ids=["own-status", "default-status"])
@pytest.mark.parametrize("T", [5, 40, 200])
def test_noalloc_down_matches_forward(T, own_status, cuda):
    import torch

    from ffn_residual_mesh_b200 import _native as N
    D, F, ld, want, down, hi, lo = setup_layer(T, cuda)
    lib = N.lib()
    for call_no in range(2):
        y32 = torch.full((T, D), float("nan"), device=cuda)
        y16 = torch.zeros(T, D, dtype=torch.float16, device=cuda)
        status = torch.full((1,), -1, dtype=torch.int32, device=cuda) if own_status else None
        N.check(call(lib, D, F, ld, T, down, hi, lo, y32, y16, status))
        torch.cuda.synchronize()
        if own_status:
            assert int(status.item()) == 0, f"call {call_no}: a pipeline wait gave up"
        else:
            code = ctypes.c_int32(-1)
            N.check(lib.ffnrm_noalloc_status(ctypes.byref(code), None))
            assert code.value == 0, f"call {call_no}: a pipeline wait gave up"
        check(y32.cpu().numpy(), y16.float().cpu().numpy(), want)


def test_noalloc_down_in_captured_graph(cuda):
    """After one eager call (the device address lookup), the call captures into a CUDA
    graph in global capture mode - where any allocation would fail the capture - and the
    replay gives the same output."""
    import torch

    from ffn_residual_mesh_b200 import _native as N
    T = 40
    D, F, ld, want, down, hi, lo = setup_layer(T, cuda)
    lib = N.lib()
    y32 = torch.full((T, D), float("nan"), device=cuda)
    y16 = torch.zeros(T, D, dtype=torch.float16, device=cuda)
    N.check(call(lib, D, F, ld, T, down, hi, lo, y32, y16, None))
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="global"):
        N.check(call(lib, D, F, ld, T, down, hi, lo, y32, y16, None))
    for _ in range(2):
        y32.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        check(y32.cpu().numpy(), y16.float().cpu().numpy(), want)
    code = ctypes.c_int32(-1)
    N.check(lib.ffnrm_noalloc_status(ctypes.byref(code), None))
    assert code.value == 0
    g.reset()


def test_noalloc_rejects_sizes_beyond_its_tile_grid(cuda):
    import torch

    from ffn_residual_mesh_b200 import _native as N
    lib = N.lib()
    buf = torch.zeros(1024 * 1024, dtype=torch.float16, device=cuda)
    y = torch.zeros(300 * 1024, device=cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    with pytest.raises(ValueError, match="tokens"):
        N.check(lib.ffnrm_down_project_noalloc(buf.data_ptr(), 1024, buf.data_ptr(), buf.data_ptr(), 1024, 1024,
                                               1024, 300, y.data_ptr(), None, None, stream))
    with pytest.raises(ValueError, match="d_model"):
        N.check(lib.ffnrm_down_project_noalloc(buf.data_ptr(), 1024, buf.data_ptr(), buf.data_ptr(), 1024, 100,
                                               1024, 4, y.data_ptr(), None, None, stream))
