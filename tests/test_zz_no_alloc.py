"""The allocation-free down projection against the context-based forward (GPU).

`ffnrm_down_project_noalloc` serves callers that cannot allocate device memory (for
example code running while a CUDA graph is captured, or behind an allocator that forbids
cudaMalloc on the serving path): its split-K scratch lives in fixed device arrays of the
library. This test calls it through the C ABI, twice in a row, and checks its output
against the existing entry point `ffnrm_ffn_forward` on the same layer and inputs, within
the tolerances of the other parity tests. It also runs alone in a fresh process.
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


@pytest.mark.parametrize("T", [5, 40])
def test_noalloc_down_matches_forward(T, cuda):
    import torch

    from ffn_residual_mesh_b200 import _native as N
    from ffn_residual_mesh_b200 import synth
    from ffn_residual_mesh_b200.engine import LayerSpec, ResidualMesh

    D, F, r = 1024, 1000, 2
    L = synth.make_layer(31, F, D)
    _, z, s = synth.make_activations(32 + T, T, D)
    gb = O.host_base(L.gate_codes, L.gate_alpha, L.gate_beta, z, s, r)
    ub = O.host_base(L.up_codes, L.up_alpha, L.up_beta, z, s, r)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)

    # existing entry point
    ctx = ResidualMesh(D, F, r, 1, T)
    ctx.load_layer(0, LayerSpec(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.down, L.gate_beta, L.up_beta))
    y_ref = torch.empty(T, D, device=cuda)
    ctx.forward(0, dev(z), dev(s), dev(gb.astype(np.float32)), dev(ub.astype(np.float32)), y32=y_ref)
    torch.cuda.synchronize()

    # same h, split into fp16 hi + lo, as the input of the allocation-free call
    ref = O.ffn_forward(L.gate_codes, L.up_codes, L.gate_alpha, L.up_alpha, L.gate_beta, L.up_beta, L.down, z, s, r,
                        gate_base=gb, up_base=ub)
    h = ref["h"].astype(np.float32)
    h_hi = h.astype(np.float16)
    h_lo = (h - h_hi.astype(np.float32)).astype(np.float16)
    ld = (F + 7) // 8 * 8
    pad = lambda a: np.pad(a, ((0, 0), (0, ld - a.shape[1])))
    down_d, hi_d, lo_d = dev(pad(L.down)), dev(pad(h_hi)), dev(pad(h_lo))
    lib = N.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        y32 = torch.full((T, D), float("nan"), device=cuda)
        y16 = torch.zeros(T, D, dtype=torch.float16, device=cuda)
        status = torch.full((1,), -1, dtype=torch.int32, device=cuda)
        rc = lib.ffnrm_down_project_noalloc(down_d.data_ptr(), ld, hi_d.data_ptr(), lo_d.data_ptr(), ld, D, F, T,
                                            y32.data_ptr(), y16.data_ptr(), status.data_ptr(), ctypes.c_void_p(stream))
        N.check(rc)
        torch.cuda.synchronize()
        assert int(status.item()) == 0, f"call {call}: pipeline wait gave up"
        got, want = y32.cpu().numpy(), y_ref.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_l2(got, want) < 1e-5, f"call {call}"
        assert np.abs(got - want).max() < Y_MAX_ABS
        assert rel_l2(y16.float().cpu().numpy(), want) < Y_REL_L2
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
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
