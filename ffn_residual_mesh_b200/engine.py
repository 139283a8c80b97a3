"""Host-side engine over the C ABI: one ``ResidualMesh`` per device (or per d_ff shard).

It mirrors the reference's in-process operator surface for this path:

* ``residual(...)``        — the GPU residual contraction
  (``residual_kernel``, src/exact_residual_cuda_runner.cu:122-159; Triton
  ``residual_direct_kernel``, scripts/benchmark_cpu_base_gpu_full_ffn.py:80-104);
* ``forward(...)``         — merge + SwiGLU + down with HBM-resident base sums
  (scripts/benchmark_gpu_full_ffn_density.py:120-121,161-162);
* ``forward_host(...)``    — the same with host-streamed base sums
  (src/exact_cpu_base_gpu_full_ffn_runner.cu:291-347).

Arguments may be torch tensors (device or pinned host), numpy arrays (host) or
raw integer addresses. Shape errors raise ``ValueError`` like the reference's
Python adapter (scripts/native_radix_cpu.py:74-79).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _native as N


def _addr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("arrays must be C-contiguous")
        return x.ctypes.data
    ptr = getattr(x, "data_ptr", None)
    if ptr is not None:
        if not x.is_contiguous():
            raise ValueError("tensors must be contiguous")
        return ptr()
    raise TypeError(f"unsupported buffer type {type(x)!r}")


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _shape(x):
    return tuple(x.shape) if x is not None else None


@dataclass
class LayerSpec:
    """Weights of one layer in the reference's terms (host numpy arrays)."""
    gate_codes: np.ndarray          # [F, D] Q4 codes (0..15), or packed low codes (see codes_format)
    up_codes: np.ndarray
    gate_alpha: np.ndarray          # [F, G]
    up_alpha: np.ndarray
    down: np.ndarray                # [D, F] fp16 (or [D, ld] with down_ld)
    gate_beta: np.ndarray | None = None
    up_beta: np.ndarray | None = None
    codes_format: int = N.CODES_Q4_BYTES
    gate_high: np.ndarray | None = None
    up_high: np.ndarray | None = None
    keep_fallback: bool = False


class ResidualMesh:
    """Device context holding a stack of FFN layers for the exact base/residual split."""

    def __init__(self, d_model: int, d_ff: int, residual_bits: int, n_layers: int, max_tokens: int,
                 base_tile_rows: int = 256, device: int = 0):
        self.lib = N.lib()
        self.d_model, self.d_ff, self.r = d_model, d_ff, residual_bits
        self.groups = d_model // 32
        self.n_layers, self.max_tokens, self.tile_rows, self.device = n_layers, max_tokens, base_tile_rows, device
        cfg = N.Config(d_model, d_ff, residual_bits, n_layers, max_tokens, base_tile_rows)
        handle = ctypes.c_void_p()
        N.check(self.lib.ffnrm_create(ctypes.byref(handle), device, ctypes.byref(cfg)))
        self.handle = handle

    # -- lifetime ---------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "handle", None):
            N.check(self.lib.ffnrm_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- weights ------------------------------------------------------------
    def load_layer(self, layer: int, spec: LayerSpec) -> None:
        """Copy one layer's weights into HBM in the device layouts. Arrays may be host
        numpy arrays or torch tensors (host or on this context's device); the library
        decodes and packs them on the GPU."""
        F, D, G = self.d_ff, self.d_model, self.groups
        keep = []

        def arr(a, dtype, shape=None):
            if a is None:
                return None
            if hasattr(a, "data_ptr"):  # torch tensor: used in place
                import torch
                want = {np.uint8: torch.uint8, np.float32: torch.float32}[dtype]
                if a.dtype != want or not a.is_contiguous():
                    raise ValueError(f"expected a contiguous {want} tensor, got {a.dtype}")
                if shape is not None and tuple(a.shape) != shape:
                    raise ValueError(f"expected shape {shape}, got {tuple(a.shape)}")
                keep.append(a)
                return a.data_ptr()
            v = np.ascontiguousarray(a, dtype=dtype)
            if shape is not None and v.shape != shape:
                raise ValueError(f"expected shape {shape}, got {v.shape}")
            keep.append(v)
            return v.ctypes.data

        if spec.codes_format == N.CODES_Q4_BYTES:
            cshape = (F, D)
        elif spec.codes_format == N.CODES_QLO2_ROWPACKED:
            cshape = (F, D // 4)
        else:
            cshape = None
        codes = [arr(spec.gate_codes, np.uint8, cshape), arr(spec.up_codes, np.uint8, cshape)]
        if spec.codes_format == N.CODES_BITPLANES:
            for a in (spec.gate_codes, spec.up_codes):
                size = a.numel() if hasattr(a, "numel") else np.asarray(a).size
                if size != self.r * F * D // 8:
                    raise ValueError("bitplane payload length does not match d_ff, d_model and residual_bits")
        down = spec.down
        if hasattr(down, "data_ptr"):
            import torch
            if down.dtype != torch.float16 or down.dim() != 2 or down.shape[0] != D or down.shape[1] < F \
                    or down.stride(1) != 1:
                raise ValueError(f"down must be fp16 [{D}, >= {F}] with unit column stride, got {down.dtype} "
                                 f"{tuple(down.shape)}")
            down_ptr, down_ld = down.data_ptr(), down.stride(0)
            keep.append(down)
        else:
            down = np.asarray(down)
            if down.dtype != np.float16 or down.ndim != 2 or down.shape[0] != D or down.shape[1] < F:
                raise ValueError(f"down must be fp16 [{D}, >= {F}], got {down.dtype} {down.shape}")
            down = np.ascontiguousarray(down)
            keep.append(down)
            down_ptr, down_ld = down.ctypes.data, down.shape[1]
        w = N.LayerWeights(
            spec.codes_format, codes[0], codes[1],
            arr(spec.gate_high, np.uint8), arr(spec.up_high, np.uint8),
            arr(spec.gate_alpha, np.float32, (F, G)), arr(spec.up_alpha, np.float32, (F, G)),
            arr(spec.gate_beta, np.float32, (F, G)), arr(spec.up_beta, np.float32, (F, G)),
            down_ptr, down_ld, int(spec.keep_fallback))
        N.check(self.lib.ffnrm_load_layer(self.handle, layer, ctypes.byref(w)))

    def layer_bytes(self, layer: int) -> tuple[int, int]:
        res, down = ctypes.c_int64(), ctypes.c_int64()
        N.check(self.lib.ffnrm_layer_bytes(self.handle, layer, ctypes.byref(res), ctypes.byref(down)))
        return res.value, down.value

    @property
    def launches(self) -> int:
        return int(self.lib.ffnrm_launch_count(self.handle))

    def check_device_error(self, stream=None) -> None:
        """Synchronise and raise TimeoutError if a kernel gave up on a bounded wait."""
        N.check(self.lib.ffnrm_check_device_error(self.handle, _stream(stream)))

    def profile(self, enable: bool) -> None:
        """Start (and clear) or stop live per-kernel CUDA-event timing."""
        N.check(self.lib.ffnrm_profile_enable(self.handle, int(enable)))

    def profile_read(self) -> dict:
        """{kernel: (total device ms, launches)} since profiling was enabled."""
        out = {}
        for name, kind in (("residual", N.KERNEL_RESIDUAL), ("down", N.KERNEL_DOWN), ("reduce", N.KERNEL_REDUCE)):
            ms, n = ctypes.c_double(), ctypes.c_int64()
            N.check(self.lib.ffnrm_profile_read(self.handle, kind, ctypes.byref(ms), ctypes.byref(n)))
            out[name] = (ms.value, n.value)
        return out

    # -- compute ------------------------------------------------------------
    def _check_act(self, z, s) -> int:
        if z is None or len(z.shape) != 2 or z.shape[1] != self.d_model:
            raise ValueError(f"z must have shape (T,{self.d_model}), got {_shape(z)}")
        T = int(z.shape[0])
        if tuple(s.shape) not in {(T, self.groups)}:
            raise ValueError(f"s must have shape ({T},{self.groups}), got {_shape(s)}")
        return T

    def _check_tf(self, name, x, T):
        if x is not None and tuple(x.shape) != (T, self.d_ff):
            raise ValueError(f"{name} must have shape ({T},{self.d_ff}), got {_shape(x)}")

    def residual(self, layer, z, s, gate_res, up_res, dots=None, fallback_tiles=None, stream=None) -> None:
        """Exact residual gate/up contraction (device buffers); rows of flagged
        fallback tiles receive the unsplit exact projection instead."""
        T = self._check_act(z, s)
        self._check_tf("gate_res", gate_res, T)
        self._check_tf("up_res", up_res, T)
        if dots is not None and tuple(dots.shape) != (2, T, self.d_ff, self.groups):
            raise ValueError("dots must have shape (2, T, d_ff, d_model/32)")
        N.check(self.lib.ffnrm_residual(self.handle, layer, _addr(z), _addr(s), T, _addr(gate_res),
                                        _addr(up_res), _addr(dots), _addr(fallback_tiles), _stream(stream)))

    def forward(self, layer, z, s, gate_base, up_base, fallback_tiles=None, y32=None, y16=None,
                stream=None) -> None:
        """Full split FFN with HBM-resident base sums (device buffers)."""
        T = self._check_act(z, s)
        self._check_tf("gate_base", gate_base, T)
        self._check_tf("up_base", up_base, T)
        for name, y in (("y32", y32), ("y16", y16)):
            if y is not None and tuple(y.shape) != (T, self.d_model):
                raise ValueError(f"{name} must have shape ({T},{self.d_model})")
        N.check(self.lib.ffnrm_ffn_forward(self.handle, layer, _addr(z), _addr(s), T, _addr(gate_base),
                                           _addr(up_base), _addr(fallback_tiles), _addr(y32), _addr(y16),
                                           _stream(stream)))

    def forward_host(self, layer, z, s, gate_base, up_base, y16, fallback_tiles=None, stream=None) -> None:
        """Full split FFN, host buffers in and out, base sums streamed on a side stream."""
        T = self._check_act(z, s)
        self._check_tf("gate_base", gate_base, T)
        self._check_tf("up_base", up_base, T)
        if tuple(y16.shape) != (T, self.d_model):
            raise ValueError(f"y16 must have shape ({T},{self.d_model})")
        N.check(self.lib.ffnrm_ffn_forward_host(self.handle, layer, _addr(z), _addr(s), T, _addr(gate_base),
                                                _addr(up_base), _addr(fallback_tiles), _addr(y16),
                                                _stream(stream)))

    def forward_host_partial(self, layer, z, s, gate_base, up_base, y32, fallback_tiles=None, stream=None) -> None:
        """Host-streamed forward of one d_ff shard: host inputs, device fp32 partial out."""
        T = self._check_act(z, s)
        self._check_tf("gate_base", gate_base, T)
        self._check_tf("up_base", up_base, T)
        if tuple(y32.shape) != (T, self.d_model):
            raise ValueError(f"y32 must have shape ({T},{self.d_model})")
        N.check(self.lib.ffnrm_ffn_forward_host_partial(self.handle, layer, _addr(z), _addr(s), T, _addr(gate_base),
                                                        _addr(up_base), _addr(fallback_tiles), _addr(y32),
                                                        _stream(stream)))


def host_register(array) -> None:
    """Page-lock a host buffer (numpy array) for async copies."""
    N.check(N.lib().ffnrm_host_register(_addr(array), array.nbytes))


def host_unregister(array) -> None:
    N.check(N.lib().ffnrm_host_unregister(_addr(array)))


def cast_f16(src, dst, stream=None) -> None:
    N.check(N.lib().ffnrm_cast_f16(_addr(src), _addr(dst), int(np.prod(src.shape)), _stream(stream)))
