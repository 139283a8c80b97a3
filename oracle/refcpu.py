"""ctypes view of ``oracle/_ref/libref_cpu.so`` (the reference's AVX2 CPU evaluator).

TEST INFRASTRUCTURE / CPU BASELINE ONLY (tests, smoke, bench.py's CPU leg).
Built by ``oracle/Makefile`` from the reference sources; see ``ref_cpu_driver.cpp``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "_ref" / "libref_cpu.so"
_P = ctypes.c_void_p


def available() -> bool:
    return LIB_PATH.exists()


def _lib():
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.ref_ffn_create.restype = _P
    lib.ref_ffn_create.argtypes = [ctypes.c_int] * 3 + [_P] * 7
    lib.ref_ffn_destroy.argtypes = [_P]
    lib.ref_ffn_gate_up.argtypes = [_P, _P, _P, ctypes.c_int, _P, _P, _P]
    lib.ref_ffn_forward.argtypes = [_P, _P, _P, ctypes.c_int, _P]
    lib.ref_fused_base.restype = ctypes.c_int
    lib.ref_fused_base.argtypes = [ctypes.c_int] * 5 + [_P] * 8
    return lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


class RefFfn:
    """The reference's CPU FFN (direct_q4 gate/up + SwiGLU + fp16 down) for one layer."""

    def __init__(self, gate_q, up_q, gate_alpha, up_alpha, gate_beta, up_beta, down=None,
                 threads: int | None = None):
        self.lib = _lib()
        self.rows, self.hidden = gate_q.shape
        self.threads = threads or os.cpu_count() or 1
        self._keep = [np.ascontiguousarray(a) for a in (gate_q, up_q)] + [
            np.ascontiguousarray(a, dtype=np.float32) for a in (gate_alpha, up_alpha, gate_beta, up_beta)]
        self._keep.append(None if down is None else np.ascontiguousarray(down, dtype=np.float16).view(np.uint16))
        self.handle = self.lib.ref_ffn_create(self.rows, self.hidden, self.threads, *[_ptr(a) for a in self._keep])

    def gate_up(self, z: np.ndarray, s: np.ndarray, with_dots: bool = False):
        z = np.ascontiguousarray(z, dtype=np.int8)
        s = np.ascontiguousarray(s, dtype=np.float32)
        T = z.shape[0]
        g = np.empty((T, self.rows), np.float32)
        u = np.empty_like(g)
        dots = np.empty((2, T, self.rows, self.hidden // 32), np.int32) if with_dots else None
        self.lib.ref_ffn_gate_up(self.handle, _ptr(z), _ptr(s), T, _ptr(g), _ptr(u), _ptr(dots))
        return (g, u, dots) if with_dots else (g, u)

    def forward(self, z: np.ndarray, s: np.ndarray) -> np.ndarray:
        z = np.ascontiguousarray(z, dtype=np.int8)
        s = np.ascontiguousarray(s, dtype=np.float32)
        y = np.empty((z.shape[0], self.hidden), np.float32)
        self.lib.ref_ffn_forward(self.handle, _ptr(z), _ptr(s), z.shape[0], _ptr(y))
        return y

    def close(self):
        if self.handle:
            self.lib.ref_ffn_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


def fused_base(table, high_sum, alpha, beta, z, s, block: int, threads: int = 1, prefetch: int = 4):
    """Reference ``fused_base`` (radix table, r = 2) for one token -> (base[rows], P_hi[rows, groups])."""
    lib = _lib()
    rows, groups = high_sum.shape
    arrs = [np.ascontiguousarray(table, dtype=np.uint8), np.ascontiguousarray(high_sum, dtype=np.int16),
            np.ascontiguousarray(alpha, dtype=np.float32), np.ascontiguousarray(beta, dtype=np.float32),
            np.ascontiguousarray(z, dtype=np.int8).reshape(-1), np.ascontiguousarray(s, dtype=np.float32).reshape(-1)]
    out = np.empty(rows, np.float32)
    dots = np.empty((rows, groups), np.int32)
    rc = lib.ref_fused_base(rows, groups * 32, block, threads, prefetch, *[_ptr(a) for a in arrs], _ptr(out), _ptr(dots))
    if rc:
        raise ValueError("reference fused_base rejected the shape")
    return out, dots
