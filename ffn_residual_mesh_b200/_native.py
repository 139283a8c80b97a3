"""ctypes binding of ``libffnrm.so`` (declared in ``include/ffnrm.h``).

The product path always goes through this library; there is no CPU fallback.
Importing the package on a machine without the built library raises
``NativeLibraryMissing`` at the first call that needs it.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_int, c_int32, c_int64, c_size_t, c_uint8, c_uint16, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libffnrm.so"

OK, ERR_ARG, ERR_CUDA, ERR_STATE, ERR_NOMEM, ERR_TIMEOUT = 0, 1, 2, 3, 4, 5
CODES_Q4_BYTES, CODES_QLO2_ROWPACKED, CODES_BITPLANES = 0, 1, 2
KERNEL_RESIDUAL, KERNEL_DOWN, KERNEL_REDUCE = 0, 1, 2
IPC_HANDLE_BYTES = 64

# Every symbol include/ffnrm.h declares, with its ctypes signature.
SIGNATURES = {
    "ffnrm_create": (c_int, [POINTER(c_void_p), c_int, c_void_p]),
    "ffnrm_destroy": (c_int, [c_void_p]),
    "ffnrm_load_layer": (c_int, [c_void_p, c_int, c_void_p]),
    "ffnrm_residual": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p]),
    "ffnrm_ffn_forward": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_void_p]),
    "ffnrm_ffn_forward_host": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_void_p]),
    "ffnrm_ffn_forward_host_partial": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                                               c_void_p, c_void_p, c_void_p]),
    "ffnrm_host_register": (c_int, [c_void_p, c_size_t]),
    "ffnrm_host_unregister": (c_int, [c_void_p]),
    "ffnrm_cast_f16": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "ffnrm_peer_create": (c_int, [POINTER(c_void_p), c_int, c_int, c_int, c_int64, c_void_p]),
    "ffnrm_peer_connect": (c_int, [c_void_p, c_void_p]),
    "ffnrm_ffn_forward_reduced": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_void_p]),
    "ffnrm_peer_allreduce": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
    "ffnrm_peer_check": (c_int, [c_void_p, c_void_p]),
    "ffnrm_peer_destroy": (c_int, [c_void_p]),
    "ffnrm_layer_bytes": (c_int, [c_void_p, c_int, POINTER(c_int64), POINTER(c_int64)]),
    "ffnrm_launch_count": (c_int64, [c_void_p]),
    "ffnrm_check_device_error": (c_int, [c_void_p, c_void_p]),
    "ffnrm_down_project_noalloc": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int, c_int, c_int,
                                           c_void_p, c_void_p, c_void_p, c_void_p]),
    "ffnrm_noalloc_status": (c_int, [c_void_p, c_void_p]),
    "ffnrm_profile_enable": (c_int, [c_void_p, c_int]),
    "ffnrm_profile_read": (c_int, [c_void_p, c_int, POINTER(ctypes.c_double), POINTER(c_int64)]),
    "ffnrm_base_producer_create": (c_int, [POINTER(c_void_p), c_int]),
    "ffnrm_base_producer_destroy": (c_int, [c_void_p]),
    "ffnrm_base_from_table": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_int,
                                      c_void_p, c_int64, c_void_p]),
    "ffnrm_table_dots": (c_int, [c_void_p, c_void_p, c_void_p]),
    "ffnrm_last_error": (c_char_p, []),
    "ffnrm_version": (c_char_p, []),
}


class Config(ctypes.Structure):
    _fields_ = [("d_model", c_int32), ("d_ff", c_int32), ("residual_bits", c_int32), ("n_layers", c_int32),
                ("max_tokens", c_int32), ("base_tile_rows", c_int32)]


class LayerWeights(ctypes.Structure):
    _fields_ = [("codes_format", c_int32), ("gate_codes", c_void_p), ("up_codes", c_void_p),
                ("gate_high", c_void_p), ("up_high", c_void_p), ("gate_alpha", c_void_p), ("up_alpha", c_void_p),
                ("gate_beta", c_void_p), ("up_beta", c_void_p), ("down", c_void_p), ("down_ld", c_int64),
                ("keep_fallback", c_int32)]


class NativeLibraryMissing(RuntimeError):
    pass


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise NativeLibraryMissing(
                f"{LIB_PATH} is not built; run `python -m ffn_residual_mesh_b200.build` (there is no CPU fallback)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int) -> None:
    """Map a status code to the reference's error conventions."""
    if rc == OK:
        return
    msg = (lib().ffnrm_last_error() or b"").decode()
    if rc == ERR_ARG:
        raise ValueError(msg)
    if rc == ERR_NOMEM:
        raise MemoryError(msg)
    if rc == ERR_TIMEOUT:
        raise TimeoutError(msg)
    raise RuntimeError(f"ffnrm error {rc}: {msg}")
