"""The C-ABI library loads and exports every symbol include/ffnrm.h declares (CPU)."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT


def declared_functions():
    text = (ROOT / "include" / "ffnrm.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(ffnrm_[a-z_0-9]+)\s*\(", text, flags=re.M)))


def test_library_builds_and_exports_all_symbols():
    from ffn_residual_mesh_b200 import _native as N
    from ffn_residual_mesh_b200 import build
    build.build()
    lib = ctypes.CDLL(str(N.LIB_PATH))
    names = declared_functions()
    assert len(names) >= 14
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(N.SIGNATURES), "binding table out of sync with the header"
    assert N.lib().ffnrm_version().startswith(b"ffnrm")


def test_errors_without_device_are_loud():
    """On a machine without a GPU, creating a context fails with a CUDA error
    instead of falling back to the CPU."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from ffn_residual_mesh_b200.engine import ResidualMesh
    with pytest.raises((RuntimeError, ValueError)):
        ResidualMesh(256, 64, 2, 1, 1)


def test_argument_validation_before_device_use():
    from ffn_residual_mesh_b200.engine import ResidualMesh
    with pytest.raises(ValueError):
        ResidualMesh(100, 64, 2, 1, 1)
