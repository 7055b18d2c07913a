"""The C ABI library and the pybind11 surface load and export what they declare (no GPU)."""

import ctypes
import importlib
import inspect
import os
import re

import pytest

from orchard_b200 import _lib

REFERENCE_SURFACE = ["initialize", "is_available", "get_device_name", "run_matmul", "run_matmul_simd",
                     "run_rmsnorm", "run_rope", "run_gemv_q8_0", "run_gemv_q4_0", "run_gemm_q4_0",
                     "run_add", "run_mul", "run_silu", "run_softmax", "run_embedding"]


def test_library_built():
    assert os.path.exists(_lib.LIB_PATH), "run `python -m orchard_b200.build`"


def test_every_header_symbol_exported():
    names = _lib.header_symbols()
    assert len(names) >= 40
    h = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in names if not hasattr(h, n)]
    assert not missing, missing


def test_ctypes_signatures_cover_header():
    assert set(_lib.header_symbols()) == set(_lib._SIGS)


def test_status_strings_and_version():
    L = _lib.lib()
    assert L.orch_version() >= 100
    assert L.orch_status_string(0) == b"ok"
    assert b"invalid" in L.orch_status_string(1)


def test_host_side_argument_checks_without_gpu():
    """Argument validation runs before any device work."""
    L = _lib.lib()
    rc = L.orch_gemm_q4_0_ex(None, None, None, 1, None, 1, 4096, 4096, 1, None)
    assert rc == 1 and b"null" in L.orch_last_error()
    rc = L.orch_rope_ex(1, 1, 1, 1, 1, 1, 1, 3, 1, 1, None)
    assert rc == 1 and b"even" in L.orch_last_error()
    assert L.orch_binary_ex(7, 1, 1, 1, 1, 4, None) == 1
    assert L.orch_init(0, b"/nonexistent/kernels") == 1


def test_orchard_core_surface_matches_reference():
    oc = importlib.import_module("orchard_b200.orchard_core")
    for name in REFERENCE_SURFACE:
        assert hasattr(oc.MetalBackend, name), name
    assert [m for m in ("Float32", "Float16", "Int8") if hasattr(oc.DType, m)] == ["Float32", "Float16", "Int8"]
    assert int(oc.DType.Float32) == 0 and int(oc.DType.Float16) == 1 and int(oc.DType.Int8) == 2
    for name in ("copy_from_host", "copy_to_host", "shape", "numel", "size_bytes"):
        assert hasattr(oc.Tensor, name)


def test_orchard_core_fails_loudly_without_gpu():
    oc = importlib.import_module("orchard_b200.orchard_core")
    b = oc.MetalBackend()
    if b.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError):
        b.initialize("")
    with pytest.raises(RuntimeError):
        oc.Tensor(b, [16], oc.DType.Float32)
