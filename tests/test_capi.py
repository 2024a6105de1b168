"""CPU checks of the C ABI: the library loads, exports every function include/ce4b200.h
declares, and rejects bad arguments on the host before any GPU work."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "ce4b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(ce4b_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_abi() -> None:
    names = declared_functions()
    assert "ce4b_model_forward" in names and "ce4b_bf16_gemm" in names
    assert len(names) >= 15


def test_library_exports_every_declared_function() -> None:
    from ce4b200 import _lib

    lib = _lib.library()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # Every declared function has a typed binding in the Python layer.
    assert set(declared_functions()) <= set(_lib.SIGNATURES)


def test_version_and_empty_error() -> None:
    from ce4b200 import _lib

    assert b"sm_100a" in _lib.library().ce4b_version()


def test_host_side_argument_checks_need_no_gpu() -> None:
    from ce4b200 import _lib

    lib = _lib.library()
    # Null output and bad extents are rejected before any CUDA call.
    assert lib.ce4b_bf16_gemm(None, None, None, 0, 16, 16, None) == _lib.CE4B_ERR_INVALID_ARGUMENT
    assert "positive" in _lib.last_error()
    assert lib.ce4b_dense_block_workspace_size(0, 512, 1536) == -1
    assert lib.ce4b_dense_block_workspace_size(100, 512, 1536) == 128 * 512 * 2 + 128 * 1536 * 2
    handle = ctypes.c_void_p()
    assert lib.ce4b_model_create(None, 0, 16, ctypes.byref(handle)) == _lib.CE4B_ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _lib.check(_lib.CE4B_ERR_UNSUPPORTED)


def test_model_create_validates_config_on_host() -> None:
    from ce4b200 import _lib

    lib = _lib.library()
    handle = ctypes.c_void_p()
    bad = _lib.ModelConfigStruct(
        arch=_lib.ARCH_DENSE, d_model=100, depth=2, history_length=8, expansion_ratio=3.0,
        rms_norm_eps=1e-6, policy_size=1858, policy_storage_size=1888,
        precision=_lib.PRECISION_BF16,
    )
    assert lib.ce4b_model_create(ctypes.byref(bad), 0, 16, ctypes.byref(handle)) == _lib.CE4B_ERR_INVALID_ARGUMENT
    assert "multiple of 64" in _lib.last_error()
    bad.d_model, bad.history_length = 128, 9
    assert lib.ce4b_model_create(ctypes.byref(bad), 0, 16, ctypes.byref(handle)) == _lib.CE4B_ERR_INVALID_ARGUMENT


def test_safetensors_loader_reports_missing_file() -> None:
    from ce4b200 import _lib

    handle = ctypes.c_void_p()
    status = _lib.library().ce4b_model_load_safetensors(b"/nonexistent/model.safetensors", 0, 8, 0, ctypes.byref(handle))
    assert status == _lib.CE4B_ERR_IO
    assert "cannot open" in _lib.last_error()


def test_bounded_wait_selftest_checks_arguments_on_the_host() -> None:
    import ctypes

    from ce4b200 import _lib

    waited = ctypes.c_int64(0)
    lib = _lib.library()
    assert lib.ce4b_selftest_bounded_wait(2, 1000, ctypes.byref(waited), None) == _lib.CE4B_ERR_INVALID_ARGUMENT
    assert "kind" in _lib.last_error()
    assert lib.ce4b_selftest_bounded_wait(0, 10**9, ctypes.byref(waited), None) == _lib.CE4B_ERR_INVALID_ARGUMENT
    assert "limit" in _lib.last_error()
