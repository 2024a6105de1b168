"""ctypes binding of libce4b200.so (the C ABI declared in include/ce4b200.h).

The shared library is built in-tree (``make -C chess-engine-4_b200``) and loaded from
this package directory. There is no fallback: if the library is missing, every entry
point raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libce4b200.so"

CE4B_OK = 0
CE4B_ERR_INVALID_ARGUMENT = 1
CE4B_ERR_CUDA = 2
CE4B_ERR_UNSUPPORTED = 3
CE4B_ERR_IO = 4
CE4B_ERR_DEVICE_TIMEOUT = 5
CE4B_ERR_NOT_READY = 6

ARCH_DENSE = 0
ARCH_MOE64A2 = 1
PRECISION_BF16 = 0
PRECISION_MXFP8 = 1

INPUT_F32_PLANES = 0
INPUT_BF16_PLANES = 1
INPUT_LC0 = 2
INPUT_PACKED_F32 = 3
INPUT_PACKED_BF16 = 4

DTYPE_BF16 = 0
DTYPE_F32 = 1


class ModelConfigStruct(ctypes.Structure):
    _fields_ = [
        ("arch", ctypes.c_int32),
        ("d_model", ctypes.c_int32),
        ("depth", ctypes.c_int32),
        ("history_length", ctypes.c_int32),
        ("expansion_ratio", ctypes.c_float),
        ("rms_norm_eps", ctypes.c_float),
        ("policy_size", ctypes.c_int32),
        ("policy_storage_size", ctypes.c_int32),
        ("precision", ctypes.c_int32),
    ]


class ModelInfoStruct(ctypes.Structure):
    _fields_ = [
        ("d_model", ctypes.c_int32),
        ("depth", ctypes.c_int32),
        ("history_length", ctypes.c_int32),
        ("policy_size", ctypes.c_int32),
        ("maximum_batch_size", ctypes.c_int32),
        ("hidden_dim", ctypes.c_int32),
        ("expert_hidden_dim", ctypes.c_int32),
        ("arch", ctypes.c_int32),
        ("weight_bytes", ctypes.c_int64),
        ("workspace_bytes", ctypes.c_int64),
    ]


class Mxfp8TapStruct(ctypes.Structure):
    _fields_ = [("layer", ctypes.c_int32)] + [
        (name, ctypes.c_void_p)
        for name in (
            "a_codes_dev", "a_scales_dev", "n_bf16_dev", "n_codes_dev", "n_scales_dev",
            "h_bf16_dev", "h_codes_dev", "h_scales_dev",
        )
    ]


class Ce4bError(RuntimeError):
    """A libce4b200 call failed on the device or in CUDA."""

    def __init__(self, status: int, message: str) -> None:
        super().__init__(message)
        self.status = status


_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_fp = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ce4b_last_error": (ctypes.c_char_p, []),
    "ce4b_version": (ctypes.c_char_p, []),
    "ce4b_check_device_error": (_i32, [_i32, ctypes.POINTER(_i32)]),
    "ce4b_model_create": (
        _i32,
        [ctypes.POINTER(ModelConfigStruct), _i32, _i32, ctypes.POINTER(_vp)],
    ),
    "ce4b_model_set_tensor": (
        _i32,
        [_vp, ctypes.c_char_p, _vp, _i32, _i32, ctypes.POINTER(_i64), _i32],
    ),
    "ce4b_model_finalize": (_i32, [_vp]),
    "ce4b_model_load_safetensors": (
        _i32,
        [ctypes.c_char_p, _i32, _i32, _i32, ctypes.POINTER(_vp)],
    ),
    "ce4b_model_info_get": (_i32, [_vp, ctypes.POINTER(ModelInfoStruct)]),
    "ce4b_model_forward": (
        _i32,
        [_vp, _i32, _vp, _vp, _i32, _vp, _vp, _vp, _i32, _i32, _vp, _vp],
    ),
    "ce4b_model_evaluate": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp]),
    "ce4b_model_evaluate_async": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp, _vp]),
    "ce4b_model_set_trace": (_i32, [_vp, _vp, _i32]),
    "ce4b_model_set_task_trace": (_i32, [_vp, _vp, _i32]),
    "ce4b_nccl_unique_id": (_i32, [_vp, _i32]),
    "ce4b_policy_softmax": (_i32, [_vp, _i32, _i32, _vp, _vp, ctypes.c_float, _vp, _vp]),
    "ce4b_model_evaluate_legal": (_i32, [_vp, _vp, _i32, _vp, _vp, ctypes.c_float, _vp, _vp, _vp]),
    "ce4b_model_enable_expert_parallel": (_i32, [_vp, _i32, _i32, _vp]),
    "ce4b_expert_parallel_plan": (_i32, [_i32, _i32, _vp, _vp, _vp, _vp, _vp, _i32, ctypes.POINTER(_i32)]),
    "ce4b_model_task_count": (_i32, [_vp, _i32, ctypes.POINTER(_i32)]),
    "ce4b_model_set_latency_path": (_i32, [_vp, _i32]),
    "ce4b_model_set_direct_io": (_i32, [_vp, _i32]),
    "ce4b_model_uses_latency_path": (_i32, [_vp, _i32, ctypes.POINTER(_i32)]),
    "ce4b_model_set_mxfp8_tap": (_i32, [_vp, ctypes.POINTER(Mxfp8TapStruct)]),
    "ce4b_model_set_routing_tap": (_i32, [_vp, _vp, _i32]),
    "ce4b_model_trace_label": (_i32, [_vp, _i32, ctypes.c_char_p, _i32]),
    "ce4b_model_destroy": (None, [_vp]),
    "ce4b_selftest_bounded_wait": (_i32, [_i32, _i64, ctypes.POINTER(_i64), _vp]),
    "ce4b_bf16_gemm": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "ce4b_rmsnorm_forward": (_i32, [_vp, _vp, _vp, _i32, _i32, _f32, _vp]),
    "ce4b_swiglu_forward": (_i32, [_vp, _vp, _i32, _i32, _vp]),
    "ce4b_residual_add": (_i32, [_vp, _vp, _i64, _vp]),
    "ce4b_dense_block_workspace_size": (_i64, [_i32, _i32, _i32]),
    "ce4b_dense_block_forward": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _f32, _i32, _vp],
    ),
    "ce4b_moe_route": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _vp]),
    "ce4b_moe_dispatch_capacity": (_i32, [_i32]),
    "ce4b_moe_route_dispatch_workspace_size": (_i64, [_i32]),
    "ce4b_moe_route_dispatch": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _vp],
    ),
    "ce4b_moe_workspace_size": (_i64, [_i32, _i32, _i32]),
    "ce4b_moe_forward": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp],
    ),
    "ce4b_quantize_mxfp8": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp]),
    "ce4b_quantize_mxfp8_transpose": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp]),
    "ce4b_mxfp8_gemm": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "ce4b_dense_block_forward_static": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _f32, _i32, _vp],
    ),
}

_LIB: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    """Load (once) and return the shared library with typed entry points."""

    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.is_file():
        raise RuntimeError(
            f"libce4b200.so is not built ({LIB_PATH}); run `make -C chess-engine-4_b200`"
        )
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


def last_error() -> str:
    message = library().ce4b_last_error()
    return message.decode() if message else ""


def check(status: int) -> None:
    """Raise the exception the reference raises for the same kind of failure."""

    if status == CE4B_OK:
        return
    message = last_error()
    if status in (CE4B_ERR_INVALID_ARGUMENT, CE4B_ERR_UNSUPPORTED):
        raise ValueError(message)
    if status == CE4B_ERR_IO:
        raise OSError(message)
    raise Ce4bError(status, message)


def nccl_unique_id() -> bytes:
    """128-byte NCCL unique id for ce4b_model_enable_expert_parallel (made by rank 0)."""

    buf = ctypes.create_string_buffer(128)
    check(library().ce4b_nccl_unique_id(buf, 128))
    return buf.raw


def check_device_error(device: int) -> int:
    code = ctypes.c_int(0)
    check(library().ce4b_check_device_error(device, ctypes.byref(code)))
    return code.value
