"""Python access to the C MXFP8 oracle (oracle/mxfp8.c) — TEST INFRASTRUCTURE ONLY.

The shared library is built by ``make -C oracle`` (``__graft_entry__.build()`` does it);
if it is missing or older than its source it is rebuilt here with the system C compiler.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libce4oracle.so"
_lib: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        src = HERE / "mxfp8.c"
        if not LIB.is_file() or LIB.stat().st_mtime < src.stat().st_mtime:
            subprocess.run(["make", "-C", os.fspath(HERE)], check=True, capture_output=True)
        lib = ctypes.CDLL(os.fspath(LIB))
        lib.ce4o_e8m0_round_up.restype = ctypes.c_uint8
        lib.ce4o_e8m0_round_up.argtypes = [ctypes.c_float]
        lib.ce4o_e4m3_rne_satfinite.restype = ctypes.c_uint8
        lib.ce4o_e4m3_rne_satfinite.argtypes = [ctypes.c_float]
        lib.ce4o_e4m3_value.restype = ctypes.c_float
        lib.ce4o_e4m3_value.argtypes = [ctypes.c_uint8]
        lib.ce4o_quantize_mxfp8.restype = None
        lib.ce4o_quantize_mxfp8.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_void_p, ctypes.c_void_p]
        _lib = lib
    return _lib


def quantize(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """BF16 [rows, cols] (multiples of 128) -> (E4M3 codes uint8 [rows, cols],
    E8M0 scales uint8 [rows/128, cols/128, 32, 16])."""

    x = x.detach().to("cpu", torch.bfloat16).contiguous()
    rows, cols = x.shape
    if rows % 128 or cols % 128:
        raise ValueError("dimensions must be multiples of 128")
    values = np.empty((rows, cols), dtype=np.uint8)
    scales = np.empty((rows // 128, cols // 128, 32, 16), dtype=np.uint8)
    library().ce4o_quantize_mxfp8(
        x.view(torch.int16).numpy().ctypes.data, rows, cols, values.ctypes.data, scales.ctypes.data
    )
    return torch.from_numpy(values), torch.from_numpy(scales)


def e4m3_table() -> torch.Tensor:
    """float32 value of every E4M3 code (NaN for 0x7F / 0xFF)."""

    lib = library()
    return torch.tensor([lib.ce4o_e4m3_value(c) for c in range(256)], dtype=torch.float32)


def unswizzle_scales(scales: torch.Tensor) -> torch.Tensor:
    """[rows/128, cols/128, 32, 16] tile layout -> [rows, cols/32] row-major codes."""

    rt, ct = scales.shape[:2]
    s = scales.reshape(rt, ct, 32, 4, 4)  # [rt, ct, r%32, r/32, kb]
    s = s.permute(0, 3, 2, 1, 4)          # [rt, r/32, r%32, ct, kb]
    return s.reshape(rt * 128, ct * 4)


def dequantize(values: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """FP32 matrix value = E4M3(code) * 2^(scale - 127) per 32-column block."""

    v = e4m3_table()[values.long()]
    s = unswizzle_scales(scales).float() - 127.0
    return v * torch.exp2(s).repeat_interleave(32, dim=1)
