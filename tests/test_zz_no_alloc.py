"""The allocation-free dense-block entry point against the allocating one.

``ce4b_dense_block_forward_static`` serves callers that cannot allocate device memory
(for example an engine thread in a process whose allocator is frozen after start-up, or
a plugin that is handed only its input and output buffers): its scratch lives in a fixed
8 MiB array inside the library instead of a caller-provided workspace. It runs the same
kernels as ``ce4b_dense_block_forward``, so two calls in a row, each with different
inputs and row counts, must reproduce that entry point's output exactly; once the first
call on the device has loaded the library's device image, further calls must leave the
device's free memory unchanged; and a call whose scratch would not fit must fail with a
clear error. This file sorts last so that a run stopping at the first failure has
already run every other test.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _block_inputs(rows: int, d: int, h: int, seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
    nw = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    wgu = (0.05 * torch.randn(2 * h, d, device="cuda", generator=g)).bfloat16()
    wd = (0.05 * torch.randn(d, h, device="cuda", generator=g)).bfloat16()
    return x, nw, wgu, wd


def _static_call(x, nw, wgu, wd, out, rows, d, h) -> int:
    from ce4b200 import _lib

    return _lib.library().ce4b_dense_block_forward_static(
        x.data_ptr(), nw.data_ptr(), wgu.data_ptr(), wd.data_ptr(), out.data_ptr(),
        rows, d, h, 1e-6, _lib.PRECISION_BF16, torch.cuda.current_stream().cuda_stream,
    )


def test_static_scratch_block_matches_allocating_entry_point() -> None:
    from ce4b200 import _lib, kernels

    for rows, d, h, seed in ((300, 512, 1536, 1), (129, 128, 384, 2)):
        x, nw, wgu, wd = _block_inputs(rows, d, h, seed)
        expected = kernels.dense_block_forward(x, nw, wgu, wd, precision="bf16")
        out = torch.full_like(x, float("nan"))
        _lib.check(_static_call(x, nw, wgu, wd, out, rows, d, h))
        torch.cuda.synchronize()
        torch.testing.assert_close(out, expected, atol=0, rtol=0)
    assert _lib.check_device_error(torch.cuda.current_device()) == 0


def test_static_scratch_call_leaves_free_memory_unchanged() -> None:
    from ce4b200 import _lib

    rows, d, h = 1024, 512, 1536
    x, nw, wgu, wd = _block_inputs(rows, d, h, 4)
    out = torch.empty_like(x)
    # The first call on the device loads the library's device image (the 8 MiB array).
    _lib.check(_static_call(x, nw, wgu, wd, out, rows, d, h))
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    _lib.check(_static_call(x, nw, wgu, wd, out, rows, d, h))
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


def test_static_scratch_rejects_oversized_blocks() -> None:
    from ce4b200 import _lib

    rows, d, h = 4096, 512, 1536  # 16 MiB of scratch > 8 MiB
    # Buffers hold all 4096 rows, so a regression in the size check fails an assertion
    # instead of launching kernels past the end of a smaller buffer.
    x, nw, wgu, wd = _block_inputs(rows, d, h, 3)
    out = torch.empty_like(x)
    status = _static_call(x, nw, wgu, wd, out, rows, d, h)
    torch.cuda.synchronize()
    assert status == _lib.CE4B_ERR_INVALID_ARGUMENT
    assert "static scratch" in _lib.last_error()
