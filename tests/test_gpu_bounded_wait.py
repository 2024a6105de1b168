"""The bounded in-kernel waits give up instead of hanging: a kernel that waits for a
counter nobody publishes, or for an mbarrier nobody arrives on, returns after its limit
with the timeout code in the device error word, and the context stays usable."""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind,code", [(0, 7), (1, 1)])
def test_wait_that_never_ends_times_out_with_its_code(kind: int, code: int) -> None:
    from ce4b200 import _lib

    lib = _lib.library()
    dev = torch.cuda.current_device()
    assert _lib.check_device_error(dev) == 0
    limit_ns = 2_000_000  # 2 ms
    waited = ctypes.c_int64(0)
    _lib.check(lib.ce4b_selftest_bounded_wait(kind, limit_ns, ctypes.byref(waited),
                                              torch.cuda.current_stream().cuda_stream))
    assert limit_ns <= waited.value < limit_ns + 50_000_000
    assert _lib.check_device_error(dev) == code  # read and cleared
    assert _lib.check_device_error(dev) == 0
    # The context is still usable.
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2

