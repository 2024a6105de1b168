"""CPU checks of the MXFP8 oracle (oracle/mxfp8.c) against the format definitions and
against the reference's own torch restatement of its quantiser
(third_party/ThunderKittens/kernels/gemm/mxfp8_b200/test_quantize.py:10-41), which agrees
with the kernel except for all-zero blocks (the kernel's 1e-12 floor gives scale code 88,
the restatement's -127 clamp gives 0)."""

from __future__ import annotations

import math

import pytest
import torch


def _lib():
    from oracle import mxfp8

    return mxfp8.library()


def test_e4m3_conversion_matches_torch_float8() -> None:
    lib = _lib()
    g = torch.Generator().manual_seed(0)
    values = torch.cat([
        torch.randn(20000, generator=g) * 40,
        torch.randn(20000, generator=g) * 2**-7,   # subnormal range
        torch.tensor([0.0, -0.0, 448.0, -448.0, 2**-9, 2**-10, 3 * 2**-11, 464.0, 1e30]),
    ])
    ours = torch.tensor([lib.ce4o_e4m3_rne_satfinite(float(v)) for v in values], dtype=torch.uint8)
    ref = values.clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(ours, ref)


@pytest.mark.parametrize("value", [1e-12, 2**-39, 1.0, 1.5, 2**20 + 1, 3.4e38, 7e-41])
def test_e8m0_rounds_up_to_a_power_of_two(value: float) -> None:
    code = _lib().ce4o_e8m0_round_up(value)
    if value < 2.0**127:
        assert 2.0 ** (code - 127) >= value * (1 - 1e-7)
    if code > 0 and code < 254:
        assert 2.0 ** (code - 128) < value
    if value >= 2.0**127:
        assert code == 254


def _torch_restatement(v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's torch restatement of the quantiser (unswizzled scales)."""

    m, n = v.shape
    v = v.float()
    amax = v.abs().view(m, n // 32, 32).amax(dim=-1)
    sc = torch.clamp(torch.ceil(torch.log2(amax / 448.0)), min=-127.0)
    q = (v / (2 ** sc.repeat_interleave(32, dim=-1))).to(torch.float8_e4m3fn)
    return q.view(torch.uint8), (sc + 127).to(torch.uint8)


def test_quantizer_matches_reference_restatement_on_nonzero_blocks() -> None:
    from oracle import mxfp8

    g = torch.Generator().manual_seed(1)
    x = (torch.randn(256, 512, generator=g) * torch.exp(torch.randn(256, 1, generator=g) * 3)).bfloat16()
    x[5, 64:96] = 0  # one all-zero block
    codes, scales = mxfp8.quantize(x)
    ref_codes, ref_scales = _torch_restatement(x)
    flat = mxfp8.unswizzle_scales(scales)
    zero = torch.zeros_like(flat, dtype=torch.bool)
    zero[5, 2] = True
    assert int(flat[5, 2]) == 88 and int(ref_scales[5, 2]) == 0
    assert torch.equal(flat[~zero], ref_scales[~zero])
    mask = ~zero.repeat_interleave(32, dim=1)
    assert torch.equal(codes[mask], ref_codes[mask])
    deq = mxfp8.dequantize(codes, scales)
    rel = (deq - x.float()).abs() / x.float().abs().clamp_min(1e-30)
    # Values within 16x of their block maximum stay in E4M3's normal range: 3 mantissa bits.
    block_amax = x.float().abs().view(256, 16, 32).amax(-1).repeat_interleave(32, dim=1)
    normal = x.float().abs() >= block_amax / 16
    assert float(rel[normal & (x.float() != 0)].max()) <= 2**-4 + 1e-6
    assert math.isclose(float(deq[5, 64:96].abs().max()), 0.0)
