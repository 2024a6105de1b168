"""GPU parity of the dense path: tcgen05 GEMM, kernel ops and the full model forward
against the CPU oracle (oracle/dense.py) on seeded inputs and weights."""

from __future__ import annotations

import pytest
import torch

from helpers import (
    ARGMAX_AGREEMENT,
    POLICY_ATOL,
    POLICY_RTOL,
    WDL_PROB_ATOL,
    argmax_agreement,
    assert_policy_close,
    dense_model,
)

pytestmark = pytest.mark.gpu


def _gemm_ref(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return (a.double() @ b.double().T).float()


@pytest.mark.parametrize(
    "m,n,k",
    [(128, 128, 64), (256, 256, 512), (4096, 3072, 512), (300, 160, 200), (1, 16, 8), (129, 1888, 512),
     (1000, 512, 7168)],
)
def test_bf16_gemm_matches_fp64_reference(m: int, n: int, k: int) -> None:
    from ce4b200 import kernels

    g = torch.Generator(device="cuda").manual_seed(m * 7 + n * 3 + k)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    b = torch.randn(n, k, device="cuda", generator=g).bfloat16()
    c = kernels.bf16_gemm(a, b)
    torch.cuda.synchronize()
    ref = _gemm_ref(a, b)
    # One BF16 rounding of an FP32-accumulated dot product of length k.
    torch.testing.assert_close(c.float(), ref, atol=1e-3 * k**0.5, rtol=8e-3)


def test_kernel_ops_match_torch() -> None:
    from ce4b200 import kernels

    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(333, 512, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(512, device="cuda", generator=g)).bfloat16()
    out = kernels.rmsnorm_forward(x, w, 1e-6)
    xf = x.float()
    ref = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).bfloat16()
    torch.testing.assert_close(out.float(), ref.float(), atol=2e-2, rtol=1e-2)

    gu = torch.randn(77, 2 * 384, device="cuda", generator=g).bfloat16()
    hidden = kernels.swiglu_forward(gu)
    gf, uf = gu.float()[:, :384], gu.float()[:, 384:]
    torch.testing.assert_close(hidden.float(), (torch.nn.functional.silu(gf) * uf).bfloat16().float(),
                               atol=1e-2, rtol=1e-2)

    a = torch.randn(50, 64, device="cuda", generator=g).bfloat16()
    r = torch.randn(50, 64, device="cuda", generator=g).bfloat16()
    expected = (a.float() + r.float()).bfloat16()
    kernels.residual_add(a, r)
    torch.testing.assert_close(a, expected)


@pytest.mark.parametrize("rows,d,h", [(256, 128, 384), (300, 512, 1536), (64, 192, 320)])
def test_dense_block_forward(rows: int, d: int, h: int) -> None:
    from ce4b200 import kernels

    g = torch.Generator(device="cuda").manual_seed(rows + d)
    x = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
    nw = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).bfloat16()
    wgu = (0.05 * torch.randn(2 * h, d, device="cuda", generator=g)).bfloat16()
    wd = (0.05 * torch.randn(d, h, device="cuda", generator=g)).bfloat16()
    out = kernels.dense_block_forward(x, nw, wgu, wd, precision="bf16")
    torch.cuda.synchronize()
    xf = x.float().cpu()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * nw.float().cpu()).bfloat16().float()
    gu = n @ wgu.float().cpu().T
    gg, uu = gu[:, :h].bfloat16().float(), gu[:, h:].bfloat16().float()
    hid = (gg / (1 + torch.exp(-gg)) * uu).bfloat16().float()
    ref = (xf + (hid @ wd.float().cpu().T).bfloat16().float()).bfloat16().float()
    torch.testing.assert_close(out.float().cpu(), ref, atol=3e-2, rtol=2e-2)


def _dense_case(d: int, depth: int, ratio: float, batch: int, hist: int = 8, wseed: int = 0, pseed: int = 1):
    from ce4b200 import synthetic

    weights = synthetic.make_dense_weights(
        d_model=d, depth=depth, hidden_dim=int(d * ratio), seed=wseed, history_length=hist
    )
    lc0 = synthetic.make_lc0_planes(batch, pseed)
    planes = synthetic.lc0_to_dense(lc0)
    return weights, lc0, planes


@pytest.mark.parametrize(
    "d,depth,ratio,batch,hist",
    [(128, 6, 3.0, 256, 8), (512, 12, 3.0, 256, 8), (64, 2, 2.0, 7, 8), (128, 2, 3.0, 129, 2),
     (512, 12, 3.0, 4096, 8)],
)
def test_dense_model_matches_oracle(d: int, depth: int, ratio: float, batch: int, hist: int) -> None:
    from oracle import dense as oracle

    weights, _, planes = _dense_case(d, depth, ratio, batch, hist)
    model = dense_model(weights, d=d, depth=depth, ratio=ratio, hist=hist).cuda()
    out = model(planes.cuda())
    torch.cuda.synchronize()
    ref16 = oracle.forward(weights, planes, depth=depth, history_length=hist, mode="bf16")
    ref32 = oracle.forward(weights, planes, depth=depth, history_length=hist, mode="fp32")
    # Full contract against the reference's BF16 forward (same rounding points).
    assert_policy_close(out.policy_logits, ref16[0], atol=POLICY_ATOL, rtol=POLICY_RTOL)
    # Argmax agreement both ways: raw (the picked moves are identical) and tolerance-aware
    # (the picked move's reference logit is within POLICY_ATOL of the reference maximum),
    # beside the reference's own BF16-vs-FP32 raw agreement for scale.
    raw = argmax_agreement(out.policy_logits, ref16[0], tol=0.0)
    tol_aware = argmax_agreement(out.policy_logits, ref16[0])
    own_raw = argmax_agreement(ref16[0], ref32[0], tol=0.0)
    print(f"d{d}x{depth} B={batch}: argmax raw {raw:.4f}, tolerance-aware {tol_aware:.4f}; "
          f"reference BF16 vs FP32 raw {own_raw:.4f}")
    assert tol_aware >= ARGMAX_AGREEMENT
    torch.testing.assert_close(
        torch.softmax(out.wdl_logits.cpu(), -1), oracle.wdl_probabilities(ref16[1]),
        atol=WDL_PROB_ATOL, rtol=0,
    )
    torch.testing.assert_close(out.moves_left.cpu(), ref16[2], atol=POLICY_ATOL, rtol=POLICY_RTOL)
    # Against the FP32 portable model: no further from it than the reference's own BF16
    # rounding is (BF16 vs FP32 argmax agreement is itself ~96 % at d512 x 12).
    own = (ref16[0] - ref32[0]).abs().max().item()
    ours = (out.policy_logits.cpu() - ref32[0]).abs().max().item()
    assert ours <= 1.5 * own + 2e-3, (ours, own)
    wdl_gap = (torch.softmax(out.wdl_logits.cpu(), -1) - oracle.wdl_probabilities(ref32[1])).abs().max()
    assert wdl_gap <= WDL_PROB_ATOL


def test_dense_model_at_c4_depth_is_as_close_as_bf16_allows() -> None:
    """d1024 x 16 (the c4 tower). Through 16 BF16 layers the logits depend on FP32
    accumulation order: on this case two CPU runs of the reference's exact BF16 rounding
    points that differ only in matmul accumulation (FP32 vs FP64) already differ by up to
    0.043, with only half of the positions inside the 2e-2 / 1e-2 bar in every logit, and
    the reference's BF16 path sits up to 0.043 from its FP32 form. The elementwise bar
    against the BF16 restatement is therefore not a property any implementation with a
    different accumulation order has at this depth. The test requires instead that the
    GPU forward is no further from the FP32 portable model (the function both approximate)
    than the reference's own BF16 path is, in max-abs, in the fraction of logits beyond the
    bar, in WDL probabilities and moves-left, and that it agrees with the BF16 reference's
    best move (tolerance-aware) on >= 99.5 % of positions."""
    from oracle import dense as oracle

    d, depth, ratio, batch = 1024, 16, 3.0, 512
    weights, _, planes = _dense_case(d, depth, ratio, batch)
    model = dense_model(weights, d=d, depth=depth, ratio=ratio).cuda()
    out = model(planes.cuda())
    torch.cuda.synchronize()
    ref16 = oracle.forward(weights, planes, depth=depth, mode="bf16")
    ref32 = oracle.forward(weights, planes, depth=depth, mode="fp32")
    ours = out.policy_logits.cpu()

    def beyond(a, b):
        return float(((a - b).abs() > POLICY_ATOL + POLICY_RTOL * b.abs()).float().mean())

    own_max = float((ref16[0] - ref32[0]).abs().max())
    our_max = float((ours - ref32[0]).abs().max())
    own_beyond, our_beyond = beyond(ref16[0], ref32[0]), beyond(ours, ref32[0])
    sm = lambda t: torch.softmax(t.float(), -1)  # noqa: E731
    own_wdl = float((sm(ref16[1]) - sm(ref32[1])).abs().max())
    our_wdl = float((sm(out.wdl_logits.cpu()) - sm(ref32[1])).abs().max())
    own_ml = float((ref16[2] - ref32[2]).abs().max())
    our_ml = float((out.moves_left.cpu() - ref32[2]).abs().max())
    tol_aware = argmax_agreement(out.policy_logits, ref16[0])
    print(f"d1024x16 B={batch} vs FP32: max {our_max:.4f} (reference BF16 {own_max:.4f}), beyond the bar "
          f"{our_beyond:.4f} ({own_beyond:.4f}), wdl {our_wdl:.4f} ({own_wdl:.4f}), moves-left {our_ml:.4f} "
          f"({own_ml:.4f}); vs BF16: max {float((ours - ref16[0]).abs().max()):.4f}, beyond "
          f"{beyond(ours, ref16[0]):.4f}, argmax raw {argmax_agreement(ours, ref16[0], tol=0.0):.4f}, "
          f"tolerance-aware {tol_aware:.4f}")
    assert our_max <= 1.1 * own_max + 2e-3
    assert our_beyond <= 1.2 * own_beyond + 1e-3
    assert our_wdl <= 1.2 * own_wdl + 1e-3
    assert our_ml <= 1.2 * own_ml + 2e-3
    assert tol_aware >= ARGMAX_AGREEMENT


def test_input_layouts_agree() -> None:
    from ce4b200 import synthetic

    d, depth, ratio, batch = 128, 2, 3.0, 200
    weights = synthetic.make_dense_weights(d_model=d, depth=depth, hidden_dim=int(d * ratio), seed=4)
    lc0 = synthetic.make_lc0_planes(batch, 9, aux_constant=True)
    planes = synthetic.lc0_to_dense(lc0).cuda()
    packed, scalars = synthetic.lc0_to_packed(lc0)
    model = dense_model(weights, d=d, depth=depth, ratio=ratio).cuda()
    a = model(planes.clone())
    b = model(planes.clone().bfloat16())
    c = model.forward_packed(packed.cuda(), scalars.cuda())
    e = model.forward_lc0(synthetic.lc0_planes_tensor(lc0).cuda(), wdl_probs=False)
    for other in (b, c, e):
        torch.testing.assert_close(other.policy_logits, a.policy_logits, atol=0, rtol=0)
        torch.testing.assert_close(other.wdl_logits, a.wdl_logits, atol=0, rtol=0)
        torch.testing.assert_close(other.moves_left, a.moves_left, atol=0, rtol=0)


def test_forward_normalizes_rule50_in_place_like_reference() -> None:
    from ce4b200 import synthetic

    weights = synthetic.make_dense_weights(d_model=64, depth=1, hidden_dim=128, seed=2)
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(3, 5)).cuda()
    before = planes.clone()
    model = dense_model(weights, d=64, depth=1, ratio=2.0).cuda()
    model(planes)
    torch.cuda.synchronize()
    expected = before.clone()
    expected[:, 109] /= 99.0
    torch.testing.assert_close(planes, expected)


@pytest.mark.parametrize(
    "d,depth,ratio,batch",
    [
        (512, 12, 3.0, 4096),  # the benchmark shape
        (512, 3, 3.0, 200),  # ragged last row block
        (1024, 2, 3.0, 300),  # four 256-column input tiles per row block
        (256, 4, 3.0, 300),
        (128, 2, 3.0, 7),  # 128-column input tiles, one partial row block
        (512, 2, 2.0, 300),  # h = 1024: down tiles in 64-deep stages (h % 96 != 0), K split
        (512, 2, 2.0, 2048),  # same, one K part per down tile
    ],
)
def test_persistent_forward_matches_folded_restatement(d: int, depth: int, ratio: float, batch: int) -> None:
    """Dense BF16 models run as one persistent kernel that folds each RMSNorm weight into
    the next linear (bf16(W * diag(w))) and scales the FP32 accumulator by the row's
    rsqrt(mean(x^2) + eps). Against a CPU restatement of exactly that arithmetic only the
    FP32 accumulation order differs, so the bound is tighter than against the reference's
    rounding points (test_dense_model_matches_oracle)."""

    from oracle import dense as oracle

    weights, _, planes = _dense_case(d, depth, ratio, batch)
    model = dense_model(weights, d=d, depth=depth, ratio=ratio).cuda()
    model.set_latency_path(False)  # small batches too: this test is about the persistent kernel
    out = model(planes.cuda())
    torch.cuda.synchronize()
    policy, wdl, ml = oracle.forward(weights, planes, depth=depth, mode="bf16", fold_norm=True)
    ref_policy = oracle.forward(weights, planes, depth=depth, mode="bf16")[0]
    ours = out.policy_logits.cpu()
    mean_folded = float((ours - policy).abs().mean())
    mean_ref = float((ours - ref_policy).abs().mean())
    # The restatement captures the kernel's arithmetic: the output sits closer to it than
    # to the reference's rounding points (both within one BF16 ulp of the logits per row).
    assert mean_folded <= mean_ref, (mean_folded, mean_ref)
    assert float((ours - policy).abs().max()) <= 2e-2
    assert argmax_agreement(out.policy_logits, policy) >= ARGMAX_AGREEMENT
    torch.testing.assert_close(out.moves_left.cpu(), ml, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("d,depth,batch", [(512, 3, 1000), (256, 2, 300)])
def test_persistent_forward_is_deterministic(d: int, depth: int, batch: int) -> None:
    """Both tower kernels fix every summation order (K-split partial tiles are a sum of two
    terms), so repeated forwards give bit-identical outputs. (The forward normalises its
    input planes in place, as the reference's does, so every call gets a fresh copy.)"""

    weights, _, planes = _dense_case(d, depth, 3.0, batch)
    model = dense_model(weights, d=d, depth=depth, ratio=3.0).cuda()
    x = planes.cuda()
    first = model(x.clone())
    torch.cuda.synchronize()
    ref = [t.clone() for t in (first.policy_logits, first.wdl_logits, first.moves_left)]
    for _ in range(3):
        again = model(x.clone())
        torch.cuda.synchronize()
        for a, b in zip(ref, (again.policy_logits, again.wdl_logits, again.moves_left)):
            assert torch.equal(a, b)


def test_persistent_forward_schedules_and_batch_size() -> None:
    """The persistent forward picks a schedule by batch size: small batches (at most ~9 row
    blocks) split the input tiles into 8 K parts and the down tiles into 4, larger ones use
    2 and 1, and large ones make the down tiles 256 columns wide. Within a K split the
    parts are summed in fixed order and the tile width only assigns columns to CTAs, so a
    position's outputs are the same bits for every batch with the same K split; across
    K splits they agree to FP32 accumulation order."""

    torch.manual_seed(0)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    big = 128 * sms + 256  # 256-wide down tiles: (big / 128) * (512 / 256) >= 2 * SMs
    weights, _, planes = _dense_case(512, 2, 3.0, big)
    model = dense_model(weights, d=512, depth=2, ratio=3.0).cuda()
    x = planes.cuda()

    def run(rows):
        out = model(x[:rows].clone())
        torch.cuda.synchronize()
        return [t[:200].clone() for t in (out.policy_logits, out.wdl_logits, out.moves_left)]

    small_a, small_b = run(200), run(700)  # 8 input / 4 down K parts
    medium_a, medium_b = run(1536), run(2048)  # 2 / 1, 128-wide down tiles
    wide = run(big)  # 2 / 1, 256-wide down tiles
    for a, b in zip(small_a, small_b):
        assert torch.equal(a, b)
    for a, b, c in zip(medium_a, medium_b, wide):
        assert torch.equal(a, b)
        assert torch.equal(a, c)
    for a, b in zip(small_a, medium_a):
        torch.testing.assert_close(a.float(), b.float(), atol=2e-2, rtol=1e-2)
