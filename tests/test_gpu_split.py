"""GPU: work partitioning (split-K and multi-wave persistent scheduling) must
not change results.  Every plan the scheduler can pick -- forced split
factors, both kernels, repeated calls -- is compared with a float64 PyTorch
reference of the same f16 operand staging at a tight tolerance."""
import pytest
import torch

from burn_image_b200 import _lib as L
from burn_image_b200 import q4

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def problem(M, K, N, block):
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N + K)
    words = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device=DEV,
                          dtype=torch.int64).to(torch.int32).contiguous()
    scales = (torch.rand((K // block, N), generator=g, device=DEV) * 0.019 + 0.001).contiguous()
    x = torch.randn((M, K), generator=g, device=DEV)
    return words, scales, x


@pytest.mark.parametrize("folded", [False, True])
@pytest.mark.parametrize("S", [1, 2, 4, 8])
@pytest.mark.parametrize("M,K,N", [(256, 9728, 2560), (512, 4096, 4096), (4352, 12288, 3072)])
def test_partitioning_does_not_change_results(M, K, N, S, folded, monkeypatch):
    monkeypatch.setenv("BQ4_FORCE_KSPLIT", str(S))
    q4.set_numerics(L.NUMERICS_FOLDED if folded else L.NUMERICS_EXACT)
    try:
        _check_partitioning(M, K, N, folded)
    finally:
        q4.set_numerics(L.NUMERICS_AUTO)


def _check_partitioning(M, K, N, folded):
    block = 128
    words, scales, x = problem(M, K, N, block)
    pw = q4.PreparedQ4Weight(words, scales, K, N, block, L.LAYOUT_ROW, DEV)
    W = pw.dequantize().double()
    if folded:  # f16(q * f16(scale))
        s_rep = scales.double().repeat_interleave(block, 0)
        W = ((W / s_rep).half() * scales.half().repeat_interleave(block, 0)).double()
    ref = x.half().double() @ W
    first = None
    for _ in range(3):
        y = pw.linear(x)
        torch.cuda.synchronize()
        q4.poll_device_error()
        rf = (torch.linalg.norm(y.double() - ref) / torch.linalg.norm(ref)).item()
        assert rf < 5e-5, f"rel_frob {rf}"  # f32 accumulation over K <= 12288
        if first is None:
            first = y.clone()
        else:
            assert torch.equal(first, y)


@pytest.mark.parametrize("M,K,N", [(256, 2560, 512), (4352, 3072, 1024)])
def test_numerics_modes_both_within_tolerance(M, K, N):
    """EXACT and FOLDED staging (and AUTO) all meet the 5e-3 relative
    Frobenius bound against a float64 reference of the exact weights."""
    words, scales, x = problem(M, K, N, 128)
    pw = q4.PreparedQ4Weight(words, scales, K, N, 128, L.LAYOUT_ROW, DEV)
    ref = x.double() @ pw.dequantize().double()
    errs = {}
    for mode in (L.NUMERICS_EXACT, L.NUMERICS_FOLDED, L.NUMERICS_AUTO):
        q4.set_numerics(mode)
        try:
            y = pw.linear(x)
            torch.cuda.synchronize()
        finally:
            q4.set_numerics(L.NUMERICS_AUTO)
        errs[mode] = (torch.linalg.norm(y.double() - ref) / torch.linalg.norm(ref)).item()
        assert errs[mode] <= 5e-3
    assert errs[L.NUMERICS_EXACT] < errs[L.NUMERICS_FOLDED]
    print(f"numerics M{M}: exact {errs[1]:.3e} folded {errs[2]:.3e} auto {errs[0]:.3e}")


@pytest.mark.parametrize("M,K,N", [(4352, 12288, 3072), (1024, 3072, 9216), (300, 1024, 640)])
def test_unit_order_does_not_change_results(M, K, N, monkeypatch):
    """N-tile-fastest and M-tile-fastest unit orders only reschedule whole
    tiles, so the outputs are bit-identical.  (With a stream-K tail the order
    also decides which tiles are cut in two, which moves rounding; that plan
    is compared with whole tiles in test_gpu_streamk.py.)"""
    monkeypatch.setenv("BQ4_NO_STREAMK", "1")
    words, scales, x = problem(M, K, N, 128)
    pw = q4.PreparedQ4Weight(words, scales, K, N, 128, L.LAYOUT_ROW, DEV)
    outs = []
    for order in ("0", "1"):
        monkeypatch.setenv("BQ4_FORCE_NFAST", order)
        outs.append(pw.linear(x))
        torch.cuda.synchronize()
        q4.poll_device_error()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("M,K,N,S", [(1024, 3072, 1024, 1), (4352, 3072, 3072, 1), (256, 2560, 2560, 5), (600, 1536, 768, 2)])
def test_exact_with_a_in_tmem_at_256_tokens(M, K, N, S, monkeypatch):
    """Exact numerics with the dequantized weight tile in TMEM and 256-token
    tiles (BQ4_EXACT_TA256=1: one TMEM partial, drained by the scaler before
    the next K block's MMAs): the same products and summation order as the
    plan with A in shared memory, so the results agree to the last bits."""
    block = 128
    words, scales, x = problem(M, K, N, block)
    pw = q4.PreparedQ4Weight(words, scales, K, N, block, L.LAYOUT_ROW, DEV)
    ref = x.half().double() @ pw.dequantize().double()
    monkeypatch.setenv("BQ4_FORCE_KSPLIT", str(S))
    monkeypatch.setenv("BQ4_FORCE_BT", "256")
    monkeypatch.setenv("BQ4_NO_STREAMK", "1")
    q4.set_numerics(L.NUMERICS_EXACT)
    try:
        smem = pw.linear(x).clone()
        monkeypatch.setenv("BQ4_EXACT_TA256", "1")
        info = pw.plan_info(M)
        assert info["exact"] == 1 and info["ta"] == 1 and info["bt"] == 256, info
        a = pw.linear(x).clone()
        b = pw.linear(x).clone()
    finally:
        q4.set_numerics(L.NUMERICS_AUTO)
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert torch.equal(a, b)
    rf = (torch.linalg.norm(a.double() - ref) / torch.linalg.norm(ref)).item()
    assert rf < 5e-5, f"rel_frob {rf}"
    rs = (torch.linalg.norm(a.double() - smem.double()) / torch.linalg.norm(smem.double())).item()
    assert rs < 1e-6, f"rel to the shared-memory plan {rs}"
