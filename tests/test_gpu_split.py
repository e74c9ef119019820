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
    if folded:
        monkeypatch.setenv("BQ4_FORCE_FOLDED", "1")
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
