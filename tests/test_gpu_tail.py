"""GPU: the split-K tail launch.

When whole tiles leave the last wave partial, the planner can run the full
waves as one launch and the remaining tiles as a second launch in which each
tile is cut into K ranges, one cluster of CTAs per tile reducing through the
workspace (opt-in, BQ4_SPLIT_TAIL=1: measured no faster).  Checked here:

- the planner picks it for the c1 shape (152 tiles on 148 SMs: 4 tail tiles);
- results match a float64 reference of the same staging, tightly;
- they match whole tiles (BQ4_NO_TAIL=1) up to summation order;
- repeated calls give the same bits;
- f16 activations read in place and f16 outputs at a row pitch give the bits
  of the f32 path.
"""
import pytest
import torch

from burn_image_b200 import _lib as L
from burn_image_b200 import q4

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _problem(M, K, N, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    words = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device=DEV,
                          dtype=torch.int64).to(torch.int32).contiguous()
    scales = (torch.rand((K // 128, N), generator=g, device=DEV) * 0.019 + 0.001).contiguous()
    x = torch.randn((M, K), generator=g, device=DEV)
    bias = torch.randn(N, generator=g, device=DEV) * 0.02
    return q4.PreparedQ4Weight(words, scales, K, N, 128, L.LAYOUT_ROW, DEV), scales, x, bias


def _rel(a, b):
    return (torch.linalg.norm(a.double() - b.double()) / torch.linalg.norm(b.double())).item()


@pytest.fixture(autouse=True)
def _split_tail(monkeypatch):
    monkeypatch.setenv("BQ4_SPLIT_TAIL", "1")


def test_tail_plan_and_results(monkeypatch):
    M, K, N = 512, 2560, 9728  # c1: 2 x 76 tiles of 256 tokens
    pw, scales, x, bias = _problem(M, K, N, seed=3)
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    plan = pw.plan_info(M)
    tiles = 2 * (N // 128)
    assert plan["exact"] == 0 and plan["sk_tiles"] == 0
    assert plan["tail_tiles"] == tiles % sms and plan["tail_split"] >= 2
    y = pw.linear(x, bias, L.ACT_GELU_TANH)
    y2 = pw.linear(x, bias, L.ACT_GELU_TANH)
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert torch.equal(y, y2)
    # the folded staging in float64: f16(x) . f16(q * f16(s)) + bias, then GELU-tanh
    W = pw.dequantize().double()
    s_rep = scales.double().repeat_interleave(128, 0)
    Wf = ((W / s_rep).half() * scales.half().repeat_interleave(128, 0)).double()
    ref = torch.nn.functional.gelu(x.half().double() @ Wf + bias.double(), approximate="tanh")
    assert _rel(y, ref) < 5e-5
    monkeypatch.setenv("BQ4_NO_TAIL", "1")
    assert pw.plan_info(M)["tail_tiles"] == 0
    y_whole = pw.linear(x, bias, L.ACT_GELU_TANH)
    torch.cuda.synchronize()
    assert _rel(y, y_whole) < 1e-5  # the same sums, split in K and added


def test_tail_with_f16_activations_and_rows():
    # the chained entry point (f16 x, f16 y at a row pitch) on a tail plan
    M, K, N = 512, 2560, 9728
    pw, _, x, bias = _problem(M, K, N, seed=5)
    assert pw.plan_info(M)["tail_tiles"] > 0
    out = torch.zeros((M, N + 64), dtype=torch.float16, device=DEV)
    pw.linear_ex(x.half(), bias, out=out[:, :N])
    y32 = pw.linear(x, bias)
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert torch.equal(out[:, :N], y32.half())
    assert out[:, N:].abs().sum().item() == 0.0
