"""GPU: the stream-K tail.

When whole tiles would leave the last wave partial, the planner deals the
last full wave plus the remainder to the CTAs as equal ranges of 128-K
stages (for exact numerics and the gated pair, where it measured faster).  A tile cut between CTAs c-1 and c is finished by c from the partial
c-1 published through the workspace.  Checked here:

- the planner picks the tail on such shapes;
- results match a float64 reference of the same f16 staging, tightly;
- they match the whole-tile plan (BQ4_NO_STREAMK=1) up to summation order;
- repeated calls give the same bits;
- f16 activations, whose flags are zeroed by their own kernel, agree bit for
  bit with f32 activations;
- the gated pair and a reduced SM budget work the same way;
- folded plans keep whole tiles.
"""
import numpy as np
import pytest
import torch

import oracle as O
from burn_image_b200 import _lib as L
from burn_image_b200 import q4

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _exact_numerics():
    # the tail is planned for exact numerics (and the gated pair); AUTO stages folded weights
    q4.set_numerics(L.NUMERICS_EXACT)
    yield
    q4.set_numerics(L.NUMERICS_AUTO)


def _problem(M, K, N, block, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    words = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device=DEV,
                          dtype=torch.int64).to(torch.int32).contiguous()
    scales = (torch.rand((K // block, N), generator=g, device=DEV) * 0.019 + 0.001).contiguous()
    x = torch.randn((M, K), generator=g, device=DEV)
    bias = torch.randn(N, generator=g, device=DEV) * 0.02
    return q4.PreparedQ4Weight(words, scales, K, N, block, L.LAYOUT_ROW, DEV), words, scales, x, bias


def _ref(pw, scales, x, block, exact):
    W = pw.dequantize().double()
    if not exact:  # f16(q * f16(scale))
        s_rep = scales.double().repeat_interleave(block, 0)
        W = ((W / s_rep).half() * scales.half().repeat_interleave(block, 0)).double()
    return x.half().double() @ W


def _rel(a, b):
    return (torch.linalg.norm(a.double() - b.double()) / torch.linalg.norm(b.double())).item()


# (M, K, N, block), exact numerics (set by the fixture: the plans that take the tail):
# 150 tiles; 64-blocks (two K blocks per stage); a longer K.  K is large
# enough on each that the planner's cost model prefers the stream-K tail.
SHAPES = [(200, 1024, 19200, 128), (200, 768, 19200, 64), (256, 2048, 19200, 128)]


@pytest.mark.parametrize("M,K,N,block", SHAPES)
def test_streamk_plan_and_results(M, K, N, block, monkeypatch):
    pw, words, scales, x, bias = _problem(M, K, N, block, seed=M + N + block)
    plan = pw.plan_info(M)
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    tiles = -(-M // plan["bt"]) * (N // 128)
    assert tiles > sms and tiles % sms
    assert plan["ksplit"] == 1 and plan["ta"] == 0 and plan["sk_tiles"] == sms + tiles % sms
    assert plan["dp_tiles"] == tiles - plan["sk_tiles"]
    ref = _ref(pw, scales, x, block, plan["exact"] == 1) + bias.double()
    first = None
    for _ in range(2):
        y = pw.linear(x, bias)
        torch.cuda.synchronize()
        q4.poll_device_error()
        assert _rel(y, ref) < 5e-5  # f32 accumulation of f16 products
        if first is None:
            first = y.clone()
        else:
            assert torch.equal(first, y)
    monkeypatch.setenv("BQ4_NO_STREAMK", "1")
    assert pw.plan_info(M)["sk_tiles"] == 0
    y_whole = pw.linear(x, bias)
    torch.cuda.synchronize()
    # the same sums cut in two and added: f32 accumulation rounding over K,
    # about sqrt(K) ulps (1.5e-6 measured at K = 2560)
    assert _rel(first, y_whole) < 1e-5


def test_streamk_against_the_oracle():
    # a small problem made multi-wave by an SM budget of 20 CTAs
    M, K, N, block = 200, 1024, 2816, 128
    pw, words, scales, x, bias = _problem(M, K, N, block, seed=5)
    q4.set_sm_budget(20)
    try:
        assert pw.plan_info(M)["sk_tiles"] > 0
        y = pw.linear(x, bias, L.ACT_GELU_TANH)
        torch.cuda.synchronize()
        q4.poll_device_error()
    finally:
        q4.set_sm_budget(0)
    y = y.cpu().numpy()
    W = O.unpack(words.cpu().numpy().view(np.uint32), scales.cpu().numpy(), K, N, block, O.LAYOUT_ROW)
    ref = O.linear_f64(x.cpu().numpy(), W, bias.cpu().numpy(), O.ACT_GELU_TANH)
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel <= 5e-3, f"rel_frob {rel}, max_abs {np.abs(y - ref).max()}"


def test_streamk_f16_activations_bit_identical():
    M, K, N, block = 200, 1024, 19200, 128
    pw, _, _, x, bias = _problem(M, K, N, block, seed=7)
    assert pw.plan_info(M)["sk_tiles"] > 0
    y32 = pw.linear(x, bias)
    y16in = pw.linear_ex(x.half(), bias)
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert torch.equal(y32, y16in)


def test_streamk_gated_pair():
    M, K, N, block = 256, 1024, 9728, 128  # 2 x 76 = 152 tiles of 128 tokens x 2 weights
    pg, _, sg, x, bg = _problem(M, K, N, block, seed=11)
    pu, _, su, _, bu = _problem(M, K, N, block, seed=12)
    plan = pg.plan_info(M, gated=True)
    assert plan["sk_tiles"] > 0 and plan["bt"] == 128
    exact = plan["exact"] == 1
    g = _ref(pg, sg, x, block, exact) + bg.double()
    u = _ref(pu, su, x, block, exact) + bu.double()
    ref = g * torch.sigmoid(g) * u
    y = q4.linear_gated(pg, pu, x, bg, bu)
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert _rel(y, ref) < 5e-5


def test_streamk_under_an_sm_budget():
    M, K, N, block = 200, 2560, 19200, 128
    pw, _, scales, x, _ = _problem(M, K, N, block, seed=13)
    q4.set_sm_budget(100)  # 150 tiles over 100 CTAs: the last wave plus the rest dealt
    try:
        plan = pw.plan_info(M)
        tiles = -(-M // plan["bt"]) * (N // 128)
        assert plan["grid"] == 100 and plan["sk_tiles"] == 100 + tiles % 100
        assert plan["dp_tiles"] == tiles - plan["sk_tiles"]
        y = pw.linear(x)
        torch.cuda.synchronize()
        q4.poll_device_error()
    finally:
        q4.set_sm_budget(0)
    assert _rel(y, _ref(pw, scales, x, block, plan["exact"] == 1)) < 5e-5


def test_folded_plans_keep_whole_tiles(monkeypatch):
    M, K, N = 512, 2560, 9728  # folded: 256-token TMEM-operand tiles, 152 of them
    q4.set_numerics(L.NUMERICS_FOLDED)
    pw, *_ = _problem(M, K, N, 128, seed=17)
    plan = pw.plan_info(M)
    assert plan["exact"] == 0 and plan["sk_tiles"] == 0
    monkeypatch.setenv("BQ4_FORCE_BT", "128")  # folded 128-token tiles, A in shared memory
    plan = pw.plan_info(M)
    assert plan["ta"] == 0 and plan["sk_tiles"] == 0
