"""GPU: the packed-F16 kernels (patches/burn-cubecl-0.21.0/src/kernel/packed_f16.rs)
against the oracle and the reference's own golden vectors.

- widening: all 65536 binary16 patterns bit-exact; strided views;
- row select: the reference's golden case, both kernel paths, and an index
  out of range (zero row, BQ4_EINVAL_ARG);
- rhs matmul (kind::tf32): the reference's golden case exactly, random
  shapes within 5e-3 of the f64 oracle and within 2e-5 of an f64 reference
  fed the same tf32 activations, the prepared weight with bias and GELU, the
  reference's throughput-smoke value;
- conv2d (implicit GEMM for stride 1, gathered rows otherwise): the golden
  case exactly, padding / dilation / stride / ragged channel counts against
  the oracle, prepared == one-shot bit for bit, the throughput-smoke value.
"""
import numpy as np
import pytest
import torch

import oracle as O
from burn_image_b200 import _lib as L
from burn_image_b200 import f16 as F
from burn_image_b200 import q4
from burn_image_b200.q4 import Bq4Error

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _h(values, shape=None):
    t = torch.tensor(np.asarray(values, np.float32), dtype=torch.float16, device=DEV)
    return t.reshape(shape) if shape is not None else t


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _tf32(x: np.ndarray, mode: str) -> np.ndarray:
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    if mode == "rna":
        b = b + 0x1000
    return (b & 0xFFFFE000).astype(np.uint32).view(np.float32).reshape(x.shape)


def test_widen_exhaustive_bit_exact():
    h = torch.arange(1 << 16, dtype=torch.int32).to(torch.int16).view(torch.float16).to(DEV)
    got = F.packed_f16_to_f32(h)
    torch.cuda.synchronize()
    exp = O.f16_widen_bits(np.arange(1 << 16, dtype=np.uint32).astype(np.uint16))
    assert np.array_equal(got.cpu().view(torch.int32).numpy().view(np.uint32), exp)


def test_widen_strided_views():
    t = (torch.randn((6, 10, 12), device=DEV) * 30).half()
    for v in (t.transpose(0, 2), t[:, 2:9:3, 1:], t[1], t.permute(1, 0, 2)[3:], t[..., 5]):
        got = F.packed_f16_to_f32(v)
        torch.cuda.synchronize()
        exp = O.f16_widen_bits(_bits(v)).view(np.float32)
        assert np.array_equal(got.cpu().numpy().view(np.uint32), exp.view(np.uint32)), v.shape


def test_select_rows():
    # packed_f16.rs test :828-846
    table = _h([1.0, 2.0, 3.0, 4.0, 5.0, 6.0, -1.0, -2.0, -3.0, 7.0, 8.0, 9.0], (4, 3))
    got = F.packed_f16_select_rows(table, 0, torch.tensor([2, 0], dtype=torch.int32, device=DEV))
    assert got.cpu().numpy().ravel().tolist() == [-1.0, -2.0, -3.0, 1.0, 2.0, 3.0]
    for cols in (24, 13):  # 16-byte rows and the scalar path
        tab = (torch.randn((100, cols), device=DEV) * 4).half()
        idx = torch.randint(0, 100, (57,), dtype=torch.int32, device=DEV)
        got = F.packed_f16_select_rows(tab, 0, idx)
        torch.cuda.synchronize()
        exp = O.f16_widen_bits(_bits(tab)[idx.cpu().numpy()])
        assert np.array_equal(got.cpu().numpy().view(np.uint32), exp)
    bad = F.packed_f16_select_rows(tab, 0, torch.tensor([1, 100, -1], dtype=torch.int32, device=DEV))
    torch.cuda.synchronize()
    with pytest.raises(Bq4Error, match="EINVAL_ARG"):
        q4.poll_device_error()
    assert bad[1:].abs().sum().item() == 0.0
    with pytest.raises(Bq4Error, match="EINVAL_ARG"):
        F.packed_f16_select_rows(tab, 1, idx)


def test_rhs_matmul_golden():
    # packed_f16.rs test :791-826: checkpoint [4, 3] used through its transposed view
    lhs = torch.tensor([[1.0, 2.0, 3.0], [-1.0, 0.5, 2.0]], device=DEV)
    rhs = _h([1.0, 0.0, 2.0, 0.0, 1.0, -1.0, 2.0, -1.0, 0.5, -1.0, 2.0, 1.0], (4, 3)).t()
    out = F.packed_f16_rhs_matmul(lhs, rhs)
    torch.cuda.synchronize()
    assert out.cpu().numpy().ravel().tolist() == [7.0, -1.0, 1.5, 6.0, 3.0, -1.5, -1.5, 4.0]


def _check_matmul(x, rhs, got):
    K, N = rhs.shape
    bits = _bits(rhs)  # contiguous [K][N]
    xn = x.cpu().numpy().reshape(-1, K)
    ref = O.f16_matmul_f64(xn, bits, K, N, N, 1)
    g = got.cpu().numpy().reshape(-1, N)
    rel = O.rel_frobenius(g, ref)
    assert rel <= 5e-3, f"rel_frob {rel}, max_abs {np.abs(g - ref).max()}"
    # the same sums of tf32 activations in f64: only f32 accumulation differs
    tight = min(O.rel_frobenius(g, O.f16_matmul_f64(_tf32(xn, m), bits, K, N, N, 1)) for m in ("trunc", "rna"))
    assert tight <= 2e-5, f"rel vs tf32-staged reference {tight}"


# (M, K, N, stored): token tiles of 64/128/256 and split-K, K not a multiple of
# 4 (staged rows) or of 64 (zero chunks), N not a multiple of 128, both views
@pytest.mark.parametrize("M,K,N,stored", [(1, 64, 128, "kn"), (37, 70, 45, "nk"), (300, 512, 384, "nk"),
                                          (1000, 1000, 640, "kn"), (4352, 512, 1536, "kn")])
def test_rhs_matmul_against_oracle(M, K, N, stored):
    g = torch.Generator(device=DEV).manual_seed(M + K + N)
    x = torch.randn((M, K), generator=g, device=DEV)
    w = (torch.randn((K, N), generator=g, device=DEV) * K ** -0.5).half()
    rhs = w if stored == "kn" else w.t().contiguous().t()  # the [N, K] checkpoint's transposed view
    got = F.packed_f16_rhs_matmul(x, rhs)
    torch.cuda.synchronize()
    q4.poll_device_error()
    _check_matmul(x, w, got)


def test_prepared_weight_linear_with_epilogue():
    M, K, N = 260, 768, 1152
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn((M, K), generator=g, device=DEV)
    w = (torch.randn((N, K), generator=g, device=DEV) * K ** -0.5).half()  # stored [out, in]
    bias = torch.randn(N, generator=g, device=DEV)
    pw = F.PreparedF16Weight(w.t())
    assert pw.plan_info(M)["exact"] == 0
    y = pw.linear(x, bias, L.ACT_GELU_TANH)
    one = F.packed_f16_rhs_matmul(x, w.t())
    torch.cuda.synchronize()
    q4.poll_device_error()
    W = O.f16_widen_bits(_bits(w.t())).view(np.float32).reshape(K, N)
    ref = O.linear_f64(x.cpu().numpy(), W, bias.cpu().numpy(), O.ACT_GELU_TANH)
    assert O.rel_frobenius(y.cpu().numpy(), ref) <= 5e-3
    # the prepared weight without epilogue == the one-shot call
    assert torch.equal(pw.linear(x), one)
    # K % 4 != 0 through the prepared weight (rows re-pitched by the host mirror)
    w2 = (torch.randn((66, 40), generator=g, device=DEV) * 0.1).half()
    x2 = torch.randn((9, 66), generator=g, device=DEV)
    y2 = F.PreparedF16Weight(w2).linear(x2)
    _check_matmul(x2, w2, y2)


def test_wide_tiles(monkeypatch):
    # 256 x 256 tiles (two N tiles per token tile) once they fill a wave and the
    # K loop is 16+ stages (K >= 512); an odd N-tile count (1100 = 8.6 tiles)
    # pairs the last tile with a zero one
    M, K, N = 9000, 512, 1100
    g = torch.Generator(device=DEV).manual_seed(21)
    x = torch.randn((M, K), generator=g, device=DEV)
    w = (torch.randn((K, N), generator=g, device=DEV) * K ** -0.5).half()
    bias = torch.randn(N, generator=g, device=DEV)
    pw = F.PreparedF16Weight(w)
    plan = pw.plan_info(M)
    assert plan["wide"] == 1 and plan["bt"] == 256 and plan["ksplit"] == 1
    y = pw.linear(x, bias, L.ACT_SILU)
    torch.cuda.synchronize()
    q4.poll_device_error()
    W = O.f16_widen_bits(_bits(w)).view(np.float32).reshape(K, N)
    ref = O.linear_f64(x.cpu().numpy(), W, bias.cpu().numpy(), O.ACT_SILU)
    assert O.rel_frobenius(y.cpu().numpy(), ref) <= 5e-3
    # the same K order per output either way: bit-identical to 128-row tiles
    monkeypatch.setenv("BQ4_NO_WIDE", "1")
    assert pw.plan_info(M)["wide"] == 0
    assert torch.equal(y, pw.linear(x, bias, L.ACT_SILU))
    _check_matmul(x[:500], w, pw.linear(x[:500]))
    monkeypatch.delenv("BQ4_NO_WIDE")
    assert F.PreparedF16Weight(w[:384]).plan_info(M)["wide"] == 0  # K = 384: too short a K loop


def test_rhs_matmul_throughput_smoke_value():
    # packed_f16.rs :876-943 at its size: ones [4096, 4096] x f16(1/4096) -> 1 within 1e-3
    n = 4096
    lhs = torch.ones((n, n), device=DEV)
    rhs = torch.full((n, n), 1.0 / n, device=DEV).half().t()
    out = F.packed_f16_rhs_matmul(lhs, rhs)
    torch.cuda.synchronize()
    assert abs(out[0, 0].item() - 1.0) <= 1e-3
    assert out.min().item() == 1.0 and out.max().item() == 1.0  # 4096 * 2^-12, exact in f32


def test_conv2d_golden():
    # packed_f16.rs test :848-873
    x = torch.arange(1, 10, dtype=torch.float32, device=DEV).reshape(1, 1, 3, 3)
    w = _h([1.0, 0.0, 0.0, -1.0, 0.5, 0.5, 0.5, 0.5], (2, 1, 2, 2))
    b = torch.tensor([0.5, -1.0], device=DEV)
    out = F.packed_f16_conv2d(x, w, b, F.ConvOptions((1, 1), (0, 0), (1, 1), 1))
    torch.cuda.synchronize()
    assert out.cpu().numpy().ravel().tolist() == [-3.5, -3.5, -3.5, -3.5, 5.0, 7.0, 11.0, 13.0]


# (B, C, H, W, O, k, stride, padding, dilation)
CONV = [(1, 64, 20, 20, 128, 3, (1, 1), (1, 1), (1, 1)),     # VAE-like 3x3, padding 1
        (2, 16, 17, 13, 200, 3, (1, 1), (1, 1), (1, 1)),     # 16 channels (padded to 32), 200 outputs
        (1, 32, 9, 30, 64, 1, (1, 1), (0, 0), (1, 1)),       # 1x1
        (1, 48, 15, 15, 96, 3, (1, 1), (2, 2), (2, 2)),      # dilation 2
        (2, 24, 16, 16, 130, 3, (2, 2), (1, 1), (1, 1)),     # stride 2: gathered rows
        (1, 3, 33, 31, 64, 3, (2, 1), (1, 0), (1, 1)),       # RGB input, mixed strides
        (1, 32, 12, 12, 40, 3, (1, 1), (1, 1), (1, 1)),      # 9 x 32 = 288 K: a zero chunk
        (1, 512, 12, 12, 512, 3, (1, 1), (1, 1), (1, 1))]    # the mid-block width


@pytest.mark.parametrize("B,C,H,W,O_,k,stride,padding,dilation", CONV)
def test_conv2d_against_oracle(B, C, H, W, O_, k, stride, padding, dilation):
    g = torch.Generator(device=DEV).manual_seed(B * 1000 + C + O_ + k)
    x = torch.randn((B, C, H, W), generator=g, device=DEV)
    w = (torch.randn((O_, C, k, k), generator=g, device=DEV) * (C * k * k) ** -0.5).half()
    b = torch.randn(O_, generator=g, device=DEV)
    opt = F.ConvOptions(stride, padding, dilation, 1)
    pw = F.PreparedF16ConvWeight(w)
    got = pw.conv2d(x, b, opt)
    one = F.packed_f16_conv2d(x, w, b, opt)
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert torch.equal(got, one)
    wb = _bits(w).reshape(O_, C, k, k)
    xn = x.cpu().numpy()
    ref = O.f16_conv2d_f64(xn, wb, b.cpu().numpy(), stride, padding, dilation)
    gn = got.cpu().numpy()
    assert gn.shape == ref.shape
    rel = O.rel_frobenius(gn, ref)
    assert rel <= 5e-3, f"rel_frob {rel}, max_abs {np.abs(gn - ref).max()}"
    tight = O.rel_frobenius(gn, O.f16_conv2d_f64(_tf32(xn, "rna"), wb, b.cpu().numpy(), stride, padding, dilation))
    assert tight <= 2e-5, f"rel vs tf32-staged reference {tight}"


def test_conv2d_throughput_smoke_value():
    # packed_f16.rs :945-1026 at its size: 512 -> 512, 3x3, padding 1, 64 x 64,
    # weight f16(1/4608): the centre sample is 1 within 2e-3
    C, S = 512, 64
    x = torch.ones((1, C, S, S), device=DEV)
    w = torch.full((C, C, 3, 3), 1.0 / (C * 9), device=DEV).half()
    out = F.packed_f16_conv2d(x, w, None, F.ConvOptions((1, 1), (1, 1), (1, 1), 1))
    torch.cuda.synchronize()
    assert abs(out[0, 0, S // 2, S // 2].item() - 1.0) <= 2e-3
    # every interior position sees all 9 taps; the corners 4 of them
    assert abs(out[0, :, 1:-1, 1:-1] - out[0, 0, S // 2, S // 2]).max().item() <= 1e-6
    assert abs(out[0, 0, 0, 0].item() - 4.0 / 9.0 * out[0, 0, S // 2, S // 2].item()) <= 1e-5


def test_argument_checks():
    w = _h(np.ones(2 * 4 * 9), (2, 4, 3, 3))
    x = torch.ones((1, 4, 5, 5), device=DEV)
    with pytest.raises(Bq4Error, match="EUNSUPPORTED"):
        F.packed_f16_conv2d(x, w, None, F.ConvOptions((1, 1), (1, 1), (1, 1), 2))
    with pytest.raises(Bq4Error, match="EINVAL_SHAPE"):
        F.packed_f16_conv2d(x, w, None, F.ConvOptions((1, 1), (0, 0), (3, 3), 1))  # kernel beyond the input
    with pytest.raises(Bq4Error, match="EINVAL_SHAPE"):
        F.packed_f16_rhs_matmul(torch.ones((2, 5), device=DEV), _h(np.ones(12), (4, 3)))
    pw = F.PreparedF16Weight(_h(np.ones(64 * 128), (64, 128)))
    with pytest.raises(Bq4Error, match="EINVAL_ARG"):
        pw.linear_ex(torch.ones((4, 64), device=DEV).half())  # f16 activations: f32 only
    with pytest.raises(Bq4Error, match="EINVAL_ARG"):
        q4.linear_gated(pw, pw, torch.ones((4, 64), device=DEV))  # the gated pair takes packed-Q4 weights
    # a gated pair must share one prepared form: N-packed (pre-expanded) with row layout is refused
    K, N = 128, 128
    words = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), device=DEV, dtype=torch.int64).to(torch.int32)
    scales = torch.rand((K // 128, N), device=DEV) * 0.01 + 0.001
    row = q4.PreparedQ4Weight(words, scales, K, N, 128, L.LAYOUT_ROW, DEV)
    npk = q4.PreparedQ4Weight(torch.randint(-2 ** 31, 2 ** 31 - 1, (K, N // 8), device=DEV,
                                            dtype=torch.int64).to(torch.int32).contiguous(),
                              (torch.rand((K, N // 128), device=DEV) * 0.01 + 0.001).contiguous(),
                              K, N, 128, L.LAYOUT_NPACKED, DEV)
    with pytest.raises(Bq4Error, match="EINVAL_ARG"):
        q4.linear_gated(row, npk, torch.ones((4, K), device=DEV))
