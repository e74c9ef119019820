"""GPU: QK-norm + RoPE (the step between the q/k projections and attention,
crates/burn_boogu/src/model/attention.rs:114-133, 916-928).

- bq4_qk_norm_rope (standalone, any even head_dim) against the oracle, and on
  the reference's own fused-preparation fixture (native_flash.rs:2897-2960)
  at that test's bar, max-abs <= 1e-6;
- bq4_linear_qk_norm_rope: the q/k/v projection with the norm and rotation
  in the GEMM epilogue (head_dim 128) on each kernel variant that carries
  it, and through the standalone kernel (head_dim 120, the real model's),
  against the oracle (linear in f64, then the norm/rotation) within 5e-3 and
  against a float64 reference of the same f16 staging within 5e-5; the fused
  result against the unfused composition within 1e-5.
"""
import numpy as np
import pytest
import torch

import oracle as O
from burn_image_b200 import _lib as L
from burn_image_b200 import q4
from burn_image_b200.q4 import Bq4Error

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
EPS = 1.0e-5


def _tables(M, hd, seed):
    rng = np.random.default_rng(seed)
    ids = np.stack([np.zeros(M, np.int64), rng.integers(0, 64, M), rng.integers(0, 64, M)], 1)
    third = hd // 3 // 2 * 2
    axes = [hd - 2 * third, third, third]
    cos, sin = O.rope_tables(ids, axes, 10000.0)
    return torch.from_numpy(cos).to(DEV), torch.from_numpy(sin).to(DEV)


@pytest.mark.parametrize("hd,heads,dtype_in,dtype_out", [(120, 5, torch.float32, torch.float32),
                                                         (128, 3, torch.float32, torch.float16),
                                                         (64, 4, torch.float16, torch.float32),
                                                         (256, 2, torch.float16, torch.float16)])
def test_standalone_against_oracle(hd, heads, dtype_in, dtype_out):
    M = 37
    g = torch.Generator(device=DEV).manual_seed(hd + heads)
    x = torch.randn((M, heads * hd + 8), generator=g, device=DEV) * 2.0  # row pitch wider than the heads
    xin = x.to(dtype_in)
    gamma = torch.rand(hd, generator=g, device=DEV) + 0.5
    cos, sin = _tables(M, hd, hd)
    y = q4.qk_norm_rope(xin, heads, hd, gamma, EPS, cos, sin, out_dtype=dtype_out)
    torch.cuda.synchronize()
    ref = O.qk_norm_rope_f64(xin.float().cpu().numpy(), heads, hd, gamma.cpu().numpy(), EPS, cos.cpu().numpy(),
                             sin.cpu().numpy())
    err = np.abs(y.float().cpu().numpy() - ref).max()
    bound = 5e-6 if dtype_out == torch.float32 else 4e-3  # f32 rounding / one f16 rounding of |y| < 4
    assert err <= bound, f"max_abs {err}"


def test_standalone_in_place_and_without_rope():
    M, heads, hd = 20, 3, 120
    x = torch.randn((M, heads * hd), device=DEV)
    ref = O.qk_norm_rope_f64(x.cpu().numpy(), heads, hd, None, EPS)
    q4.qk_norm_rope(x, heads, hd, None, EPS, out=x)  # in place, no gamma, no rotation
    torch.cuda.synchronize()
    assert np.abs(x.cpu().numpy() - ref).max() <= 5e-6


def test_standalone_meets_reference_fixture_bar():
    # native_flash.rs:2897-2960 (inputs from :2697-2710), the query tensor, head_dim 120
    hd, heads = 120, 4
    idx = np.arange(heads * 3 * hd)
    xq = ((((idx + 31) * 19 + 7) % 53 - 26.0) / 17.0).astype(np.float32).reshape(1, heads, 3, hd)
    gi = np.arange(hd)
    gamma = (((((gi + 43) * 19 + 7) % 53 - 26.0) / 17.0).astype(np.float32) * np.float32(0.25) + np.float32(1.0))
    phase = (((np.arange(3 * hd) // 2) % 17).astype(np.float32) / np.float32(19.0)).reshape(3, hd)
    cos, sin = np.cos(phase), np.sin(phase)
    x = xq.transpose(0, 2, 1, 3).reshape(3, heads * hd)
    expected = O.qk_norm_rope_f64(x, heads, hd, gamma, EPS, cos, sin)  # pinned to that test's composition
    y = q4.qk_norm_rope(torch.from_numpy(x).to(DEV), heads, hd, torch.from_numpy(gamma).to(DEV), EPS,
                        torch.from_numpy(cos).to(DEV), torch.from_numpy(sin).to(DEV))
    torch.cuda.synchronize()
    assert np.abs(y.cpu().numpy() - expected).max() <= 1.0e-6


def _projection(M, K, hq, hk, hv, hd, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    N = (hq + hk + hv) * hd
    words = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device=DEV,
                          dtype=torch.int64).to(torch.int32).contiguous()
    scales = (torch.rand((K // 128, N), generator=g, device=DEV) * 0.019 + 0.001).contiguous()
    pw = q4.PreparedQ4Weight(words, scales, K, N, 128, L.LAYOUT_ROW, DEV)
    x = torch.randn((M, K), generator=g, device=DEV)
    bias = torch.randn(N, generator=g, device=DEV) * 0.02
    gq = torch.rand(hd, generator=g, device=DEV) + 0.5
    gk = torch.rand(hd, generator=g, device=DEV) + 0.5
    cos, sin = _tables(M, hd, seed)
    return pw, words, scales, x, bias, gq, gk, cos, sin


def _norm_sections(lin, hq, hk, hd, gq, gk, cos, sin):
    out = lin.copy()
    c, s = cos.cpu().numpy(), sin.cpu().numpy()
    out[:, :hq * hd] = O.qk_norm_rope_f64(lin[:, :hq * hd], hq, hd, gq.cpu().numpy(), EPS, c, s)
    out[:, hq * hd:(hq + hk) * hd] = O.qk_norm_rope_f64(lin[:, hq * hd:(hq + hk) * hd], hk, hd, gk.cpu().numpy(),
                                                       EPS, c, s)
    return out


# (M, K, hq, hk, hv, hd): 256-token tiles (M = 200, 300), 128-token tiles (M <= 64),
# folded TMEM-operand tiles (M > 256), and head_dim 120 (linear + standalone kernel)
@pytest.mark.parametrize("M,K,hq,hk,hv,hd", [(200, 512, 4, 2, 2, 128), (60, 512, 3, 3, 2, 128),
                                             (300, 1024, 4, 2, 2, 128), (77, 512, 4, 2, 2, 120)])
def test_projection_against_oracle(M, K, hq, hk, hv, hd):
    pw, words, scales, x, bias, gq, gk, cos, sin = _projection(M, K, hq, hk, hv, hd, seed=M + K + hd)
    y = pw.linear_qk_norm_rope(x, hq, hk, hd, bias, gq, gk, EPS, cos, sin)
    torch.cuda.synchronize()
    q4.poll_device_error()
    N = (hq + hk + hv) * hd
    W = O.unpack(words.cpu().numpy().view(np.uint32), scales.cpu().numpy(), K, N, 128, O.LAYOUT_ROW)
    lin = O.linear_f64(x.cpu().numpy(), W, bias.cpu().numpy())
    ref = _norm_sections(lin, hq, hk, hd, gq, gk, cos, sin)
    got = y.cpu().numpy()
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel <= 5e-3, f"rel_frob {rel}, max_abs {np.abs(got - ref).max()}"
    # tight: the same f16 activation staging in float64 (exact or folded weights, as planned)
    exact = pw.plan_info(M)["exact"] == 1
    Wt = pw.dequantize().double()
    if not exact:
        s_rep = scales.double().repeat_interleave(128, 0)
        Wt = ((Wt / s_rep).half() * scales.half().repeat_interleave(128, 0)).double()
    lin_t = (x.half().double() @ Wt + bias.double()).cpu().numpy()
    ref_t = _norm_sections(lin_t.astype(np.float32), hq, hk, hd, gq, gk, cos, sin)
    rel_t = np.linalg.norm(got - ref_t) / np.linalg.norm(ref_t)
    assert rel_t <= 5e-5, f"rel_frob vs staged reference {rel_t}"


@pytest.mark.parametrize("M", [200, 4352])
def test_fused_epilogue_matches_unfused_composition(M):
    hq, hk, hv, hd, K = 6, 6, 6, 128, 1024
    pw, _, _, x, bias, gq, gk, cos, sin = _projection(M, K, hq, hk, hv, hd, seed=M)
    for xd, yd in ((torch.float32, torch.float32), (torch.float16, torch.float16)):
        xin = x.to(xd)
        fused = pw.linear_qk_norm_rope(xin, hq, hk, hd, bias, gq, gk, EPS, cos, sin, out_dtype=yd)
        lin = pw.linear_ex(xin, bias, out_dtype=torch.float32)
        comp = lin.clone()
        q4.qk_norm_rope(lin[:, :hq * hd], hq, hd, gq, EPS, cos, sin, out=comp[:, :hq * hd])
        q4.qk_norm_rope(lin[:, hq * hd:(hq + hk) * hd], hk, hd, gk, EPS, cos, sin, out=comp[:, hq * hd:(hq + hk) * hd])
        torch.cuda.synchronize()
        q4.poll_device_error()
        rel = (torch.linalg.norm(fused.double() - comp.to(yd).double()) / torch.linalg.norm(comp.double())).item()
        assert rel <= (1e-5 if yd == torch.float32 else 1e-3), f"{xd}->{yd}: rel {rel}"
        # v heads pass through (the plain plan may split K, so equal up to summation order)
        fv, lv = fused[:, (hq + hk) * hd:].double(), lin[:, (hq + hk) * hd:].to(yd).double()
        assert (torch.linalg.norm(fv - lv) / torch.linalg.norm(lv)).item() <= (1e-6 if yd == torch.float32 else 1e-3)


def test_fused_epilogue_with_stream_k_tail():
    # exact numerics, 150 head tiles on 148 SMs: the planner deals the last wave as stage ranges
    M, K, hd = 200, 1024, 128
    hq, hk, hv = 50, 50, 50
    pw, _, _, x, bias, gq, gk, cos, sin = _projection(M, K, hq, hk, hv, hd, seed=9)
    q4.set_numerics(L.NUMERICS_EXACT)
    try:
        assert pw.plan_info(M)["sk_tiles"] > 0
        y = pw.linear_qk_norm_rope(x, hq, hk, hd, bias, gq, gk, EPS, cos, sin)
        lin = pw.linear_ex(x, bias)
    finally:
        q4.set_numerics(L.NUMERICS_AUTO)
    comp = lin.clone()
    q4.qk_norm_rope(lin[:, :hq * hd], hq, hd, gq, EPS, cos, sin, out=comp[:, :hq * hd])
    q4.qk_norm_rope(lin[:, hq * hd:(hq + hk) * hd], hk, hd, gk, EPS, cos, sin, out=comp[:, hq * hd:(hq + hk) * hd])
    torch.cuda.synchronize()
    q4.poll_device_error()
    rel = (torch.linalg.norm(y.double() - comp.double()) / torch.linalg.norm(comp.double())).item()
    assert rel <= 1e-5, f"rel {rel}"


def test_argument_checks():
    pw, _, _, x, bias, gq, gk, cos, sin = _projection(16, 256, 2, 1, 1, 128, seed=1)
    with pytest.raises(Bq4Error, match="EINVAL_SHAPE"):
        pw.linear_qk_norm_rope(x, 3, 2, 128)  # 5 heads of 128 do not fit N = 512
    with pytest.raises(Bq4Error, match="EINVAL_ARG"):
        pw.linear_qk_norm_rope(x, 2, 1, 128, cos=cos)  # cos without sin
    with pytest.raises(Bq4Error, match="EINVAL_SHAPE"):
        q4.qk_norm_rope(x[:, :255], 1, 255)  # odd head_dim
