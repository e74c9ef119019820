"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Bars: dequantization bit-exact; linear outputs within relative Frobenius
error 5e-3 of the oracle's f64-accumulated result (max-abs printed), plus a
tight check against an emulation of the kernel's f16 operand staging.
Ordered from the simplest kernel to the full GEMM so `-x` stops early.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from burn_image_b200 import _lib as L
from burn_image_b200 import q4
from conftest import gen_bias, gen_q4, gen_x

pytestmark = pytest.mark.gpu

TOL = 5e-3  # north-star relative Frobenius tolerance
DEV = torch.device("cuda", 0)


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).to(DEV)


def p(t):
    return ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)


def decode_q(words, K, N, layout):
    """Logical int q [K][N] from raw words (test helper)."""
    q = np.zeros((K, N), np.int32)
    if layout == O.LAYOUT_ROW:
        for lane in range(8):
            nib = ((words >> np.uint32(4 * lane)) & np.uint32(0xF)).astype(np.int32)
            q[lane::8, :] = np.where(nib >= 8, nib - 16, nib)
    else:
        for lane in range(8):
            nib = ((words >> np.uint32(4 * lane)) & np.uint32(0xF)).astype(np.int32)
            q[lane::8, :] = np.where(nib >= 8, nib - 16, nib).T
    return q


def scales_kn(scales, K, N, block, layout):
    s = scales if layout == O.LAYOUT_ROW else scales.T
    return np.repeat(np.ascontiguousarray(s), block, axis=0)[:K]


def staged_weight(words, scales, K, N, block, layout, exact=None):
    """Emulation of the kernel's weight staging: exact plans (blocks of
    64/128) keep q * scale exact (the scale multiplies the f32 accumulator);
    folded plans stage f16(q * f16(scale)).  exact=None: exact for every
    block of 64/128 (the EXACT numerics mode)."""
    if exact if exact is not None else block >= 64:
        return O.unpack(words, scales, K, N, block, layout)
    q = decode_q(words, K, N, layout).astype(np.float16)
    s = scales_kn(scales, K, N, block, layout).astype(np.float16)
    return (q * s).astype(np.float16).astype(np.float32)


def report(name, got, ref):
    rf = O.rel_frobenius(got, ref)
    ma = float(np.abs(np.asarray(got, np.float64) - ref).max()) if ref.size else 0.0
    print(f"{name}: rel_frob={rf:.3e} max_abs={ma:.3e}")
    return rf


# ---------------------------------------------------------------- dequant

def unpack_any(w, s, K, N, block, layout):
    """Oracle unpack; the N-packed layout is the transpose of a column-layout
    tensor of shape [K rows][N inner]."""
    if layout == L.LAYOUT_NPACKED:
        return O.unpack(w, s, N, K, block, O.LAYOUT_COL).T.copy()
    return O.unpack(w, s, K, N, block, layout)


@pytest.mark.parametrize("layout", [O.LAYOUT_ROW, O.LAYOUT_COL, L.LAYOUT_NPACKED])
@pytest.mark.parametrize("block", [8, 16, 32, 64, 128])
def test_dequant_raw_bit_exact(layout, block, rng):
    K, N = 256, 384 if layout == L.LAYOUT_NPACKED else 136
    w, s = gen_q4(K, N, block, layout, rng)
    ref = unpack_any(w, s, K, N, block, layout)
    wd, sd = dev(w), dev(s)
    out = torch.empty((K, N), dtype=torch.float32, device=DEV)
    L.check(L.lib().bq4_dequant_raw(p(wd), p(sd), K, N, block, layout, p(out), L.LAYOUT_ROW, stream()))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref)
    out_t = torch.empty((N, K), dtype=torch.float32, device=DEV)
    L.check(L.lib().bq4_dequant_raw(p(wd), p(sd), K, N, block, layout, p(out_t), L.LAYOUT_COL, stream()))
    torch.cuda.synchronize()
    assert np.array_equal(out_t.cpu().numpy(), ref.T)


@pytest.mark.parametrize("K,N,block,layout", [
    (256, 136, 128, O.LAYOUT_ROW), (192, 264, 32, O.LAYOUT_COL), (3360, 200, 32, O.LAYOUT_ROW),
    (96, 8, 8, O.LAYOUT_COL), (640, 384, 64, O.LAYOUT_ROW), (128, 1, 16, O.LAYOUT_COL)])
def test_prepare_then_dequant_bit_exact(K, N, block, layout, rng):
    """The one-time re-layout loses nothing: dequantizing the prepared weight
    (padding included) is bit-identical to the oracle unpack."""
    w, s = gen_q4(K, N, block, layout, rng)
    ref = O.unpack(w, s, K, N, block, layout)
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, block, layout, DEV)
    got = pw.dequantize(L.LAYOUT_ROW).cpu().numpy()
    assert np.array_equal(got, ref)
    assert np.array_equal(pw.dequantize(L.LAYOUT_COL).cpu().numpy(), ref.T)
    # host pointers are accepted too (uploaded by the library)
    pw2 = q4.PreparedQ4Weight(torch.from_numpy(w.view(np.int32)), torch.from_numpy(s), K, N, block, layout, DEV)
    assert np.array_equal(pw2.dequantize().cpu().numpy(), ref)


def test_nibble_minus8_decodes_two_complement():
    w = np.full((1, 8), 0x88888888, np.uint32)
    s = np.full((1, 8), 0.5, np.float32)
    pw = q4.PreparedQ4Weight(dev(w), dev(s), 8, 8, 8, O.LAYOUT_ROW, DEV)
    assert np.all(pw.dequantize().cpu().numpy() == -4.0)


# ---------------------------------------------------------------- linear, golden fixtures

@pytest.mark.parametrize("name", ["random_row_b128", "random_col_b32_gelu", "random_row_b8_silu"])
def test_linear_golden_fixtures(name):
    import os
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", name + ".npz")))
    M, K, N, blk, lay, act, with_bias = [int(v) for v in g["meta"]]
    pw = q4.PreparedQ4Weight(dev(g["words"]), dev(g["scales"]), K, N, blk, lay, DEV)
    bias = dev(g["bias"]) if with_bias else None
    y = pw.linear(dev(g["x"]), bias, act).cpu().numpy()
    q4.poll_device_error()
    assert report(name, y, g["y"]) <= TOL


def test_exact_representable_fixture_gpu():
    """crates/bevy_image/src/browser_boogu/runtime.rs:4777 -- max-abs <= 5e-4."""
    import os
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "exact_row_4x128.npz")))
    pw = q4.PreparedQ4Weight(dev(g["words"]), dev(g["scales"]), 128, 128, int(g["block"]), O.LAYOUT_ROW, DEV)
    y = pw.linear(dev(g["lhs"])).cpu().numpy()
    assert np.all(np.isfinite(y))
    assert np.abs(y - g["expected"]).max() <= 5e-4


def test_wave_fixture_gpu():
    """crates/burn_boogu/src/artifacts.rs:10501-10584 thresholds on the GPU path:
    the plain [input=128, output=128] tensor packed (and blocked) along its
    last axis is used directly as the matmul rhs (BQ4_LAYOUT_NPACKED)."""
    import os
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "wave_block128.npz")))
    pw = q4.PreparedQ4Weight(dev(g["words"]), dev(g["scales"]), 128, 128, 128, L.LAYOUT_NPACKED, DEV)
    x = g["input"].reshape(1, 128)
    y = pw.linear(dev(x)).cpu().numpy()[0]
    v = g["values"].reshape(128, 128)  # [input k][output n]
    ref = x[0].astype(np.float64) @ v.astype(np.float64)
    err = np.sqrt(((y - ref) ** 2).sum() / (ref ** 2).sum())
    cos = (y * ref).sum() / np.linalg.norm(y) / np.linalg.norm(ref)
    assert err < 0.08 and cos > 0.996
    # rank-3 input agrees with rank-2 (< 1e-5)
    y3 = pw.linear(dev(x.reshape(1, 1, 128))).cpu().numpy().reshape(-1)
    assert np.abs(y3 - y).max() < 1e-5


# ---------------------------------------------------------------- linear sweeps

CASES = [
    # M, K, N, block, layout, act, bias, aux
    (1, 256, 128, 128, O.LAYOUT_ROW, O.ACT_NONE, False, False),
    (5, 512, 136, 64, O.LAYOUT_COL, O.ACT_NONE, True, False),
    (64, 1024, 256, 128, O.LAYOUT_ROW, O.ACT_GELU_TANH, True, False),
    (100, 384, 200, 32, O.LAYOUT_ROW, O.ACT_SILU, True, True),
    (129, 640, 384, 16, O.LAYOUT_COL, O.ACT_NONE, False, True),
    (256, 2560, 512, 128, O.LAYOUT_COL, O.ACT_NONE, True, False),
    (300, 3360, 264, 32, O.LAYOUT_ROW, O.ACT_GELU_TANH, True, False),
    (517, 1024, 640, 8, O.LAYOUT_ROW, O.ACT_NONE, True, False),
    (1000, 768, 1024, 128, O.LAYOUT_COL, O.ACT_GELU_TANH, False, False),
]


@pytest.mark.parametrize("M,K,N,block,layout,act,with_bias,with_aux", CASES)
def test_linear_parity(M, K, N, block, layout, act, with_bias, with_aux, rng):
    w, s = gen_q4(K, N, block, layout, rng)
    x = gen_x(M, K, rng)
    bias = gen_bias(N, rng) if with_bias else None
    aux = rng.standard_normal((M, N), dtype=np.float32) if with_aux else None
    W = O.unpack(w, s, K, N, block, layout)
    ref = O.linear_f64(x, W, bias, act, aux)
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, block, layout, DEV)
    y = pw.linear(dev(x), dev(bias) if bias is not None else None, act,
                  dev(aux) if aux is not None else None).cpu().numpy()
    q4.poll_device_error()
    assert np.all(np.isfinite(y))
    assert report(f"M{M}K{K}N{N}b{block}", y, ref) <= TOL
    # tight check: the same staging emulated on the CPU (f16 x, f16 weights)
    Ws = staged_weight(w, s, K, N, block, layout, exact=pw.plan_info(M)["exact"] == 1)
    xs = x.astype(np.float16).astype(np.float32)
    ref_s = O.linear_f64(xs, Ws, bias, act, aux)
    tight = 2e-3 if act != O.ACT_NONE else 1e-5  # GELU/SiLU use approximate tanh/exp
    assert report("  staged", y, ref_s) <= tight


def test_column_layout_kernel_rel_rmse():
    """crates/burn_qwen3_vl/src/artifacts.rs:1877-2049: Qwen column layout
    through qwen_linear_forward; kernel rel-RMSE vs the dequantized f32
    matmul < 1e-4 (the exact-weight kernel keeps q * scale exact), quantized
    vs raw rel-RMSE < 0.12, cosine > 0.993, rank-3 equals rank-2 (< 1e-5)."""
    import os
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "col_layout_256x128.npz")))
    packed = q4.PackedQ4(g["words"].reshape(-1), g["scales"].reshape(-1), (256, 128), q4.QuantScheme())
    lin = q4.Q4Linear(q4.QuantizedTensor.from_packed(packed, DEV, stored="nk"))
    x = g["input"].reshape(1, 128)
    y = q4.qwen_linear_forward(lin, dev(x)).cpu().numpy()[0]
    y3 = q4.qwen_linear_forward(lin, dev(x.reshape(1, 1, 128))).cpu().numpy().reshape(-1)
    assert np.abs(y3 - y).max() < 1e-5
    W = O.unpack(g["words"], g["scales"], 128, 256, 128, O.LAYOUT_COL)
    quant_ref = O.linear_f64(x, W)[0].astype(np.float64)
    raw_ref = g["raw"].reshape(256, 128).astype(np.float64) @ x[0].astype(np.float64)
    kernel_rmse = np.sqrt(((y - quant_ref) ** 2).sum() / (quant_ref ** 2).sum())
    rmse = np.sqrt(((y - raw_ref) ** 2).sum() / (raw_ref ** 2).sum())
    cos = (y * raw_ref).sum() / np.linalg.norm(y) / np.linalg.norm(raw_ref)
    print(f"column layout: kernel rel-RMSE={kernel_rmse:.3e} rel-RMSE={rmse:.3e} cos={cos:.5f}")
    assert kernel_rmse < 1e-4 and rmse < 0.12 and cos > 0.993


@pytest.mark.parametrize("M,K,N,block", [(33, 200, 256, 8), (130, 512, 384, 128)])
def test_npacked_linear_parity(M, K, N, block, rng):
    """Plain [K,N] PackedU32(0) rhs (blocks along N) via q_matmul."""
    w, s = gen_q4(K, N, block, L.LAYOUT_NPACKED, rng)
    x = gen_x(M, K, rng)
    W = unpack_any(w, s, K, N, block, L.LAYOUT_NPACKED)
    ref = O.linear_f64(x, W)
    qt = q4.QuantizedTensor(dev(w), dev(s), (K, N), q4.QuantScheme(store_packed_dim=0, level=(block,)),
                            transposed_view=False)
    y = q4.q_matmul(dev(x), qt).cpu().numpy()
    assert report(f"npacked M{M}", y, ref) <= TOL
    y2 = qt.prepared().linear(dev(x)).cpu().numpy()
    assert np.array_equal(y, y2)


def test_linear_strided_input(rng):
    """ldx > K (a column slice of a wider activation, as the o-projection
    reads the attention output)."""
    M, K, N, block = 77, 512, 256, 128
    w, s = gen_q4(K, N, block, O.LAYOUT_ROW, rng)
    big = gen_x(M, 3 * K, rng)
    W = O.unpack(w, s, K, N, block, O.LAYOUT_ROW)
    ref = O.linear_f64(np.ascontiguousarray(big[:, K:2 * K]), W)
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, block, O.LAYOUT_ROW, DEV)
    xt = dev(big)[:, K:2 * K]
    y = torch.empty((M, N), dtype=torch.float32, device=DEV)
    ws = q4.Workspace.get(DEV, pw.workspace_bytes(M))
    L.check(L.lib().bq4_linear(pw.handle, p(xt), M, 3 * K, None, 0, None, p(y), p(ws), ws.numel(), stream()))
    assert report("strided", y.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("M,K,N,block", [(7, 256, 128, 128), (96, 2560, 512, 128), (200, 1024, 384, 32)])
def test_linear_gated_parity(M, K, N, block, rng):
    wg, sg = gen_q4(K, N, block, O.LAYOUT_COL, rng)
    wu, su = gen_q4(K, N, block, O.LAYOUT_COL, rng)
    x = gen_x(M, K, rng)
    bg, bu = gen_bias(N, rng), gen_bias(N, rng)
    ref = O.linear_gated_f64(x, O.unpack(wg, sg, K, N, block, 0), O.unpack(wu, su, K, N, block, 0), bg, bu)
    g = q4.PreparedQ4Weight(dev(wg), dev(sg), K, N, block, 0, DEV)
    u = q4.PreparedQ4Weight(dev(wu), dev(su), K, N, block, 0, DEV)
    y = q4.linear_gated(g, u, dev(x), dev(bg), dev(bu)).cpu().numpy()
    q4.poll_device_error()
    assert report(f"gated M{M}", y, ref) <= TOL


def test_q_matmul_entry_parity(rng):
    """The reference-shaped op: raw packed buffers + scheme, rank-3 lhs."""
    K, N, block = 384, 256, 64
    w, s = gen_q4(K, N, block, O.LAYOUT_ROW, rng)
    x = gen_x(2 * 45, K, rng)
    ref = O.linear_f64(x, O.unpack(w, s, K, N, block, O.LAYOUT_ROW))
    qt = q4.QuantizedTensor(dev(w), dev(s), (K, N), q4.QuantScheme(store_packed_dim=1, level=(block, 1)))
    y = q4.q_matmul(dev(x).reshape(2, 45, K), qt)
    assert tuple(y.shape) == (2, 45, N)
    assert report("q_matmul", y.reshape(-1, N).cpu().numpy(), ref) <= TOL
    with pytest.raises(q4.Bq4Error):
        q4.q_matmul(dev(x), q4.QuantizedTensor(dev(w), dev(s), (K, N), q4.QuantScheme(level=(256,))))


def test_linear_forward_adapters(rng):
    """linear_forward / qwen_linear_forward: bias fused, rank >= 2 enforced."""
    K, N = 256, 128
    vals = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    packed = q4.quantize_q4s_block128_f32(vals, (N, K))
    lin = q4.Q4Linear(q4.QuantizedTensor.from_packed(packed, DEV), dev(gen_bias(N, rng)))
    x = gen_x(6, K, rng)
    W = O.unpack(packed.words.reshape(N, K // 8), packed.scales.reshape(N, 1 * K // 128), K, N, 128, 0)
    ref = O.linear_f64(x, W, lin.bias.cpu().numpy())
    y = q4.qwen_linear_forward(lin, dev(x).reshape(2, 3, K))
    assert report("qwen_linear_forward", y.reshape(6, N).cpu().numpy(), ref) <= TOL
    with pytest.raises(q4.Bq4Error):
        q4.linear_forward(lin, dev(x[0]))


def test_deterministic_and_split_k(rng):
    """Repeated calls are bit-identical, including the split-K fix-up path."""
    M, K, N, block = 256, 2560, 256, 128  # few tiles -> split-K engaged
    w, s = gen_q4(K, N, block, O.LAYOUT_ROW, rng)
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, block, O.LAYOUT_ROW, DEV)
    x = dev(gen_x(M, K, rng))
    a = pw.linear(x).clone()
    b = pw.linear(x).clone()
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_error_status_on_bad_args(rng):
    K, N = 256, 128
    w, s = gen_q4(K, N, 128, O.LAYOUT_ROW, rng)
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, 128, O.LAYOUT_ROW, DEV)
    x = dev(gen_x(4, K, rng))
    y = torch.empty((4, N), dtype=torch.float32, device=DEV)
    lib = L.lib()
    import os
    os.environ["BQ4_NO_SKINNY"] = "1"  # the tcgen05 plan, which needs a workspace (the few-token one needs none)
    try:
        ws = q4.Workspace.get(DEV, pw.workspace_bytes(4))
        assert pw.workspace_bytes(4) > 16
        assert lib.bq4_linear(pw.handle, p(x), 4, K, None, 0, None, p(y), p(ws), 16, stream()) == L.EWORKSPACE
    finally:
        os.environ.pop("BQ4_NO_SKINNY", None)
    assert lib.bq4_linear(pw.handle, p(x), 0, K, None, 0, None, p(y), p(ws), ws.numel(), stream()) == L.EINVAL_SHAPE
    assert lib.bq4_linear(pw.handle, p(x), 4, K - 8, None, 0, None, p(y), p(ws), ws.numel(), stream()) == L.EINVAL_SHAPE
    assert lib.bq4_linear(pw.handle, p(x), 4, K, None, 9, None, p(y), p(ws), ws.numel(), stream()) == L.EINVAL_ARG
    assert lib.bq4_linear(pw.handle, None, 4, K, None, 0, None, p(y), p(ws), ws.numel(), stream()) == L.EINVAL_ARG


# ---------------------------------------------------------------- BASELINE sizes: torch fp32 reference

@pytest.mark.parametrize("M,K,N,act", [(256, 2560, 2560, 0), (256, 2560, 512, 0), (256, 9728, 2560, 0),
                                       (512, 2560, 9728, 0), (4352, 3072, 12288, 1), (4352, 12288, 3072, 0),
                                       (18432, 3072, 9216, 0), (18432, 3072, 3072, 0)])
def test_baseline_shapes_vs_torch_fp32(M, K, N, act):
    """Full BASELINE shapes against a PyTorch fp64 product of the same op on
    the device (weights dequantized by the bit-exact kernel): configs 1-3 and
    the 1536 px edit projections of config 4 (fused qkv 18432 x 3072 -> 9216,
    o 18432 x 3072 -> 3072), which have more token tiles and different
    split / stream-K plans than any smaller case."""
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N)
    words = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device=DEV, dtype=torch.int64).to(torch.int32)
    scales = (torch.rand((K // 128, N), generator=g, device=DEV) * 0.019 + 0.001).contiguous()
    x = torch.randn((M, K), generator=g, device=DEV)
    bias = torch.randn(N, generator=g, device=DEV) * 0.02
    pw = q4.PreparedQ4Weight(words.contiguous(), scales, K, N, 128, L.LAYOUT_ROW, DEV)
    W = pw.dequantize()
    ref = torch.addmm(bias.double(), x.double(), W.double())
    if act == 1:
        ref = torch.nn.functional.gelu(ref, approximate="tanh")
    y = pw.linear(x, bias, act)
    q4.poll_device_error()
    rf = (torch.linalg.norm((y.double() - ref)) / torch.linalg.norm(ref)).item()
    print(f"baseline M{M} K{K} N{N}: rel_frob={rf:.3e} max_abs={(y.double() - ref).abs().max().item():.3e}")
    assert rf <= TOL


def test_baseline_gated_pair_vs_torch_fp64():
    """Config 2's fused gate+up pair at full size (M=256, K=2560, N=2 x 9728,
    SiLU(gate) * up, crates/burn_qwen3_vl/src/text.rs:46-52) against an fp64
    product of the bit-exact dequantized weights."""
    M, K, N = 256, 2560, 9728
    g = torch.Generator(device=DEV).manual_seed(97281)
    ws = []
    for _ in range(2):
        words = torch.randint(-2 ** 31, 2 ** 31 - 1, (N, K // 8), generator=g, device=DEV,
                              dtype=torch.int64).to(torch.int32).contiguous()
        scales = (torch.rand((N, K // 128), generator=g, device=DEV) * 0.019 + 0.001).contiguous()
        ws.append(q4.PreparedQ4Weight(words, scales, K, N, 128, L.LAYOUT_COL, DEV))
    x = torch.randn((M, K), generator=g, device=DEV)
    bg = torch.randn(N, generator=g, device=DEV) * 0.02
    bu = torch.randn(N, generator=g, device=DEV) * 0.02
    y = q4.linear_gated(ws[0], ws[1], x, bg, bu)
    q4.poll_device_error()
    xd = x.double()
    gate = torch.addmm(bg.double(), xd, ws[0].dequantize().double())
    up = torch.addmm(bu.double(), xd, ws[1].dequantize().double())
    ref = torch.nn.functional.silu(gate) * up
    rf = (torch.linalg.norm(y.double() - ref) / torch.linalg.norm(ref)).item()
    print(f"gated pair M{M} K{K} N2x{N}: rel_frob={rf:.3e} max_abs={(y.double() - ref).abs().max().item():.3e}")
    assert rf <= TOL
    assert torch.equal(y, q4.linear_gated(ws[0], ws[1], x, bg, bu))  # repeat calls: same bits
