"""CPU: pin the oracle to the reference's own known-answer tests and check the
library's host packers against it bit for bit.

Each test restates an assertion of a reference test (cited) on the same
inputs; the committed fixtures in tests/golden/ guard against regressions.
"""
import os

import numpy as np
import pytest

import oracle as O
from burn_image_b200 import Bq4Error, q4
from conftest import gen_q4

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def rel_rmse(actual, expected):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    return float(np.sqrt(((a - e) ** 2).sum() / (e ** 2).sum()))


def cosine(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float((a * b).sum() / np.linalg.norm(a) / np.linalg.norm(b))


def test_wave_block128_roundtrip_correctness():
    """crates/burn_boogu/src/artifacts.rs:10413-10498
    (packed_q4s_block128_roundtrip_and_linear_module_error_correctness)."""
    g = load("wave_block128")
    values = g["values"]
    words, scales = O.quantize_col_block128(values.reshape(128, 128))
    assert words.nbytes + scales.nbytes == values.size // 2 + values.size // 128 * 4
    assert np.array_equal(words.reshape(-1), g["words"])
    assert np.array_equal(scales.reshape(-1), g["scales"])
    # into_vec_i8 reconstruction, block-wise in flat order
    W = O.unpack(words, scales, 128, 128, 128, O.LAYOUT_COL)  # [k][n] = tensor[n][k]
    recon = W.T.reshape(-1)
    inp = g["input"]
    ref = np.array([(inp.astype(np.float64) * values.reshape(128, 128)[:, o]).sum() for o in range(128)])
    act = np.array([(inp.astype(np.float64) * recon.reshape(128, 128)[:, o]).sum() for o in range(128)])
    max_weight_error = float(np.abs(recon - values).max())
    assert np.isfinite(max_weight_error) and max_weight_error < 0.025
    assert rel_rmse(act, ref) < 0.08
    assert cosine(act, ref) > 0.996


def test_column_layout_fixture_correctness():
    """crates/burn_qwen3_vl/src/artifacts.rs:1877-2049: the source passes
    through F16 before the packer; quantized reference = dequantized matmul."""
    g = load("col_layout_256x128")
    assert np.array_equal(g["raw"].astype(np.float16).astype(np.float32), g["raw_f16"])
    words, scales = O.quantize_col_block128(g["raw_f16"].reshape(256, 128))
    assert np.array_equal(words, g["words"]) and np.array_equal(scales, g["scales"])
    W = O.unpack(words, scales, 128, 256, 128, O.LAYOUT_COL)  # [K=128][N=256]
    inp = g["input"]
    ref = g["raw"].reshape(256, 128).astype(np.float64) @ inp.astype(np.float64)
    quant = O.linear_f64(inp.reshape(1, 128), W)[0]
    assert rel_rmse(quant, ref) < 0.12
    assert cosine(quant, ref) > 0.993


def test_exact_representable_fixture_correctness():
    """crates/bevy_image/src/browser_boogu/runtime.rs:4511-4545,4777: scale is
    exactly 1/64, so the row-layout round trip is exact and the matmul is
    within 5e-4 of the f32 reference."""
    g = load("exact_row_4x128")
    words, scales, block = O.quantize_row_up_to128(g["weight"])
    assert block == 128 and np.all(scales == np.float32(1 / 64))
    assert np.array_equal(words, g["words"])
    W = O.unpack(words, scales, 128, 128, block, O.LAYOUT_ROW)
    assert np.array_equal(W, g["weight"])
    y = O.linear_f64(g["lhs"], W)
    assert np.abs(y - g["expected"]).max() <= 5e-4


def test_qwen_packed_byte_counts_correctness():
    """crates/burn_qwen3_vl/src/artifacts.rs:1603-1606,1731-1732."""
    vals = ((np.arange(256, dtype=np.float32) - 127.5) / 256.0).astype(np.float16).astype(np.float32)
    w, s = O.quantize_col_block128(vals.reshape(2, 128))
    assert w.nbytes + s.nbytes == 256 // 2 + (256 // 128) * 4
    assert s.size == 2


def test_invalid_sources_rejected_correctness():
    """crates/burn_boogu/src/artifacts.rs:10880-10886 (oracle and library)."""
    with pytest.raises(O.OracleError):
        O.quantize_col_block128(np.full((1, 128), np.nan, np.float32))
    with pytest.raises(O.OracleError):
        O.quantize_col_block128(np.zeros((1, 127), np.float32))
    with pytest.raises(Bq4Error):
        q4.quantize_q4s_block128_f32(np.full(128, np.nan, np.float32), [1, 128])
    with pytest.raises(Bq4Error):
        q4.quantize_q4s_block128_f32(np.zeros(127, np.float32), [1, 127])
    with pytest.raises(Bq4Error):
        q4.quantize_q4s_block128_f32(np.zeros(128, np.float32), [2, 128])
    with pytest.raises(Bq4Error):
        q4.quantize_q4s_block128_f32(np.zeros(0, np.float32), [])
    with pytest.raises(Bq4Error):  # output width not divisible by 8
        q4.quantize_row_layout_q4s_block_up_to128_f32(np.zeros(8 * 12, np.float32), [8, 12])
    with pytest.raises(Bq4Error):  # no exact block for input width 12
        q4.quantize_row_layout_q4s_block_up_to128_f32(np.zeros(12 * 8, np.float32), [12, 8])


@pytest.mark.parametrize("shape", [(3, 128), (5, 384), (1, 1024)])
def test_library_col_packer_matches_oracle_parity(shape, rng):
    v = (rng.standard_normal(shape) * 0.05).astype(np.float32)
    v[0, :128] = 0.0  # all-zero block -> f32::MIN_POSITIVE scale
    p = q4.quantize_q4s_block128_f32(v, shape)
    w, s = O.quantize_col_block128(v)
    assert np.array_equal(p.words, w.reshape(-1)) and np.array_equal(p.scales, s.reshape(-1))
    assert p.scales[0] == np.float32(1.17549435e-38)
    assert p.scheme.store_packed_dim == 0 and p.scheme.level == (128,)


@pytest.mark.parametrize("K,N,block", [(128, 16, 128), (3360 // 10 * 10 // 2, 8, 16), (96, 24, 32), (40, 8, 8), (64, 32, 64)])
def test_library_row_packer_matches_oracle_parity(K, N, block, rng):
    v = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    p = q4.quantize_row_layout_q4s_block_up_to128_f32(v, (K, N))
    w, s, b = O.quantize_row_up_to128(v)
    assert b == block == p.scheme.block
    assert p.scheme.level == (block, 1) and p.scheme.store_packed_dim == 1
    assert np.array_equal(p.words, w.reshape(-1)) and np.array_equal(p.scales, s.reshape(-1))


def test_row_block_policy_correctness():
    """crates/burn_boogu/src/artifacts.rs:513-525 (block choice) for the real
    Boogu widths (3360 -> 32, 13568 -> 128) and the BASELINE widths."""
    from burn_image_b200 import _lib as L
    for width, want in [(3360, 32), (13568, 128), (3072, 128), (12288, 128), (40, 8), (12, 0)]:
        assert L.lib().bq4_row_block_for(width) == want
        assert O.lib().orc_row_block_for(width) == want


@pytest.mark.parametrize("layout", [O.LAYOUT_ROW, O.LAYOUT_COL])
@pytest.mark.parametrize("block", [8, 16, 32, 64, 128])
def test_unpack_two_layouts_agree_parity(layout, block, rng):
    """The two physical layouts of one logical weight unpack identically, and
    nibble 0x8 decodes as -8 (two's complement; parity-unpinned for -8)."""
    K, N = 256, 24
    w_row, s_row = gen_q4(K, N, block, 1, np.random.default_rng(7))
    w_col, s_col = gen_q4(K, N, block, 0, np.random.default_rng(7))
    A = O.unpack(w_row, s_row, K, N, block, O.LAYOUT_ROW)
    B = O.unpack(w_col, s_col, K, N, block, O.LAYOUT_COL)
    assert np.array_equal(A, B)
    w8 = np.full((1, 8), 0x88888888, np.uint32)
    s1 = np.ones((1, 8), np.float32)
    assert np.all(O.unpack(w8, s1, 8, 8, 8, O.LAYOUT_ROW) == -8.0)


@pytest.mark.parametrize("name", ["random_row_b128", "random_col_b32_gelu", "random_row_b8_silu"])
def test_random_fixtures_reproduce(name):
    g = load(name)
    M, K, N, blk, lay, act, with_bias = [int(v) for v in g["meta"]]
    W = O.unpack(g["words"], g["scales"], K, N, blk, lay)
    y = O.linear_f64(g["x"], W, g["bias"] if with_bias else None, act)
    assert np.array_equal(y, g["y"])


def test_cpu_baseline_matches_checker(rng):
    """The timed CPU baseline (f32 SGEMM) agrees with the f64 checker."""
    K, N, M, blk = 512, 200, 50, 64
    w, s = gen_q4(K, N, blk, 1, rng)
    x = rng.standard_normal((M, K), dtype=np.float32)
    bias = rng.standard_normal(N).astype(np.float32) * 0.02
    W = O.unpack(w, s, K, N, blk, O.LAYOUT_ROW)
    for act in (O.ACT_NONE, O.ACT_GELU_TANH, O.ACT_SILU):
        ref = O.linear_f64(x, W, bias, act)
        got = O.cpu_linear(w, s, K, N, blk, O.LAYOUT_ROW, x, bias, act)
        assert O.rel_frobenius(got, ref) < 1e-5
