"""CPU: the packed-F16 oracle (oracle/bq4_oracle.c, orc_f16_*) pinned to the
reference's own tests of packed-F16 storage.

- widening: crates/burn_boogu/src/model/packed_f16.rs:574-601 require the
  bit-level widening to equal the IEEE binary16 -> binary32 conversion of the
  `half` crate for all 65536 patterns (quiet bit set on NaN); here against
  numpy's exact conversion for every non-NaN pattern and the quiet-NaN rule,
  plus the reference's list of IEEE classes;
- word order (:603-621) and the materialisation case (:709-757);
- rhs matmul, select and conv2d golden vectors of
  packed_f16_wgpu_linear_embedding_and_convolution_correctness (:763-874);
- the reference's throughput smokes (:876-1026) as value checks at a size the
  CPU oracle finishes quickly: ones times f16(1/K) sums to 1 within their bars.
"""
import numpy as np
import pytest

import oracle as O


def _f16_bits(values):
    return np.asarray(values, dtype=np.float32).astype(np.float16).view(np.uint16)


def test_widening_exhaustive():
    h = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    got = O.f16_widen_bits(h)
    exp = h.view(np.float16).astype(np.float32).view(np.uint32)
    e = (h.astype(np.uint32) >> 10) & 0x1F
    m = h.astype(np.uint32) & 0x3FF
    nan = (e == 0x1F) & (m != 0)
    # NaN: payload kept, quiet bit set (numpy keeps signalling NaNs signalling)
    exp = np.where(nan, ((h.astype(np.uint32) & 0x8000) << 16) | 0x7FC00000 | (m << 13), exp).astype(np.uint32)
    assert np.array_equal(got, exp)


def test_widening_ieee_classes():
    # packed_f16.rs:587-601: signed zero, subnormal, normal, infinity, NaN payloads
    cases = {0x0000: 0x00000000, 0x8000: 0x80000000, 0x0001: 0x33800000, 0x03FF: 0x387FC000,
             0x8001: 0xB3800000, 0x0400: 0x38800000, 0x3C00: 0x3F800000, 0x7BFF: 0x477FE000,
             0xBC00: 0xBF800000, 0x7C00: 0x7F800000, 0xFC00: 0xFF800000, 0x7C01: 0x7FC02000,
             0x7E00: 0x7FC00000, 0x7FFF: 0x7FFFE000, 0xFE01: 0xFFC02000}
    got = O.f16_widen_bits(np.array(list(cases), dtype=np.uint16))
    assert [int(v) for v in got] == list(cases.values())


def test_packed_word_order_low_then_high():
    # packed_f16.rs:603-621
    halves = np.array([0x3C00, 0xC000, 0x0001, 0x7C00, 0x7E35], dtype=np.uint16)
    padded = np.append(halves, np.uint16(0))
    words = padded[0::2].astype(np.uint32) | (padded[1::2].astype(np.uint32) << 16)
    unpacked = np.array([(int(words[i // 2]) >> ((i % 2) * 16)) & 0xFFFF for i in range(halves.size)], np.uint16)
    assert np.array_equal(unpacked, halves)  # the storage is a little-endian uint16 array
    assert np.array_equal(words.view(np.uint16)[:halves.size], halves)
    assert np.array_equal(O.f16_widen_bits(unpacked), O.f16_widen_bits(halves))


def test_rhs_matmul_golden():
    # :791-826: checkpoint [out=4, in=3] used through its transposed view
    lhs = np.array([[1.0, 2.0, 3.0], [-1.0, 0.5, 2.0]], np.float32)
    ckpt = _f16_bits([1.0, 0.0, 2.0, 0.0, 1.0, -1.0, 2.0, -1.0, 0.5, -1.0, 2.0, 1.0])
    got = O.f16_matmul_f64(lhs, ckpt, K=3, N=4, inner=1, col=3)
    assert got.astype(np.float32).ravel().tolist() == [7.0, -1.0, 1.5, 6.0, 3.0, -1.5, -1.5, 4.0]


def test_select_rows_golden():
    # :828-846
    table = _f16_bits([1.0, 2.0, 3.0, 4.0, 5.0, 6.0, -1.0, -2.0, -3.0, 7.0, 8.0, 9.0]).reshape(4, 3)
    rows = O.f16_widen_bits(table[[2, 0]]).view(np.float32)
    assert rows.ravel().tolist() == [-1.0, -2.0, -3.0, 1.0, 2.0, 3.0]


def test_conv2d_golden():
    # :848-873: input 1x1x3x3, weight [2,1,2,2], bias, stride 1, no padding
    x = np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3)
    w = _f16_bits([1.0, 0.0, 0.0, -1.0, 0.5, 0.5, 0.5, 0.5]).reshape(2, 1, 2, 2)
    got = O.f16_conv2d_f64(x, w, np.array([0.5, -1.0], np.float32))
    assert got.astype(np.float32).ravel().tolist() == [-3.5, -3.5, -3.5, -3.5, 5.0, 7.0, 11.0, 13.0]


def test_throughput_smoke_values():
    # :876-943: ones [.., 4096] times f16(1/4096) -> 1 within 1e-3
    K = 4096
    w = np.full((8, K), 1.0 / K, np.float32).astype(np.float16).view(np.uint16)  # stored [out, in]
    y = O.f16_matmul_f64(np.ones((2, K), np.float32), w, K=K, N=8, inner=1, col=K)
    assert np.abs(y - 1.0).max() <= 1e-3
    # :945-1026: 512 -> 512 channels, 3x3, padding 1, weight f16(1/4608): interior sample 1 within 2e-3
    C = 512
    wc = np.full((C, C, 3, 3), 1.0 / (C * 9), np.float32).astype(np.float16).view(np.uint16)
    out = O.f16_conv2d_f64(np.ones((1, C, 6, 6), np.float32), wc, padding=(1, 1))
    assert abs(out[0, 0, 3, 3] - 1.0) <= 2e-3


@pytest.mark.parametrize("stride,padding,dilation", [((1, 1), (1, 1), (1, 1)), ((2, 2), (1, 0), (1, 1)),
                                                     ((1, 2), (2, 1), (2, 1))])
def test_conv2d_matches_im2col_matmul(stride, padding, dilation):
    # the convolution is the matmul of its gathered input rows with the [in*kh*kw, out] weight view
    rng = np.random.default_rng(5)
    B, C, H, W, O_, kh, kw = 2, 5, 9, 7, 6, 3, 2
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    w = rng.standard_normal((O_, C, kh, kw)).astype(np.float16).view(np.uint16)
    bias = rng.standard_normal(O_).astype(np.float32)
    got = O.f16_conv2d_f64(x, w, bias, stride, padding, dilation)
    OH, OW = got.shape[2:]
    xp = np.pad(x, ((0, 0), (0, 0), (padding[0],) * 2, (padding[1],) * 2))
    rows = np.empty((B, OH, OW, C, kh, kw), np.float32)
    for ky in range(kh):
        for kx in range(kw):
            ys = ky * dilation[0] + stride[0] * np.arange(OH)
            xs = kx * dilation[1] + stride[1] * np.arange(OW)
            rows[..., ky, kx] = xp[:, :, ys][:, :, :, xs].transpose(0, 2, 3, 1)
    ref = O.f16_matmul_f64(rows.reshape(-1, C * kh * kw), w.reshape(O_, -1), K=C * kh * kw, N=O_, inner=1,
                           col=C * kh * kw, bias=bias)
    ref = ref.reshape(B, OH, OW, O_).transpose(0, 3, 1, 2)
    assert np.abs(got - ref).max() < 1e-9


def test_cpu_arms_match_checker():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((37, 70)).astype(np.float32)
    w = rng.standard_normal((70, 45)).astype(np.float16).view(np.uint16)
    y = O.cpu_f16_matmul(x, w, K=70, N=45, inner=45, col=1)
    assert O.rel_frobenius(y, O.f16_matmul_f64(x, w, 70, 45, 45, 1)) < 1e-6
    xi = rng.standard_normal((2, 6, 11, 10)).astype(np.float32)
    wc = rng.standard_normal((7, 6, 3, 3)).astype(np.float16).view(np.uint16)
    b = rng.standard_normal(7).astype(np.float32)
    for stride, pad in (((1, 1), (1, 1)), ((2, 2), (0, 1))):
        yc = O.cpu_f16_conv2d(xi, wc, b, stride, pad)
        assert O.rel_frobenius(yc, O.f16_conv2d_f64(xi, wc, b, stride, pad)) < 1e-6
