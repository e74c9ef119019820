"""GPU: weights prepared straight from a stored tensor's QFloat payload
(bq4_weight_prepare_payload, the loader hook) dequantize bit-exactly to the
oracle's unpack of the same bytes -- Qwen column layout (axis 0 seen through
its transposed view), Boogu row layout (axis 1), and a plain axis-0 [K, N]
tensor (checked through a linear) -- from host, unaligned host and device
payloads."""
import numpy as np
import pytest
import torch

import oracle as O
from burn_image_b200 import _lib as L
from burn_image_b200 import q4

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_qwen_column_payload():
    rng = np.random.default_rng(1)
    N, K = 384, 512
    packed = q4.quantize_q4s_block128_f32(rng.standard_normal((N, K)).astype(np.float32), (N, K))
    payload = packed.to_bytes()
    w = q4.PreparedQ4Weight.from_payload(payload, (N, K), packed.stored_dtype, transposed_view=True, device=DEV)
    assert (w.K, w.N, w.block, w.layout) == (K, N, 128, L.LAYOUT_COL)
    ref = O.unpack(packed.words, packed.scales, K, N, 128, O.LAYOUT_COL)
    assert np.array_equal(w.dequantize().cpu().numpy(), ref)
    # the same bytes at an odd offset of a host buffer, and from device memory
    w2 = q4.PreparedQ4Weight.from_payload(memoryview(b"\0" + payload)[1:], (N, K), packed.stored_dtype, device=DEV)
    dev_bytes = torch.frombuffer(bytearray(payload), dtype=torch.uint8).to(DEV)
    w3 = q4.PreparedQ4Weight.from_payload(dev_bytes, (N, K), packed.stored_dtype, device=DEV)
    assert np.array_equal(w2.dequantize().cpu().numpy(), ref)
    assert np.array_equal(w3.dequantize().cpu().numpy(), ref)


@pytest.mark.parametrize("K", [480, 3360])  # blocks 32 (480 = 32 * 15, 3360 = 32 * 105: real Boogu width)
def test_boogu_row_payload(K):
    rng = np.random.default_rng(K)
    N = 256
    packed = q4.quantize_row_layout_q4s_block_up_to128_f32(rng.standard_normal((K, N)).astype(np.float32), (K, N))
    assert packed.stored_dtype == "q4s-block32x1-f32-packed-axis1"
    w = q4.PreparedQ4Weight.from_payload(packed.to_bytes(), (K, N), packed.stored_dtype, device=DEV)
    assert (w.K, w.N, w.block, w.layout) == (K, N, 32, L.LAYOUT_ROW)
    ref = O.unpack(packed.words, packed.scales, K, N, 32, O.LAYOUT_ROW)
    assert np.array_equal(w.dequantize().cpu().numpy(), ref)


def test_plain_axis0_payload_through_a_linear():
    # a plain stored [K, N] tensor packed (and blocked) along N, used without a transposed view
    rng = np.random.default_rng(3)
    K, N, block = 256, 512, 64
    words = rng.integers(0, 2 ** 32, size=(K, N // 8), dtype=np.uint64).astype(np.uint32)
    scales = rng.uniform(0.001, 0.02, size=(K, N // block)).astype(np.float32)
    payload = words.astype("<u4").tobytes() + scales.astype("<f4").tobytes()
    w = q4.PreparedQ4Weight.from_payload(payload, (K, N), q4.q4s_stored_dtype(block, 0), transposed_view=False,
                                         device=DEV)
    assert w.layout == L.LAYOUT_NPACKED
    x = rng.standard_normal((40, K)).astype(np.float32)
    y = w.linear(torch.from_numpy(x).to(DEV)).cpu().numpy()
    W = O.unpack(words, scales, N, K, block, O.LAYOUT_COL).T.copy()  # N-packed = transpose of column layout
    ref = O.linear_f64(x, W)
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel <= 5e-3
