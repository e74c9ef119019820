"""GPU: packed-Q4 row selection (bq4_q_select_rows, QTensorOps::q_select on
dim 0) and the fused select + dequantize of an embedding lookup
(bq4_q_select_rows_dequant), bit-exact against the oracle, with int32 and
int64 ids, repeated and unsorted ids, and every block size; an out-of-range
id gives a zero row and BQ4_EINVAL_ARG from poll_device_error."""
import numpy as np
import pytest
import torch

import oracle as O
from burn_image_b200 import _lib as L
from burn_image_b200 import q4
from burn_image_b200.q4 import Bq4Error, QuantizedTensor, QuantScheme

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _table(rows, cols, block, seed):
    rng = np.random.default_rng(seed)
    words = rng.integers(0, 2 ** 32, size=(rows, cols // 8), dtype=np.uint64).astype(np.uint32)
    scales = rng.uniform(0.001, 0.02, size=(rows, cols // block)).astype(np.float32)
    qt = QuantizedTensor(torch.from_numpy(words.view(np.int32)).to(DEV), torch.from_numpy(scales).to(DEV),
                         (rows, cols), QuantScheme(store_packed_dim=0, level=(block,)), transposed_view=False)
    return words, scales, qt


@pytest.mark.parametrize("block", [8, 32, 128])
@pytest.mark.parametrize("ids_dtype", [torch.int32, torch.int64])
def test_select_rows_bit_exact(block, ids_dtype):
    rows, cols = 4096, 2560
    words, scales, qt = _table(rows, cols, block, seed=block)
    ids_np = np.random.default_rng(3).integers(0, rows, size=300)
    ids_np[:4] = [0, rows - 1, 7, 7]
    ids = torch.from_numpy(ids_np).to(ids_dtype).to(DEV)
    sel = q4.q_select(qt, 0, ids)
    emb = q4.embedding(qt, ids)
    torch.cuda.synchronize()
    q4.poll_device_error()
    ow, osc, of, ok = O.select_rows(words, scales, rows, cols, block, ids_np)
    assert ok
    assert np.array_equal(sel.values.cpu().numpy().view(np.uint32), ow)
    assert np.array_equal(sel.scales.cpu().numpy(), osc)
    assert sel.shape == (300, cols)
    assert np.array_equal(emb.cpu().numpy(), of)


def test_select_from_a_transposed_view_table():
    # a Qwen-layout QFloat (stored [N, K], seen as [K, N]) selects rows of the stored tensor
    rows, cols, block = 640, 512, 128
    words, scales, qt = _table(rows, cols, block, seed=5)
    qt_view = QuantizedTensor(qt.values, qt.scales, (cols, rows), qt.scheme, transposed_view=True)
    ids = torch.tensor([3, 639, 0], device=DEV)
    emb = q4.embedding(qt_view, ids)
    torch.cuda.synchronize()
    _, _, of, _ = O.select_rows(words, scales, rows, cols, block, ids.cpu().numpy())
    assert np.array_equal(emb.cpu().numpy(), of)


def test_out_of_range_id_is_reported():
    rows, cols, block = 64, 256, 64
    words, scales, qt = _table(rows, cols, block, seed=9)
    q4.poll_device_error()
    emb = q4.embedding(qt, torch.tensor([1, 64, 2], device=DEV, dtype=torch.int32))
    torch.cuda.synchronize()
    with pytest.raises(Bq4Error, match="EINVAL_ARG"):
        q4.poll_device_error()
    q4.poll_device_error()  # cleared by the previous poll
    e = emb.cpu().numpy()
    _, _, of, _ = O.select_rows(words, scales, rows, cols, block, np.array([1, 2]))
    assert np.array_equal(e[[0, 2]], of) and not e[1].any()


def test_select_argument_checks():
    _, _, qt = _table(16, 256, 64, seed=2)
    ids = torch.tensor([1], device=DEV)
    with pytest.raises(Bq4Error, match="EINVAL_ARG"):
        q4.q_select(qt, 1, ids)  # only rows, like the reference
    with pytest.raises(Bq4Error):
        q4.q_select(qt, 0, ids.float())
    lib = L.lib()
    out = torch.empty((1, 256), device=DEV)
    rc = lib.bq4_q_select_rows_dequant(qt.values.data_ptr(), qt.scales.data_ptr(), 16, 256, 48,
                                       ids.data_ptr(), 1, 1, out.data_ptr(), None)
    assert rc == L.EINVAL_BLOCK
    rc = lib.bq4_q_select_rows_dequant(qt.values.data_ptr(), qt.scales.data_ptr(), 16, 200, 64,
                                       ids.data_ptr(), 1, 1, out.data_ptr(), None)
    assert rc == L.EINVAL_SHAPE
