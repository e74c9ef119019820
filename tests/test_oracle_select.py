"""CPU: the oracle's packed-Q4 row selection (q_select on dim 0) against the
pinned unpack.  Selecting rows of a PackedU32(0) table [rows, cols] is the
column layout with N = rows and K = cols, so the dequantized selected rows
must equal rows of that unpack bit for bit."""
import numpy as np
import pytest

import oracle as O


@pytest.mark.parametrize("block", [8, 16, 32, 64, 128])
def test_select_rows_matches_unpack(block):
    rng = np.random.default_rng(block)
    rows, cols = 37, 256
    words = rng.integers(0, 2 ** 32, size=(rows, cols // 8), dtype=np.uint64).astype(np.uint32)
    scales = rng.uniform(0.001, 0.02, size=(rows, cols // block)).astype(np.float32)
    ids = np.array([5, 0, 36, 5, 12, 36, 1])
    ow, osc, of, ok = O.select_rows(words, scales, rows, cols, block, ids)
    assert ok
    assert np.array_equal(ow, words[ids]) and np.array_equal(osc, scales[ids])
    full = O.unpack(words, scales, cols, rows, block, O.LAYOUT_COL)  # [K = cols, N = rows]
    assert np.array_equal(of, full.T[ids])


def test_select_rows_out_of_range_gives_zero_row():
    rng = np.random.default_rng(1)
    rows, cols, block = 8, 128, 128
    words = rng.integers(0, 2 ** 32, size=(rows, cols // 8), dtype=np.uint64).astype(np.uint32)
    scales = rng.uniform(0.001, 0.02, size=(rows, cols // block)).astype(np.float32)
    ow, osc, of, ok = O.select_rows(words, scales, rows, cols, block, np.array([2, 8, -1]))
    assert not ok
    assert np.array_equal(ow[0], words[2])
    assert not ow[1:].any() and not osc[1:].any() and not of[1:].any()
