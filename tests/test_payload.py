"""CPU: the stored-dtype spellings of packed-Q4 tensors in the reference's
sealed artifact inventory (crates/burn_boogu/src/artifacts.rs:527-537) and
the host-side checks of the payload loader (bq4_weight_prepare_payload), which
reject a bad spelling or a payload whose size does not match the shape
(crates/burn_qwen3_vl/src/artifacts.rs:1204-1240) before touching a device."""
import ctypes

import numpy as np
import pytest

from burn_image_b200 import _lib as L
from burn_image_b200 import q4
from burn_image_b200.q4 import Bq4Error


@pytest.mark.parametrize("block", [8, 16, 32, 64, 128])
def test_spellings_round_trip(block):
    s0, s1 = q4.q4s_stored_dtype(block, 0), q4.q4s_stored_dtype(block, 1)
    assert s0 == f"q4s-block{block}-f32-packed-axis0"
    assert s1 == f"q4s-block{block}x1-f32-packed-axis1"
    assert q4.parse_stored_dtype(s0) == (block, 0)
    assert q4.parse_stored_dtype(s1) == (block, 1)


@pytest.mark.parametrize("bad", ["q4s-block12-f32-packed-axis0", "q4s-block0128-f32-packed-axis0",
                                 "q4s-block128-f32-packed-axis1", "q4s-block128x1-f32-packed-axis0",
                                 "q8s-block32-f32", "f16", "q4s-block64-f32-packed-axis0 "])
def test_other_spellings_rejected(bad):
    with pytest.raises(Bq4Error, match="EINVAL_ARG"):
        q4.parse_stored_dtype(bad)


def test_packer_payload_sizes_match_the_contract():
    rng = np.random.default_rng(0)
    col = q4.quantize_q4s_block128_f32(rng.standard_normal((96, 256)).astype(np.float32), (96, 256))
    assert col.stored_dtype == "q4s-block128-f32-packed-axis0"
    assert len(col.to_bytes()) == 96 * 256 // 2 + 96 * 256 // 128 * 4
    row = q4.quantize_row_layout_q4s_block_up_to128_f32(rng.standard_normal((480, 64)).astype(np.float32), (480, 64))
    assert row.stored_dtype == "q4s-block32x1-f32-packed-axis1"  # 480 = 32 * 15
    assert len(row.to_bytes()) == 480 * 64 // 2 + 480 // 32 * 64 * 4


def test_payload_loader_rejects_before_any_device_work():
    lib = L.lib()
    out = ctypes.c_void_p()
    payload = (ctypes.c_uint8 * 1000)()
    rc = lib.bq4_weight_prepare_payload(payload, 1000, 16, 128, b"q4s-block128-f32-packed-axis0", 1, 0,
                                        ctypes.byref(out))
    assert rc == L.EINVAL_SHAPE  # 16 x 128 at block 128 needs 1024 + 64 bytes
    assert b"needs 1088" in lib.bq4_last_error_string()
    rc = lib.bq4_weight_prepare_payload(payload, 1000, 16, 128, b"q4s-block128", 1, 0, ctypes.byref(out))
    assert rc == L.EINVAL_ARG
