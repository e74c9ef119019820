"""CPU: the C-ABI library loads, exports every symbol include/bq4.h declares,
and rejects bad arguments with status codes (no compute without a GPU)."""
import ctypes
import os
import re

import numpy as np
import pytest

from burn_image_b200 import _lib as L
from burn_image_b200 import q4

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "bq4.h")).read()
    return sorted(set(re.findall(r"^BQ4_API\s+[\w\s\*]+?\b(bq4_\w+)\(", text, re.M)))


def test_header_declares_expected_entry_points():
    syms = declared_symbols()
    for name in ("bq4_weight_prepare", "bq4_linear", "bq4_linear_gated", "bq4_dequant",
                 "bq4_dequant_raw", "bq4_q_matmul", "bq4_last_error_string"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in L.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_string():
    lib = L.lib()
    assert lib.bq4_version().decode().startswith("bq4")
    assert isinstance(lib.bq4_last_error_string(), bytes)


def test_invalid_geometry_returns_status():
    lib = L.lib()
    out = ctypes.c_void_p()
    w = np.zeros(16, np.uint32)
    s = np.ones(4, np.float32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    # block 12 invalid
    assert lib.bq4_weight_prepare(p(w), p(s), 128, 8, 12, 1, 0, ctypes.byref(out)) == L.EINVAL_BLOCK
    # K not multiple of block
    assert lib.bq4_weight_prepare(p(w), p(s), 72, 8, 64, 1, 0, ctypes.byref(out)) == L.EINVAL_BLOCK
    # K not multiple of 8
    assert lib.bq4_weight_prepare(p(w), p(s), 12, 8, 8, 1, 0, ctypes.byref(out)) == L.EINVAL_SHAPE
    # bad layout
    assert lib.bq4_weight_prepare(p(w), p(s), 128, 8, 128, 5, 0, ctypes.byref(out)) == L.EINVAL_ARG
    # NULL out
    assert lib.bq4_weight_prepare(p(w), p(s), 128, 8, 128, 1, 0, None) == L.EINVAL_ARG
    assert b"NULL" in lib.bq4_last_error_string()
    # row shard that does not fall on block boundaries: 3360 / 2 = 1680 not multiple of 128? (block 32 ok)
    assert lib.bq4_weight_prepare_shard(p(w), p(s), 3360, 8, 32, 1, 1, 0, 4, 0, ctypes.byref(out)) == L.EINVAL_BLOCK


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="CPU-only behaviour")
def test_no_gpu_fails_loudly():
    """Without an sm_100 device the library refuses instead of computing."""
    lib = L.lib()
    out = ctypes.c_void_p()
    w = np.zeros(16 * 8, np.uint32)
    s = np.ones(8, np.float32)
    rc = lib.bq4_weight_prepare(w.ctypes.data_as(ctypes.c_void_p), s.ctypes.data_as(ctypes.c_void_p),
                                128, 8, 128, 1, 0, ctypes.byref(out))
    assert rc in (L.EINVAL_ARG, L.EUNSUPPORTED, L.ECUDA)
    assert not out.value


def test_scheme_eligibility_mirror():
    """patches/burn-cubecl-0.21.0/src/ops/qtensor.rs:304-323."""
    S = q4.QuantScheme
    assert S(store_packed_dim=0, level=(128,)).eligible()
    assert S(store_packed_dim=1, level=(32, 1)).eligible()
    for b in (8, 16, 32, 64, 128):
        assert S(level=(b,)).eligible()
    assert not S(level=(256,)).eligible()
    assert not S(level=(12,)).eligible()
    assert not S(level=(32, 2)).eligible()
    assert not S(value="Q8S").eligible()
    assert not S(param="F16").eligible()
    assert not S(mode="Affine").eligible()
    assert not S(store_packed_dim=2).eligible()
