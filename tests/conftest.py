import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) CUDA device")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


# ----------------------------------------------------------------- synthetic data
# Distributions of BASELINE.json: activations ~N(0,1) f32; int4 values uniform
# in [-8, 7] drawn directly as nibbles; f32 scales |U(0.001, 0.02)|; bias ~N(0, 0.02).

def gen_q4(K: int, N: int, block: int, layout: int, rng: np.random.Generator):
    """Raw reference-packed words and scales for a K x N weight (layout 0 COL,
    1 ROW, 2 NPACKED)."""
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int64)  # logical [K][N]
    nib = (q & 0xF).astype(np.uint32)
    scales_kn = np.abs(rng.uniform(0.001, 0.02, size=(K // block, N))).astype(np.float32)
    if layout == 2:  # NPACKED: words [K][N/8] (8 consecutive N per word), scales [K][N/b]
        w = np.zeros((K, N // 8), dtype=np.uint32)
        for lane in range(8):
            w |= nib[:, lane::8] << np.uint32(4 * lane)
        s = np.abs(rng.uniform(0.001, 0.02, size=(K, N // block))).astype(np.float32)
    elif layout == 1:  # ROW: words [K/8][N]
        w = np.zeros((K // 8, N), dtype=np.uint32)
        for lane in range(8):
            w |= nib[lane::8, :] << np.uint32(4 * lane)
        s = scales_kn
    else:  # COL: words [N][K/8], scales [N][K/b]
        nt = nib.T  # [N][K]
        w = np.zeros((N, K // 8), dtype=np.uint32)
        for lane in range(8):
            w |= nt[:, lane::8] << np.uint32(4 * lane)
        s = np.ascontiguousarray(scales_kn.T)
    return np.ascontiguousarray(w), np.ascontiguousarray(s)


def gen_x(M: int, K: int, rng: np.random.Generator):
    return rng.standard_normal((M, K), dtype=np.float32)


def gen_bias(N: int, rng: np.random.Generator):
    return (rng.standard_normal(N, dtype=np.float32) * np.float32(0.02)).astype(np.float32)


@pytest.fixture
def rng():
    return np.random.default_rng(20261201)
