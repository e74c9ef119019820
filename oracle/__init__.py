"""ctypes front end of the CPU oracle (``oracle/bq4_oracle.c``).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA product and the
timed CPU baseline.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py`` (its cpu_baseline leg and ``--impl reference`` arm) import this
package; the product path in ``burn_image_b200`` never does.

Every function restates the reference algorithm; the C file cites the
reference file:line of each step.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liborc.so")

LAYOUT_COL = 0  # PackedU32(0): tensor [N,K], words [N][K/8], scales [N][K/b]
LAYOUT_ROW = 1  # PackedU32(1): tensor [K,N], words [K/8][N], scales [K/b][N]
ACT_NONE, ACT_GELU_TANH, ACT_SILU = 0, 1, 2

OK, ENONFINITE, ESHAPE, EBLOCK = 0, 1, 2, 3

_lib = None


def build() -> str:
    """Compile liborc.so with the committed Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        i64, i32, p = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p
        _lib.orc_quantize_col_block128.argtypes = [p, i64, i64, p, p]
        _lib.orc_quantize_row_up_to128.argtypes = [p, i64, i64, p, p, p]
        _lib.orc_row_block_for.argtypes = [i64]
        _lib.orc_unpack.argtypes = [p, p, i64, i64, i32, i32, p]
        _lib.orc_select_rows.argtypes = [p, p, i64, i64, i32, p, i64, p, p, p]
        _lib.orc_linear_f64.argtypes = [p, i64, i64, i64, p, i64, p, i32, p, p]
        _lib.orc_linear_f64.restype = None
        _lib.orc_linear_gated_f64.argtypes = [p, i64, i64, i64, p, p, i64, p, p, p]
        _lib.orc_linear_gated_f64.restype = None
        _lib.orc_cpu_linear.argtypes = [p, p, i64, i64, i32, i32, p, i64, i64, p, i32, p, p, i32]
        _lib.orc_cpu_threads.argtypes = []
        _lib.orc_qk_norm_rope_f64.argtypes = [p, i64, i64, i64, i64, p, ctypes.c_double, p, p, i64, p, i64]
        _lib.orc_qk_norm_rope_f64.restype = None
        _lib.orc_f16_widen_bits.argtypes = [p, i64, p]
        _lib.orc_f16_widen_bits.restype = None
        _lib.orc_f16_matmul_f64.argtypes = [p, i64, i64, p, i64, i64, i64, p, p]
        _lib.orc_f16_matmul_f64.restype = None
        _lib.orc_f16_conv2d_f64.argtypes = [p, i64, i64, i64, i64, p, i64, i64, i64, p] + [i64] * 6 + [p]
        _lib.orc_f16_conv2d_f64.restype = None
        _lib.orc_cpu_f16_matmul.argtypes = [p, i64, i64, p, i64, i64, i64, p, i32]
        _lib.orc_cpu_f16_conv2d.argtypes = [p, i64, i64, i64, i64, p, i64, i64, i64, p] + [i64] * 6 + [p, i32]
        _lib.orc_attention_f64.argtypes = [p, p, p, i64, i64, i64, i64, i64, i64, ctypes.c_double, p]
        _lib.orc_attention_f64.restype = None
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


class OracleError(ValueError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: oracle status {code}")
        self.code = code


def quantize_col_block128(values: np.ndarray):
    """Qwen column-layout packer (crates/burn_qwen3_vl/src/artifacts.rs:1301-1366).

    values: [rows, inner] float.  Returns (words u32 [rows, inner/8],
    scales f32 [rows, inner/128]) -- the reference's byte stream is
    ``words.tobytes() + scales.tobytes()``.
    """
    v = _f32(values)
    if v.ndim < 1 or v.size == 0:
        raise OracleError(ESHAPE, "quantize_col_block128")
    rows = int(np.prod(v.shape[:-1])) if v.ndim > 1 else 1
    inner = int(v.shape[-1])
    words = np.zeros((rows, max(inner // 8, 1)), dtype=np.uint32)
    scales = np.zeros((rows, max(inner // 128, 1)), dtype=np.float32)
    rc = lib().orc_quantize_col_block128(_ptr(v), rows, inner, _ptr(words), _ptr(scales))
    if rc:
        raise OracleError(rc, "quantize_col_block128")
    return words, scales


def quantize_row_up_to128(values: np.ndarray):
    """Boogu row-layout packer (crates/burn_boogu/src/artifacts.rs:7296-7385).

    values: [input K, output N] float.  Returns (words u32 [K/8, N],
    scales f32 [K/b, N], block b).
    """
    v = _f32(values)
    if v.ndim != 2:
        raise OracleError(ESHAPE, "quantize_row_up_to128")
    K, N = v.shape
    b = int(lib().orc_row_block_for(K)) or 8
    words = np.zeros((max(K // 8, 1), N), dtype=np.uint32)
    scales = np.zeros((max(K // b, 1), N), dtype=np.float32)
    blk = ctypes.c_int32(0)
    rc = lib().orc_quantize_row_up_to128(_ptr(v), K, N, _ptr(words), _ptr(scales), ctypes.byref(blk))
    if rc:
        raise OracleError(rc, "quantize_row_up_to128")
    return words, scales, int(blk.value)


def unpack(words: np.ndarray, scales: np.ndarray, K: int, N: int, block: int, layout: int) -> np.ndarray:
    """Dequantized logical weight W [K, N] (y = x . W), f32, q * scale."""
    w = np.ascontiguousarray(words, dtype=np.uint32)
    s = _f32(scales)
    out = np.empty((K, N), dtype=np.float32)
    rc = lib().orc_unpack(_ptr(w), _ptr(s), K, N, block, layout, _ptr(out))
    if rc:
        raise OracleError(rc, "unpack")
    return out


def select_rows(words: np.ndarray, scales: np.ndarray, rows: int, cols: int, block: int, ids) -> tuple:
    """q_select on dim 0 of a packed [rows, cols] table (PackedU32(0), blocks
    along the row): (selected words [n, cols/8], scales [n, cols/block],
    dequantized rows [n, cols] f32, ok).  ok is False when an index was out
    of range (its row is zero)."""
    w = np.ascontiguousarray(words, dtype=np.uint32)
    s = _f32(scales)
    idx = np.ascontiguousarray(ids, dtype=np.int64)
    n = idx.shape[0]
    ow = np.empty((n, cols // 8), dtype=np.uint32)
    osc = np.empty((n, cols // block), dtype=np.float32)
    of = np.empty((n, cols), dtype=np.float32)
    rc = lib().orc_select_rows(_ptr(w), _ptr(s), rows, cols, block, _ptr(idx), n, _ptr(ow), _ptr(osc), _ptr(of))
    if rc not in (0, 2):
        raise OracleError(rc, "select_rows")
    return ow, osc, of, rc == 0


def linear_f64(x: np.ndarray, w_kn: np.ndarray, bias=None, act: int = ACT_NONE, aux=None) -> np.ndarray:
    """f64-accumulated reference linear: act(x . W + bias) (* aux)."""
    x = _f32(x)
    w = _f32(w_kn)
    M, K = x.shape
    N = w.shape[1]
    y = np.empty((M, N), dtype=np.float32)
    lib().orc_linear_f64(_ptr(x), M, K, K, _ptr(w), N, _ptr(_f32(bias)), act, _ptr(_f32(aux)), _ptr(y))
    return y


def linear_gated_f64(x, wg_kn, wu_kn, bg=None, bu=None) -> np.ndarray:
    """f64-accumulated silu(x . Wg + bg) * (x . Wu + bu)."""
    x = _f32(x)
    M, K = x.shape
    N = wg_kn.shape[1]
    y = np.empty((M, N), dtype=np.float32)
    lib().orc_linear_gated_f64(_ptr(x), M, K, K, _ptr(_f32(wg_kn)), _ptr(_f32(wu_kn)), N,
                               _ptr(_f32(bg)), _ptr(_f32(bu)), _ptr(y))
    return y


def cpu_linear(words, scales, K, N, block, layout, x, bias=None, act=ACT_NONE, aux=None,
               threads: int = 0, out=None) -> np.ndarray:
    """Timed CPU baseline (dequantize + blocked SGEMM + epilogue, OpenMP)."""
    x = _f32(x)
    M = x.shape[0]
    y = out if out is not None else np.empty((M, N), dtype=np.float32)
    rc = lib().orc_cpu_linear(_ptr(np.ascontiguousarray(words, dtype=np.uint32)), _ptr(_f32(scales)),
                              K, N, block, layout, _ptr(x), M, x.shape[1], _ptr(_f32(bias)), act,
                              _ptr(_f32(aux)), _ptr(y), threads)
    if rc:
        raise OracleError(rc, "cpu_linear")
    return y


def cpu_threads() -> int:
    return int(lib().orc_cpu_threads())


def qk_norm_rope_f64(x: np.ndarray, heads: int, head_dim: int, gamma=None, eps: float = 1e-5,
                     cos=None, sin=None) -> np.ndarray:
    """RMS-normalise each head of x [M, heads*head_dim] (times gamma), then
    rotate interleaved pairs by the per-(token, dim) cos/sin [M, head_dim];
    f64 inside, f32 out (bq4_oracle.c orc_qk_norm_rope_f64)."""
    x = _f32(x)
    M = x.shape[0]
    assert x.shape[1] >= heads * head_dim and head_dim % 2 == 0
    g = None if gamma is None else _f32(gamma)
    c = None if cos is None else _f32(cos)
    s = None if sin is None else _f32(sin)
    y = np.zeros((M, heads * head_dim), dtype=np.float32)
    lib().orc_qk_norm_rope_f64(_ptr(x), M, heads, head_dim, x.shape[1], _ptr(g), float(eps), _ptr(c), _ptr(s),
                               head_dim if c is None else c.shape[1], _ptr(y), heads * head_dim)
    return y


def rope_tables(ids: np.ndarray, axis_dims, theta: float = 10000.0):
    """cos/sin [S, sum(axis_dims)] for position ids [S, 3]: per axis, pair p of
    that axis' dims rotates by id * theta^(-2p/dim), each value repeated for
    the two dims of the pair (crates/burn_boogu/src/model/denoiser.rs:992-1032)."""
    ids = np.asarray(ids)
    cos_parts, sin_parts = [], []
    for axis, dim in enumerate(axis_dims):
        inv = theta ** (-(2.0 * np.arange(dim // 2)) / dim)
        phase = ids[:, axis:axis + 1].astype(np.float64) * inv[None, :]
        cos_parts.append(np.repeat(np.cos(phase).astype(np.float32), 2, axis=1))
        sin_parts.append(np.repeat(np.sin(phase).astype(np.float32), 2, axis=1))
    return np.concatenate(cos_parts, 1), np.concatenate(sin_parts, 1)


def rel_frobenius(actual: np.ndarray, expected: np.ndarray) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    den = np.sqrt((e * e).sum())
    return float(np.sqrt(((a - e) ** 2).sum()) / (den if den > 0 else 1.0))


# ---------------------------------------------------------------- packed F16

def _bits(a) -> np.ndarray:
    """binary16 bit patterns (uint16) of a float16 / uint16 array."""
    a = np.asarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    return np.ascontiguousarray(a, dtype=np.uint16)


def f16_widen_bits(bits) -> np.ndarray:
    """binary32 bit patterns of binary16 bit patterns (packed_f16.rs:48-74)."""
    h = _bits(bits)
    out = np.empty(h.shape, dtype=np.uint32)
    lib().orc_f16_widen_bits(_ptr(h), h.size, _ptr(out))
    return out


def f16_matmul_f64(lhs, rhs_bits, K: int, N: int, inner: int, col: int, bias=None) -> np.ndarray:
    """lhs f32 [M, K] times the packed rhs (element (k, n) at k*inner + n*col
    of rhs_bits), f64 accumulation (packed_f16.rs:133-292)."""
    x = _f32(lhs).reshape(-1, K)
    h = _bits(rhs_bits).reshape(-1)
    out = np.empty((x.shape[0], N), dtype=np.float64)
    lib().orc_f16_matmul_f64(_ptr(x), x.shape[0], K, _ptr(h), inner, col, N, _ptr(_f32(bias)), _ptr(out))
    return out


def f16_conv2d_f64(inp, weight_bits, bias=None, stride=(1, 1), padding=(0, 0), dilation=(1, 1)) -> np.ndarray:
    """NCHW f32 input, OIHW binary16 weight, groups 1, f64 accumulation
    (packed_f16.rs:375-602)."""
    x = _f32(inp)
    B, C, H, W = x.shape
    wb = _bits(weight_bits)
    O, Cw, kh, kw = wb.shape
    assert Cw == C
    OH = (H + 2 * padding[0] - dilation[0] * (kh - 1) - 1) // stride[0] + 1
    OW = (W + 2 * padding[1] - dilation[1] * (kw - 1) - 1) // stride[1] + 1
    out = np.empty((B, O, OH, OW), dtype=np.float64)
    lib().orc_f16_conv2d_f64(_ptr(x), B, C, H, W, _ptr(wb), O, kh, kw, _ptr(_f32(bias)), stride[0], stride[1],
                             padding[0], padding[1], dilation[0], dilation[1], _ptr(out))
    return out


def cpu_f16_matmul(lhs, rhs_bits, K: int, N: int, inner: int, col: int, threads: int = 0, out=None) -> np.ndarray:
    """Timed CPU arm: rhs widened to f32 panels, blocked SGEMM (OpenMP)."""
    x = _f32(lhs).reshape(-1, K)
    y = out if out is not None else np.empty((x.shape[0], N), dtype=np.float32)
    rc = lib().orc_cpu_f16_matmul(_ptr(x), x.shape[0], K, _ptr(_bits(rhs_bits)), inner, col, N, _ptr(y), threads)
    if rc:
        raise OracleError(rc, "cpu_f16_matmul")
    return y


def cpu_f16_conv2d(inp, weight_bits, bias=None, stride=(1, 1), padding=(0, 0), dilation=(1, 1), threads: int = 0,
                   out=None) -> np.ndarray:
    """Timed CPU arm: im2col blocks times the widened OIHW panels (OpenMP)."""
    x = _f32(inp)
    B, C, H, W = x.shape
    wb = _bits(weight_bits)
    O, _, kh, kw = wb.shape
    OH = (H + 2 * padding[0] - dilation[0] * (kh - 1) - 1) // stride[0] + 1
    OW = (W + 2 * padding[1] - dilation[1] * (kw - 1) - 1) // stride[1] + 1
    y = out if out is not None else np.empty((B, O, OH, OW), dtype=np.float32)
    rc = lib().orc_cpu_f16_conv2d(_ptr(x), B, C, H, W, _ptr(wb), O, kh, kw, _ptr(_f32(bias)), stride[0], stride[1],
                                  padding[0], padding[1], dilation[0], dilation[1], _ptr(y), threads)
    if rc:
        raise OracleError(rc, "cpu_f16_conv2d")
    return y


def attention_f64(q, k, v, scale=None) -> np.ndarray:
    """softmax(scale q k^T) v per batch and query head, query head h on kv
    head h // (Hq // Hkv); q [B,Hq,Sq,D], k/v [B,Hkv,Skv,D]; f64 out."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    assert Hq % Hkv == 0 and v.shape == k.shape
    out = np.empty((B, Hq, Sq, D), dtype=np.float64)
    lib().orc_attention_f64(_ptr(q), _ptr(k), _ptr(v), B, Hq, Hkv, Sq, Skv, D,
                            float(scale if scale is not None else 1.0 / np.sqrt(D)), _ptr(out))
    return out
