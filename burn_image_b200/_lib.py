"""ctypes binding of libbq4.so (the C ABI declared in include/bq4.h).

The shared library is built in-tree by ``burn_image_b200/build.py``.  There
is no fallback: when the library is missing or the device is not an sm_100
GPU, calls raise instead of computing anything on the CPU.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbq4.so")

# bq4_status
OK, EINVAL_SHAPE, EINVAL_BLOCK, EALIGN, ECUDA, ENCCL, ETIMEOUT, EINVAL_ARG, EWORKSPACE, ENONFINITE, EUNSUPPORTED = range(11)
STATUS_NAMES = {
    0: "BQ4_OK", 1: "BQ4_EINVAL_SHAPE", 2: "BQ4_EINVAL_BLOCK", 3: "BQ4_EALIGN", 4: "BQ4_ECUDA",
    5: "BQ4_ENCCL", 6: "BQ4_ETIMEOUT", 7: "BQ4_EINVAL_ARG", 8: "BQ4_EWORKSPACE",
    9: "BQ4_ENONFINITE", 10: "BQ4_EUNSUPPORTED",
}
LAYOUT_COL, LAYOUT_ROW, LAYOUT_NPACKED, LAYOUT_F16 = 0, 1, 2, 3
ACT_NONE, ACT_GELU_TANH, ACT_SILU = 0, 1, 2
NOALLOC_SCRATCH_BYTES = 32 << 20  # BQ4_NOALLOC_SCRATCH_BYTES
NUMERICS_AUTO, NUMERICS_EXACT, NUMERICS_FOLDED = 0, 1, 2
DTYPE_F32, DTYPE_F16 = 0, 1
MAX_PEERS = 8            # BQ4_MAX_PEERS
IPC_HANDLE_BYTES = 64    # BQ4_IPC_HANDLE_BYTES

# Every symbol include/bq4.h declares, with (restype, argtypes).
_p, _i32, _i64, _sz, _u64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_uint64
_st = ctypes.c_int
SIGNATURES = {
    "bq4_version": (ctypes.c_char_p, []),
    "bq4_last_error_string": (ctypes.c_char_p, []),
    "bq4_weight_prepare": (_st, [_p, _p, _i64, _i64, _i32, _i32, _i32, ctypes.POINTER(_p)]),
    "bq4_weight_prepare_shard": (_st, [_p, _p, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(_p)]),
    "bq4_weight_free": (_st, [_p]),
    "bq4_weight_info": (_st, [_p, ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_i32),
                              ctypes.POINTER(_i32), ctypes.POINTER(_sz)]),
    "bq4_linear_workspace_size": (_st, [_p, _i64, ctypes.POINTER(_sz)]),
    "bq4_linear_plan_info": (_st, [_p, _i64, _i32, ctypes.POINTER(_i32), _i32]),
    "bq4_linear": (_st, [_p, _p, _i64, _i64, _p, _i32, _p, _p, _p, _sz, _p]),
    "bq4_linear_noalloc": (_st, [_p, _p, _i64, _i64, _p, _i32, _p, _p, _p]),
    "bq4_linear_ex_workspace_size": (_st, [_p, _i64, _i32, ctypes.POINTER(_sz)]),
    "bq4_linear_ex": (_st, [_p, _p, _i32, _i64, _i64, _p, _i32, _p, _p, _i32, _i64, _p, _sz, _p]),
    "bq4_linear_gated_workspace_size": (_st, [_p, _p, _i64, ctypes.POINTER(_sz)]),
    "bq4_linear_gated": (_st, [_p, _p, _p, _i64, _i64, _p, _p, _p, _p, _sz, _p]),
    "bq4_dequant": (_st, [_p, _p, _i32, _p]),
    "bq4_dequant_raw": (_st, [_p, _p, _i64, _i64, _i32, _i32, _p, _i32, _p]),
    "bq4_q_matmul_workspace_size": (_st, [_i64, _i64, _i64, _p, ctypes.POINTER(_sz)]),
    "bq4_q_matmul": (_st, [_p, _i64, _i64, _p, _p, _i64, _p, _p, _p, _sz, _p]),
    "bq4_quantize_col_block128": (_st, [_p, _i64, _i64, _p, _p]),
    "bq4_quantize_row_up_to128": (_st, [_p, _i64, _i64, _p, _p, ctypes.POINTER(_i32)]),
    "bq4_row_block_for": (_i32, [_i64]),
    "bq4_poll_device_error": (_st, []),
    "bq4_set_numerics": (_st, [_i32]),
    "bq4_set_sm_budget": (_st, [_i32]),
    "bq4_parse_stored_dtype": (_st, [ctypes.c_char_p, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "bq4_weight_prepare_payload": (_st, [_p, _sz, _i64, _i64, ctypes.c_char_p, _i32, _i32, ctypes.POINTER(_p)]),
    "bq4_q_select_rows": (_st, [_p, _p, _i64, _i64, _i32, _p, _i32, _i64, _p, _p, _p]),
    "bq4_q_select_rows_dequant": (_st, [_p, _p, _i64, _i64, _i32, _p, _i32, _i64, _p, _p]),
    "bq4_rms_renorm": (_st, [_p, _i32, _i64, _i64, _i64, _p, _i32, _i64, ctypes.c_float, _p]),
    "bq4_qk_norm_rope": (_st, [_p, _i32, _i64, _i64, _i64, _i64, _p, ctypes.c_float, _p, _p, _i64, _p, _i32, _i64,
                               _p]),
    "bq4_linear_qk_norm_rope_workspace_size": (_st, [_p, _i64, _i32, _i64, ctypes.POINTER(_sz)]),
    "bq4_peer_buffer_alloc": (_st, [_sz, _i32, ctypes.POINTER(_p), _p]),
    "bq4_peer_buffer_open": (_st, [_p, _i32, ctypes.POINTER(_p)]),
    "bq4_peer_buffer_close": (_st, [_p]),
    "bq4_peer_buffer_free": (_st, [_p, _i32]),
    "bq4_peer_signal_wait": (_st, [_p, _p, _i32, _i32, ctypes.c_uint32, _p]),
    "bq4_set_peer_wait_timeout_ns": (_st, [_u64]),
    "bq4_reduce_slices": (_st, [_p, _i32, _i64, _i64, _i64, _i32, ctypes.c_float, _p, _i32, _i64, _p]),
    "bq4_reduce_slices_peer": (_st, [_p, _i32, _i64, _i64, _i64, _i64, _i32, ctypes.c_float, _p, _i32, _i64, _p]),
    "bq4_reduce_slices_peer_bcast": (_st, [_p, _i32, _i64, _i64, _i64, _i64, _i32, ctypes.c_float, _p, _i32, _i64,
                                           _p]),
    "bq4_linear_rowscatter": (_st, [_p, _p, _i32, _i64, _i64, _p, _i32, _p, _i32, _i32, _i64, _p, _sz, _p]),
    "bq4_linear_qk_norm_rope": (_st, [_p, _p, _i32, _i64, _i64, _p, _i64, _i64, _i64, _p, _p, ctypes.c_float, _p, _p,
                                      _i64, _p, _i32, _i64, _p, _sz, _p]),
    "bq4_packed_f16_to_f32": (_st, [_p, _i32, ctypes.POINTER(_i64), ctypes.POINTER(_i64), _p, _p]),
    "bq4_packed_f16_select_rows": (_st, [_p, _i64, _i64, _p, _i64, _p, _p]),
    "bq4_f16_weight_prepare": (_st, [_p, _i64, _i64, _i64, _i64, _i32, ctypes.POINTER(_p)]),
    "bq4_packed_f16_rhs_matmul_workspace_size": (_st, [_i64, _i64, _i64, ctypes.POINTER(_sz)]),
    "bq4_packed_f16_rhs_matmul": (_st, [_p, _i64, _i64, _p, _i64, _i64, _i64, _p, _p, _sz, _p]),
    "bq4_f16_conv_weight_prepare": (_st, [_p, _i64, _i64, _i32, _i32, _i32, ctypes.POINTER(_p)]),
    "bq4_conv2d_workspace_size": (_st, [_p, _i64, _i64, _i64, _p, ctypes.POINTER(_sz)]),
    "bq4_conv2d": (_st, [_p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _sz, _p]),
    "bq4_packed_f16_conv2d_workspace_size": (_st, [_i64, _i64, _i64, _i64, _i64, _i32, _i32, _p,
                                                   ctypes.POINTER(_sz)]),
    "bq4_packed_f16_conv2d": (_st, [_p, _i64, _i64, _i64, _i64, _p, _i64, _i32, _i32, _p, _p, _p, _p, _sz, _p]),
    "bq4_attention_workspace_size": (_st, [_i64, _i64, _i64, _i64, _i64, _i64, ctypes.POINTER(_sz)]),
    "bq4_attention": (_st, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _p, _p, _sz, _p]),
    "bq4_launch_count": (_u64, []),
    "bq4_launch_count_reset": (None, []),
}


class QuantScheme(ctypes.Structure):
    """bq4_quant_scheme: the reference QuantScheme fields on this path."""
    _fields_ = [("value", _i32), ("mode", _i32), ("param", _i32), ("store_packed_dim", _i32),
                ("block_rank", _i32), ("block", _i32), ("rhs_transposed_view", _i32)]


class Conv2dOptions(ctypes.Structure):
    """bq4_conv2d_options: Burn ConvOptions<2> ([height, width] pairs, groups)."""
    _fields_ = [("stride", _i32 * 2), ("padding", _i32 * 2), ("dilation", _i32 * 2), ("groups", _i32)]


class Bq4Error(RuntimeError):
    """A non-OK bq4_status.  The reference unwraps its setup errors (a panic,
    patches/burn-cubecl-0.21.0/src/ops/qtensor.rs:360); here they raise."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libbq4.so not found at {LIB_PATH}; build it with `python burn_image_b200/build.py` "
                "(there is no CPU fallback)")
        _lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def check(status: int) -> None:
    if status != OK:
        raise Bq4Error(status, lib().bq4_last_error_string().decode(errors="replace"))
