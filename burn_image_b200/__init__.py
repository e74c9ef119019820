"""burn_image_b200 -- B200-native packed signed-Q4 linear (dequant-matmul +
bias / GELU-tanh / SiLU-gate epilogue) for burn_image, and the packed-F16
widening / matmul / convolution kernels beside it, behind a C ABI
(include/bq4.h, libbq4.so) with a host mirror of the reference interface.
"""
from ._lib import (ACT_GELU_TANH, ACT_NONE, ACT_SILU, LAYOUT_COL, LAYOUT_NPACKED, LAYOUT_ROW,  # noqa: F401
                   LIB_PATH, Bq4Error)
from .q4 import (PackedQ4, PreparedQ4Weight, Q4Linear, QuantizedTensor, QuantScheme,  # noqa: F401
                 feed_forward_swiglu, linear_forward, linear_gated, poll_device_error, q_matmul,
                 quantize_q4s_block128_f32, quantize_row_layout_q4s_block_up_to128_f32,
                 qwen_linear_forward)

from .f16 import (ConvOptions, PreparedF16ConvWeight, PreparedF16Weight, packed_f16_conv2d,  # noqa: F401
                  packed_f16_rhs_matmul, packed_f16_select_rows, packed_f16_to_f32)

__version__ = "0.1.0"
