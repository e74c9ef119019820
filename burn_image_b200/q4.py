"""Host-side mirror of burn_image's packed-Q4 linear interface over libbq4.

Names and argument meanings follow the reference so that parity tests read
like the reference's own tests:

* ``quantize_q4s_block128_f32`` -- Qwen column-layout packer
  (crates/burn_qwen3_vl/src/artifacts.rs:1301-1366)
* ``quantize_row_layout_q4s_block_up_to128_f32`` -- Boogu row-layout packer
  (crates/burn_boogu/src/artifacts.rs:7296-7385)
* ``QuantizedTensor`` / ``QuantScheme`` -- a QFloat tensor (packed u32 values
  plus F32 scales, patches/burn-cubecl-0.21.0/src/ops/qtensor.rs:64-158)
* ``q_matmul`` -- ``QTensorOps::q_matmul`` (qtensor.rs:303-368)
* ``Q4Linear`` + ``linear_forward`` / ``qwen_linear_forward`` -- the linear
  adapters (crates/burn_boogu/src/model/linear.rs:14-37,
  crates/burn_qwen3_vl/src/linear.rs:107-140), with the bias and activation
  fused into the kernel epilogue.

Device memory and streams come from PyTorch; all arithmetic is done by the
CUDA kernels in libbq4.so.  Tensors must live on an sm_100 CUDA device.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib as L
from ._lib import Bq4Error, check

VALUES_PER_WORD = 8
SUPPORTED_BLOCKS = (8, 16, 32, 64, 128)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream_ptr(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


# --------------------------------------------------------------------- packers

@dataclass
class PackedQ4:
    """Reference byte stream split into its two parts: ``words`` (u32, the
    first N*K/2 bytes) and ``scales`` (f32, the rest), plus the scheme."""
    words: np.ndarray
    scales: np.ndarray
    shape: tuple
    scheme: "QuantScheme"

    def to_bytes(self) -> bytes:
        return self.words.astype("<u4").tobytes() + self.scales.astype("<f4").tobytes()

    @property
    def stored_dtype(self) -> str:
        """The sealed-inventory spelling of this tensor's storage contract."""
        return q4s_stored_dtype(self.scheme.block, self.scheme.store_packed_dim)


def q4s_stored_dtype(block: int, axis: int) -> str:
    """crates/burn_boogu/src/artifacts.rs:527-537 -- the stable inventory
    spelling of one Q4S / F32-scale storage contract."""
    return f"q4s-block{block}-f32-packed-axis0" if axis == 0 else f"q4s-block{block}x1-f32-packed-axis1"


def parse_stored_dtype(stored_dtype: str) -> tuple:
    """(block, packed axis) of a packed-Q4 inventory spelling (through the C
    ABI's parser); raises for any other dtype."""
    block, axis = ctypes.c_int32(), ctypes.c_int32()
    check(L.lib().bq4_parse_stored_dtype(stored_dtype.encode(), ctypes.byref(block), ctypes.byref(axis)))
    return block.value, axis.value


def quantize_q4s_block128_f32(values, shape: Sequence[int]) -> PackedQ4:
    """Column layout (Qwen, ``PackedU32(0)``, ``Block([128])``): the last axis
    is packed, one F32 scale per contiguous 128-block."""
    v = np.ascontiguousarray(np.asarray(values, dtype=np.float32)).reshape(-1)
    shape = tuple(int(s) for s in shape)
    if len(shape) == 0:
        raise Bq4Error(L.EINVAL_SHAPE, "Q4S block tensor must have at least one dimension")
    if int(np.prod(shape)) != v.size:
        raise Bq4Error(L.EINVAL_SHAPE, f"Q4S shape {shape} describes {int(np.prod(shape))} elements, received {v.size}")
    inner = shape[-1]
    rows = v.size // inner if inner else 0
    words = np.zeros(max(v.size // 8, 1), dtype=np.uint32)
    scales = np.zeros(max(v.size // 128, 1), dtype=np.float32)
    check(L.lib().bq4_quantize_col_block128(v.ctypes.data_as(ctypes.c_void_p), rows, inner,
                                            words.ctypes.data_as(ctypes.c_void_p),
                                            scales.ctypes.data_as(ctypes.c_void_p)))
    return PackedQ4(words, scales, shape, QuantScheme(store_packed_dim=0, level=(128,)))


def quantize_row_layout_q4s_block_up_to128_f32(values, shape: Sequence[int]) -> PackedQ4:
    """Row layout (Boogu, ``PackedU32(1)``, ``Block([b,1])``) of a [input,
    output] matrix; b = largest of 128/64/32/16/8 dividing input."""
    v = np.ascontiguousarray(np.asarray(values, dtype=np.float32)).reshape(-1)
    shape = tuple(int(s) for s in shape)
    if len(shape) != 2:
        raise Bq4Error(L.EINVAL_SHAPE, f"runtime Q4S denoiser quantization requires a rank-two matrix, found {shape}")
    K, N = shape
    b = int(L.lib().bq4_row_block_for(K)) or 8
    words = np.zeros(max(K // 8 * N, 1), dtype=np.uint32)
    scales = np.zeros(max(K // b * N, 1), dtype=np.float32)
    blk = ctypes.c_int32(0)
    check(L.lib().bq4_quantize_row_up_to128(v.ctypes.data_as(ctypes.c_void_p), K, N,
                                            words.ctypes.data_as(ctypes.c_void_p),
                                            scales.ctypes.data_as(ctypes.c_void_p), ctypes.byref(blk)))
    return PackedQ4(words, scales, shape, QuantScheme(store_packed_dim=1, level=(int(blk.value), 1)))


# --------------------------------------------------------------------- scheme

@dataclass(frozen=True)
class QuantScheme:
    """The QuantScheme fields on this path (burn-std 0.21): Q4S values,
    Symmetric mode, F32 params, PackedU32(store_packed_dim), Block(level)."""
    value: str = "Q4S"
    mode: str = "Symmetric"
    param: str = "F32"
    store_packed_dim: int = 0
    level: tuple = (128,)

    @property
    def block(self) -> int:
        return int(self.level[0])

    def eligible(self) -> bool:
        """qtensor.rs:304-323 -- the packed-Q4 kernel's eligibility test."""
        lvl_ok = (len(self.level) == 1 or (len(self.level) == 2 and self.level[1] == 1)) and \
            self.level[0] in SUPPORTED_BLOCKS
        return (self.mode == "Symmetric" and self.value == "Q4S" and self.param == "F32"
                and self.store_packed_dim in (0, 1) and lvl_ok)

    def to_c(self, transposed_view: bool = True) -> L.QuantScheme:
        return L.QuantScheme(value=0 if self.value == "Q4S" else 99,
                             mode=0 if self.mode == "Symmetric" else 99,
                             param=0 if self.param == "F32" else 99,
                             store_packed_dim=self.store_packed_dim,
                             block_rank=len(self.level) if (len(self.level) == 1 or self.level[-1] == 1) else 99,
                             block=self.block, rhs_transposed_view=1 if transposed_view else 0)


# --------------------------------------------------------------------- workspace

class Workspace:
    """Grow-only device scratch per (device, stream).  The C ABI never
    allocates on compute calls; this host helper owns the memory it passes."""
    _cache: dict = {}

    @classmethod
    def get(cls, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        buf = cls._cache.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            cls._cache[key] = buf
        return buf

    @classmethod
    def clear(cls):
        cls._cache.clear()


# --------------------------------------------------------------------- weights

class PreparedQ4Weight:
    """A weight re-laid-out once into the kernels' device layout (the loader
    hook of the north star).  ``K`` input width, ``N`` output width."""

    def __init__(self, words, scales, K: int, N: int, block: int, layout: int,
                 device: Optional[torch.device] = None, shard: Optional[tuple] = None):
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda":
            raise Bq4Error(L.EINVAL_ARG, "prepared Q4 weights live on a CUDA device")
        w = torch.as_tensor(np.ascontiguousarray(words).view(np.int32)) if isinstance(words, np.ndarray) else words
        s = torch.as_tensor(np.ascontiguousarray(scales, dtype=np.float32)) if isinstance(scales, np.ndarray) else scales
        w = w.contiguous()
        s = s.contiguous()
        handle = ctypes.c_void_p()
        lib = L.lib()
        if shard is None:
            check(lib.bq4_weight_prepare(_ptr(w), _ptr(s), K, N, block, layout, dev.index, ctypes.byref(handle)))
        else:
            kind, rank, size = shard
            check(lib.bq4_weight_prepare_shard(_ptr(w), _ptr(s), K, N, block, layout, kind, rank, size,
                                               dev.index, ctypes.byref(handle)))
        self._h = handle
        k, n, b, lay, nb = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_size_t()
        check(lib.bq4_weight_info(handle, ctypes.byref(k), ctypes.byref(n), ctypes.byref(b), ctypes.byref(lay),
                                  ctypes.byref(nb)))
        self.K, self.N, self.block, self.layout, self.device_bytes = k.value, n.value, b.value, lay.value, nb.value
        self.device = dev

    @classmethod
    def from_payload(cls, payload, shape: tuple, stored_dtype: str, transposed_view: bool = True,
                     device=None) -> "PreparedQ4Weight":
        """Loader hook: prepare straight from a stored tensor's QFloat payload
        (the reference's byte stream: packed words, then F32 scales), its
        stored [rows, cols] shape and inventory dtype (bq4_weight_prepare_payload).
        ``transposed_view`` (axis-0 spellings only): the stored tensor is the
        [N, K] weight the matmul sees transposed (Qwen), else a plain [K, N]."""
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if isinstance(payload, torch.Tensor):
            buf, nbytes = payload, payload.numel() * payload.element_size()
            ptr = ctypes.c_void_p(payload.data_ptr())
        else:
            buf = np.frombuffer(bytes(payload), dtype=np.uint8)
            nbytes = buf.size
            ptr = ctypes.c_void_p(buf.ctypes.data)
        rows, cols = int(shape[0]), int(shape[1])
        handle = ctypes.c_void_p()
        check(L.lib().bq4_weight_prepare_payload(ptr, nbytes, rows, cols, stored_dtype.encode(),
                                                 1 if transposed_view else 0, dev.index, ctypes.byref(handle)))
        del buf
        self = cls.__new__(cls)
        self._h = handle
        k, n, b, lay, nb = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_size_t()
        check(L.lib().bq4_weight_info(handle, ctypes.byref(k), ctypes.byref(n), ctypes.byref(b), ctypes.byref(lay),
                                      ctypes.byref(nb)))
        self.K, self.N, self.block, self.layout, self.device_bytes = k.value, n.value, b.value, lay.value, nb.value
        self.device = dev
        return self

    @classmethod
    def from_packed(cls, packed: PackedQ4, device=None, stored: str = "nk") -> "PreparedQ4Weight":
        """stored: for a PackedU32(0) tensor, "nk" = stored [N,K] and used
        through its transposed view (Qwen); "kn" = a plain [K,N] tensor
        (packed and blocked along N)."""
        K, N, layout = physical_layout(packed.scheme, packed.shape, stored)
        return cls(packed.words, packed.scales, K, N, packed.scheme.block, layout, device)

    @property
    def handle(self):
        return self._h

    def free(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            L.lib().bq4_weight_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def dequantize(self, out_layout: int = L.LAYOUT_ROW) -> torch.Tensor:
        shape = (self.K, self.N) if out_layout == L.LAYOUT_ROW else (self.N, self.K)
        out = torch.empty(shape, dtype=torch.float32, device=self.device)
        check(L.lib().bq4_dequant(self._h, _ptr(out), out_layout, _stream_ptr(self.device)))
        return out

    def workspace_bytes(self, M: int) -> int:
        n = ctypes.c_size_t()
        check(L.lib().bq4_linear_workspace_size(self._h, M, ctypes.byref(n)))
        return n.value

    PLAN_FIELDS = ("bt", "ksplit", "grid", "exact", "ta", "stages", "sk_tiles", "dp_tiles", "workspace_256", "wide",
                   "tail_tiles", "tail_split", "skinny")

    def plan_info(self, M: int, gated: bool = False) -> dict:
        """The launch plan of bq4_linear (or of the gated pair) for M rows."""
        info = (ctypes.c_int32 * len(self.PLAN_FIELDS))()
        check(L.lib().bq4_linear_plan_info(self._h, M, 1 if gated else 0, info, len(self.PLAN_FIELDS)))
        return dict(zip(self.PLAN_FIELDS, list(info)))

    def linear(self, x: torch.Tensor, bias: Optional[torch.Tensor] = None, act: int = L.ACT_NONE,
               aux: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y = act(x . W + bias) (* aux) over the last axis of x (leading dims flattened)."""
        x2, lead = _as_rows(x, self.K, self.device)
        M = x2.shape[0]
        y = out if out is not None else torch.empty((M, self.N), dtype=torch.float32, device=self.device)
        _check_out(y, M, self.N, self.device)
        if bias is not None:
            bias = _vec(bias, self.N, self.device)
        if aux is not None:
            aux = aux.reshape(M, self.N)
            _check_out(aux, M, self.N, self.device)
        nbytes = self.workspace_bytes(M)
        ws = Workspace.get(self.device, nbytes)
        check(L.lib().bq4_linear(self._h, _ptr(x2), M, x2.stride(0), _ptr(bias), act, _ptr(aux), _ptr(y),
                                 _ptr(ws), ws.numel(), _stream_ptr(self.device)))
        return y.reshape(*lead, self.N)


    def linear_ex(self, x: torch.Tensor, bias: Optional[torch.Tensor] = None, act: int = L.ACT_NONE,
                  aux: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                  out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """bq4_linear_ex: the same linear for chained activations.  x is a
        float32 or float16 [M, K] view with unit column stride (its row pitch
        is passed on, so a column slice of a wider buffer works; float16 x
        needs K % 128 == 0 and 16-byte aligned rows and is read in place).
        The output is float32 or float16 (``out``'s dtype, else
        ``out_dtype``), written to ``out`` -- an [M, N] view with unit column
        stride, possibly a column slice of a wider buffer."""
        dt = {torch.float32: L.DTYPE_F32, torch.float16: L.DTYPE_F16}
        if x.device != self.device or x.dtype not in dt or x.dim() != 2 or x.shape[1] != self.K or x.stride(1) != 1:
            raise Bq4Error(L.EINVAL_ARG, f"x must be a float32/float16 [M, {self.K}] row view on {self.device}")
        M = x.shape[0]
        y = out if out is not None else torch.empty((M, self.N), dtype=out_dtype, device=self.device)
        if y.device != self.device or y.dtype not in dt or tuple(y.shape) != (M, self.N) or y.stride(1) != 1:
            raise Bq4Error(L.EINVAL_ARG, f"out must be a float32/float16 [{M}, {self.N}] row view on {self.device}")
        if bias is not None:
            bias = _vec(bias, self.N, self.device)
        if aux is not None:
            aux = aux.reshape(M, self.N)
            _check_out(aux, M, self.N, self.device)
        n = ctypes.c_size_t()
        check(L.lib().bq4_linear_ex_workspace_size(self._h, M, dt[x.dtype], ctypes.byref(n)))
        ws = Workspace.get(self.device, n.value) if n.value else None
        check(L.lib().bq4_linear_ex(self._h, _ptr(x), dt[x.dtype], M, x.stride(0), _ptr(bias), act, _ptr(aux),
                                    _ptr(y), dt[y.dtype], y.stride(0), _ptr(ws), ws.numel() if ws is not None else 0,
                                    _stream_ptr(self.device)))
        return y

    def linear_qk_norm_rope(self, x: torch.Tensor, q_heads: int, k_heads: int, head_dim: int,
                            bias: Optional[torch.Tensor] = None, gamma_q: Optional[torch.Tensor] = None,
                            gamma_k: Optional[torch.Tensor] = None, eps: float = 1e-5,
                            cos: Optional[torch.Tensor] = None, sin: Optional[torch.Tensor] = None,
                            out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """bq4_linear_qk_norm_rope: the q/k/v projection (features = q heads,
        k heads, v heads of head_dim) with QK-norm + RoPE on the q and k heads;
        fused into the GEMM epilogue when head_dim == 128.  x as linear_ex;
        gamma_q/gamma_k [head_dim], cos/sin [M, head_dim] float32."""
        dt = {torch.float32: L.DTYPE_F32, torch.float16: L.DTYPE_F16}
        if x.device != self.device or x.dtype not in dt or x.dim() != 2 or x.shape[1] != self.K or x.stride(1) != 1:
            raise Bq4Error(L.EINVAL_ARG, f"x must be a float32/float16 [M, {self.K}] row view on {self.device}")
        M = x.shape[0]
        y = out if out is not None else torch.empty((M, self.N), dtype=out_dtype, device=self.device)
        if y.device != self.device or y.dtype not in dt or tuple(y.shape) != (M, self.N) or y.stride(1) != 1:
            raise Bq4Error(L.EINVAL_ARG, f"out must be a float32/float16 [{M}, {self.N}] row view on {self.device}")
        if bias is not None:
            bias = _vec(bias, self.N, self.device)
        for t in (gamma_q, gamma_k, cos, sin):
            if t is not None and (t.dtype != torch.float32 or t.device != self.device or t.stride(-1) != 1):
                raise Bq4Error(L.EINVAL_ARG, "gamma/cos/sin must be float32 on the weight's device")
        ld_rope = cos.stride(0) if cos is not None else 0
        n = ctypes.c_size_t()
        check(L.lib().bq4_linear_qk_norm_rope_workspace_size(self._h, M, dt[x.dtype], head_dim, ctypes.byref(n)))
        ws = Workspace.get(self.device, n.value) if n.value else None
        check(L.lib().bq4_linear_qk_norm_rope(self._h, _ptr(x), dt[x.dtype], M, x.stride(0), _ptr(bias), q_heads,
                                              k_heads, head_dim, _ptr(gamma_q), _ptr(gamma_k), ctypes.c_float(eps),
                                              _ptr(cos), _ptr(sin), ld_rope, _ptr(y), dt[y.dtype], y.stride(0),
                                              _ptr(ws), ws.numel() if ws is not None else 0,
                                              _stream_ptr(self.device)))
        return y


def rms_renorm(x: torch.Tensor, out: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """out[m,:] = x[m,:] / sqrt(mean(x[m,:]^2) + eps) in one kernel (the
    between-block step of the layer-stack workload); x and out are float32 or
    float16 [M, H] row views with unit column stride."""
    dt = {torch.float32: L.DTYPE_F32, torch.float16: L.DTYPE_F16}
    if x.dim() != 2 or out.shape != x.shape or x.stride(1) != 1 or out.stride(1) != 1 \
            or x.dtype not in dt or out.dtype not in dt:
        raise Bq4Error(L.EINVAL_ARG, "rms_renorm needs float32/float16 [M, H] row views of one shape")
    check(L.lib().bq4_rms_renorm(_ptr(x), dt[x.dtype], x.shape[0], x.shape[1], x.stride(0), _ptr(out),
                                 dt[out.dtype], out.stride(0), ctypes.c_float(eps), _stream_ptr(x.device)))
    return out


def qk_norm_rope(x: torch.Tensor, heads: int, head_dim: int, gamma: Optional[torch.Tensor] = None,
                 eps: float = 1e-5, cos: Optional[torch.Tensor] = None, sin: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """QK-norm + RoPE (attention.rs:114-133, 916-928) on x [M, >= heads*head_dim]
    (float32/float16 row view): per head x / sqrt(mean(x^2) + eps) * gamma,
    then the interleaved-pair rotation by cos/sin [M, head_dim] (float32).
    Writes `out` (may be x itself) or a new [M, heads*head_dim] tensor."""
    dt = {torch.float32: L.DTYPE_F32, torch.float16: L.DTYPE_F16}
    if x.dim() != 2 or x.stride(1) != 1 or x.dtype not in dt:
        raise Bq4Error(L.EINVAL_ARG, "qk_norm_rope needs a float32/float16 [M, W] row view")
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, heads * head_dim), dtype=out_dtype or x.dtype, device=x.device)
    if out.dim() != 2 or out.stride(1) != 1 or out.dtype not in dt or out.shape[0] != M:
        raise Bq4Error(L.EINVAL_ARG, "out must be a float32/float16 [M, W] row view")
    for t in (gamma, cos, sin):
        if t is not None and (t.dtype != torch.float32 or t.device != x.device or t.stride(-1) != 1):
            raise Bq4Error(L.EINVAL_ARG, "gamma/cos/sin must be float32 on the device of x")
    ld_rope = cos.stride(0) if cos is not None else 0
    if cos is not None and (sin is None or sin.stride(0) != ld_rope):
        raise Bq4Error(L.EINVAL_ARG, "cos and sin must be given together with the same row pitch")
    check(L.lib().bq4_qk_norm_rope(_ptr(x), dt[x.dtype], M, heads, head_dim, x.stride(0), _ptr(gamma),
                                   ctypes.c_float(eps), _ptr(cos), _ptr(sin), ld_rope, _ptr(out), dt[out.dtype],
                                   out.stride(0), _stream_ptr(x.device)))
    return out


def set_sm_budget(sms: int) -> None:
    """Cap the SMs a GEMM launch occupies (0 = all), leaving room for
    kernels on other streams such as overlapping NCCL collectives."""
    check(L.lib().bq4_set_sm_budget(int(sms)))


def physical_layout(scheme: QuantScheme, shape: tuple, stored: str = "nk"):
    """(K, N, bq4 layout) of a packed tensor of stored `shape`."""
    if scheme.store_packed_dim == 1:
        K, N = shape
        return K, N, L.LAYOUT_ROW
    if stored == "nk":
        N, K = shape[-2], shape[-1]
        return K, N, L.LAYOUT_COL
    K, N = shape[-2], shape[-1]
    return K, N, L.LAYOUT_NPACKED


def linear_gated(gate: PreparedQ4Weight, up: PreparedQ4Weight, x: torch.Tensor,
                 gate_bias: Optional[torch.Tensor] = None, up_bias: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """silu(x . Wg + bg) * (x . Wu + bu) in one kernel (SwiGLU front half)."""
    x2, lead = _as_rows(x, gate.K, gate.device)
    M = x2.shape[0]
    y = out if out is not None else torch.empty((M, gate.N), dtype=torch.float32, device=gate.device)
    _check_out(y, M, gate.N, gate.device)
    n = ctypes.c_size_t()
    check(L.lib().bq4_linear_gated_workspace_size(gate.handle, up.handle, M, ctypes.byref(n)))
    ws = Workspace.get(gate.device, n.value)
    gb = _vec(gate_bias, gate.N, gate.device) if gate_bias is not None else None
    ub = _vec(up_bias, gate.N, gate.device) if up_bias is not None else None
    check(L.lib().bq4_linear_gated(gate.handle, up.handle, _ptr(x2), M, x2.stride(0), _ptr(gb), _ptr(ub),
                                   _ptr(y), _ptr(ws), ws.numel(), _stream_ptr(gate.device)))
    return y.reshape(*lead, gate.N)


def _as_rows(x: torch.Tensor, K: int, device: torch.device):
    if x.device != device or x.dtype != torch.float32:
        raise Bq4Error(L.EINVAL_ARG, f"x must be float32 on {device}, got {x.dtype} on {x.device}")
    if x.dim() < 1 or x.shape[-1] != K:
        raise Bq4Error(L.EINVAL_SHAPE, f"x last dim {tuple(x.shape)} != K={K}")
    lead = tuple(x.shape[:-1])
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1 or x2.stride(0) < K:
        x2 = x2.contiguous()
    return x2, lead


def _check_out(t: torch.Tensor, M: int, N: int, device: torch.device):
    if t.device != device or t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != M * N:
        raise Bq4Error(L.EINVAL_ARG, f"output/aux must be contiguous float32 [{M},{N}] on {device}")


def _vec(v: torch.Tensor, n: int, device: torch.device) -> torch.Tensor:
    if v.device != device or v.dtype != torch.float32 or v.numel() != n:
        raise Bq4Error(L.EINVAL_ARG, f"bias must be float32 [{n}] on {device}")
    return v.contiguous()


# --------------------------------------------------------------------- QFloat tensor + q_matmul

@dataclass
class QuantizedTensor:
    """A QFloat tensor as burn-cubecl stores it: u32 ``values`` and F32
    ``scales`` on the device, a logical ``shape`` and its ``scheme``.
    ``shape`` is the logical [K, N] the matmul sees (the Qwen weight is the
    transposed view of its stored [N, K] tensor)."""
    values: torch.Tensor
    scales: torch.Tensor
    shape: tuple
    scheme: QuantScheme
    transposed_view: bool = True  # PackedU32(0) only: stored [N,K] seen as [K,N] (Qwen)
    _prepared: Optional[PreparedQ4Weight] = field(default=None, repr=False)

    @classmethod
    def from_packed(cls, packed: PackedQ4, device, stored: str = "nk") -> "QuantizedTensor":
        dev = torch.device(device)
        values = torch.as_tensor(packed.words.view(np.int32)).to(dev)
        scales = torch.as_tensor(packed.scales).to(dev)
        K, N, layout = physical_layout(packed.scheme, packed.shape, stored)
        return cls(values, scales, (K, N), packed.scheme, layout == L.LAYOUT_COL)

    @property
    def layout(self) -> int:
        if self.scheme.store_packed_dim == 1:
            return L.LAYOUT_ROW
        return L.LAYOUT_COL if self.transposed_view else L.LAYOUT_NPACKED

    def prepared(self) -> PreparedQ4Weight:
        if self._prepared is None:
            K, N = self.shape
            self._prepared = PreparedQ4Weight(self.values, self.scales, K, N, self.scheme.block, self.layout,
                                              self.values.device)
        return self._prepared


def q_matmul(lhs: torch.Tensor, rhs: QuantizedTensor) -> torch.Tensor:
    """QTensorOps::q_matmul for an f32 lhs [..., M, K] and a packed-Q4 rhs
    [K, N] (batch-broadcast over the leading dims, like the weight reshaped
    to rank D in linear_forward).  Ineligible schemes raise (the reference
    would select its generic quantized path, which has no B200 counterpart).
    Goes through the C ABI entry ``bq4_q_matmul`` (prepare + GEMM per call)."""
    if lhs.dtype != torch.float32:
        raise Bq4Error(L.EINVAL_ARG, f"lhs dtype {lhs.dtype} is not F32")
    if not (lhs.is_cuda and rhs.values.is_cuda and rhs.scales.is_cuda):
        raise Bq4Error(L.EINVAL_ARG, "q_matmul runs on the GPU only: lhs and the packed rhs must be CUDA tensors")
    if not rhs.scheme.eligible():
        raise Bq4Error(L.EINVAL_ARG, f"scheme {rhs.scheme} is not eligible for the packed-Q4 kernel")
    K, N = rhs.shape
    if lhs.dim() < 2 or lhs.shape[-1] != K:
        raise Bq4Error(L.EINVAL_SHAPE, f"lhs {tuple(lhs.shape)} does not match rhs [{K},{N}]")
    lead = tuple(lhs.shape[:-1])
    x = lhs.reshape(-1, K).contiguous()  # qtensor.rs:345-349 makes lhs contiguous
    M = x.shape[0]
    out = torch.empty((M, N), dtype=torch.float32, device=lhs.device)
    nbytes = ctypes.c_size_t()
    with torch.cuda.device(lhs.device):
        sch = rhs.scheme.to_c(rhs.transposed_view)
        check(L.lib().bq4_q_matmul_workspace_size(M, K, N, ctypes.byref(sch), ctypes.byref(nbytes)))
        ws = Workspace.get(lhs.device, nbytes.value)
        check(L.lib().bq4_q_matmul(_ptr(x), M, K, _ptr(rhs.values), _ptr(rhs.scales), N, ctypes.byref(sch),
                                   _ptr(out), _ptr(ws), ws.numel(), _stream_ptr(lhs.device)))
    return out.reshape(*lead, N)


# --------------------------------------------------------------------- quantized row selection

def _stored_rows(qt: QuantizedTensor):
    """(rows, cols) of the stored rank-2 PackedU32(0) tensor behind qt."""
    if qt.scheme.store_packed_dim != 0:
        raise Bq4Error(L.EINVAL_ARG, "quantized row selection requires PackedU32(0) (blocks along the row)")
    K, N = qt.shape
    return (N, K) if qt.transposed_view else (K, N)


def _ids(indices: torch.Tensor, device: torch.device):
    if indices.dim() != 1:
        raise Bq4Error(L.EINVAL_SHAPE, "quantized select indices must be rank one")
    if indices.dtype not in (torch.int32, torch.int64):
        raise Bq4Error(L.EINVAL_ARG, f"indices must be int32 or int64, got {indices.dtype}")
    return indices.to(device).contiguous()


def q_select(qt: QuantizedTensor, dim: int, indices: torch.Tensor) -> QuantizedTensor:
    """QTensorOps::q_select (patches/burn-cubecl-0.21.0/src/ops/qtensor.rs:267-293):
    rows of the stored rank-2 packed-Q4 tensor, kept packed (values and scales
    of each selected row copied, nothing widened).  Same restrictions as the
    reference: dim 0, Q4S, Block level, F32 scales, PackedU32(0).  The result
    is a plain stored [n, cols] tensor.  An out-of-range index gives a zero row
    and is reported by poll_device_error()."""
    if dim != 0:
        raise Bq4Error(L.EINVAL_ARG, "quantized select only supports rows (dim 0)")
    if not (qt.scheme.value == "Q4S" and qt.scheme.param == "F32"):
        raise Bq4Error(L.EINVAL_ARG, "quantized row selection requires packed Q4S with F32 scales")
    rows, cols = _stored_rows(qt)
    block = qt.scheme.block
    dev = qt.values.device
    ids = _ids(indices, dev)
    n = ids.shape[0]
    out_v = torch.empty((n, cols // 8), dtype=torch.int32, device=dev)
    out_s = torch.empty((n, cols // block), dtype=torch.float32, device=dev)
    check(L.lib().bq4_q_select_rows(_ptr(qt.values), _ptr(qt.scales), rows, cols, block, _ptr(ids),
                                    1 if ids.dtype == torch.int64 else 0, n, _ptr(out_v), _ptr(out_s),
                                    _stream_ptr(dev)))
    return QuantizedTensor(out_v, out_s, (n, cols), qt.scheme, transposed_view=False)


def embedding(qt: QuantizedTensor, indices: torch.Tensor) -> torch.Tensor:
    """Embedding lookup on a packed-Q4 table: q_select of the rows, then their
    dequantization (dequantize.rs:6-33), fused in one pass; f32 [n, cols],
    bit-exact."""
    rows, cols = _stored_rows(qt)
    dev = qt.values.device
    ids = _ids(indices, dev)
    out = torch.empty((ids.shape[0], cols), dtype=torch.float32, device=dev)
    check(L.lib().bq4_q_select_rows_dequant(_ptr(qt.values), _ptr(qt.scales), rows, cols, qt.scheme.block,
                                            _ptr(ids), 1 if ids.dtype == torch.int64 else 0, ids.shape[0],
                                            _ptr(out), _stream_ptr(dev)))
    return out


# --------------------------------------------------------------------- linear adapters

class Q4Linear:
    """A linear layer whose weight is a packed-Q4 QFloat tensor ([input,
    output] logical) with an optional F32 bias -- the nn::Linear / QwenLinear
    the adapters receive."""

    def __init__(self, weight: QuantizedTensor, bias: Optional[torch.Tensor] = None):
        self.weight = weight
        self.bias = bias

    @property
    def dims(self):
        return self.weight.shape


def linear_forward(linear: Q4Linear, input: torch.Tensor, act: int = L.ACT_NONE) -> torch.Tensor:
    """crates/burn_boogu/src/model/linear.rs:14-37 -- rank >= 2 input, matmul
    against the prepared Q4 weight, bias added (fused into the epilogue)."""
    if input.dim() < 2:
        raise Bq4Error(L.EINVAL_SHAPE, "Boogu linear projections require rank >= 2")
    return linear.weight.prepared().linear(input, linear.bias, act)


def qwen_linear_forward(linear: Q4Linear, input: torch.Tensor, act: int = L.ACT_NONE) -> torch.Tensor:
    """crates/burn_qwen3_vl/src/linear.rs:107-140 -- same contract for the
    Qwen column layout (transposed view of the stored [N, K] weight)."""
    if input.dim() < 2:
        raise Bq4Error(L.EINVAL_SHAPE, "Qwen linear projections require rank >= 2")
    return linear.weight.prepared().linear(input, linear.bias, act)


def feed_forward_swiglu(l1: Q4Linear, l3: Q4Linear, l2: Q4Linear, x: torch.Tensor) -> torch.Tensor:
    """crates/burn_boogu/src/model/feed_forward.rs:32-36:
    linear_2(silu(linear_1(x)) * linear_3(x)), with the gate fused."""
    gated = linear_gated(l1.weight.prepared(), l3.weight.prepared(), x, l1.bias, l3.bias)
    return linear_forward(l2, gated)


def set_numerics(mode: int) -> None:
    """Operand staging for subsequent calls: NUMERICS_AUTO (exact weights up
    to M = 64 rows, the reference's f16 staging above), NUMERICS_EXACT or
    NUMERICS_FOLDED (see include/bq4.h)."""
    check(L.lib().bq4_set_numerics(mode))


def poll_device_error() -> None:
    """Raise if a kernel's bounded device-side wait expired since the last poll."""
    check(L.lib().bq4_poll_device_error())
