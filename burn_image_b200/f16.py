"""Host-side mirror of burn_image's packed-F16 kernels over libbq4.

The reference keeps F16 weights (the VAE's, and the F16 profiles' tables) as
raw binary16 bits bound as u32 words and widens them at the point of use
(patches/burn-cubecl-0.21.0/src/kernel/packed_f16.rs).  Names and argument
meanings follow that file:

* ``packed_f16_to_f32(input)`` -- strided widening (:88-131)
* ``packed_f16_select_rows(tensor, dim, indices)`` -- row gather (:296-358)
* ``packed_f16_rhs_matmul(lhs, rhs)`` -- f32 lhs times an f16 rhs view (:133-292)
* ``packed_f16_conv2d(input, weight, bias, options)`` -- NCHW x OIHW,
  groups 1 (:421-602), with ``ConvOptions`` as Burn's ConvOptions<2>

A float16 torch tensor's storage is exactly this packed format (two values
per little-endian u32 word, even index in the low half), so these functions
take float16 tensors and pass their storage, offset and strides on.

``PreparedF16Weight`` / ``PreparedF16ConvWeight`` prepare a weight once (the
loader re-layout into MMA-ready tf32 tiles); the one-shot functions above
prepare into the workspace on every call, like the reference's unprepared
calls.  All arithmetic runs in the CUDA kernels of libbq4.so.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib as L
from ._lib import Bq4Error, check
from .q4 import PreparedQ4Weight, Workspace, _ptr, _stream_ptr


def _f16(t: torch.Tensor, what: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or t.dtype != torch.float16 or t.device.type != "cuda":
        raise Bq4Error(L.EINVAL_ARG, f"{what} must be a float16 CUDA tensor (packed-F16 storage)")
    return t


def _f32(t: torch.Tensor, what: str, device: torch.device) -> torch.Tensor:
    if t.dtype != torch.float32 or t.device != device:
        raise Bq4Error(L.EINVAL_ARG, f"{what} must be float32 on {device}, got {t.dtype} on {t.device}")
    return t


@dataclass
class ConvOptions:
    """Burn ConvOptions<2>: [height, width] stride, padding and dilation; groups."""
    stride: Sequence[int] = (1, 1)
    padding: Sequence[int] = (0, 0)
    dilation: Sequence[int] = (1, 1)
    groups: int = 1

    def to_c(self) -> L.Conv2dOptions:
        o = L.Conv2dOptions()
        o.stride[0], o.stride[1] = int(self.stride[0]), int(self.stride[1])
        o.padding[0], o.padding[1] = int(self.padding[0]), int(self.padding[1])
        o.dilation[0], o.dilation[1] = int(self.dilation[0]), int(self.dilation[1])
        o.groups = int(self.groups)
        return o

    def output_hw(self, in_h: int, in_w: int, kh: int, kw: int) -> tuple:
        oh = (in_h + 2 * self.padding[0] - self.dilation[0] * (kh - 1) - 1) // self.stride[0] + 1
        ow = (in_w + 2 * self.padding[1] - self.dilation[1] * (kw - 1) - 1) // self.stride[1] + 1
        return oh, ow


def packed_f16_to_f32(input: torch.Tensor) -> torch.Tensor:
    """Widen a float16 tensor (any strides) to a contiguous float32 tensor,
    bit-exactly (NaN payloads kept, quiet bit set)."""
    t = _f16(input, "input")
    out = torch.empty(tuple(t.shape), dtype=torch.float32, device=t.device)
    if t.numel() == 0:
        return out
    rank = t.dim()
    shape = (ctypes.c_int64 * max(rank, 1))(*t.shape)
    strides = (ctypes.c_int64 * max(rank, 1))(*t.stride())
    check(L.lib().bq4_packed_f16_to_f32(_ptr(t), rank, shape, strides, _ptr(out), _stream_ptr(t.device)))
    return out


def packed_f16_select_rows(tensor: torch.Tensor, dim: int, indices: torch.Tensor) -> torch.Tensor:
    """Rows ``indices`` of a contiguous float16 matrix, as float32 [n, cols]."""
    t = _f16(tensor, "tensor")
    if t.dim() != 2:
        raise Bq4Error(L.EINVAL_SHAPE, "packed-F16 select requires a matrix")
    if dim != 0:
        raise Bq4Error(L.EINVAL_ARG, "packed-F16 select only supports row selection")
    if not t.is_contiguous():
        raise Bq4Error(L.EINVAL_ARG, "packed-F16 select table must be contiguous")
    if indices.dtype != torch.int32 or indices.dim() != 1 or indices.device != t.device:
        raise Bq4Error(L.EINVAL_ARG, "packed-F16 select requires rank-one int32 indices on the table's device")
    idx = indices.contiguous()
    rows, cols = t.shape
    out = torch.empty((idx.numel(), cols), dtype=torch.float32, device=t.device)
    check(L.lib().bq4_packed_f16_select_rows(_ptr(t), rows, cols, _ptr(idx), idx.numel(), _ptr(out),
                                             _stream_ptr(t.device)))
    return out


def _rhs_view(rhs: torch.Tensor):
    r = _f16(rhs, "rhs")
    if r.dim() < 2 or any(d != 1 for d in r.shape[:-2]):
        raise Bq4Error(L.EINVAL_SHAPE, "packed-F16 matmul supports one broadcast weight matrix")
    K, N = r.shape[-2], r.shape[-1]
    return r, K, N, r.stride(-2), r.stride(-1)


def packed_f16_rhs_matmul(lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    """lhs float32 [..., K] times a float16 rhs [.., K, N] (any strides, e.g.
    the transposed view of a stored [N, K] checkpoint) -> float32 [..., N]."""
    r, K, N, inner, col = _rhs_view(rhs)
    x = _f32(lhs, "lhs", r.device)
    if x.dim() != r.dim():
        raise Bq4Error(L.EINVAL_SHAPE, "packed-F16 matmul ranks differ")
    if x.shape[-1] != K:
        raise Bq4Error(L.EINVAL_SHAPE, "packed-F16 matmul inner dimensions differ")
    lead = tuple(x.shape[:-1])
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=torch.float32, device=r.device)
    if M == 0:
        return out.reshape(*lead, N)
    n = ctypes.c_size_t()
    check(L.lib().bq4_packed_f16_rhs_matmul_workspace_size(M, K, N, ctypes.byref(n)))
    ws = Workspace.get(r.device, n.value)
    check(L.lib().bq4_packed_f16_rhs_matmul(_ptr(x2), M, K, _ptr(r), inner, col, N, _ptr(out), _ptr(ws),
                                            ws.numel(), _stream_ptr(r.device)))
    return out.reshape(*lead, N)


def packed_f16_conv2d(input: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                      options: ConvOptions) -> torch.Tensor:
    """One groups=1 NCHW convolution from float16 OIHW weight storage, f32
    accumulation; the weight is prepared into the workspace on every call."""
    w = _f16(weight, "weight")
    if w.dim() != 4 or not w.is_contiguous():
        raise Bq4Error(L.EINVAL_ARG, "packed-F16 convolution requires a contiguous OIHW weight")
    x = _f32(input, "input", w.device)
    if x.dim() != 4:
        raise Bq4Error(L.EINVAL_SHAPE, "packed-F16 convolution requires NCHW input")
    x = x.contiguous()
    B, C, H, W = x.shape
    O, Cw, kh, kw = w.shape
    if Cw != C:
        raise Bq4Error(L.EINVAL_SHAPE, f"weight in_channels {Cw} != input channels {C}")
    b = None if bias is None else _f32(bias, "bias", w.device).contiguous()
    opt = options.to_c()
    oh, ow = options.output_hw(H, W, kh, kw)
    out = torch.empty((B, O, max(oh, 0), max(ow, 0)), dtype=torch.float32, device=w.device)
    n = ctypes.c_size_t()
    check(L.lib().bq4_packed_f16_conv2d_workspace_size(B, C, H, W, O, kh, kw, ctypes.byref(opt), ctypes.byref(n)))
    ws = Workspace.get(w.device, n.value)
    check(L.lib().bq4_packed_f16_conv2d(_ptr(x), B, C, H, W, _ptr(w), O, kh, kw, _ptr(b), ctypes.byref(opt),
                                        _ptr(out), _ptr(ws), ws.numel(), _stream_ptr(w.device)))
    return out


class PreparedF16Weight(PreparedQ4Weight):
    """A packed-F16 matmul rhs [K, N] prepared once into MMA-ready tf32
    tiles.  ``linear`` / ``linear_ex`` (float32 x) / ``plan_info`` work as for
    Q4 weights: y = act(x . W + bias) with the epilogue fused."""

    def __init__(self, rhs: torch.Tensor, device: Optional[torch.device] = None):
        r, K, N, inner, col = _rhs_view(rhs)
        dev = torch.device(device) if device is not None else r.device
        handle = ctypes.c_void_p()
        lib = L.lib()
        check(lib.bq4_f16_weight_prepare(_ptr(r), K, N, inner, col, dev.index, ctypes.byref(handle)))
        self._h = handle
        self.K, self.N, self.block, self.layout = K, N, 0, L.LAYOUT_F16
        nb = ctypes.c_size_t()
        check(lib.bq4_weight_info(handle, None, None, None, None, ctypes.byref(nb)))
        self.device_bytes = nb.value
        self.device = dev

    def linear(self, x: torch.Tensor, bias: Optional[torch.Tensor] = None, act: int = L.ACT_NONE,
               aux: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.K % 4 == 0:
            return super().linear(x, bias, act, aux, out)
        # token rows are read by TMA in place: give them a 16-byte pitch
        lead = tuple(x.shape[:-1])
        xp = torch.zeros((max(x.numel() // max(self.K, 1), 0), (self.K + 3) // 4 * 4), dtype=torch.float32,
                         device=self.device)
        xp[:, :self.K] = _f32(x, "x", self.device).reshape(-1, self.K)
        return self.linear_ex(xp[:, :self.K], bias, act, aux, out).reshape(*lead, self.N)


class PreparedF16ConvWeight(PreparedQ4Weight):
    """An OIHW packed-F16 convolution weight prepared once; ``conv2d`` runs
    bq4_conv2d (implicit GEMM for stride 1, gathered rows otherwise)."""

    def __init__(self, weight: torch.Tensor, device: Optional[torch.device] = None):
        w = _f16(weight, "weight")
        if w.dim() != 4 or not w.is_contiguous():
            raise Bq4Error(L.EINVAL_ARG, "packed-F16 convolution requires a contiguous OIHW weight")
        dev = torch.device(device) if device is not None else w.device
        O, C, kh, kw = w.shape
        handle = ctypes.c_void_p()
        lib = L.lib()
        check(lib.bq4_f16_conv_weight_prepare(_ptr(w), O, C, kh, kw, dev.index, ctypes.byref(handle)))
        self._h = handle
        self.out_channels, self.in_channels, self.kernel = O, C, (kh, kw)
        k, nb = ctypes.c_int64(), ctypes.c_size_t()
        check(lib.bq4_weight_info(handle, ctypes.byref(k), None, None, None, ctypes.byref(nb)))
        self.K, self.N, self.block, self.layout, self.device_bytes = k.value, O, 0, L.LAYOUT_F16, nb.value
        self.device = dev

    def conv2d(self, input: torch.Tensor, bias: Optional[torch.Tensor] = None,
               options: Optional[ConvOptions] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        options = options or ConvOptions()
        x = _f32(input, "input", self.device)
        if x.dim() != 4 or x.shape[1] != self.in_channels:
            raise Bq4Error(L.EINVAL_SHAPE, f"input must be NCHW with {self.in_channels} channels")
        x = x.contiguous()
        B, _, H, W = x.shape
        oh, ow = options.output_hw(H, W, *self.kernel)
        y = out if out is not None else torch.empty((B, self.out_channels, max(oh, 0), max(ow, 0)),
                                                    dtype=torch.float32, device=self.device)
        b = None if bias is None else _f32(bias, "bias", self.device).contiguous()
        opt = options.to_c()
        n = ctypes.c_size_t()
        check(L.lib().bq4_conv2d_workspace_size(self._h, B, H, W, ctypes.byref(opt), ctypes.byref(n)))
        ws = Workspace.get(self.device, n.value)
        check(L.lib().bq4_conv2d(_ptr(x), B, H, W, self._h, _ptr(b), ctypes.byref(opt), _ptr(y), _ptr(ws),
                                 ws.numel(), _stream_ptr(self.device)))
        return y


def attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scale: Optional[float] = None,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax(scale * q k^T) v, no mask, as Burn's ``attention`` with default
    options (the reference's consumer of the q/k/v projection).  query
    [B, Hq, Sq, D], key / value [B, Hkv, Skv, D], float16 on one device;
    query head h attends with kv head h // (Hq // Hkv).  Returns float32
    [B, Hq, Sq, D].  scale None: 1 / sqrt(D)."""
    q = _f16(query, "query").contiguous()
    k = _f16(key, "key").contiguous()
    v = _f16(value, "value").contiguous()
    if q.dim() != 4 or k.dim() != 4 or v.shape != k.shape or q.shape[0] != k.shape[0] or q.shape[3] != k.shape[3]:
        raise Bq4Error(L.EINVAL_SHAPE, "attention takes q [B,Hq,Sq,D], k and v [B,Hkv,Skv,D]")
    if k.device != q.device or v.device != q.device:
        raise Bq4Error(L.EINVAL_ARG, "q, k and v must be on one device")
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    y = out if out is not None else torch.empty((B, Hq, Sq, D), dtype=torch.float32, device=q.device)
    n = ctypes.c_size_t()
    check(L.lib().bq4_attention_workspace_size(B, Hq, Hkv, Sq, Skv, D, ctypes.byref(n)))
    ws = Workspace.get(q.device, n.value)
    check(L.lib().bq4_attention(_ptr(q), _ptr(k), _ptr(v), B, Hq, Hkv, Sq, Skv, D, float(scale or 0.0), _ptr(y),
                                _ptr(ws), ws.numel(), _stream_ptr(q.device)))
    return y
