"""Tensor-parallel packed-Q4 linears over torch.distributed (NCCL on NVLink).

Column-parallel (qkv, up): each rank holds N/P output features of the
weight, with their scale columns; the output stays sharded.  Row-parallel
(o, down): each rank holds K/P input features, cut on quant-block
boundaries (K/P % block == 0); partial f32 outputs are summed with one
all-reduce, the bias is added once (by rank 0's epilogue).

The reference runs single-device (it has no distributed code); this module
is the B200 multi-GPU layer around the same op.  Shards are prepared
straight from the full reference-packed buffers by the C ABI
(bq4_weight_prepare_shard), so no host round trip is needed.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _lib as L
from .q4 import PreparedQ4Weight, Workspace, _ptr, _stream_ptr

COLUMN, ROW = 0, 1


def column_shard_bounds(N: int, rank: int, size: int):
    """Output-feature range [n0, n1) of `rank` in a column-parallel split."""
    if N % size:
        raise ValueError(f"column shard: N={N} not divisible by {size}")
    n = N // size
    return rank * n, (rank + 1) * n


def row_shard_bounds(K: int, block: int, rank: int, size: int):
    """Input-feature range [k0, k1) of `rank` in a row-parallel split; the
    cut must fall on quant-block (and 8-value word) boundaries."""
    if K % size or (K // size) % block or (K // size) % 8:
        raise ValueError(f"row shard: K={K} over {size} ranks does not fall on block-{block} boundaries")
    k = K // size
    return rank * k, (rank + 1) * k


def slice_raw(words: np.ndarray, scales: np.ndarray, K: int, N: int, block: int, layout: int,
              n0: int, n1: int, k0: int, k1: int):
    """Host slice of reference-packed buffers to the window [k0,k1) x [n0,n1),
    in the same physical layout (used for host-side sharding and tests)."""
    if layout == L.LAYOUT_ROW:
        w = words.reshape(K // 8, N)[k0 // 8:k1 // 8, n0:n1]
        s = scales.reshape(K // block, N)[k0 // block:k1 // block, n0:n1]
    else:
        w = words.reshape(N, K // 8)[n0:n1, k0 // 8:k1 // 8]
        s = scales.reshape(N, K // block)[n0:n1, k0 // block:k1 // block]
    return np.ascontiguousarray(w), np.ascontiguousarray(s)


# Pass as `group` to build an unsharded linear or stack on every rank (token
# parallelism: each rank runs the whole weight on its own tokens).
LOCAL = "local"


def _world(group):
    if group == LOCAL:
        return 0, 1
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


class ColumnParallelQ4Linear:
    def __init__(self, words: torch.Tensor, scales: torch.Tensor, K: int, N: int, block: int, layout: int,
                 device: torch.device, bias: Optional[torch.Tensor] = None, act: int = L.ACT_NONE, group=None):
        self.rank, self.size = _world(group)
        self.group = group
        self.n0, self.n1 = column_shard_bounds(N, self.rank, self.size)
        self.weight = PreparedQ4Weight(words, scales, K, N, block, layout, device,
                                       shard=(COLUMN, self.rank, self.size))
        self.bias = None if bias is None else bias[self.n0:self.n1].contiguous()
        self.act = act

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x [M, K] (replicated) -> local output columns [M, N/P]."""
        return self.weight.linear(x, self.bias, self.act, out=out)

    def forward_ex(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Same, with float16 or float32 activations in and out."""
        return self.weight.linear_ex(x, self.bias, self.act, out=out)


class RowParallelQ4Linear:
    def __init__(self, words: torch.Tensor, scales: torch.Tensor, K: int, N: int, block: int, layout: int,
                 device: torch.device, bias: Optional[torch.Tensor] = None, group=None):
        self.rank, self.size = _world(group)
        self.group = group
        self.k0, self.k1 = row_shard_bounds(K, block, self.rank, self.size)
        self.weight = PreparedQ4Weight(words, scales, K, N, block, layout, device,
                                       shard=(ROW, self.rank, self.size))
        self.bias = bias if self.rank == 0 else None  # added once, before the sum

    def forward(self, x_local: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x_local [M, K/P] (this rank's input columns, may be a strided view)
        -> full output [M, N] summed over ranks."""
        w = self.weight
        M = x_local.shape[0]
        y = out if out is not None else torch.empty((M, w.N), dtype=torch.float32, device=w.device)
        if x_local.stride(-1) != 1:
            x_local = x_local.contiguous()
        ws = Workspace.get(w.device, w.workspace_bytes(M))
        L.check(L.lib().bq4_linear(w.handle, _ptr(x_local), M, x_local.stride(0), _ptr(self.bias), L.ACT_NONE,
                                   None, _ptr(y), _ptr(ws), ws.numel(), _stream_ptr(w.device)))
        if self.size > 1:
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y

    def forward_scatter(self, x_local: torch.Tensor, ex: "PeerExchange", b: int) -> None:
        """This rank's partial product, written by the GEMM epilogue straight
        into the receive buffer b of each output row's owner rank
        (bq4_linear_rowscatter), then the cross-rank signal/wait: afterwards
        every rank holds all partials of its own rows."""
        w = self.weight
        M = x_local.shape[0]
        dt = {torch.float32: L.DTYPE_F32, torch.float16: L.DTYPE_F16}
        n = ctypes.c_size_t()
        L.check(L.lib().bq4_linear_ex_workspace_size(w.handle, M, dt[x_local.dtype], ctypes.byref(n)))
        ws = Workspace.get(w.device, n.value) if n.value else None
        L.check(L.lib().bq4_linear_rowscatter(w.handle, _ptr(x_local), dt[x_local.dtype], M, x_local.stride(0),
                                              _ptr(self.bias), L.ACT_NONE, ex.targets(b), ex.size, ex.rank, ex.H,
                                              _ptr(ws), ws.numel() if ws is not None else 0, _stream_ptr(w.device)))
        ex.signal_wait()

    def forward_local(self, x_local: torch.Tensor, ex: "PeerExchange", b: int) -> None:
        """The pull form: this rank's whole partial product [M, H] f32 goes
        into its own shared buffer b (a plain bq4_linear_ex, local HBM
        stores), then the cross-rank signal/wait; afterwards every owner can
        read its rows from every rank's buffer (PeerExchange.reduce_pull)."""
        w = self.weight
        M = x_local.shape[0]
        dt = {torch.float32: L.DTYPE_F32, torch.float16: L.DTYPE_F16}
        n = ctypes.c_size_t()
        L.check(L.lib().bq4_linear_ex_workspace_size(w.handle, M, dt[x_local.dtype], ctypes.byref(n)))
        ws = Workspace.get(w.device, n.value) if n.value else None
        L.check(L.lib().bq4_linear_ex(w.handle, _ptr(x_local), dt[x_local.dtype], M, x_local.stride(0),
                                      _ptr(self.bias), L.ACT_NONE, None, ctypes.c_void_p(ex.local[b]), L.DTYPE_F32,
                                      ex.H, _ptr(ws), ws.numel() if ws is not None else 0, _stream_ptr(w.device)))
        ex.signal_wait()

    def forward_ex(self, x_local: torch.Tensor, out: torch.Tensor, async_op: bool = False):
        """Same, with float16 or float32 activations; the partial sums are
        reduced in ``out``'s dtype.  With ``async_op`` the all-reduce is only
        enqueued and its work handle returned (``wait()`` makes the current
        stream wait for it); otherwise returns ``out``."""
        self.weight.linear_ex(x_local, self.bias, L.ACT_NONE, out=out)
        if self.size > 1:
            work = dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group, async_op=async_op)
            if async_op:
                return work
        return None if async_op else out


class _DeviceArray:
    """A device pointer presented through the CUDA array interface, so that
    torch can view memory it did not allocate (the shared buffers)."""

    def __init__(self, ptr: int, shape, dtype: torch.dtype):
        typestr = {torch.float16: "<f2", torch.float32: "<f4"}[dtype]
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerExchange:
    """Receive buffers and flags shared between the ranks of `group` through
    CUDA IPC (bq4_peer_buffer_*), for the row-parallel exchange over NVLink
    peer memory: two [P][rows][H] f32 receive buffers used alternately (the
    barrier of one exchange proves every rank has finished reading the buffer
    before it), and one [P] u32 flag array per rank for bq4_peer_signal_wait.
    """

    def __init__(self, device: torch.device, group, rows: int, H: int, acts: int = 0):
        self.device, self.group = device, group
        self.rank, self.size = _world(group)
        self.rows, self.H = rows, H
        lib = L.lib()
        # buffers 0, 1: f32 partials; 2: flags; 3, 3 + acts: [M][H] f16 activation copies that
        # peers write into (reduce_bcast)
        sizes = [self.size * rows * H * 4] * 2 + [4 * L.MAX_PEERS] + [self.size * rows * H * 2] * acts
        self.local, handles = [], []
        for n in sizes:
            ptr, h = ctypes.c_void_p(), (ctypes.c_uint8 * L.IPC_HANDLE_BYTES)()
            L.check(lib.bq4_peer_buffer_alloc(n, device.index, ctypes.byref(ptr), h))
            self.local.append(ptr.value)
            handles.append(bytes(h))
        everyone = [None] * self.size
        dist.all_gather_object(everyone, handles, group=group)
        self.peer = [[None] * self.size for _ in sizes]  # [buffer][rank] -> device pointer mapped here
        self.opened = []
        for r in range(self.size):
            for b in range(len(sizes)):
                if r == self.rank:
                    self.peer[b][r] = self.local[b]
                    continue
                ptr = ctypes.c_void_p()
                h = (ctypes.c_uint8 * L.IPC_HANDLE_BYTES).from_buffer_copy(everyone[r][b])
                L.check(lib.bq4_peer_buffer_open(h, device.index, ctypes.byref(ptr)))
                self.peer[b][r] = ptr.value
                self.opened.append(ptr.value)
        self.epoch = 0

    def targets(self, b: int):
        """y_ranks argument of bq4_linear_rowscatter for receive buffer b."""
        return (ctypes.c_void_p * self.size)(*self.peer[b])

    def signal_wait(self):
        self.epoch += 1
        flags = (ctypes.c_void_p * self.size)(*self.peer[2])
        L.check(L.lib().bq4_peer_signal_wait(ctypes.c_void_p(self.local[2]), flags, self.size, self.rank,
                                             ctypes.c_uint32(self.epoch), _stream_ptr(self.device)))

    def reduce(self, b: int, out: torch.Tensor, renorm: bool, eps: float = 1e-6):
        """Sum this rank's rows of receive buffer b over the ranks (rank
        order), optionally RMS-renormalised, into `out` [rows, H] (f16/f32)."""
        dt = {torch.float32: L.DTYPE_F32, torch.float16: L.DTYPE_F16}
        L.check(L.lib().bq4_reduce_slices(ctypes.c_void_p(self.local[b]), self.size, self.rows, self.H, self.H,
                                          1 if renorm else 0, ctypes.c_float(eps), _ptr(out), dt[out.dtype],
                                          out.stride(0), _stream_ptr(self.device)))

    def view(self, b: int, shape, dtype: torch.dtype) -> torch.Tensor:
        """This rank's buffer b as a tensor (no copy; valid until close)."""
        return torch.as_tensor(_DeviceArray(self.local[b], tuple(shape), dtype), device=self.device)

    def reduce_bcast(self, b: int, dst: int, renorm: bool, eps: float = 1e-6):
        """As reduce_pull, writing this rank's rows of the result (f16) into
        every rank's activation buffer dst over peer memory (in place of an
        all-gather); a signal_wait afterwards makes every rank's copy whole."""
        src = (ctypes.c_void_p * self.size)(*self.peer[b])
        outs = (ctypes.c_void_p * self.size)(*self.peer[dst])
        L.check(L.lib().bq4_reduce_slices_peer_bcast(src, self.size, self.rank * self.rows, self.rows, self.H, self.H,
                                                     1 if renorm else 0, ctypes.c_float(eps), outs, L.DTYPE_F16,
                                                     self.H, _stream_ptr(self.device)))

    def reduce_pull(self, b: int, out: torch.Tensor, renorm: bool, eps: float = 1e-6):
        """As reduce, reading this rank's rows of every rank's buffer b (each
        rank's whole partial product, written by forward_local) over peer
        memory."""
        dt = {torch.float32: L.DTYPE_F32, torch.float16: L.DTYPE_F16}
        src = (ctypes.c_void_p * self.size)(*self.peer[b])
        L.check(L.lib().bq4_reduce_slices_peer(src, self.size, self.rank * self.rows, self.rows, self.H, self.H,
                                               1 if renorm else 0, ctypes.c_float(eps), _ptr(out), dt[out.dtype],
                                               out.stride(0), _stream_ptr(self.device)))

    def close(self):
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = L.lib()
        for p in self.opened:
            lib.bq4_peer_buffer_close(ctypes.c_void_p(p))
        self.opened = []
        dist.barrier(group=self.group)
        for p in self.local:
            lib.bq4_peer_buffer_free(ctypes.c_void_p(p), self.device.index)
        self.local = []


class DiTQ4Stack:
    """The DiT-shaped layer stack of the benchmark: per block a fused qkv
    (column-parallel, hidden -> 3*hidden), o (row-parallel over the v slice,
    hidden -> hidden, bias), up (column-parallel, hidden -> mlp, bias +
    GELU-tanh) and down (row-parallel, mlp -> hidden, bias), then the
    activations are renormalised (RMS over the hidden axis).  Attention
    itself is outside the Q4 path; the o-projection reads the rank's value
    columns of the qkv output as its input shard.  For P > 1 the fused qkv
    weight's columns are ordered so that rank r's contiguous column shard is
    [q_r | k_r | v_r] (each hidden / P wide, Megatron-style), hence v_r -- the
    last hidden / P columns of the shard -- is the slice of v whose rows of
    the o weight rank r holds: the sharded stack computes the unsharded one."""

    def __init__(self, blocks: int, hidden: int, qkv: int, mlp: int, device: torch.device, seed: int = 0,
                 block: int = 128, group=None, act_dtype: torch.dtype = torch.float32, chunks: int = 1,
                 exchange: str = "nccl"):
        self.device = device
        # exchange "p2p" (P > 1, float16 activations): the row-parallel
        # partials go to each row's owner through the GEMM epilogue over NVLink
        # peer memory, the owner sums (and renormalises) its rows, and an NCCL
        # all-gather of float16 rows rebuilds the replicated activations
        # (_forward_p2p); "pull": each rank's GEMM writes its partials into
        # its own shared buffer and each owner reads its rows from every
        # rank's buffer (same sums in the same order); "bcast": "pull" with
        # each owner writing its reduced rows into every rank's copy of the
        # activations instead of an all-gather; "nccl": a float32 all-reduce
        # of the partials.
        self.exchange = exchange
        self.group = group
        self._peer = None
        # act_dtype float16: activations stay in the GEMM's operand format
        # between linears (bq4_linear_ex), the renorm is one kernel.  The
        # row-parallel partials (P > 1) are still summed in float32: float16
        # partial sums overflow on this workload (its random weights have a
        # nonzero mean, so activations grow to ~1e5 between renorms).
        # chunks > 1 pipelines token chunks so that each chunk's all-reduces
        # overlap the other chunks' GEMMs.
        self.act_dtype = act_dtype
        self.chunks = max(1, int(chunks))
        self.hidden, self.qkv, self.mlp = hidden, qkv, mlp
        self.rank, self.size = _world(group)
        self.layers = []
        g = torch.Generator(device=device)
        for b in range(blocks):
            g.manual_seed(seed * 1000003 + b)
            mk = lambda K, N: _random_packed(K, N, block, g, device)  # noqa: E731
            bias = lambda N: torch.randn(N, generator=g, device=device) * 0.02  # noqa: E731
            wq, sq = mk(hidden, qkv)
            if self.size > 1:
                perm = _qkv_rank_order(hidden, qkv, self.size, device)
                wq, sq = wq[:, perm].contiguous(), sq[:, perm].contiguous()
            wo, so = mk(hidden, hidden)
            wu, su = mk(hidden, mlp)
            wd, sd = mk(mlp, hidden)
            bo, bu, bd = bias(hidden), bias(mlp), bias(hidden)
            layer = dict(
                qkv=ColumnParallelQ4Linear(wq, sq, hidden, qkv, block, L.LAYOUT_ROW, device, group=group),
                o=RowParallelQ4Linear(wo, so, hidden, hidden, block, L.LAYOUT_ROW, device, bo, group=group),
                up=ColumnParallelQ4Linear(wu, su, hidden, mlp, block, L.LAYOUT_ROW, device, bu, L.ACT_GELU_TANH,
                                          group=group),
                down=RowParallelQ4Linear(wd, sd, mlp, hidden, block, L.LAYOUT_ROW, device, bd, group=group))
            self.layers.append(layer)
            del wq, sq, wo, so, wu, su, wd, sd
        self.bufs = {}

    def flops_per_token(self) -> int:
        h, q, m = self.hidden, self.qkv, self.mlp
        return 2 * len(self.layers) * (h * q + h * h + h * m + m * h)

    def _buf(self, name, shape, dtype=torch.float32):
        t = self.bufs.get(name)
        if t is None or tuple(t.shape) != tuple(shape) or t.dtype != dtype:
            t = torch.empty(shape, dtype=dtype, device=self.device)
            self.bufs[name] = t
        return t

    def forward(self, x: torch.Tensor, on_linear=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The stack on x [M, hidden]; the renormalised float32 output goes to
        ``out`` when given (else an internal buffer reused by the next call)."""
        if self.act_dtype == torch.float16:
            if self.exchange in ("p2p", "pull", "bcast") and self.size > 1:
                return self._forward_p2p(x, on_linear, out)
            return self._forward_chained(x, on_linear, out)
        M = x.shape[0]
        P = self.size
        qkv_local = self.qkv // P
        hid_local = self.hidden // P
        for layer in self.layers:
            t = self._buf("qkv", (M, qkv_local))
            _timed(on_linear, "qkv", lambda: layer["qkv"].forward(x, out=t))
            v = t[:, qkv_local - hid_local:]
            o = self._buf("o", (M, self.hidden))
            _timed(on_linear, "o", lambda: layer["o"].forward(v, out=o))
            u = self._buf("up", (M, self.mlp // P))
            _timed(on_linear, "up", lambda: layer["up"].forward(o, out=u))
            d = self._buf("down", (M, self.hidden))
            _timed(on_linear, "down", lambda: layer["down"].forward(u, out=d))
            x = d * torch.rsqrt(d.pow(2).mean(-1, keepdim=True) + 1e-6)
        if out is not None:
            out.copy_(x)
            return out
        return x


    def _forward_chained(self, x: torch.Tensor, on_linear=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The stack with float16 activations between linears (float32 where
        a row-parallel partial sum is reduced), in token chunks.  Per block and chunk: [renorm of the previous block's output,
        qkv, o (row-parallel partial, all-reduce enqueued)] then [wait, up,
        down (partial, all-reduce enqueued)]; each phase runs over all chunks
        before the next, so a chunk's all-reduce overlaps the other chunks'
        GEMMs.  Returns the renormalised float32 output of the last block."""
        from .q4 import rms_renorm
        M = x.shape[0]
        P, C = self.size, self.chunks
        qkv_local, hid_local, mlp_local = self.qkv // P, self.hidden // P, self.mlp // P
        bounds = [(M * c // C, M * (c + 1) // C) for c in range(C)]
        f16 = torch.float16
        o_dtype = f16 if P == 1 else torch.float32   # row-parallel outputs are reduced in float32
        d_dtype = torch.float32                       # down output: the renorm's input
        xin = self._buf("x16", (M, self.hidden), f16)
        t = self._buf("qkv16", (M, qkv_local), f16)
        o = self._buf("o_c", (M, self.hidden), o_dtype)
        u = self._buf("up16", (M, mlp_local), f16)
        d = self._buf("down_c", (M, self.hidden), d_dtype)
        pending = [None] * C
        first = True
        for layer in self.layers:
            works = []
            for c, (a, b) in enumerate(bounds):
                if first:
                    xc = x[a:b]
                else:
                    if pending[c] is not None:
                        pending[c].wait()
                    xc = rms_renorm(d[a:b], xin[a:b])
                _timed(on_linear, "qkv", lambda: layer["qkv"].forward_ex(xc, out=t[a:b]))
                v = t[a:b, qkv_local - hid_local:]
                works.append(_timed(on_linear, "o", lambda: layer["o"].forward_ex(v, out=o[a:b], async_op=True)))
            first = False
            for c, (a, b) in enumerate(bounds):
                if works[c] is not None:
                    works[c].wait()
                _timed(on_linear, "up", lambda: layer["up"].forward_ex(o[a:b], out=u[a:b]))
                pending[c] = _timed(on_linear, "down",
                                    lambda: layer["down"].forward_ex(u[a:b], out=d[a:b], async_op=True))
        if out is None:
            out = self._buf("out32", (M, self.hidden), torch.float32)
        for c, (a, b) in enumerate(bounds):
            if pending[c] is not None:
                pending[c].wait()
            rms_renorm(d[a:b], out[a:b])
        return out


    def _forward_p2p(self, x: torch.Tensor, on_linear=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The float16-chained stack with the row-parallel exchange over peer
        memory.  Rank r owns token rows [r*M/P, (r+1)*M/P).  Per block: qkv
        (column-parallel) -> o partials scattered to the row owners -> owners
        sum them into float16 rows -> all-gather -> up (column-parallel) ->
        down partials scattered -> owners sum and renormalise -> all-gather.
        Same arithmetic as _forward_chained with a float32 all-reduce (the
        owner adds the partials in rank order; the renorm and float16
        rounding are the same kernels' math).  Returns the renormalised
        float32 output of the last block."""
        M = x.shape[0]
        P, r = self.size, self.rank
        if M % P:
            raise ValueError(f"p2p exchange: M={M} not divisible by {P} ranks")
        R = M // P
        bcast = self.exchange == "bcast"
        pull = self.exchange in ("pull", "bcast")
        if self._peer is None or self._peer.rows != R:
            if self._peer is not None:
                self._peer.close()
            self._peer = PeerExchange(self.device, self.group, R, self.hidden, acts=2 if bcast else 0)
        ex = self._peer
        qkv_local, hid_local, mlp_local = self.qkv // P, self.hidden // P, self.mlp // P
        f16 = torch.float16
        t = self._buf("qkv16", (M, qkv_local), f16)
        if bcast:  # peers write their rows of o and of the next block's input straight into these
            o16 = ex.view(3, (M, self.hidden), f16)
            xin = ex.view(4, (M, self.hidden), f16)
        else:
            o16 = self._buf("o16", (M, self.hidden), f16)
            xin = self._buf("x16", (M, self.hidden), f16)
        u = self._buf("up16", (M, mlp_local), f16)
        if out is None:
            out = self._buf("out32", (M, self.hidden), torch.float32)
        mine = slice(r * R, (r + 1) * R)
        n = len(self.layers)
        for i, layer in enumerate(self.layers):
            xc = x if i == 0 else xin
            _timed(on_linear, "qkv", lambda: layer["qkv"].forward_ex(xc, out=t))
            v = t[:, qkv_local - hid_local:]
            dst = out if i == n - 1 else xin
            if pull:
                _timed(on_linear, "o", lambda: layer["o"].forward_local(v, ex, 0))
                if bcast:
                    ex.reduce_bcast(0, 3, renorm=False)
                    ex.signal_wait()
                else:
                    ex.reduce_pull(0, o16[mine], renorm=False)
            else:
                _timed(on_linear, "o", lambda: layer["o"].forward_scatter(v, ex, 0))
                ex.reduce(0, o16[mine], renorm=False)
            if not bcast:
                dist.all_gather_into_tensor(o16, o16[mine], group=self.group)
            _timed(on_linear, "up", lambda: layer["up"].forward_ex(o16, out=u))
            if pull:
                _timed(on_linear, "down", lambda: layer["down"].forward_local(u, ex, 1))
                if bcast and i < n - 1:
                    ex.reduce_bcast(1, 4, renorm=True)
                    ex.signal_wait()
                else:
                    ex.reduce_pull(1, dst[mine], renorm=True)
            else:
                _timed(on_linear, "down", lambda: layer["down"].forward_scatter(u, ex, 1))
                ex.reduce(1, dst[mine], renorm=True)
            if not (bcast and i < n - 1):
                dist.all_gather_into_tensor(dst, dst[mine], group=self.group)
        return out

    def close(self):
        """Release the peer-exchange buffers (collective over the group)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None


def _timed(cb, name, fn):
    if cb is None:
        return fn()
    cb(name, True)
    r = fn()
    cb(name, False)
    return r


def _qkv_rank_order(hidden: int, qkv: int, P: int, device: torch.device) -> torch.Tensor:
    """Column order of a fused [q | k | v] weight (each section `hidden` wide)
    whose r-th contiguous N shard is [q_r | k_r | v_r]."""
    if qkv != 3 * hidden or hidden % P:
        raise ValueError(f"qkv={qkv} must be 3 x hidden={hidden} with hidden divisible by {P} ranks")
    part = hidden // P
    r = torch.arange(P, device=device).view(P, 1, 1)
    sec = torch.arange(3, device=device).view(1, 3, 1)
    j = torch.arange(part, device=device).view(1, 1, part)
    return (sec * hidden + r * part + j).reshape(-1)


def _random_packed(K: int, N: int, block: int, g: torch.Generator, device: torch.device):
    """Row-layout raw buffers: uniform nibbles in [-8, 7] (random u32 words)
    and scales |U(0.001, 0.02)|."""
    words = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device=device,
                          dtype=torch.int64).to(torch.int32)
    scales = torch.rand((K // block, N), generator=g, device=device) * 0.019 + 0.001
    return words.contiguous(), scales.contiguous()
