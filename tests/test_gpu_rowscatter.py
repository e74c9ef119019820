"""GPU, one device: the row-scatter GEMM (bq4_linear_rowscatter), the
row-parallel layer's epilogue that writes each output row's partial product
into the receive buffer of the rank that owns the row.

The receive buffers of all "ranks" are plain buffers on this one device, so
the kernel's addressing is checked without peer memory: owner r of rows
[r R, (r+1) R) (R = M / nranks) must hold, at rows [rank R, (rank+1) R) of its
buffer, exactly the rows the plain linear (bq4_linear_ex, f32 output) computes
for them, and no other row of any buffer may change.  Row-slice sizes that are
not multiples of the token tile put owner boundaries inside tiles.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from burn_image_b200 import _lib as L
from burn_image_b200 import q4
from conftest import gen_bias, gen_q4

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).to(DEV)


@pytest.mark.parametrize("M,K,N,nranks,rank,x_f16", [(520, 1024, 768, 4, 2, True), (600, 768, 384, 8, 5, True),
                                                     (264, 512, 640, 2, 0, False), (4352, 3072, 3072, 4, 3, True)])
def test_rowscatter_rows_land_at_their_owner(M, K, N, nranks, rank, x_f16, rng):
    w, s = gen_q4(K, N, 128, O.LAYOUT_ROW, rng)
    bias = dev(gen_bias(N, rng))
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, 128, O.LAYOUT_ROW, DEV)
    x = torch.randn((M, K), generator=torch.Generator(device=DEV).manual_seed(M + K), device=DEV)
    if x_f16:
        x = x.half()
    ref = pw.linear_ex(x, bias)  # f32 [M, N]
    R = M // nranks
    sentinel = float("nan")
    bufs = [torch.full((M, N), sentinel, device=DEV) for _ in range(nranks)]
    targets = (ctypes.c_void_p * L.MAX_PEERS)(*[b.data_ptr() for b in bufs], *([None] * (L.MAX_PEERS - nranks)))
    dt = L.DTYPE_F16 if x_f16 else L.DTYPE_F32
    n = ctypes.c_size_t()
    L.check(L.lib().bq4_linear_ex_workspace_size(pw.handle, M, dt, ctypes.byref(n)))
    ws = torch.empty(max(n.value, 256), dtype=torch.uint8, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    for _ in range(2):  # a repeated call writes the same bits
        L.check(L.lib().bq4_linear_rowscatter(pw.handle, ctypes.c_void_p(x.data_ptr()), dt, M, x.stride(0),
                                              ctypes.c_void_p(bias.data_ptr()), L.ACT_NONE, targets, nranks, rank, N,
                                              ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream))
        torch.cuda.synchronize()
        q4.poll_device_error()
        for r in range(nranks):
            got = bufs[r][rank * R:(rank + 1) * R]
            want = ref[r * R:(r + 1) * R]
            rel = (torch.linalg.norm(got.double() - want.double()) / torch.linalg.norm(want.double())).item()
            assert rel <= 1e-6, f"owner {r}: rel {rel}"
            others = torch.cat([bufs[r][:rank * R], bufs[r][(rank + 1) * R:]])
            assert bool(torch.isnan(others).all()), f"owner {r}: rows outside this rank's slot were written"


@pytest.mark.parametrize("nranks,rank,renorm,f16", [(4, 1, False, True), (8, 7, True, True), (2, 0, True, False)])
def test_reduce_slices_peer_matches_reduce_slices(nranks, rank, renorm, f16):
    """bq4_reduce_slices_peer (the pull exchange: rank s's slice is rows
    [rank R, (rank+1) R) of rank s's own [M][H] partial buffer) against
    bq4_reduce_slices on the same rows gathered into one [P][R][H] receive
    buffer: the same sums in the same order, so the same bits.  All "ranks"
    are buffers on this one device."""
    R, H = 40, 3072
    M = nranks * R
    g = torch.Generator(device=DEV).manual_seed(nranks * 10 + rank)
    parts = [torch.randn((M, H), generator=g, device=DEV) * 100 for _ in range(nranks)]
    recv = torch.stack([p[rank * R:(rank + 1) * R] for p in parts]).contiguous()  # [P][R][H]
    odt = torch.float16 if f16 else torch.float32
    dt = L.DTYPE_F16 if f16 else L.DTYPE_F32
    a = torch.empty((R, H), dtype=odt, device=DEV)
    b = torch.empty((R, H), dtype=odt, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    L.check(L.lib().bq4_reduce_slices(ctypes.c_void_p(recv.data_ptr()), nranks, R, H, H, 1 if renorm else 0,
                                      ctypes.c_float(1e-6), ctypes.c_void_p(a.data_ptr()), dt, H, stream))
    src = (ctypes.c_void_p * nranks)(*[p.data_ptr() for p in parts])
    L.check(L.lib().bq4_reduce_slices_peer(src, nranks, rank * R, R, H, H, 1 if renorm else 0, ctypes.c_float(1e-6),
                                           ctypes.c_void_p(b.data_ptr()), dt, H, stream))
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert torch.equal(a, b)
    want = sum(p[rank * R:(rank + 1) * R].double() for p in parts)
    if renorm:
        want = want / torch.sqrt((want * want).mean(dim=1, keepdim=True) + 1e-6)
    rel = (torch.linalg.norm(b.double() - want) / torch.linalg.norm(want)).item()
    assert rel <= (1e-3 if f16 else 1e-6), rel


@pytest.mark.parametrize("nranks,rank,renorm", [(4, 2, False), (8, 0, True)])
def test_reduce_slices_peer_bcast_writes_every_copy(nranks, rank, renorm):
    """bq4_reduce_slices_peer_bcast writes this rank's reduced rows into every
    rank's [M][H] f16 activation copy at rows [rank R, (rank+1) R), with the
    bits bq4_reduce_slices_peer gives, and leaves every other row alone."""
    R, H = 24, 1024
    M = nranks * R
    g = torch.Generator(device=DEV).manual_seed(nranks + 100 * rank)
    parts = [torch.randn((M, H), generator=g, device=DEV) for _ in range(nranks)]
    src = (ctypes.c_void_p * nranks)(*[p.data_ptr() for p in parts])
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    ref = torch.empty((R, H), dtype=torch.float16, device=DEV)
    L.check(L.lib().bq4_reduce_slices_peer(src, nranks, rank * R, R, H, H, 1 if renorm else 0, ctypes.c_float(1e-6),
                                           ctypes.c_void_p(ref.data_ptr()), L.DTYPE_F16, H, stream))
    copies = [torch.full((M, H), float("nan"), dtype=torch.float16, device=DEV) for _ in range(nranks)]
    outs = (ctypes.c_void_p * nranks)(*[c.data_ptr() for c in copies])
    L.check(L.lib().bq4_reduce_slices_peer_bcast(src, nranks, rank * R, R, H, H, 1 if renorm else 0,
                                                 ctypes.c_float(1e-6), outs, L.DTYPE_F16, H, stream))
    torch.cuda.synchronize()
    q4.poll_device_error()
    for c in copies:
        assert torch.equal(c[rank * R:(rank + 1) * R], ref)
        assert bool(torch.isnan(torch.cat([c[:rank * R], c[(rank + 1) * R:]])).all())
