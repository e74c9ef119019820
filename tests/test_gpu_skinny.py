"""GPU parity of the few-token kernel (csrc/bq4_skinny.cu) through the C ABI.

The planner sends decode- and prompt-shaped calls (up to 256 rows) to a
bandwidth-bound kernel that streams the weights from HBM into registers and
runs mma.sync tensor-core steps; BQ4_FORCE_SKINNY=1 makes it take every call
that fits, BQ4_NO_SKINNY=1 none, BQ4_SKINNY_KS / BQ4_SKINNY_STAGES pin its K
splits per cluster and the depth of its weight ring.  Bars as elsewhere: relative
Frobenius <= 5e-3 against the oracle's f64 result, and a tight check against
the same f16 operand staging emulated on the CPU.
"""
import ctypes
import os
from contextlib import contextmanager

import numpy as np
import pytest
import torch

import oracle as O
from burn_image_b200 import _lib as L
from burn_image_b200 import q4
from conftest import gen_bias, gen_q4, gen_x

pytestmark = pytest.mark.gpu
TOL = 5e-3
DEV = torch.device("cuda", 0)


@contextmanager
def env(**kv):
    old = {k: os.environ.get(k) for k in kv}
    try:
        for k, v in kv.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = str(v)
        yield
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).to(DEV)


def staged_weight(words, scales, K, N, block, layout, exact):
    W = O.unpack(words, scales, K, N, block, layout)
    if exact:
        return W
    s = np.repeat(scales if layout == O.LAYOUT_ROW else scales.T, block, axis=0)[:K].astype(np.float64)
    q = np.rint(W / np.where(s == 0, 1, s))
    s16 = s.astype(np.float16)
    return (q.astype(np.float16) * s16).astype(np.float16).astype(np.float32)


def rel(got, ref):
    return O.rel_frobenius(got, ref)


CASES = [
    # M, K, N, block, layout, act, bias, aux
    (1, 2560, 512, 128, O.LAYOUT_COL, O.ACT_NONE, True, False),
    (1, 256, 136, 128, O.LAYOUT_ROW, O.ACT_NONE, False, False),
    (3, 384, 264, 64, O.LAYOUT_ROW, O.ACT_GELU_TANH, True, False),
    (8, 1024, 384, 32, O.LAYOUT_COL, O.ACT_SILU, True, True),
    (9, 640, 200, 16, O.LAYOUT_ROW, O.ACT_NONE, True, False),
    (16, 3360, 264, 32, O.LAYOUT_ROW, O.ACT_NONE, True, False),
    (17, 512, 128, 8, O.LAYOUT_COL, O.ACT_NONE, False, True),
    (33, 1152, 640, 128, O.LAYOUT_ROW, O.ACT_GELU_TANH, True, False),
    (64, 768, 256, 128, O.LAYOUT_COL, O.ACT_NONE, True, False),
    (100, 512, 384, 32, O.LAYOUT_ROW, O.ACT_NONE, True, True),
    (256, 2560, 512, 128, O.LAYOUT_COL, O.ACT_NONE, True, False),
]


@pytest.mark.parametrize("M,K,N,block,layout,act,with_bias,with_aux", CASES)
def test_skinny_linear_parity(M, K, N, block, layout, act, with_bias, with_aux, rng):
    w, s = gen_q4(K, N, block, layout, rng)
    x = gen_x(M, K, rng)
    bias = gen_bias(N, rng) if with_bias else None
    aux = rng.standard_normal((M, N), dtype=np.float32) if with_aux else None
    W = O.unpack(w, s, K, N, block, layout)
    ref = O.linear_f64(x, W, bias, act, aux)
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, block, layout, DEV)
    # exact numerics (AUTO's choice up to 64 rows) need 128-blocks in this kernel;
    # 64-blocks then go to the tcgen05 GEMM, so they are run folded here
    q4.set_numerics(L.NUMERICS_FOLDED if block == 64 and M <= 64 else L.NUMERICS_AUTO)
    try:
        with env(BQ4_FORCE_SKINNY=1, BQ4_NO_SKINNY=None):
            info = pw.plan_info(M)
            assert info["skinny"] == 1, info
            y = pw.linear(dev(x), dev(bias) if bias is not None else None, act,
                          dev(aux) if aux is not None else None).cpu().numpy()
    finally:
        q4.set_numerics(L.NUMERICS_AUTO)
    q4.poll_device_error()
    assert np.all(np.isfinite(y))
    rf = rel(y, ref)
    print(f"skinny M{M} K{K} N{N} b{block}: rel_frob={rf:.3e} max_abs={np.abs(y - ref).max():.3e}")
    assert rf <= TOL
    Ws = staged_weight(w, s, K, N, block, layout, exact=info["exact"] == 1)
    ref_s = O.linear_f64(x.astype(np.float16).astype(np.float32), Ws, bias, act, aux)
    tight = 2e-3 if act != O.ACT_NONE else 1e-5
    assert rel(y, ref_s) <= tight


@pytest.mark.parametrize("M,exact,KS", [(1, 1, 4), (5, 0, 4), (12, 1, 3), (16, 0, 2), (9, 1, 1)])
def test_skinny_three_ctas_per_sm(M, exact, KS, rng):
    """The variant compiled for three CTAs per SM (BQ4_SKINNY_MINB=3: one
    weight, up to 16 tokens, a smaller register and shared-memory budget)
    gives the oracle's result, deterministically, at every K split."""
    K, N, block = 2560, 640, 128
    w, s = gen_q4(K, N, block, O.LAYOUT_ROW, rng)
    x = gen_x(M, K, rng)
    bias = gen_bias(N, rng)
    ref = O.linear_f64(x, O.unpack(w, s, K, N, block, O.LAYOUT_ROW), bias)
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, block, O.LAYOUT_ROW, DEV)
    xd, bd = dev(x), dev(bias)
    q4.set_numerics(L.NUMERICS_EXACT if exact else L.NUMERICS_FOLDED)
    try:
        with env(BQ4_SKINNY_MINB=3, BQ4_SKINNY_KS=KS):
            info = pw.plan_info(M)
            assert info["skinny"] == 1 and info["ksplit"] == KS and info["exact"] == exact, info
            a = pw.linear(xd, bd).clone()
            b = pw.linear(xd, bd).clone()
    finally:
        q4.set_numerics(L.NUMERICS_AUTO)
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert torch.equal(a, b)
    assert rel(a.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("KS,STAGES", [(1, 0), (2, 2), (4, 3), (8, 0), (3, 2), (1, 2)])
def test_skinny_ring_depths_and_cluster_splits(KS, STAGES, rng):
    """Every cluster K split and weight-ring depth gives the same result
    within rounding; each one is deterministic."""
    M, K, N, block = 12, 2048, 384, 128
    w, s = gen_q4(K, N, block, O.LAYOUT_COL, rng)
    x = gen_x(M, K, rng)
    bias = gen_bias(N, rng)
    ref = O.linear_f64(x, O.unpack(w, s, K, N, block, O.LAYOUT_COL), bias)
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, block, O.LAYOUT_COL, DEV)
    xd, bd = dev(x), dev(bias)
    with env(BQ4_FORCE_SKINNY=1, BQ4_SKINNY_KS=KS, BQ4_SKINNY_STAGES=STAGES or None):
        info = pw.plan_info(M)
        assert info["skinny"] == 1 and info["ksplit"] == KS, info
        a = pw.linear(xd, bd).clone()
        b = pw.linear(xd, bd).clone()
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert torch.equal(a, b)
    assert rel(a.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("M,numerics", [(4, L.NUMERICS_EXACT), (4, L.NUMERICS_FOLDED), (48, L.NUMERICS_EXACT),
                                        (200, L.NUMERICS_FOLDED)])
def test_skinny_matches_tcgen05_path(M, numerics, rng):
    """The few-token kernel and the tcgen05 GEMM stage the operands the same
    way, so they agree far inside the parity bar (only the f32 summation
    order differs)."""
    K, N, block = 1536, 640, 128
    w, s = gen_q4(K, N, block, O.LAYOUT_ROW, rng)
    x = dev(gen_x(M, K, rng))
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, block, O.LAYOUT_ROW, DEV)
    q4.set_numerics(numerics)
    try:
        with env(BQ4_FORCE_SKINNY=1, BQ4_NO_SKINNY=None):
            assert pw.plan_info(M)["skinny"] == 1
            a = pw.linear(x).clone()
        with env(BQ4_NO_SKINNY=1, BQ4_FORCE_SKINNY=None):
            assert pw.plan_info(M)["skinny"] == 0
            b = pw.linear(x).clone()
    finally:
        q4.set_numerics(L.NUMERICS_AUTO)
    q4.poll_device_error()
    d = (torch.linalg.norm(a.double() - b.double()) / torch.linalg.norm(b.double())).item()
    print(f"skinny vs tcgen05 M{M} numerics {numerics}: {d:.3e}")
    assert d <= 1e-5


@pytest.mark.parametrize("M,K,N,block", [(1, 2560, 512, 128), (7, 256, 128, 32), (16, 2560, 1024, 128)])
def test_skinny_gated_parity(M, K, N, block, rng):
    wg, sg = gen_q4(K, N, block, O.LAYOUT_COL, rng)
    wu, su = gen_q4(K, N, block, O.LAYOUT_COL, rng)
    x = gen_x(M, K, rng)
    bg, bu = gen_bias(N, rng), gen_bias(N, rng)
    ref = O.linear_gated_f64(x, O.unpack(wg, sg, K, N, block, 0), O.unpack(wu, su, K, N, block, 0), bg, bu)
    g = q4.PreparedQ4Weight(dev(wg), dev(sg), K, N, block, 0, DEV)
    u = q4.PreparedQ4Weight(dev(wu), dev(su), K, N, block, 0, DEV)
    with env(BQ4_FORCE_SKINNY=1):
        assert g.plan_info(M, gated=True)["skinny"] == 1
        y = q4.linear_gated(g, u, dev(x), dev(bg), dev(bu)).cpu().numpy()
    q4.poll_device_error()
    assert rel(y, ref) <= TOL


def test_skinny_f16_chain_and_pitches(rng):
    """bq4_linear_ex through the few-token kernel: f16 activations read in
    place from a column slice of a wider buffer, f16 output into a column
    slice, against the f32 entry point (the same rounding, so the f16 output
    equals the f32 output rounded to f16)."""
    M, K, N, block = 10, 1024, 256, 128
    w, s = gen_q4(K, N, block, O.LAYOUT_ROW, rng)
    x = gen_x(M, K, rng)
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, block, O.LAYOUT_ROW, DEV)
    wide = torch.zeros((M, 3 * K), dtype=torch.float16, device=DEV)
    wide[:, K:2 * K] = dev(x).half()
    out = torch.zeros((M, 2 * N), dtype=torch.float16, device=DEV)
    with env(BQ4_FORCE_SKINNY=1):
        assert pw.plan_info(M)["skinny"] == 1
        pw.linear_ex(wide[:, K:2 * K], out=out[:, N:])
        y32 = pw.linear(dev(x))
    torch.cuda.synchronize()
    q4.poll_device_error()
    assert torch.equal(out[:, N:], y32.half())
    assert torch.count_nonzero(out[:, :N]) == 0


def test_skinny_strided_f32_input(rng):
    """ldx > K and an unaligned row start (scalar staging path)."""
    M, K, N, block = 6, 520, 136, 8
    w, s = gen_q4(K, N, block, O.LAYOUT_ROW, rng)
    big = gen_x(M, 3 * K + 1, rng)
    xs = np.ascontiguousarray(big[:, K + 1:2 * K + 1])
    ref = O.linear_f64(xs, O.unpack(w, s, K, N, block, O.LAYOUT_ROW))
    pw = q4.PreparedQ4Weight(dev(w), dev(s), K, N, block, O.LAYOUT_ROW, DEV)
    bigd = dev(big)
    y = torch.empty((M, N), dtype=torch.float32, device=DEV)
    ws = q4.Workspace.get(DEV, max(pw.workspace_bytes(M), 256))
    with env(BQ4_FORCE_SKINNY=1):
        assert pw.plan_info(M)["skinny"] == 1
        L.check(L.lib().bq4_linear(pw.handle, ctypes.c_void_p(bigd.data_ptr() + (K + 1) * 4), M, 3 * K + 1, None,
                                   0, None, ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                   ws.numel(), ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)))
    q4.poll_device_error()
    assert rel(y.cpu().numpy(), ref) <= TOL


def test_default_plan_routes_decode_shapes_to_skinny():
    """Under the default planner the decode-shaped calls take the few-token
    kernel and need no workspace."""
    g = torch.Generator(device=DEV).manual_seed(5)
    K, N = 2560, 9728
    words = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device=DEV,
                          dtype=torch.int64).to(torch.int32)
    scales = torch.rand((K // 128, N), generator=g, device=DEV) * 0.019 + 0.001
    pw = q4.PreparedQ4Weight(words.contiguous(), scales.contiguous(), K, N, 128, L.LAYOUT_ROW, DEV)
    for M in (1, 16):
        info = pw.plan_info(M)
        assert info["skinny"] == 1, (M, info)
        assert pw.workspace_bytes(M) == 0
        x = torch.randn((M, K), generator=g, device=DEV)
        W = pw.dequantize()
        ref = x.half().double() @ W.double()
        y = pw.linear(x)
        q4.poll_device_error()
        assert (torch.linalg.norm(y.double() - ref) / torch.linalg.norm(ref)).item() <= 1e-5
