"""GPU: bq4_linear_noalloc, the entry point for callers that cannot allocate
device memory (their runtime owns all device memory, or they must not call
the device-synchronizing cudaMalloc), against the workspace-taking
bq4_linear.

It runs the same GEMM with its scratch in a static device array of
BQ4_NOALLOC_SCRATCH_BYTES instead of a caller-provided workspace.  When
bq4_linear's plan fits that array the two entry points run the same plan
and their outputs must be bit-identical; when it does not because of the
stream-K partial slots, the no-alloc call plans whole tiles instead and the
outputs agree within the parity tolerance.  Each case calls it twice in a
row, since calls share (and reuse) that array.  Kept in a file that pytest
collects last; it also passes when run alone.
"""
import ctypes

import numpy as np
import pytest
import torch

from burn_image_b200 import _lib as L
from burn_image_b200 import q4

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TOL = 5e-3  # relative Frobenius, the parity tolerance of the other GPU tests


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)


def _problem(M, K, N, block, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    words = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device=DEV,
                          dtype=torch.int64).to(torch.int32).contiguous()
    scales = (torch.rand((K // block, N), generator=g, device=DEV) * 0.019 + 0.001).contiguous()
    x = torch.randn((M, K), generator=g, device=DEV)
    bias = torch.randn(N, generator=g, device=DEV) * 0.02
    return q4.PreparedQ4Weight(words, scales, K, N, block, L.LAYOUT_ROW, DEV), x, bias


def _rel(a, b):
    return (torch.linalg.norm(a.double() - b.double()) / torch.linalg.norm(b.double())).item()


def _run_pair(pw, x, bias, act, M, N):
    """bq4_linear's output and two consecutive bq4_linear_noalloc outputs."""
    lib = L.lib()
    K = pw.K
    y_ref = torch.empty((M, N), dtype=torch.float32, device=DEV)
    ws = q4.Workspace.get(DEV, pw.workspace_bytes(M))
    L.check(lib.bq4_linear(pw.handle, _p(x), M, K, _p(bias), act, None, _p(y_ref), _p(ws), ws.numel(), _stream()))
    outs = []
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device=DEV)
        L.check(lib.bq4_linear_noalloc(pw.handle, _p(x), M, K, _p(bias), act, None, _p(y), _stream()))
        torch.cuda.synchronize()
        q4.poll_device_error()
        assert torch.isfinite(y).all()
        outs.append(y)
    return y_ref, outs


# exact-weight path (M <= 64), folded path (block 32), and a split-K plan (few tiles):
# the default plan fits the static array, so the same kernel runs the same plan on the
# same inputs and the outputs must be bit-identical
@pytest.mark.parametrize("M,K,N,block,act", [(48, 512, 256, 128, 1), (300, 1024, 640, 32, 0),
                                             (256, 2560, 2560, 128, 2)])
def test_noalloc_matches_workspace_entry_twice(M, K, N, block, act):
    pw, x, bias = _problem(M, K, N, block, seed=M + K + N)
    assert pw.workspace_bytes(M) <= L.NOALLOC_SCRATCH_BYTES
    y_ref, outs = _run_pair(pw, x, bias, act, M, N)
    for y in outs:
        assert torch.equal(y, y_ref)


def test_noalloc_drops_stream_k_tail_to_fit():
    """A plan whose stream-K partial slots push the workspace past the static
    array: the entry point re-plans with whole tiles, which fit.  The tiling
    then differs from bq4_linear's, so the outputs agree within the parity
    tolerance (and the two no-alloc calls agree bit for bit)."""
    q4.set_numerics(L.NUMERICS_EXACT)  # stream-K tails are planned for exact numerics
    try:
        found = None
        for M, K, N in [(2048, 4096, 2560), (2048, 4096, 2304), (1536, 6144, 2560), (2560, 3072, 2560)]:
            pw, x, bias = _problem(M, K, N, 128, seed=M + N)
            info = pw.plan_info(M)
            if (info["sk_tiles"] > 0 and pw.workspace_bytes(M) > L.NOALLOC_SCRATCH_BYTES
                    and M * K * 2 + (1 << 20) <= L.NOALLOC_SCRATCH_BYTES):
                found = (pw, x, bias, M, N)
                break
        assert found is not None, "no candidate shape plans a stream-K tail beyond the static array"
        pw, x, bias, M, N = found
        y_ref, outs = _run_pair(pw, x, bias, 0, M, N)
        assert _rel(outs[0], y_ref) <= TOL
        assert torch.equal(outs[0], outs[1])
    finally:
        q4.set_numerics(L.NUMERICS_AUTO)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    M, K, N = 8192, 4096, 256  # the f16 copy of x alone is 64 MiB
    pw, x, _ = _problem(64, K, N, 128, seed=3)
    x = torch.zeros((M, K), dtype=torch.float32, device=DEV)
    y = torch.empty((M, N), dtype=torch.float32, device=DEV)
    assert pw.workspace_bytes(M) > L.NOALLOC_SCRATCH_BYTES
    rc = L.lib().bq4_linear_noalloc(pw.handle, _p(x), M, K, None, 0, None, _p(y), _stream())
    assert rc == L.EWORKSPACE
    assert b"static limit" in L.lib().bq4_last_error_string()
