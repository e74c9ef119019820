"""GPU: a bounded device-side wait that runs out returns an error status.

bq4_peer_signal_wait publishes an epoch into every peer's flag array and
waits, bounded, until every peer has published it into this rank's array.
Here it runs as rank 0 of two ranks on ONE GPU with no second process: the
"peer" flag array is a second local buffer that nothing ever writes into this
rank's slot, so the wait must run out.  With the bound set to 50 ms the
kernel records BQ4_ETIMEOUT in the device error word and returns (it does
not trap), bq4_poll_device_error reports it, and the context stays usable:
a linear launched afterwards still computes the right result.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

import oracle as O
from burn_image_b200 import _lib as L
from burn_image_b200 import q4
from conftest import gen_q4, gen_x

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)


def test_peer_wait_runs_out_and_reports_timeout(rng):
    lib = L.lib()
    assert lib.bq4_poll_device_error() == L.OK  # start from a clear error word
    flags = torch.zeros(2, dtype=torch.int32, device=DEV)      # this rank's array: nobody signals slot 1
    other = torch.zeros(2, dtype=torch.int32, device=DEV)      # stands in for rank 1's array
    peers = (ctypes.c_void_p * 2)(ctypes.c_void_p(flags.data_ptr()), ctypes.c_void_p(other.data_ptr()))
    L.check(lib.bq4_set_peer_wait_timeout_ns(50_000_000))      # 50 ms
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        L.check(lib.bq4_peer_signal_wait(ctypes.c_void_p(flags.data_ptr()), peers, 2, 0, 1, _stream()))
        rc = lib.bq4_poll_device_error()  # synchronizes
        elapsed = time.perf_counter() - t0
    finally:
        L.check(lib.bq4_set_peer_wait_timeout_ns(0))  # back to the default bound
    assert rc == L.ETIMEOUT
    assert b"bounded wait" in lib.bq4_last_error_string()
    assert 0.04 <= elapsed < 5.0, elapsed
    # the signal half ran: rank 0 published epoch 1 into slot 0 of the "peer" array
    assert other.cpu().tolist() == [1, 0]
    assert lib.bq4_poll_device_error() == L.OK  # the poll cleared the word

    # the context is still usable
    K, N, M = 256, 128, 16
    w, s = gen_q4(K, N, 128, O.LAYOUT_ROW, rng)
    x = gen_x(M, K, rng)
    pw = q4.PreparedQ4Weight(torch.from_numpy(w.view(np.int32)).to(DEV), torch.from_numpy(s).to(DEV), K, N, 128,
                             O.LAYOUT_ROW, DEV)
    y = pw.linear(torch.from_numpy(x).to(DEV)).cpu().numpy()
    ref = O.linear_f64(x, O.unpack(w, s, K, N, 128, O.LAYOUT_ROW))
    assert O.rel_frobenius(y, ref) <= 5e-3


def test_peer_wait_passes_when_signalled():
    """The same wait with the flag already set returns without an error."""
    lib = L.lib()
    assert lib.bq4_poll_device_error() == L.OK
    flags = torch.tensor([0, 1], dtype=torch.int32, device=DEV)  # rank 1 has published epoch 1
    other = torch.zeros(2, dtype=torch.int32, device=DEV)
    peers = (ctypes.c_void_p * 2)(ctypes.c_void_p(flags.data_ptr()), ctypes.c_void_p(other.data_ptr()))
    L.check(lib.bq4_set_peer_wait_timeout_ns(50_000_000))
    try:
        L.check(lib.bq4_peer_signal_wait(ctypes.c_void_p(flags.data_ptr()), peers, 2, 0, 1, _stream()))
        rc = lib.bq4_poll_device_error()
    finally:
        L.check(lib.bq4_set_peer_wait_timeout_ns(0))
    assert rc == L.OK
    assert other.cpu().tolist() == [1, 0]
