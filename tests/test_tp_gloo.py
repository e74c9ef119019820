"""CPU, world size 2 over gloo: the tensor-parallel decomposition of the Q4
linears (burn_image_b200/tp.py) is exact.

Each rank slices the reference-packed buffers with the product's sharding
helpers, computes its shard with the CPU oracle, and the collective the
product uses (all-gather of column-parallel outputs, all-reduce of
row-parallel partials) reproduces the unsharded result.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import gen_bias, gen_q4, gen_x


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, layout, results):
    import oracle as O
    from burn_image_b200 import tp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)  # identical data on every rank
        M, K, N, block = 9, 256, 64, 64
        words, scales = gen_q4(K, N, block, layout, rng)
        x = gen_x(M, K, rng)
        bias = gen_bias(N, rng)
        W = O.unpack(words, scales, K, N, block, layout)
        full = O.linear_f64(x, W, bias)

        # column parallel: this rank's output columns, then all-gather
        n0, n1 = tp.column_shard_bounds(N, rank, world)
        w_c, s_c = tp.slice_raw(words, scales, K, N, block, layout, n0, n1, 0, K)
        W_c = O.unpack(w_c, s_c, K, n1 - n0, block, layout)
        y_c = torch.from_numpy(O.linear_f64(x, W_c, bias[n0:n1]))
        parts = [torch.empty_like(y_c) for _ in range(world)]
        dist.all_gather(parts, y_c)
        col = torch.cat(parts, dim=1).numpy()

        # row parallel: this rank's input rows, bias added once, all-reduce
        k0, k1 = tp.row_shard_bounds(K, block, rank, world)
        w_r, s_r = tp.slice_raw(words, scales, K, N, block, layout, 0, N, k0, k1)
        W_r = O.unpack(w_r, s_r, k1 - k0, N, block, layout)
        y_r = torch.from_numpy(O.linear_f64(np.ascontiguousarray(x[:, k0:k1]), W_r,
                                            bias if rank == 0 else None).astype(np.float64))
        dist.all_reduce(y_r)
        row = y_r.numpy()
        if rank == 0:
            results["col"] = float(np.abs(col - full).max())
            results["row"] = float(np.abs(row - full).max())
            results["scale"] = float(np.abs(full).max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layout", [0, 1])
def test_tensor_parallel_decomposition_gloo(layout):
    world = 2
    with mp.get_context("spawn").Manager() as mgr:  # no fork of this multi-threaded process
        results = mgr.dict()
        mp.spawn(_worker, args=(world, _free_port(), layout, results), nprocs=world, join=True)
        res = dict(results)
    assert res["col"] <= 1e-6 * max(1.0, res["scale"])
    assert res["row"] <= 1e-5 * max(1.0, res["scale"])


def test_shard_bounds_rules():
    from burn_image_b200 import tp
    assert tp.column_shard_bounds(9216, 3, 8) == (3456, 4608)
    assert tp.row_shard_bounds(12288, 128, 7, 8) == (10752, 12288)
    with pytest.raises(ValueError):
        tp.row_shard_bounds(3360, 32, 0, 4)  # 840 is not a multiple of 32: real Boogu widths cannot split 4-way
    with pytest.raises(ValueError):
        tp.column_shard_bounds(3072, 0, 5)


@pytest.mark.parametrize("P", [1, 2, 4, 8])
def test_stack_qkv_order_gives_each_rank_its_value_slice(P):
    # the DiT stack's o-projection reads the last hidden/P columns of a rank's
    # contiguous qkv shard as its v slice; with the rank order of the fused
    # weight's columns the sharded block equals the unsharded one
    from burn_image_b200.tp import _qkv_rank_order
    rng = np.random.default_rng(P)
    H, M = 16, 5
    x = rng.standard_normal((M, H))
    wqkv = rng.standard_normal((H, 3 * H))
    wo = rng.standard_normal((H, H))
    ref = (x @ wqkv)[:, 2 * H:] @ wo  # o(v)
    perm = _qkv_rank_order(H, 3 * H, P, torch.device("cpu")).numpy()
    assert sorted(perm.tolist()) == list(range(3 * H))
    wp = wqkv[:, perm]
    shard, part = 3 * H // P, H // P
    total = sum((x @ wp[:, r * shard:(r + 1) * shard])[:, shard - part:] @ wo[r * part:(r + 1) * part]
                for r in range(P))
    assert np.allclose(total, ref)
