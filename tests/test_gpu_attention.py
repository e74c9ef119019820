"""GPU: attention on the q/k/v projection output (bq4_attention), against the
oracle (pinned to the reference's attention test, native_flash.rs:2784-2843).

Inputs are binary16, so the oracle runs on the same f16 values; the kernels
add the tf32 rounding of the softmax probabilities and f32 accumulation.

- the reference test's grouped-query fixture (4 query heads on 2 kv heads);
- random shapes with grouped heads, the model's head_dim 120 and 128,
  sequence lengths off the tile sizes, an explicit scale;
- head_dim 128 (the fused kernel) against the unfused composition;
- a DiT-size head set (24 heads, 4352 tokens) checked on a slice of query rows;
- repeated calls give the same bits; argument errors.
"""
import numpy as np
import pytest
import torch

import oracle as O
from burn_image_b200 import f16 as F
from burn_image_b200 import q4
from burn_image_b200.q4 import Bq4Error

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TOL = 5e-3


def _deterministic(shape, offset):
    n = int(np.prod(shape))
    idx = np.arange(n, dtype=np.int64)
    return ((((idx + offset) * 19 + 7) % 53) - 26.0).astype(np.float32).reshape(shape) / np.float32(17.0)


def _check(q, k, v, scale=None, rows=None):
    out = F.attention(q, k, v, scale)
    torch.cuda.synchronize()
    q4.poll_device_error()
    qn = q.float().cpu().numpy()
    if rows is not None:
        qn = qn[:, :, rows]
    ref = O.attention_f64(qn, k.float().cpu().numpy(), v.float().cpu().numpy(), scale)
    got = out.cpu().numpy() if rows is None else out.cpu().numpy()[:, :, rows]
    rel = O.rel_frobenius(got, ref)
    assert rel <= TOL, f"rel_frob {rel}, max_abs {np.abs(got - ref).max()}"
    return out, rel


def test_reference_gqa_fixture():
    h = lambda a: torch.from_numpy(a).to(DEV).half()  # noqa: E731
    q = h(_deterministic([1, 4, 3, 120], 2))
    k = h(_deterministic([1, 2, 5, 120], 7))
    v = h(_deterministic([1, 2, 5, 120], 11))
    _, rel = _check(q, k, v)
    assert rel <= 2e-3


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv,D,scale", [(1, 4, 2, 300, 260, 128, None), (2, 3, 3, 77, 131, 120, None),
                                                     (1, 2, 1, 513, 1000, 64, 0.05)])
def test_random_shapes(B, Hq, Hkv, Sq, Skv, D, scale):
    g = torch.Generator(device=DEV).manual_seed(Sq + Skv + D)
    q = torch.randn((B, Hq, Sq, D), generator=g, device=DEV).half()
    k = torch.randn((B, Hkv, Skv, D), generator=g, device=DEV).half()
    v = torch.randn((B, Hkv, Skv, D), generator=g, device=DEV).half()
    out, _ = _check(q, k, v, scale)
    assert torch.equal(out, F.attention(q, k, v, scale))


def test_fused_matches_unfused(monkeypatch):
    # head_dim 128 runs the fused kernel; BQ4_ATTN_UNFUSED=1 the GEMM + softmax composition
    g = torch.Generator(device=DEV).manual_seed(5)
    q = torch.randn((2, 4, 200, 128), generator=g, device=DEV).half()
    k = torch.randn((2, 2, 333, 128), generator=g, device=DEV).half()
    v = torch.randn((2, 2, 333, 128), generator=g, device=DEV).half()
    fused = F.attention(q, k, v)
    monkeypatch.setenv("BQ4_ATTN_UNFUSED", "1")
    unfused = F.attention(q, k, v)
    torch.cuda.synchronize()
    q4.poll_device_error()
    rel = (torch.linalg.norm(fused.double() - unfused.double()) / torch.linalg.norm(unfused.double())).item()
    assert rel <= 3e-3, f"rel {rel}"


@pytest.mark.parametrize("Sq,Skv", [(512, 384), (256, 40), (384, 64), (640, 129), (129, 200)])
def test_two_query_tiles(Sq, Skv, monkeypatch):
    # more than 128 query rows: two 128-row tiles per CTA (the last CTA's second tile may be
    # partly or wholly past Sq); full key blocks, one block of fewer than 64 keys, the 64- and
    # 128-key edges.  Against the oracle, and against one tile per CTA (BQ4_ATTN_ONE_TILE=1),
    # which sums the probabilities in another order and takes every exponential from
    # ex2.approx: the two-tile kernel's polynomial exponentials (relative error 7.5e-5) move
    # about 1 % of those f16 probabilities by one ulp.
    g = torch.Generator(device=DEV).manual_seed(Sq * 7 + Skv)
    q = torch.randn((1, 4, Sq, 128), generator=g, device=DEV).half()
    k = torch.randn((1, 2, Skv, 128), generator=g, device=DEV).half()
    v = torch.randn((1, 2, Skv, 128), generator=g, device=DEV).half()
    two, _ = _check(q, k, v)
    monkeypatch.setenv("BQ4_ATTN_ONE_TILE", "1")
    one, _ = _check(q, k, v)
    rel = (torch.linalg.norm(two.double() - one.double()) / torch.linalg.norm(one.double())).item()
    assert rel <= 2e-4, f"rel {rel}"
    if Sq == 512:
        # every polynomial share gives the oracle's result; without it the tiles match one tile per CTA closely
        monkeypatch.delenv("BQ4_ATTN_ONE_TILE")
        for poly in ("0", "2", "3"):
            monkeypatch.setenv("BQ4_ATTN_POLY", poly)
            out, _ = _check(q, k, v)
            if poly == "0":
                rel0 = (torch.linalg.norm(out.double() - one.double()) / torch.linalg.norm(one.double())).item()
                assert rel0 <= 1e-5, f"rel {rel0}"


def test_running_max_jumps():
    # scores grow along the keys, so a row's block max passes its running max by more than
    # the 2^8 margin in later blocks: O is rescaled in TMEM between blocks
    g = torch.Generator(device=DEV).manual_seed(3)
    Sq, Skv = 300, 1000
    q = (torch.randn((1, 2, Sq, 128), generator=g, device=DEV) * 0.25 + 1.0).half()
    ramp = torch.linspace(0.0, 3.0, Skv, device=DEV)[:, None]
    k = ((torch.randn((1, 1, Skv, 128), generator=g, device=DEV) * 0.25 + 1.0) * ramp).half()
    v = torch.randn((1, 1, Skv, 128), generator=g, device=DEV).half()
    _check(q, k, v)


def test_dit_size_slice():
    # 24 heads of 128 over 4352 tokens (the DiT block at 1024 px); query rows sampled
    g = torch.Generator(device=DEV).manual_seed(11)
    q = (torch.randn((1, 24, 4352, 128), generator=g, device=DEV) * 0.5).half()
    k = (torch.randn((1, 24, 4352, 128), generator=g, device=DEV) * 0.5).half()
    v = torch.randn((1, 24, 4352, 128), generator=g, device=DEV).half()
    _check(q, k, v, rows=np.array([0, 1, 255, 256, 2047, 4095, 4351]))


def test_argument_checks():
    q = torch.zeros((1, 3, 8, 64), device=DEV).half()
    k = torch.zeros((1, 2, 8, 64), device=DEV).half()
    with pytest.raises(Bq4Error, match="EINVAL_SHAPE"):
        F.attention(q, k, k)  # 3 query heads on 2 kv heads
    q6 = torch.zeros((1, 2, 8, 6), device=DEV).half()
    k6 = torch.zeros((1, 2, 8, 6), device=DEV).half()
    with pytest.raises(Bq4Error, match="EINVAL_SHAPE"):
        F.attention(q6, k6, k6)  # head_dim not a multiple of 4
    # the fused kernel's limits (32-bit row coordinates, B*Hkv on grid z) are checked before any launch
    qw = torch.zeros((1, 65536, 1, 128), device=DEV).half()
    with pytest.raises(Bq4Error, match="EINVAL_SHAPE"):
        F.attention(qw, qw, qw)  # B*Hkv = 65536
