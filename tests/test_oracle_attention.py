"""CPU: the attention oracle (oracle/bq4_oracle.c orc_attention_f64) pinned to
the reference's own attention test,
crates/burn_boogu/src/model/native_flash.rs:2784-2843.

That test builds deterministic q [1, 4, 3, 120], k and v [1, 2, 5, 120]
(generator native_flash.rs:2697-2710, offsets 2, 7, 11), repeats each kv head
for its two query heads, and takes Burn's `attention` with default options
(no mask, scale 1/sqrt(head_dim)) as the expected result, at max-abs <= 2e-6.
The same inputs and composition are restated here in float32 and the oracle
(which maps query head h to kv head h // 2 itself) must meet that bar.
"""
import numpy as np

import oracle as O

HEAD_DIM = 120  # BOOGU_ATTENTION_HEAD_DIM, native_flash.rs:33


def _deterministic(shape, offset):
    n = int(np.prod(shape))
    idx = np.arange(n, dtype=np.int64)
    return ((((idx + offset) * 19 + 7) % 53) - 26.0).astype(np.float32).reshape(shape) / np.float32(17.0)


def _softmax_attention_f32(q, k, v):
    s = np.einsum("bhid,bhjd->bhij", q, k).astype(np.float32) / np.float32(np.sqrt(q.shape[-1]))
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(-1, keepdims=True)
    return np.einsum("bhij,bhjd->bhid", p, v).astype(np.float32)


def test_oracle_meets_reference_gqa_attention_fixture():
    q = _deterministic([1, 4, 3, HEAD_DIM], 2)
    k = _deterministic([1, 2, 5, HEAD_DIM], 7)
    v = _deterministic([1, 2, 5, HEAD_DIM], 11)
    # key.reshape([1,2,1,5,D]).repeat_dim(2,2).reshape([1,4,5,D]): kv head h // 2
    expected = _softmax_attention_f32(q, np.repeat(k, 2, axis=1), np.repeat(v, 2, axis=1))
    got = O.attention_f64(q, k, v)
    assert np.abs(got - expected).max() <= 2.0e-6


def test_oracle_scale_and_single_key():
    rng = np.random.default_rng(4)
    q = rng.standard_normal((2, 3, 4, 16)).astype(np.float32)
    k = rng.standard_normal((2, 3, 1, 16)).astype(np.float32)
    v = rng.standard_normal((2, 3, 1, 16)).astype(np.float32)
    # one key: every query returns its value row, whatever the scale
    out = O.attention_f64(q, k, v, scale=7.0)
    assert np.allclose(out, np.broadcast_to(v, out.shape), atol=1e-12)
    k2 = rng.standard_normal((2, 3, 6, 16)).astype(np.float32)
    v2 = rng.standard_normal((2, 3, 6, 16)).astype(np.float32)
    a = O.attention_f64(q, k2, v2, scale=0.5)
    b = O.attention_f64(q * 0.5, k2, v2, scale=1.0)
    assert np.abs(a - b).max() < 1e-12
