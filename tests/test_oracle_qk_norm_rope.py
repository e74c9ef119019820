"""CPU: the QK-norm + RoPE oracle (oracle/bq4_oracle.c orc_qk_norm_rope_f64)
pinned to the reference's own test of the fused strict QK-norm/RoPE
preparation, crates/burn_boogu/src/model/native_flash.rs:2897-2960.

That test builds deterministic query/key tensors, gammas and phases (the
generator is native_flash.rs:2697-2710, head_dim 120 from :33), composes the
expected result as `input / sqrt(mean(input^2) + eps) * gamma` followed by the
interleaved-pair rotation, and requires max-abs <= 1e-6.  The same inputs and
composition are restated here in float32 and the oracle must meet that bar.
"""
import numpy as np
import pytest

import oracle as O

HEAD_DIM = 120  # BOOGU_ATTENTION_HEAD_DIM, native_flash.rs:33
EPS = 1.0e-5


def _deterministic(shape, offset):
    # native_flash.rs:2697-2710: ((index + offset) * 19 + 7) % 53, then (v - 26) / 17
    n = int(np.prod(shape))
    idx = np.arange(n, dtype=np.int64)
    return (((idx + offset) * 19 + 7) % 53 - 26.0).astype(np.float32).reshape(shape) / np.float32(17.0)


def _composed_f32(x_bshd, gamma, cos, sin):
    # the test's `normalize` and `rope` closures, in float32 ([batch, seq, heads, dim])
    x = x_bshd.astype(np.float32)
    rms = np.sqrt(np.mean(np.square(x), axis=3, keepdims=True, dtype=np.float32) + np.float32(EPS))
    v = x / rms * gamma[None, None, None, :]
    rot = np.empty_like(v)
    rot[..., 0::2] = -v[..., 1::2]
    rot[..., 1::2] = v[..., 0::2]
    return v * cos[:, :, None, :] + rot * sin[:, :, None, :]


@pytest.mark.parametrize("name,heads,offset,goffset", [("query", 4, 31, 43), ("key", 2, 37, 47)])
def test_oracle_meets_reference_fused_prep_fixture(name, heads, offset, goffset):
    x_bhsd = _deterministic([1, heads, 3, HEAD_DIM], offset)  # [batch, heads, seq, dim]
    gamma = _deterministic([HEAD_DIM], goffset) * np.float32(0.25) + np.float32(1.0)
    phases = ((np.arange(3 * HEAD_DIM) // 2) % 17).astype(np.float32) / np.float32(19.0)
    phase = phases.reshape(1, 3, HEAD_DIM)
    cos, sin = np.cos(phase), np.sin(phase)
    x_bshd = x_bhsd.transpose(0, 2, 1, 3)  # permute([0, 2, 1, 3])
    expected = _composed_f32(x_bshd, gamma, cos, sin).reshape(3, heads * HEAD_DIM)
    got = O.qk_norm_rope_f64(x_bshd.reshape(3, heads * HEAD_DIM), heads, HEAD_DIM, gamma, EPS, cos[0], sin[0])
    max_abs = float(np.abs(got - expected).max())
    assert max_abs <= 1.0e-6, f"{name}: max_abs {max_abs}"


def test_rope_tables_pair_layout():
    # denoiser.rs:992-1032: per axis, each pair's cos/sin repeated for both dims
    ids = np.array([[0, 3, 5], [1, 7, 2]])
    cos, sin = O.rope_tables(ids, [40, 40, 40], 10000.0)
    assert cos.shape == (2, 120) and sin.shape == (2, 120)
    assert np.array_equal(cos[:, 0::2], cos[:, 1::2]) and np.array_equal(sin[:, 0::2], sin[:, 1::2])
    assert np.allclose(cos[0, :40], 1.0) and np.allclose(sin[0, :40], 0.0)  # id 0 on axis 0
    inv = 10000.0 ** (-(2.0 * np.arange(20)) / 40)
    assert np.allclose(cos[1, 80:120:2], np.cos(2 * inv), atol=1e-7)


def test_without_gamma_or_rope_is_plain_rms_norm():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((7, 3 * 64)).astype(np.float32)
    got = O.qk_norm_rope_f64(x, 3, 64, None, EPS)
    xr = x.reshape(7, 3, 64).astype(np.float64)
    ref = (xr / np.sqrt((xr ** 2).mean(-1, keepdims=True) + EPS)).reshape(7, 192)
    assert np.abs(got - ref).max() < 1e-6
