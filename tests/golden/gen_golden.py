"""Generate the committed golden fixtures under tests/golden/.

The reference (Rust) cannot run here, so the fixtures are the reference's own
known-answer inputs -- built from the formulas in its tests -- together with
the outputs of the CPU oracle (oracle/bq4_oracle.c).  tests/test_oracle_golden.py
pins the oracle to the reference's assertions on these inputs; the GPU tests
compare the CUDA path against the stored outputs.

  wave_block128       crates/burn_boogu/src/artifacts.rs:10413-10498
  col_layout_256x128  crates/burn_qwen3_vl/src/artifacts.rs:1877-2049 (f16 source)
  exact_row_4x128     crates/bevy_image/src/browser_boogu/runtime.rs:4511-4545,4729-4777
  random_*            seeded synthetic cases (BASELINE.json distributions)

Run:  python tests/golden/gen_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

import oracle as O  # noqa: E402
from conftest import gen_bias, gen_q4, gen_x  # noqa: E402


def wave_values():
    idx = np.arange(128 * 128, dtype=np.int64)
    a = ((idx * 37 % 509).astype(np.float32) - np.float32(254.0)) / np.float32(1536.0)
    b = ((idx % 128).astype(np.float32) - np.float32(63.5)) / np.float32(8192.0)
    return (a + b).astype(np.float32)


def wave_input():
    i = np.arange(128, dtype=np.int64)
    return (((i * 19 % 97).astype(np.float32) - np.float32(48.0)) / np.float32(128.0)).astype(np.float32)


def col_raw(output_width=256, input_width=128):
    idx = np.arange(output_width * input_width, dtype=np.int64)
    a = ((idx * 37 % 509).astype(np.float32) - np.float32(254.0)) / np.float32(1536.0)
    b = ((idx % input_width).astype(np.float32) - np.float32(63.5)) / np.float32(8192.0)
    return (a + b).astype(np.float32)


def exact_lhs(rows, inner):
    i = np.arange(rows * inner, dtype=np.int64)
    return (((i * 17) % 29).astype(np.float32) - np.float32(14.0)) * np.float32(1.0 / 128.0)


def exact_weight(inner, output):
    i = np.arange(inner * output, dtype=np.int64)
    inp, out = i // output, i % output
    return (((inp + out * 3) % 15).astype(np.float32) - np.float32(7.0)) * np.float32(1.0 / 64.0)


def sequential_f32_matmul(lhs, w, rows, inner, output):
    """q4_probe_reference_matmul: f32 accumulation in k order."""
    res = np.zeros((rows, output), dtype=np.float32)
    for r in range(rows):
        acc = np.zeros(output, dtype=np.float32)
        for k in range(inner):
            acc = (acc + np.float32(lhs[r * inner + k]) * w[k * output:(k + 1) * output]).astype(np.float32)
        res[r] = acc
    return res


RANDOM_CASES = [
    # name, M, K, N, block, layout, act, bias
    ("random_row_b128", 37, 256, 136, 128, O.LAYOUT_ROW, O.ACT_NONE, True),
    ("random_col_b32_gelu", 19, 192, 264, 32, O.LAYOUT_COL, O.ACT_GELU_TANH, True),
    ("random_row_b8_silu", 70, 96, 128, 8, O.LAYOUT_ROW, O.ACT_SILU, False),
]


def main():
    rng = np.random.default_rng(1234)
    out = {}

    v = wave_values()
    w, s = O.quantize_col_block128(v.reshape(128, 128))
    out["wave_block128"] = dict(values=v, input=wave_input(), words=w.reshape(-1), scales=s.reshape(-1))

    raw = col_raw()
    raw_f16 = raw.astype(np.float16).astype(np.float32)  # convert_dtype(DType::F16)
    w, s = O.quantize_col_block128(raw_f16.reshape(256, 128))
    out["col_layout_256x128"] = dict(raw=raw, raw_f16=raw_f16, input=wave_input(), words=w, scales=s)

    lhs = exact_lhs(4, 128)
    wt = exact_weight(128, 128)
    w, s, b = O.quantize_row_up_to128(wt.reshape(128, 128))
    exp = sequential_f32_matmul(lhs, wt, 4, 128, 128)
    out["exact_row_4x128"] = dict(lhs=lhs.reshape(4, 128), weight=wt.reshape(128, 128), words=w, scales=s,
                                  block=np.int32(b), expected=exp)

    for name, M, K, N, blk, lay, act, with_bias in RANDOM_CASES:
        w, s = gen_q4(K, N, blk, lay, rng)
        x = gen_x(M, K, rng)
        bias = gen_bias(N, rng) if with_bias else np.zeros(0, np.float32)
        W = O.unpack(w, s, K, N, blk, lay)
        y = O.linear_f64(x, W, bias if with_bias else None, act)
        out[name] = dict(words=w, scales=s, x=x, bias=bias, y=y,
                         meta=np.array([M, K, N, blk, lay, act, int(with_bias)], np.int64))

    for name, d in out.items():
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **d)
        print("wrote", name)


if __name__ == "__main__":
    main()
