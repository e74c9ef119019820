"""Benchmark of the packed-Q4 linear hot path on B200.

Default workload (the metric's layer-stack config):
the DiT-shaped stack of 24 blocks x {qkv 3072->9216, o 3072->3072 (+bias),
up 3072->12288 (+bias, GELU-tanh), down 12288->3072 (+bias)} Q4 linears,
block 128, M = 4352 tokens, activations renormalised per block.  One step =
one DMD step's pass through the stack.  At N GPUs the stack is
tensor-parallel (column-parallel qkv/up, row-parallel o/down with an NCCL
all-reduce); total work is fixed, so scaling is "strong".

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  `value` = whole-job Q4-linear TFLOP/s with
inputs resident in HBM; `e2e` = the same through the public API with the
step's input copied from pinned host memory and the output read back inside
the timed region.  `--impl reference` times the CPU restatement of the
reference's q_matmul (oracle/, OpenMP on all host cores) on a bounded sample
of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, QKV, MLP, BLOCKS, TOKENS, QBLOCK = 3072, 9216, 12288, 24, 4352, 128
METRIC = "Q4 linear TFLOP/s, DiT layer stack (24 blocks x qkv/o/up/down, M=4352, block 128)"
WORKLOAD = "dit_layer_stack_24x(qkv3072x9216,o3072x3072,up3072x12288+gelu,down12288x3072)_M4352_b128"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--blocks", type=int, default=BLOCKS)
    ap.add_argument("--tokens", type=int, default=TOKENS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--linear", default=None,
                    help="M,K,N[,act[,block]]: time one fused Q4 linear instead of the stack "
                         "(profiling / per-config rows; act 0 none, 1 gelu-tanh)")
    ap.add_argument("--gated", default=None, help="M,K,N: time one fused SiLU-gate linear pair")
    ap.add_argument("--no-rows", action="store_true", help="skip the per-config rows")
    ap.add_argument("--act-dtype", choices=["f16", "f32"], default="f16",
                    help="activations between the stack's linears: f16 (the GEMM operand format, written by "
                         "each epilogue) or f32 (staged by every call)")
    ap.add_argument("--chunks", type=int, default=1, help="token chunks of the stack pipeline (each chunk's "
                                                          "all-reduces overlap the other chunks' GEMMs)")
    ap.add_argument("--sm-budget", type=int, default=0, help="cap the SMs a GEMM occupies (0: all)")
    ap.add_argument("--tp-exchange", choices=["auto", "p2p", "pull", "bcast", "nccl"], default="auto",
                    help="row-parallel exchange at N > 1: p2p (GEMM epilogue writes each row's partial to its "
                         "owner over NVLink peer memory, owner sums + renormalises, f16 all-gather) or nccl "
                         "(f32 all-reduce of the partials); pull: each rank's GEMM writes its partials locally and "
                         "each owner reads its rows from every rank over NVLink; bcast: pull, with each owner "
                         "writing its reduced rows into every rank's activations instead of an all-gather; "
                         "auto = bcast (the fastest measured on B200 at 2 and 4 GPUs; every form checked against "
                         "nccl and the unsharded stack)")
    ap.add_argument("--rows-only", action="store_true", help="print only the per-config rows (1 GPU)")
    ap.add_argument("--config", choices=["stack", "c4"], default="stack",
                    help="c4: BASELINE configs[3], the 1536 px edit projections (M=18432: fused qkv 3072->9216 "
                         "column-sharded, o 3072->3072 row-sharded + all-reduce) at N GPUs, with a parity check "
                         "against the unsharded projections")
    ap.add_argument("--rows", default=None, help="comma-separated row names to run (with --rows-only)")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(1.0)  # let nvidia-smi start sampling before the timed region
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self, start: bool):
        if start:
            self.t_start = time.time()
        else:
            self.t_end = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        t0 = getattr(self, "t_start", 0.0)
        t1 = getattr(self, "t_end", 1e30)
        for ts, ln in self.lines:
            if not (t0 <= ts <= t1 + 0.05):  # samples read during the timed region
                continue
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                sm.append(float(parts[2]))
                smax.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[6:10]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU baseline (oracle)

def host_cores() -> int:
    """Host threads this process may run on (torchrun sets OMP_NUM_THREADS=1,
    so the CPU arms pass this count explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_sample(tokens_sample: int, repeats: int, threads: int = 0):
    """Time the CPU restatement of the reference q_matmul (dequantize + f32
    SGEMM + epilogue, OpenMP) on one block's four linears at `tokens_sample`
    rows, on `threads` host threads (all usable cores when 0).  Returns
    (TFLOP/s, seconds, threads)."""
    import numpy as np

    import oracle as O
    if threads <= 0:
        threads = host_cores()
    rng = np.random.default_rng(0)
    shapes = [(HIDDEN, QKV, 0, False), (HIDDEN, HIDDEN, 0, True), (HIDDEN, MLP, O.ACT_GELU_TANH, True),
              (MLP, HIDDEN, 0, True)]
    ws = []
    for K, N, act, has_bias in shapes:
        words = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.uint64).astype(np.uint32)
        scales = rng.uniform(0.001, 0.02, size=(K // QBLOCK, N)).astype(np.float32)
        bias = (rng.standard_normal(N) * 0.02).astype(np.float32) if has_bias else None
        ws.append((words, scales, K, N, act, bias))
    x = rng.standard_normal((tokens_sample, HIDDEN), dtype=np.float32)
    flops = 0
    t0 = time.perf_counter()
    for _ in range(repeats):
        h = x
        for i, (words, scales, K, N, act, bias) in enumerate(ws):
            inp = h if i != 1 else h[:, -HIDDEN:]
            inp = np.ascontiguousarray(inp)
            h = O.cpu_linear(words, scales, K, N, QBLOCK, O.LAYOUT_ROW, inp, bias, act, threads=threads)
            flops += 2 * tokens_sample * K * N
    dt = time.perf_counter() - t0
    return flops / dt / 1e12, dt, threads


def cpu_config1(repeats: int = 3, threads: int = 0):
    """BASELINE configs[0] on the CPU restatement (the reference's CPU
    linear, crates/burn_boogu/src/model/linear.rs:51-96): x f32 [512, 2560]
    ~N(0,1), signed-int4 weights [2560 -> 9728] in [-8, 7], block 128,
    |U(0.001, 0.02)| scales, bias ~N(0, 0.02).  Returns (TFLOP/s, seconds of
    the median call, threads)."""
    import numpy as np

    import oracle as O
    if threads <= 0:
        threads = host_cores()
    M, K, N = 512, 2560, 9728
    rng = np.random.default_rng(1)
    words = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.uint64).astype(np.uint32)
    scales = rng.uniform(0.001, 0.02, size=(K // QBLOCK, N)).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32)
    O.cpu_linear(words, scales, K, N, QBLOCK, O.LAYOUT_ROW, x, bias, 0, threads=threads)  # warm-up
    ts = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        O.cpu_linear(words, scales, K, N, QBLOCK, O.LAYOUT_ROW, x, bias, 0, threads=threads)
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    return 2 * M * K * N / t / 1e12, t, threads


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import oracle as O
    O.build()
    tokens_sample = 64
    for _ in range(args.warmup):
        cpu_sample(tokens_sample, 1)
    vals, secs = [], 0.0
    for _ in range(args.steps):
        v, dt, thr = cpu_sample(tokens_sample, 1)
        vals.append(v)
        secs += dt
    value = statistics.median(vals)
    flops_step = (2 * TOKENS * (HIDDEN * QKV + HIDDEN * HIDDEN + HIDDEN * MLP + MLP * HIDDEN) * args.blocks)
    flops_sample = 2 * tokens_sample * (HIDDEN * QKV + HIDDEN * HIDDEN + HIDDEN * MLP + MLP * HIDDEN)
    c1_value, c1_s, c1_thr = cpu_config1()
    sample = (f"one block's 4 linears (qkv/o/up+gelu/down, block 128) at {tokens_sample} of {TOKENS} tokens per step; "
              "CPU restatement of the reference q_matmul (oracle/bq4_oracle.c: dequantize + AVX2 SGEMM, OpenMP)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": secs / max(args.steps, 1) * 1e3, "higher_is_better": True, "scaling": "strong",
        "ms_per_step_note": "measured time of one step's sample (see cpu_baseline.sample); the full step "
                            "(all 24 blocks at 4352 tokens) at the same rate is ms_per_full_step_projected",
        "ms_per_full_step_projected": flops_step / (value * 1e12) * 1e3,
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens": TOKENS, "blocks": args.blocks, "sampled_tokens": tokens_sample,
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": thr, "kind": "port", "sample": sample,
                         "sample_gflop": flops_sample / 1e9,
                         "config1": {"value": c1_value, "unit": "TFLOP/s", "ms": c1_s * 1e3, "cores": c1_thr,
                                     "workload": "BASELINE configs[0]: one Q4 linear M=512, K=2560, N=9728, "
                                                 "block 128, bias (median of 3 calls)"}},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference NdArray q_matmul unavailable on this box (Rust toolchain absent); oracle port timed",
    }))


# ------------------------------------------------------------------ per-config rows

# BASELINE configs as single-GPU rows: (name, M, K, N, kind, act); kind
# "linear" = one fused linear (+bias), "gated" = silu(x.Wg+bg)*(x.Wu+bu).
ROWS = [
    ("c1_cpu_linear_512x2560x9728", 512, 2560, 9728, "linear", 0),
    # decode-shaped rows of the text encoder's largest projection (north star: the
    # bandwidth-bound path for few tokens), where HBM is the binding roof
    ("d_decode_1x2560x9728", 1, 2560, 9728, "linear", 0),
    ("d_decode_16x2560x9728", 16, 2560, 9728, "linear", 0),
    ("d_decode_gate_up_silu_16x2560x2x9728", 16, 2560, 9728, "gated", 0),
    ("d_decode_down_16x9728x2560", 16, 9728, 2560, "linear", 0),
    ("c2_text_qo_256x2560x2560", 256, 2560, 2560, "linear", 0),
    ("c2_text_kv_256x2560x512", 256, 2560, 512, "linear", 0),
    ("c2_text_gate_up_silu_256x2560x2x9728", 256, 2560, 9728, "gated", 0),
    ("c2_text_down_256x9728x2560", 256, 9728, 2560, "linear", 0),
    ("c3_dit_up_gelu_4352x3072x12288", 4352, 3072, 12288, "linear", 1),
    ("c3_dit_down_4352x12288x3072", 4352, 12288, 3072, "linear", 0),
    ("c4_edit_qkv_18432x3072x9216", 18432, 3072, 9216, "linear", 0),
    ("c4_edit_o_18432x3072x3072", 18432, 3072, 3072, "linear", 0),
    # next row of the path: the packed-Q4 embedding lookup (q_select + dequantize), 256
    # prompt tokens from a 151936 x 2560 table (rows = table rows, K = row width)
    ("f1_q4_embedding_256_of_151936x2560", 256, 2560, 151936, "select", 0),
    # the row-parallel exchange's two kernels at one rank (the multi-GPU path's
    # GEMM with its row-scatter epilogue writing the owner's receive buffer, then
    # the owner's rank-order sum + RMS renorm into f16 rows), down-projection shape
    ("e_rowscatter_down_1rank_4352x12288x3072", 4352, 12288, 3072, "rowscatter", 0),
    # next row: the DiT qkv projection with QK-norm + RoPE on its q and k heads (24 + 24 + 24
    # heads of 128), fused into the GEMM epilogue; "us_unfused" = linear + two norm passes
    ("f3_qkv_qknorm_rope_4352x3072x9216", 4352, 3072, 9216, "qknorm", 0),
    # the attention that consumes it: 24 heads of 128 over 4352 tokens, f16 q/k/v
    # (M = tokens, K = head_dim, N = heads)
    ("f3_attention_24x4352x4352x128", 4352, 128, 24, "attn", 0),
    # next row: packed-F16 storage (the VAE's weights), kind::tf32.  The reference's own
    # throughput smokes (a 4096^3 matmul; a 512 -> 512 3x3 conv at 64 x 64) and the
    # largest FLUX-VAE decoder conv (128 -> 128 channels, 3x3, 1024 x 1024).
    # (name, M, K, N, kind, act); conv rows: M = output positions, K = in * 9, N = out.
    ("f4_f16_matmul_4096x4096x4096", 4096, 4096, 4096, "f16mm", 0),
    ("f4_f16_conv3x3_512to512_64x64", 64 * 64, 512 * 9, 512, "f16conv", 0),
    ("f4_vae_conv3x3_128to128_1024x1024", 1024 * 1024, 128 * 9, 128, "f16conv", 0),
]


def _graph_time(dev, items, call):
    """Device time of one call: every item's call captured once in a CUDA
    graph, the graph replayed, total / (replays x items)."""
    import torch
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for it in items:
            call(it)  # warm-up on the capture stream (workspace, attributes)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for it in items:
            call(it)
    graph.replay()
    torch.cuda.synchronize(dev)
    reps = max(3, int(40 // len(items)))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    del graph
    return e0.elapsed_time(e1) * 1e-3 / (reps * len(items))


def config_rows(dev, peaks, names=None):
    """Device time of each BASELINE config shape, one GPU.

    Each call reads its own weight/activation/output set; the sets rotate so
    that together they exceed twice the 126 MB L2 (every call starts cold).
    The calls are captured in a CUDA graph and replayed, so the time is the
    device time of the two kernels of a call (activation staging + GEMM),
    without host submission overhead.  Roofline: t* = max(algorithmic bytes /
    measured copy bandwidth, FLOPs / measured bf16 burst peak)."""
    import torch

    from burn_image_b200 import _lib as L
    from burn_image_b200 import q4, tp
    hbm = peaks.get("hbm_gbs", 6650.0)
    tfl = peaks.get("bf16_tflops", 1590.0)
    out = {}
    for name, M, K, N, kind, act in ROWS:
        if names and name not in names:
            continue
        if kind == "select":
            out[name] = _select_row(dev, M, K, N, hbm)
            continue
        if kind in ("f16mm", "f16conv"):
            out[name] = _f16_row(dev, kind, M, K, N, hbm, tfl)
            continue
        if kind == "attn":
            out[name] = _attn_row(dev, M, K, N, hbm, tfl)
            continue
        if kind == "rowscatter":
            out[name] = _rowscatter_row(dev, M, K, N, hbm, tfl)
            continue
        nw = 2 if kind == "gated" else 1
        wbytes = nw * (N * K // 2 + N * K // QBLOCK * 4)
        set_bytes = wbytes + M * K * 4 + M * N * 4
        sets = max(2, min(64, int(2 * 126e6 // set_bytes) + 1))
        g = torch.Generator(device=dev).manual_seed(11)
        items = []
        hd = 128
        heads = N // hd // 3  # q, k and v heads (qknorm rows)
        for _ in range(sets):
            ws = [q4.PreparedQ4Weight(*tp._random_packed(K, N, QBLOCK, g, dev), K, N, QBLOCK, L.LAYOUT_ROW, dev)
                  for _ in range(nw)]
            bias = [torch.randn(N, generator=g, device=dev) * 0.02 for _ in range(nw)]
            x = torch.randn((M, K), generator=g, device=dev)
            y = torch.empty((M, N), device=dev)
            extra = None
            if kind == "qknorm":
                phase = torch.rand((M, hd), generator=g, device=dev) * 6.0
                extra = (torch.rand(hd, generator=g, device=dev) + 0.5, torch.rand(hd, generator=g, device=dev) + 0.5,
                         torch.cos(phase), torch.sin(phase))
            items.append((ws, bias, x, y, extra))

        def call(it):
            ws, bias, x, y, extra = it
            if nw == 2:
                q4.linear_gated(ws[0], ws[1], x, bias[0], bias[1], out=y)
            elif kind == "qknorm":
                gq, gk, cs, sn = extra
                ws[0].linear_qk_norm_rope(x, heads, heads, hd, bias[0], gq, gk, 1e-5, cs, sn, out=y)
            else:
                ws[0].linear(x, bias[0], act, out=y)

        def call_unfused(it):
            ws, bias, x, y, (gq, gk, cs, sn) = it
            ws[0].linear(x, bias[0], out=y)
            q4.qk_norm_rope(y[:, :heads * hd], heads, hd, gq, 1e-5, cs, sn, out=y[:, :heads * hd])
            q4.qk_norm_rope(y[:, heads * hd:2 * heads * hd], heads, hd, gk, 1e-5, cs, sn,
                            out=y[:, heads * hd:2 * heads * hd])

        def call_norm(it):  # one standalone pass over the q heads, in place (HBM-bound)
            ws, bias, x, y, (gq, gk, cs, sn) = it
            q4.qk_norm_rope(y[:, :heads * hd], heads, hd, gq, 1e-5, cs, sn, out=y[:, :heads * hd])

        t = _graph_time(dev, items, call)
        t_gemm = None
        if M <= 256 and kind in ("linear", "gated"):
            # the same calls on the tcgen05 GEMM (the few-token kernel switched off)
            os.environ["BQ4_NO_SKINNY"] = "1"
            try:
                t_gemm = _graph_time(dev, items, call)
            finally:
                os.environ.pop("BQ4_NO_SKINNY", None)
        t_unfused = _graph_time(dev, items, call_unfused) if kind == "qknorm" else None
        t_norm = _graph_time(dev, items, call_norm) if kind == "qknorm" else None
        q4.poll_device_error()
        flops = 2 * M * K * N * nw
        nbytes = wbytes + M * K * 4 + M * N * 4 + nw * N * 4 + (2 * M * hd * 4 if kind == "qknorm" else 0)
        t_star = max(nbytes / (hbm * 1e9), flops / (tfl * 1e12))
        bound = "hbm" if nbytes / (hbm * 1e9) > flops / (tfl * 1e12) else "tensor"
        out[name] = {"us": t * 1e6, "tflops": flops / t / 1e12, "gbs": nbytes / t / 1e9, "bound": bound,
                     "t_star_us": t_star * 1e6, "frac": t_star / t, "sets": sets,
                     "kernel": "few-token (mma.sync)" if ws_plan_skinny(items[0][0][0], M, nw) else "tcgen05 GEMM"}
        if t_gemm is not None:
            out[name]["us_tcgen05_gemm"] = t_gemm * 1e6
        if t_unfused is not None:
            # the standalone pass: reads and writes M x heads x 128 f32 and reads the two tables
            norm_bytes = 2 * M * heads * hd * 4 + 2 * M * hd * 4
            out[name]["us_unfused"] = t_unfused * 1e6
            out[name]["norm_pass"] = {"us": t_norm * 1e6, "gbs": norm_bytes / t_norm / 1e9,
                                      "frac_hbm": norm_bytes / t_norm / 1e9 / hbm}
        del items
        torch.cuda.empty_cache()
    return out


def _rowscatter_row(dev, M, K, N, hbm, tfl):
    """One rank of the row-parallel peer exchange: bq4_linear_rowscatter
    (f16 activations, f32 partial rows written by the epilogue into the
    receive buffer) and bq4_reduce_slices (sum in rank order, RMS renorm,
    f16 rows), graph-replayed over rotating sets; times of the two and of
    the plain f16-in / f16-out linear of the same shape for comparison."""
    import ctypes

    import torch

    from burn_image_b200 import _lib as L
    from burn_image_b200 import q4, tp
    g = torch.Generator(device=dev).manual_seed(17)
    lib = L.lib()
    sets = 2
    items = []
    for _ in range(sets):
        pw = q4.PreparedQ4Weight(*tp._random_packed(K, N, QBLOCK, g, dev), K, N, QBLOCK, L.LAYOUT_ROW, dev)
        x = torch.randn((M, K), generator=g, device=dev).half()
        recv = torch.empty((M, N), device=dev)
        y16 = torch.empty((M, N), dtype=torch.float16, device=dev)
        items.append((pw, x, recv, y16))
    n = ctypes.c_size_t()
    L.check(lib.bq4_linear_ex_workspace_size(items[0][0].handle, M, L.DTYPE_F16, ctypes.byref(n)))
    ws = q4.Workspace.get(dev, max(n.value, 256))

    def stream():
        return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def scatter(it):
        pw, x, recv, _ = it
        targets = (ctypes.c_void_p * 1)(ctypes.c_void_p(recv.data_ptr()))
        L.check(lib.bq4_linear_rowscatter(pw.handle, ctypes.c_void_p(x.data_ptr()), L.DTYPE_F16, M, K, None,
                                          L.ACT_NONE, targets, 1, 0, N, ctypes.c_void_p(ws.data_ptr()),
                                          ws.numel(), stream()))

    def reduce(it):
        _, _, recv, y16 = it
        L.check(lib.bq4_reduce_slices(ctypes.c_void_p(recv.data_ptr()), 1, M, N, N, 1, ctypes.c_float(1e-6),
                                      ctypes.c_void_p(y16.data_ptr()), L.DTYPE_F16, N, stream()))

    def plain(it):
        pw, x, _, y16 = it
        pw.linear_ex(x, out=y16)

    t_sc = _graph_time(dev, items, scatter)
    t_red = _graph_time(dev, items, reduce)
    t_plain = _graph_time(dev, items, plain)
    q4.poll_device_error()
    flops = 2 * M * K * N
    red_bytes = M * N * 4 + M * N * 2
    t_star = max((K * N // 2 + K // QBLOCK * N * 4 + M * K * 2 + M * N * 4) / (hbm * 1e9), flops / (tfl * 1e12))
    return {"us": t_sc * 1e6, "tflops": flops / t_sc / 1e12, "bound": "tensor", "t_star_us": t_star * 1e6,
            "frac": t_star / t_sc, "sets": sets, "kernel": "tcgen05 GEMM, row-scatter epilogue",
            "us_plain_f16_linear": t_plain * 1e6,
            "reduce_slices": {"us": t_red * 1e6, "gbs": red_bytes / t_red / 1e9,
                              "frac_hbm": red_bytes / t_red / 1e9 / hbm}}


def ws_plan_skinny(pw, M, nw):
    """1 when the planner sends this call to the few-token kernel."""
    return pw.plan_info(M, gated=nw == 2)["skinny"] == 1


def _select_row(dev, n, cols, rows, hbm):
    """Embedding lookup row: n random ids into a packed table of `rows` x
    `cols` (block 128, PackedU32(0)); graph-replayed over 64 id sets and
    outputs, whose footprint exceeds L2, so the selected rows come from HBM."""
    import torch

    from burn_image_b200 import q4
    g = torch.Generator(device=dev).manual_seed(13)
    values = torch.randint(-2 ** 31, 2 ** 31 - 1, (rows, cols // 8), generator=g, device=dev,
                           dtype=torch.int64).to(torch.int32)
    scales = torch.rand((rows, cols // QBLOCK), generator=g, device=dev) * 0.019 + 0.001
    qt = q4.QuantizedTensor(values, scales, (rows, cols), q4.QuantScheme(store_packed_dim=0, level=(QBLOCK,)),
                            transposed_view=False)
    sets = 64  # selected rows + outputs of one replay cycle: ~190 MB, more than the 126 MB L2
    ids = [torch.randint(0, rows, (n,), generator=g, device=dev, dtype=torch.int64) for _ in range(sets)]
    outs = [torch.empty((n, cols), device=dev) for _ in range(sets)]
    lib = q4.L.lib()

    def call(i, stream):
        q4.check(lib.bq4_q_select_rows_dequant(values.data_ptr(), scales.data_ptr(), rows, cols, QBLOCK,
                                               ids[i].data_ptr(), 1, n, outs[i].data_ptr(), stream))

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(sets):
            call(i, side.cuda_stream)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(sets):
            call(i, side.cuda_stream)
    graph.replay()
    torch.cuda.synchronize(dev)
    reps = 5
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    q4.poll_device_error()
    t = e0.elapsed_time(e1) * 1e-3 / (reps * sets)
    nbytes = n * (cols // 2 + cols // QBLOCK * 4) + n * cols * 4 + n * 8
    t_star = nbytes / (hbm * 1e9)
    del graph
    return {"us": t * 1e6, "tflops": 0.0, "gbs": nbytes / t / 1e9, "bound": "hbm", "t_star_us": t_star * 1e6,
            "frac": t_star / t, "sets": sets}


def _attn_cpu_arm(S, D, rows=256):
    """The oracle's attention (f64, all host threads) on one head: `rows`
    query rows against all S keys; TFLOP/s of the 4 rows S D FLOPs."""
    import time

    import numpy as np

    import oracle as O
    rng = np.random.default_rng(5)
    rows = min(rows, S)
    q = (rng.standard_normal((1, 1, rows, D)) * 0.5).astype(np.float16).astype(np.float32)
    k = (rng.standard_normal((1, 1, S, D)) * 0.5).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((1, 1, S, D)).astype(np.float16).astype(np.float32)
    O.attention_f64(q[:, :, :8], k, v)
    t0 = time.perf_counter()
    O.attention_f64(q, k, v)
    dt = time.perf_counter() - t0
    return {"tflops": 4.0 * rows * S * D / dt / 1e12, "cores": O.cpu_threads(), "kind": "port",
            "sample": f"1 head, {rows} of {S} query rows"}


def _attn_row(dev, S, D, H, hbm, tfl):
    """Attention row: softmax(q k^T / sqrt(D)) v over H heads of S tokens,
    f16 q/k/v, f32 out, graph-replayed on two input sets.  head_dim 128 runs
    the fused kernel (f16 MMAs): roofline = the measured bf16 burst peak for
    the 4 S^2 D H FLOPs against q, k, v read once and out written once.  It
    also needs S^2 H exponentials, which bound it before the tensor core
    does.  cpu: the oracle's attention on a one-head sample."""
    import torch

    from burn_image_b200 import f16 as F
    from burn_image_b200 import q4
    g = torch.Generator(device=dev).manual_seed(19)
    items = []
    for _ in range(2):
        q = (torch.randn((1, H, S, D), generator=g, device=dev) * 0.5).half()
        k = (torch.randn((1, H, S, D), generator=g, device=dev) * 0.5).half()
        v = torch.randn((1, H, S, D), generator=g, device=dev).half()
        items.append((q, k, v, torch.empty((1, H, S, D), device=dev)))

    def call(it):
        F.attention(it[0], it[1], it[2], out=it[3])

    t = _graph_time(dev, items, call)
    q4.poll_device_error()
    flops = 4.0 * H * S * S * D
    nbytes = 3 * H * S * D * 2 + H * S * D * 4
    t_star = max(nbytes / (hbm * 1e9), flops / (tfl * 1e12))
    del items
    torch.cuda.empty_cache()
    row = {"us": t * 1e6, "tflops": flops / t / 1e12, "gbs": nbytes / t / 1e9, "bound": "tensor",
           "t_star_us": t_star * 1e6, "frac": t_star / t, "peak_tflops": tfl, "kernel": "fused (f16 MMA)",
           "exp_per_s": H * S * S / t, "sets": 2}
    try:
        row["cpu"] = _attn_cpu_arm(S, D)
    except Exception as e:  # noqa: BLE001 -- the CPU arm is informational
        row["cpu"] = {"tflops": None, "sample": f"failed: {e}"}
    return row


def _f16_row(dev, kind, M, K, N, hbm, tfl):
    """Packed-F16 rows (kind::tf32): the prepared-weight matmul, or the whole
    bq4_conv2d call (NCHW staging + implicit GEMM) on a square image of
    sqrt(M) x sqrt(M) with padding 1.  Graph-replayed over enough sets that
    each call starts cold.  Roofline: tf32 at half the measured bf16 burst
    peak (the nominal dense tf32 : bf16 ratio) against the algorithmic HBM
    bytes: f32 input read, f16 weights read once, f32 output written (conv:
    plus the staged copy written and read).  cpu: the oracle's f32 arm on all
    host threads (rhs widened once, blocked SGEMM; the conv as im2col blocks),
    over a sample of the rows."""
    import math
    import time

    import numpy as np
    import torch

    import oracle as O
    from burn_image_b200 import f16 as F
    from burn_image_b200 import q4
    g = torch.Generator(device=dev).manual_seed(17)
    if kind == "f16mm":
        set_bytes = M * K * 4 + K * N * 4 + M * N * 4
    else:
        S = int(math.isqrt(M))
        cin, cout = K // 9, N
        set_bytes = M * cin * 4 * 2 + M * cout * 4 + K * N * 4
    sets = max(2, min(16, int(2 * 126e6 // set_bytes) + 1))
    items = []
    for _ in range(sets):
        if kind == "f16mm":
            w = (torch.randn((N, K), generator=g, device=dev) * K ** -0.5).half()
            items.append((F.PreparedF16Weight(w.t()), torch.randn((M, K), generator=g, device=dev),
                          torch.empty((M, N), device=dev)))
        else:
            w = (torch.randn((cout, cin, 3, 3), generator=g, device=dev) * K ** -0.5).half()
            items.append((F.PreparedF16ConvWeight(w), torch.randn((1, cin, S, S), generator=g, device=dev),
                          torch.empty((1, cout, S, S), device=dev), torch.randn(cout, generator=g, device=dev)))
    opt = F.ConvOptions((1, 1), (1, 1), (1, 1), 1)

    def call(it):
        if kind == "f16mm":
            it[0].linear(it[1], out=it[2])
        else:
            it[0].conv2d(it[1], it[3], opt, out=it[2])

    t = _graph_time(dev, items, call)
    q4.poll_device_error()
    flops = 2.0 * M * K * N
    if kind == "f16mm":
        nbytes = M * K * 4 + K * N * 2 + M * N * 4
    else:
        hp = (S + 2) ** 2
        cp = (cin + 31) // 32 * 32
        nbytes = M * cin * 4 + 2 * hp * cp * 4 + K * N * 2 + M * cout * 4 + cout * 4
    tf32 = tfl / 2.0
    t_star = max(nbytes / (hbm * 1e9), flops / (tf32 * 1e12))
    row = {"us": t * 1e6, "tflops": flops / t / 1e12, "gbs": nbytes / t / 1e9,
           "bound": "tensor" if flops / (tf32 * 1e12) >= nbytes / (hbm * 1e9) else "hbm",
           "t_star_us": t_star * 1e6, "frac": t_star / t, "peak_tf32_tflops": tf32, "sets": sets}
    del items
    torch.cuda.empty_cache()
    # CPU arm on a row sample (about a second of work)
    try:
        rng = np.random.default_rng(3)
        if kind == "f16mm":
            rows = min(M, 512)
            x = rng.standard_normal((rows, K)).astype(np.float32)
            wb = (rng.standard_normal((N, K)) * K ** -0.5).astype(np.float16).view(np.uint16)
            O.cpu_f16_matmul(x[:16], wb, K, N, 1, K)
            t0 = time.perf_counter()
            O.cpu_f16_matmul(x, wb, K, N, 1, K)
            dt = time.perf_counter() - t0
            cflops, sample = 2.0 * rows * K * N, f"{rows} of {M} rows"
        else:
            hs = min(S, max(8, int(4096 // S)))
            x = rng.standard_normal((1, cin, hs, S)).astype(np.float32)
            wb = (rng.standard_normal((cout, cin, 3, 3)) * K ** -0.5).astype(np.float16).view(np.uint16)
            t0 = time.perf_counter()
            O.cpu_f16_conv2d(x, wb, None, (1, 1), (1, 1))
            dt = time.perf_counter() - t0
            cflops, sample = 2.0 * hs * S * K * N, f"{hs} of {S} image rows"
        row["cpu"] = {"tflops": cflops / dt / 1e12, "cores": O.cpu_threads(), "kind": "port", "sample": sample}
    except Exception as e:  # noqa: BLE001 -- the CPU arm is informational
        row["cpu"] = {"tflops": None, "sample": f"failed: {e}"}
    return row


# ------------------------------------------------------------------ GPU arm

def run_ours(args):
    import torch
    import torch.distributed as dist

    from burn_image_b200 import _lib as L
    from burn_image_b200 import tp

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = L.lib()

    import torch as _t
    act_dtype = _t.float16 if args.act_dtype == "f16" else _t.float32
    chunks = max(1, args.chunks)
    if args.sm_budget > 0:
        from burn_image_b200 import q4 as _q
        _q.set_sm_budget(args.sm_budget)
    exchange = args.tp_exchange
    if exchange == "auto":
        # measured on B200 (stack, TFLOP/s, push / pull / bcast): 2 GPUs 1491-1531 / 1451-1475 /
        # 1570-1587; 4 GPUs 1671 / 1683-1691 / 1832; 8 GPUs 1762 / 1788 / (not run: same code path)
        exchange = "bcast"
    if not (world > 1 and args.act_dtype == "f16" and chunks == 1):
        exchange = "nccl"
    stack = tp.DiTQ4Stack(args.blocks, HIDDEN, QKV, MLP, dev, seed=1, block=QBLOCK, group=group,
                          act_dtype=act_dtype, chunks=chunks, exchange=exchange)
    M = args.tokens
    g = torch.Generator(device=dev).manual_seed(42)
    x0 = torch.randn((M, HIDDEN), generator=g, device=dev)
    flops_step = stack.flops_per_token() * M
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # warm-up
    for _ in range(args.warmup):
        stack.forward(x0)
    barrier()

    # ---- timed region: inputs resident in HBM
    events = []

    def on_linear(name, start):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        if start:
            events.append([name, ev, None])
        else:
            events[-1][2] = ev

    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    lib.bq4_launch_count_reset()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    clocks.mark(True)
    torch.cuda.nvtx.range_push("timed")
    t_start.record(stream)
    for _ in range(args.steps):
        y = stack.forward(x0)
    t_end.record(stream)
    torch.cuda.nvtx.range_pop()
    barrier()
    clocks.mark(False)
    launches = int(lib.bq4_launch_count())
    clk = clocks.stop()
    elapsed_ms = t_start.elapsed_time(t_end)
    t = torch.tensor([elapsed_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = t.item()
    ms_step = elapsed_ms / args.steps
    value = flops_step / (ms_step * 1e-3) / 1e12

    # ---- roofline: a separate pass with CUDA events around every linear call
    # (staging, if any, + GEMM), local rank; kept out of the timed region
    for _ in range(args.steps):
        stack.forward(x0, on_linear)
    barrier()
    per = {}
    for name, a, b in events:
        per.setdefault(name, []).append(a.elapsed_time(b))
    lin_ms = sum(sum(v) for v in per.values())
    lin_flops = flops_step * args.steps / world  # this rank's share
    achieved_tflops = lin_flops / (lin_ms * 1e-3) / 1e12

    # ---- the same stack with exact-weight numerics (scale on the f32 accumulator)
    from burn_image_b200 import q4 as _q4
    _q4.set_numerics(L.NUMERICS_EXACT)
    for _ in range(2):
        stack.forward(x0)
    barrier()
    x_start = torch.cuda.Event(enable_timing=True)
    x_end = torch.cuda.Event(enable_timing=True)
    x_start.record(stream)
    for _ in range(args.steps):
        stack.forward(x0)
    x_end.record(stream)
    barrier()
    _q4.set_numerics(L.NUMERICS_AUTO)
    t = torch.tensor([x_start.elapsed_time(x_end)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    value_exact = flops_step / (t.item() / args.steps * 1e-3) / 1e12

    # ---- token-parallel alternative (N > 1): every rank runs the unsharded
    # stack on its M/N tokens, no collective; same metric, max over ranks
    value_tokens = None
    if world > 1:
        local = tp.DiTQ4Stack(args.blocks, HIDDEN, QKV, MLP, dev, seed=1, block=QBLOCK, group=tp.LOCAL,
                              act_dtype=act_dtype, chunks=1)
        a0, a1 = M * rank // world, M * (rank + 1) // world
        xl = x0[a0:a1]
        for _ in range(args.warmup):
            local.forward(xl)
        barrier()
        l_start = torch.cuda.Event(enable_timing=True)
        l_end = torch.cuda.Event(enable_timing=True)
        l_start.record(stream)
        for _ in range(args.steps):
            local.forward(xl)
        l_end.record(stream)
        barrier()
        t = torch.tensor([l_start.elapsed_time(l_end)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        value_tokens = flops_step / (t.item() / args.steps * 1e-3) / 1e12
        del local

    # ---- multi-GPU correctness: the sharded stack against the unsharded one
    # (every rank runs both on the same input; 2 blocks, same weights)
    tp_parity = None
    if world > 1:
        nb = 2
        sh = tp.DiTQ4Stack(nb, HIDDEN, QKV, MLP, dev, seed=7, block=QBLOCK, group=group, act_dtype=act_dtype,
                           chunks=1, exchange=exchange)
        un = tp.DiTQ4Stack(nb, HIDDEN, QKV, MLP, dev, seed=7, block=QBLOCK, group=tp.LOCAL, act_dtype=act_dtype,
                           chunks=1)
        ys = sh.forward(x0).clone()
        yu = un.forward(x0).clone()
        barrier()
        d = (ys.double() - yu.double())
        rel = (torch.linalg.norm(d) / torch.linalg.norm(yu.double())).item()
        mx = torch.tensor([rel, d.abs().max().item()], device=dev, dtype=torch.float64)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tp_parity = {"blocks": nb, "rel_frob": mx[0].item(), "max_abs": mx[1].item(), "bar": 5e-3,
                     "ok": bool(mx[0].item() <= 5e-3),
                     "what": "sharded stack (this run's exchange) vs the unsharded stack on every rank, same "
                             "weights and input; max over ranks"}
        sh.close()
        del sh, un

    # ---- e2e: through the public API with host buffers.  Every step copies its
    # input from pinned host memory and reads its output back; the copies run
    # on a copy stream, double-buffered, so step i+1's upload and step i's
    # read-back overlap step i+1's compute (the timed region still holds all
    # of them: it ends when the last read-back has landed).
    x_host = x0.cpu().pin_memory()
    y_host = torch.empty((M, HIDDEN), dtype=torch.float32).pin_memory()
    xd = [torch.empty_like(x0) for _ in range(2)]
    yd = [torch.empty((M, HIDDEN), dtype=torch.float32, device=dev) for _ in range(2)]
    copy = torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready = [ev(), ev()]
    in_free = [ev(), ev()]
    out_ready = [ev(), ev()]
    out_free = [ev(), ev()]
    for e in in_free + out_free:
        e.record(stream)
    barrier()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    copy.wait_stream(stream)
    with torch.cuda.stream(copy):
        xd[0].copy_(x_host, non_blocking=True)
        in_ready[0].record(copy)
    for i in range(args.steps):
        b = i % 2
        if i + 1 < args.steps:  # upload the next step's input
            with torch.cuda.stream(copy):
                copy.wait_event(in_free[1 - b])
                xd[1 - b].copy_(x_host, non_blocking=True)
                in_ready[1 - b].record(copy)
        stream.wait_event(in_ready[b])
        stream.wait_event(out_free[b])
        stack.forward(xd[b], out=yd[b])
        in_free[b].record(stream)
        out_ready[b].record(stream)
        with torch.cuda.stream(copy):  # read this step's output back
            copy.wait_event(out_ready[b])
            y_host.copy_(yd[b], non_blocking=True)
            out_free[b].record(copy)
    stream.wait_stream(copy)
    e_end.record(stream)
    barrier()
    e_ms = e_start.elapsed_time(e_end)
    t = torch.tensor([e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = flops_step / (t.item() / args.steps * 1e-3) / 1e12
    assert torch.isfinite(y_host).all(), "non-finite output"

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    # The stack's linears are timed in a step of ~19 ms at the full SM clock
    # (the bench's clock samples), so the denominator is the burst bf16 peak;
    # the sustained peak was measured at 1380 MHz under the power cap.
    peak = peaks.get("bf16_tflops")
    peak_src = "measured burst bf16 (MEASURED_PEAKS.json)"
    if peak is None:
        peak, peak_src = 1590.0, "fallback burst"
    # algorithmic bytes of one GEMM launch, mean over a block's four: f16 activations in and
    # out (chained), Q4 nibbles + f32 scales, f32 bias (this rank's shard)
    P = world
    lin = [(TOKENS, HIDDEN, QKV // P, 0), (TOKENS, HIDDEN // P, HIDDEN, 1), (TOKENS, HIDDEN, MLP // P, 1),
           (TOKENS, MLP // P, HIDDEN, 1)]
    alg_bytes = sum(m * k * 2 + k * n // 2 + k // QBLOCK * n * 4 + m * n * 2 + b * n * 4 for m, k, n, b in lin) / 4
    traffic = None
    try:
        tj = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
        traffic = tj.get(WORKLOAD if world == 1 else f"{WORKLOAD}_tp{world}")
    except Exception:
        pass

    rows = None
    if rank == 0 and world == 1 and not args.no_rows:
        rows = config_rows(dev, peaks)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            import oracle as O
            O.build()
            v, dt, thr = cpu_sample(64, 2)
            c1_value, c1_s, c1_thr = cpu_config1()
            cpu = {"value": v, "unit": "TFLOP/s", "cores": thr, "kind": "port",
                   "sample": f"one block's 4 linears at 64 of {M} tokens, x2 ({dt:.1f} s); CPU restatement of the "
                             "reference q_matmul (dequantize + AVX2 SGEMM, OpenMP)",
                   "config1": {"value": c1_value, "unit": "TFLOP/s", "ms": c1_s * 1e3, "cores": c1_thr,
                               "workload": "BASELINE configs[0]: one Q4 linear M=512, K=2560, N=9728, block 128, "
                                           "bias (median of 3 calls)"}}
        except Exception as e:  # pragma: no cover
            cpu = {"value": None, "unit": "TFLOP/s", "cores": 0, "kind": "port", "sample": f"failed: {e}"}

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 operands, f32 accumulate (Q4 weights)", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens": M, "blocks": args.blocks, "block": QBLOCK,
                       "parallelism": f"tp{world}" if world > 1 else "single",
                       "activations": ("f16 between linears (written by each epilogue, read in place)"
                                       if args.act_dtype == "f16" else "f32 between linears"),
                       "token_chunks": chunks, "sm_budget": args.sm_budget or None,
                       "tp_exchange": exchange if world > 1 else None,
                       "l2": "inputs larger than L2 (1.44 GB of Q4 weights streamed per step)"},
            "roofline": {"bound": "tensor", "achieved": achieved_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved_tflops / peak, "traffic": traffic,
                         "algorithmic_bytes_per_gemm_launch": alg_bytes,
                         "traffic_over_algorithmic": (traffic / alg_bytes) if traffic else None,
                         "peak_source": peak_src,

                         "kernel": "q4_gemm_ws_kernel (+ activation staging where a call has f32 input), CUDA "
                                   "events around every linear call in a separate pass, rank 0"},
            "numerics": "auto: f16(q*scale) staging (the reference kernel's) at this M; "
                        "value_exact = the same stack with q exact and the scale on the f32 accumulator",
            "value_exact": value_exact,
            "per_linear_ms": {k: sum(v) / len(v) for k, v in per.items()},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": M * HIDDEN * 4,
                    "d2h_bytes_per_step": M * HIDDEN * 4},
            "gpu_launches": launches,
            "clocks": clk,
            "cpu_baseline": cpu,
            "rows": rows,
            "value_token_parallel": value_tokens,
            "tp_parity": tp_parity,
            "token_parallel": None if value_tokens is None else (
                "the alternative to tensor parallelism: each GPU runs the unsharded stack on M/N tokens, no "
                "collective; same metric and FLOPs, max over ranks"),
        }
        print(json.dumps(out))
    if world > 1:
        stack.close()
        dist.barrier()
        dist.destroy_process_group()


def run_c4(args):
    """per step, the fused qkv projection (column-parallel:
    each rank its 9216/N output features) and the o projection (row-parallel:
    each rank its 3072/N input features, the rank's v columns of the qkv
    output, then an all-reduce of the f32 partials), M = 18432 f32 tokens.
    Attention is not on the Q4 path, so the o projection reads the v section
    of the qkv output directly.  FLOPs per step = 2 M 3072 (9216 + 3072)."""
    import torch
    import torch.distributed as dist

    from burn_image_b200 import _lib as L
    from burn_image_b200 import q4, tp

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    M, H, QN = 18432, HIDDEN, QKV
    g = torch.Generator(device=dev).manual_seed(4)
    wq, sq = tp._random_packed(H, QN, QBLOCK, g, dev)
    wo, so = tp._random_packed(H, H, QBLOCK, g, dev)
    bo = torch.randn(H, generator=g, device=dev) * 0.02
    x = torch.randn((M, H), generator=g, device=dev)
    if world > 1:
        perm = tp._qkv_rank_order(H, QN, world, dev)
        wq_s, sq_s = wq[:, perm].contiguous(), sq[:, perm].contiguous()
    else:
        wq_s, sq_s = wq, sq
    qkv = tp.ColumnParallelQ4Linear(wq_s, sq_s, H, QN, QBLOCK, L.LAYOUT_ROW, dev, group=group)
    o = tp.RowParallelQ4Linear(wo, so, H, H, QBLOCK, L.LAYOUT_ROW, dev, bo, group=group)
    qn_l, h_l = QN // world, H // world
    t = torch.empty((M, qn_l), device=dev)
    y = torch.empty((M, H), device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        qkv.forward(x, out=t)
        o.forward(t[:, qn_l - h_l:], out=y)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.mark(True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    clocks.mark(False)
    clk = clocks.stop()
    tt = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = tt.item() / args.steps
    flops = 2 * M * H * (QN + H)
    # algorithmic bytes per step and rank: x f32 in, the Q4 shards, qkv f32 out, o's
    # v-slice in and f32 partial out (the all-reduce traffic is reported apart)
    nbytes = (M * H * 4 + H * qn_l // 2 + H // QBLOCK * qn_l * 4 + M * qn_l * 4 + M * h_l * 4 + h_l * H // 2 +
              h_l // QBLOCK * H * 4 + M * H * 4)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    tfl = peaks.get("bf16_tflops", 1590.0)
    # parity: the unsharded projections of the same weights and input, on every rank
    ref_q = q4.PreparedQ4Weight(wq, sq, H, QN, QBLOCK, L.LAYOUT_ROW, dev)
    ref_o = q4.PreparedQ4Weight(wo, so, H, H, QBLOCK, L.LAYOUT_ROW, dev)
    tr = ref_q.linear(x)
    yr = ref_o.linear(tr[:, QN - H:], bo)
    step()
    barrier()
    d = y.double() - yr.double()
    par = torch.tensor([(torch.linalg.norm(d) / torch.linalg.norm(yr.double())).item(), d.abs().max().item()],
                       device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(par, op=dist.ReduceOp.MAX)
    if rank == 0:
        value = flops / (ms * 1e-3) / 1e12
        print(json.dumps({
            "metric": "Q4 linear TFLOP/s, 1536 px edit projections (fused qkv + o, M=18432)", "value": value,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16 operands, f32 accumulate (Q4 weights)", "data": "synthetic",
            "config": {"workload": "c4_edit_qkv18432x3072x9216_colTP+o18432x3072x3072_rowTP+allreduce_b128",
                       "parallelism": f"tp{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2 (x 226 MB f32)"},
            "gbs_per_rank": nbytes / (ms * 1e-3) / 1e9,
            "allreduce_bytes_per_step": M * H * 4 if world > 1 else 0,
            "roofline": {"bound": "tensor", "achieved_per_gpu": value / world, "peak": tfl, "unit": "TFLOP/s",
                         "frac": value / world / tfl, "peak_source": "measured burst bf16 (MEASURED_PEAKS.json)"},
            "parity": {"rel_frob": par[0].item(), "max_abs": par[1].item(), "bar": 5e-3,
                       "ok": bool(par[0].item() <= 5e-3),
                       "what": "sharded output vs the unsharded projections of the same weights, max over ranks"},
            "clocks": clk}))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_linear(args):
    """One fused linear (or gated pair) on cuda:0, events around each call."""
    import torch

    from burn_image_b200 import _lib as L
    from burn_image_b200 import q4, tp
    dev = torch.device("cuda", 0)
    gated = args.gated is not None
    f = [int(v) for v in (args.gated or args.linear).split(",")]
    M, K, N = f[:3]
    act = f[3] if len(f) > 3 and not gated else 0
    block = f[4] if len(f) > 4 else QBLOCK
    g = torch.Generator(device=dev).manual_seed(7)
    w, s = tp._random_packed(K, N, block, g, dev)
    pw = q4.PreparedQ4Weight(w, s, K, N, block, L.LAYOUT_ROW, dev)
    if gated:
        w2, s2 = tp._random_packed(K, N, block, g, dev)
        pu = q4.PreparedQ4Weight(w2, s2, K, N, block, L.LAYOUT_ROW, dev)
    # inputs larger than L2 are rotated between iterations (several copies)
    copies = max(1, min(8, int(2 * 126e6 // (M * K * 4)) + 1))
    xs = [torch.randn((M, K), generator=g, device=dev) for _ in range(copies)]
    y = torch.empty((M, N), dtype=torch.float32, device=dev)
    bias = torch.randn(N, generator=g, device=dev) * 0.02

    def call(i):
        if gated:
            q4.linear_gated(pw, pu, xs[i % copies], out=y)
        else:
            pw.linear(xs[i % copies], bias, act, out=y)

    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        ev[i][0].record(st)
        call(i)
        ev[i][1].record(st)
    torch.cuda.synchronize()
    q4.poll_device_error()
    ms = sorted(a.elapsed_time(b) for a, b in ev)
    med = ms[len(ms) // 2]
    flops = 2 * M * K * N * (2 if gated else 1)
    nbytes = (N * K // 2 + N * K // block * 4) * (2 if gated else 1) + M * K * 4 + M * N * 4
    print(json.dumps({"metric": "Q4 linear TFLOP/s", "value": flops / med / 1e9, "unit": "TFLOP/s",
                      "ms": med, "gbs": nbytes / med / 1e6, "shape": [M, K, N], "act": act, "block": block,
                      "gated": gated, "steps": args.steps}))


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.rows_only:
        import torch
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        except Exception:
            pass
        names = set(args.rows.split(",")) if args.rows else None
        print(json.dumps({"rows": config_rows(torch.device("cuda", 0), peaks, names)}))
    elif args.linear or args.gated:
        run_linear(args)
    elif args.config == "c4":
        run_c4(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
