"""CPU: the host-side parts of bench.py that need no GPU -- the defaults of
its command line, the parsing of the nvidia-smi clock samples taken during
the timed region, and the two CPU arms (the oracle's q_matmul restatement and
its attention) on small samples."""
import sys

import bench


def test_defaults_keep_the_contract(monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse()
    assert a.gpus == 1 and a.impl == "ours"
    assert a.warmup >= 3 and a.steps >= 1
    assert a.blocks == bench.BLOCKS and a.tokens == bench.TOKENS


class _Done:
    stdout = iter(())

    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0

    def kill(self):
        pass


def _sample(ts, sm, smax, active=(), gpu=0):
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    flags = ["Active" if n in active else "Not Active" for n in names]
    return ts, ", ".join(["2026/01/01 00:00:00.000", str(gpu), str(sm), str(smax), "700.0", "0x0"] + flags)


def test_clock_sampler_window_median_and_reasons():
    c = bench.ClockSampler(0)
    c.proc = _Done()
    c.lines = [_sample(0.5, 900, 1965, ("hw_slowdown",)),  # before the timed region: ignored
               _sample(1.0, 1900, 1965), _sample(1.2, 1950, 1965, ("sw_power_cap",)),
               _sample(1.4, 1930, 1965), (1.5, "malformed"), _sample(9.0, 500, 1965, ("hw_thermal_slowdown",))]
    c.t_start, c.t_end = 1.0, 1.45
    got = c.stop()
    assert got["sm_mhz"] == 1930 and got["sm_max_mhz"] == 1965
    assert got["reasons"] == ["sw_power_cap"] and got["samples"] == 3


def test_clock_sampler_without_nvidia_smi():
    got = bench.ClockSampler(0).stop()
    assert got["sm_mhz"] is None and got["reasons"] == ["nvidia-smi unavailable"]


def test_cpu_arms_on_small_samples():
    tf, dt, threads = bench.cpu_sample(4, 1, threads=2)
    assert tf > 0 and dt > 0 and threads == 2
    arm = bench._attn_cpu_arm(256, 64, rows=16)
    assert arm["tflops"] > 0 and arm["kind"] == "port" and arm["sample"] == "1 head, 16 of 256 query rows"
