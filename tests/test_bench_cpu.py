"""bench.py's host side on the CPU: the argument defaults the driver relies on,
the metric and workload it names, and the clock record's summary."""
import importlib.util
import os

import pytest

from torch2riscv_accelerator_b200.config import CONFIGS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_defaults(bench):
    a = bench.build_parser().parse_args([])
    assert (a.gpus, a.steps, a.warmup, a.impl, a.config, a.batch) == (1, 13, 3, "ours", "Qwen3-0.6B", 1)
    assert a.sustain > 0 and a.parallel == "tp" and a.workload == "bench"


def test_metric_and_prompt(bench):
    c2 = CONFIGS["Qwen3-0.6B"]
    a = bench.build_parser().parse_args([])
    assert bench.metric_of(c2, a) == bench.METRIC
    # the context filled to its last warmup + steps positions: T = 2048 at the last timed step
    assert bench.prompt_len(c2, a) == 2048 - 3 - 13
    a = bench.build_parser().parse_args(["--steps", "20", "--warmup", "3"])
    assert bench.prompt_len(c2, a) == 2025
    b = bench.build_parser().parse_args(["--batch", "128"])
    assert bench.metric_of(c2, b) != bench.METRIC
    assert bench.metric_of(CONFIGS["SmolLM2-135M"], a) != bench.METRIC


def test_config_names_the_split(bench):
    c2 = CONFIGS["Qwen3-0.6B"]
    a = bench.build_parser().parse_args([])
    one = bench.config_of(c2, a, 1)
    assert one["global_batch"] == 1 and one["prompt"] == 2032 and "batch 1" in one["workload"]
    tp = bench.config_of(c2, a, 8, tp=True)
    assert tp["parallelism"] == "tp8" and tp["global_batch"] == 1
    ep = bench.config_of(CONFIGS["Granite-3.1-1B-A400M"], a, 2, ep=True)
    assert ep["parallelism"] == "ep2" and ep["global_batch"] == 1


def test_clock_summary(bench):
    clk = bench.Clocks(0)
    assert clk.summary()["samples"] == 0
    clk.max_mhz = 1965
    clk.samples = [(1965, 0), (1950, 0x4), (1965, 0)]
    s = clk.summary()
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
    clk.samples.append((1200, 0x8 | 0x40))
    assert clk.summary()["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_power_cap"]
