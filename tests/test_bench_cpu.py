"""The bench's measurement bookkeeping on the CPU: the clock record of the timed region (nvidia-smi samples read
back, reasons kept, the nearest samples when the region is shorter than the sampling interval) and the choice of
the bf16 peak a tensor-core kernel is compared with (burst, or sustained when the power cap held the clock)."""
from __future__ import annotations

import importlib.util
import pathlib

ROOT = pathlib.Path(__file__).resolve().parent.parent


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _line(sm, mx=1965, cap=False, thermal=False):
    state = lambda on: "Active" if on else "Not Active"   # noqa: E731
    return f"0, {sm}, {mx}, 980.5, 0x4, {state(False)}, {state(thermal)}, {state(False)}, {state(cap)}\n"


def test_clock_summary_inside_and_nearest():
    b = _bench()
    c = b.ClockSampler([0], enabled=False)
    c.lines = [(0.9, _line(1965)), (1.05, _line(1300, cap=True)), (1.15, _line(1200, cap=True)),
               (1.25, _line(1250, cap=True)), (1.6, _line(1965))]
    c.t0, c.t1 = 1.0, 1.3
    s = c.summary()
    assert s["window"] == "timed region" and s["samples"] == 3
    assert s["sm_mhz"] == 1250 and s["sm_max_mhz"] == 1965 and s["reasons"] == ["sw_power_cap"]
    # a region between two samples: the last one before it and the first one after it, within 0.3 s
    c.lines = [(0.8, _line(1900, thermal=True)), (0.95, _line(1965)), (1.2, _line(1940))]
    c.t0, c.t1 = 1.0, 1.1
    s = c.summary()
    assert s["window"] == "nearest" and s["samples"] == 2 and s["reasons"] == []
    assert s["sm_mhz"] == (1965 + 1940) / 2


def test_tensor_peak_choice():
    b = _bench()
    burst, sustained = 1656.1, 1408.7
    full = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}
    flagged = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}
    held = {"sm_mhz": 1140.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}
    none = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
    assert b.tensor_peak(70.0, full, burst, sustained) == (burst, "bf16_tflops")
    assert b.tensor_peak(70.0, flagged, burst, sustained) == (burst, "bf16_tflops")   # the flag at full clock
    assert b.tensor_peak(70.0, held, burst, sustained) == (sustained, "bf16_tflops_sustained")
    assert b.tensor_peak(2000.0, full, burst, sustained) == (sustained, "bf16_tflops_sustained")
    assert b.tensor_peak(70.0, none, burst, sustained) == (burst, "bf16_tflops")       # no sampler
