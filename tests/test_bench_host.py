"""Host-side logic of bench.py that needs no GPU: the clock sampler.

The sampler is driven by a fake NVML module (read-only queries only), so the
test checks the polling thread, the reason-bit decoding and the summary that
bench.py writes under "clocks".
"""

from __future__ import annotations

import sys
import time
import types

import torch

import bench


def _fake_nvml(sm_mhz: list[int], masks: list[int]):
    state = {"i": 0}
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1
    m.nvmlClocksEventReasonHwSlowdown = 0x8
    m.nvmlClocksEventReasonHwThermalSlowdown = 0x40
    m.nvmlClocksEventReasonSwThermalSlowdown = 0x20
    m.nvmlClocksEventReasonSwPowerCap = 0x4
    m.nvmlInit = lambda: None
    m.nvmlShutdown = lambda: None
    m.nvmlDeviceGetHandleByUUID = lambda uuid: ("uuid", uuid)
    m.nvmlDeviceGetHandleByIndex = lambda i: ("index", i)
    m.nvmlDeviceGetMaxClockInfo = lambda h, c: 1965

    def clock(h, c):
        i = state["i"]
        state["i"] = i + 1
        return sm_mhz[min(i, len(sm_mhz) - 1)]

    def reasons(h):
        return masks[min(max(state["i"] - 1, 0), len(masks) - 1)]

    m.nvmlDeviceGetClockInfo = clock
    m.nvmlDeviceGetCurrentClocksEventReasons = reasons
    return m


def test_clock_sampler_polls_nvml_and_decodes_reasons(monkeypatch):
    fake = _fake_nvml([1965, 1965, 1900, 1965], [0, 0, 0x4, 0])
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.ClockSampler(torch.device("cuda", 0), period_s=0.001) as clk:
        clk.wait_first()
        time.sleep(0.05)
    s = clk.summary()
    assert s["source"].startswith("nvml")
    assert s["samples"] >= 4
    assert s["sm_max_mhz"] == 1965.0
    assert s["sm_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_sampler_flags_thermal_slowdown(monkeypatch):
    fake = _fake_nvml([1400], [0x40 | 0x4])
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.ClockSampler(torch.device("cuda", 0), period_s=0.001) as clk:
        clk.wait_first()
        time.sleep(0.01)
    s = clk.summary()
    assert s["sm_mhz"] == 1400.0
    assert s["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]


def test_clock_sampler_parses_nvidia_smi_lines():
    clk = bench.ClockSampler(torch.device("cuda", 0))
    clk.lines = ["0, 1800, 1965, 900.1, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
                 "0, 1965, 1965, 700.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
                 "garbage"]
    s = clk.summary()
    assert s["samples"] == 2
    assert s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]
