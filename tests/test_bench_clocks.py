"""bench.py's clock sampler, on a fake NVML: samples are taken while the
timed region runs and the reasons that were active are reported."""
import sys
import time
import types
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def fake_nvml(clocks, reasons):
    nv = types.SimpleNamespace()
    nv.NVML_CLOCK_SM = 1
    nv.nvmlClocksEventReasonHwSlowdown = 0x8
    nv.nvmlClocksEventReasonHwThermalSlowdown = 0x40
    nv.nvmlClocksEventReasonSwThermalSlowdown = 0x20
    nv.nvmlClocksEventReasonSwPowerCap = 0x4
    state = {"i": 0, "uuid": None}
    nv.nvmlInit = lambda: None

    def by_uuid(u):
        state["uuid"] = u
        return "h"
    nv.nvmlDeviceGetHandleByUUID = by_uuid
    nv.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965

    def clock(h, kind):
        state["i"] += 1
        return clocks[min(state["i"] - 1, len(clocks) - 1)]
    nv.nvmlDeviceGetClockInfo = clock
    nv.nvmlDeviceGetCurrentClocksEventReasons = lambda h: reasons[min(state["i"], len(reasons) - 1)]
    return nv, state


def test_nvml_sampling(monkeypatch):
    nv, state = fake_nvml([1965, 1965, 1900, 1965] + [1965] * 100, [0, 0, 0x4] + [0] * 100)
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda d: types.SimpleNamespace(uuid="abc-123"))
    s = bench.ClockSampler("cpu")
    s.start()
    time.sleep(0.06)
    info = s.stop()
    assert state["uuid"] == "GPU-abc-123"
    assert info["source"] == "nvml, 5 ms"
    assert info["samples"] >= 5
    assert info["sm_max_mhz"] == 1965
    assert info["sm_mhz"] == 1965
    assert info["reasons"] == ["sw_power_cap"]


def test_no_nvml_and_no_smi_gives_none(monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", None)  # import fails
    monkeypatch.setattr(bench.subprocess, "Popen",
                        lambda *a, **k: (_ for _ in ()).throw(FileNotFoundError("nvidia-smi")))
    s = bench.ClockSampler("cpu")
    s.start()
    assert s.stop() is None
