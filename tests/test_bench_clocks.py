"""bench.py's clock record: the sampler finds the GPU by PCI bus id (so a
renumbered CUDA_VISIBLE_DEVICES cannot point it at another GPU), uses only
read-only NVML queries, reads from the launching thread as well as its own
thread, and reports the median SM clock and the throttle reasons seen
(gpu_idle dropped).  Runs on CPU against a fake NVML."""
import sys
import types

import torch

import bench


def _fake_nvml(clocks, reasons, seen):
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1
    m.nvmlInit = lambda: seen.append("init")

    def by_bus(bus):
        seen.append(bus)
        return "handle"
    m.nvmlDeviceGetHandleByPciBusId = by_bus
    m.nvmlDeviceGetMaxClockInfo = lambda h, c: 1965
    it = iter(clocks)
    m.nvmlDeviceGetClockInfo = lambda h, c: next(it, clocks[-1])
    m.nvmlDeviceGetCurrentClocksEventReasons = lambda h: reasons
    # anything that changes a GPU setting must not be reachable
    for name in ("nvmlDeviceSetGpuLockedClocks", "nvmlDeviceResetGpuLockedClocks",
                 "nvmlDeviceSetApplicationsClocks", "nvmlDeviceSetPowerManagementLimit"):
        setattr(m, name, lambda *a, _n=name: seen.append("SET " + _n))
    return m


def test_clock_sampler_by_bus_id_and_summary(monkeypatch):
    seen = []
    # bit 0 gpu_idle, bit 2 sw_power_cap
    monkeypatch.setitem(sys.modules, "pynvml",
                        _fake_nvml([1965, 1950, 1965], 0b101, seen))
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x9a,
                                  pci_device_id=0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda d: props)
    clk = bench.ClockSampler(0)
    assert seen == ["init", "00000000:9a:00.0"]
    # launching-thread readings alone are enough for a summary
    for _ in range(3):
        assert clk.sample()
    s = clk.summary()
    assert s["sm_mhz"] == 1965 and s["sm_max_mhz"] == 1965
    assert s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
    assert not any(x.startswith("SET") for x in seen)


def test_clock_sampler_thread_and_main_thread_together(monkeypatch):
    seen = []
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml([1965], 0, seen))
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1b,
                                  pci_device_id=0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda d: props)
    with bench.ClockSampler(0) as clk:
        for _ in range(50):
            clk.sample()
    s = clk.summary()
    assert s["samples"] >= 50 and s["reasons"] == []


def test_clock_sampler_without_nvml(monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", None)     # import fails
    with bench.ClockSampler(0) as clk:
        assert not clk.sample()
    s = clk.summary()
    assert s["sm_mhz"] is None and s["samples"] == 0
