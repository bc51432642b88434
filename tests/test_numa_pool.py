"""NUMA placement of the pinned V pool: the GPU's local CPUs come from NVML
(read-only queries, looked up by PCI bus id) and the pool is first-touched
from them.  Runs on CPU against a fake NVML."""
import os
import sys
import types

import pytest
import torch

from amass_kv_b200 import tier as T


def _fake_nvml(words, seen):
    m = types.ModuleType("pynvml")
    m.nvmlInit = lambda: seen.append("init")
    m.nvmlShutdown = lambda: seen.append("shutdown")

    def by_bus(bus):
        seen.append(bus)
        return "handle"
    m.nvmlDeviceGetHandleByPciBusId = by_bus
    m.nvmlDeviceGetCpuAffinity = lambda h, n: words[:n]
    return m


def test_gpu_local_cpus_decodes_affinity(monkeypatch):
    seen = []
    monkeypatch.setitem(sys.modules, "pynvml",
                        _fake_nvml([0b1010, 1 << 3], seen))
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1b,
                                  pci_device_id=0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda d: props)
    monkeypatch.setattr(os, "cpu_count", lambda: 128)
    cpus = T.gpu_local_cpus(0)
    assert cpus == [1, 3, 67]
    assert seen == ["init", "00000000:1b:00.0", "shutdown"]


def test_gpu_local_cpus_without_nvml(monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", None)
    assert T.gpu_local_cpus(0) is None


@pytest.mark.skipif(not hasattr(os, "sched_setaffinity"), reason="linux only")
def test_affinity_scope_restores():
    before = os.sched_getaffinity(0)
    threads = torch.get_num_threads()
    one = [min(before)]
    with T._cpu_affinity(one):
        assert os.sched_getaffinity(0) == set(one)
        assert torch.get_num_threads() == 1
    assert os.sched_getaffinity(0) == before
    assert torch.get_num_threads() == threads
    with T._cpu_affinity([10 ** 6]):          # no overlap: leave it alone
        assert os.sched_getaffinity(0) == before
