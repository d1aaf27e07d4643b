"""fp64_emu.host's CPU placement helpers on the CPU, against a fake NVML:
the GPU-local core mask is decoded, the process is bound to those cores
only inside gpu_local_allocation, and without NVML nothing changes."""
import os
import sys
import types

import pytest

torch = pytest.importorskip("torch")


@pytest.fixture
def fake_gpu(monkeypatch):
    """A fake NVML whose device reports two of this process's usable cores as
    local, and a fake device 0."""
    usable = sorted(os.sched_getaffinity(0))
    local = [usable[0], usable[2]] if len(usable) >= 3 else usable[:1]
    mask = [0] * ((os.cpu_count() + 63) // 64)
    for c in local:
        mask[c // 64] |= 1 << (c % 64)
    calls = []
    nv = types.SimpleNamespace(
        nvmlInit=lambda: calls.append("init"),
        nvmlShutdown=lambda: calls.append("shutdown"),
        nvmlDeviceGetHandleByUUID=lambda u: ("handle", u),
        nvmlDeviceGetCpuAffinity=lambda h, n: mask[:n],
    )
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda i: types.SimpleNamespace(uuid="1234-abcd"))
    return local, calls


def test_local_cores_from_the_mask(fake_gpu):
    from fp64_emu.host import gpu_local_cpus
    local, calls = fake_gpu
    assert gpu_local_cpus() == local
    assert calls == ["init", "shutdown"]


def test_binding_only_inside_the_allocation_context(fake_gpu):
    from fp64_emu.host import gpu_local_allocation
    local, _ = fake_gpu
    before = os.sched_getaffinity(0)
    with gpu_local_allocation() as loc:
        assert loc.cpus == local
        assert os.sched_getaffinity(0) == set(local)
    assert os.sched_getaffinity(0) == before


def test_no_nvml_changes_nothing(monkeypatch):
    from fp64_emu.host import gpu_local_allocation, gpu_local_cpus
    monkeypatch.setitem(sys.modules, "pynvml", None)   # import fails
    before = os.sched_getaffinity(0)
    assert gpu_local_cpus(0) is None
    with gpu_local_allocation(0) as loc:
        assert loc.cpus is None
        assert os.sched_getaffinity(0) == before
    assert os.sched_getaffinity(0) == before
