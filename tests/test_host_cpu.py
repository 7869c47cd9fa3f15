"""Host-side logic on the CPU: the placement of the pinned buffers (fnx.hostmem: the sysfs
CPU-list parser and the binding rule, with the device's locality and the process affinity
faked) and bench.py's clock record from nvidia-smi samples."""
import pytest

from fnx import hostmem


@pytest.mark.parametrize("text,want", [
    ("0-3", {0, 1, 2, 3}),
    ("0-3,8,10-11\n", {0, 1, 2, 3, 8, 10, 11}),
    ("5", {5}),
    ("", set()),
    ("0-1,,4", {0, 1, 4}),
])
def test_parse_cpulist(text, want):
    assert hostmem._parse_cpulist(text) == want


def _fake(monkeypatch, local, allowed):
    calls = []
    monkeypatch.setattr(hostmem, "device_locality",
                        lambda dev: {"pci": "0000:9c:00.0", "numa_node": 1 if local else None, "cpus": set(local)})
    monkeypatch.setattr(hostmem.os, "sched_getaffinity", lambda pid: set(allowed))
    monkeypatch.setattr(hostmem.os, "sched_setaffinity", lambda pid, cpus: calls.append(set(cpus)))
    return calls


def test_bind_restricts_to_the_local_cpus(monkeypatch):
    calls = _fake(monkeypatch, local={4, 5, 6, 7, 40}, allowed=range(8))
    r = hostmem.bind_to_device("cuda:0")
    assert calls == [{4, 5, 6, 7}]            # only CPUs the process may already run on
    assert r == {"pci": "0000:9c:00.0", "numa_node": 1, "cpus": 4, "bound": True}


def test_bind_is_a_no_op_when_every_cpu_is_local(monkeypatch):
    calls = _fake(monkeypatch, local=range(32), allowed=range(16))
    r = hostmem.bind_to_device("cuda:0")
    assert calls == [] and r["bound"] is False and r["cpus"] == 16


def test_bind_is_a_no_op_without_locality(monkeypatch):
    # no sysfs locality (or none overlapping the allowed CPUs): nothing changes
    calls = _fake(monkeypatch, local=(), allowed=range(16))
    r = hostmem.bind_to_device("cuda:0")
    assert calls == [] and r == {"pci": "0000:9c:00.0", "numa_node": None, "cpus": 16, "bound": False}
    calls = _fake(monkeypatch, local={100, 101}, allowed=range(16))
    assert hostmem.bind_to_device("cuda:0")["bound"] is False and calls == []


def test_clock_sampler_summary():
    """bench.py's clock record: the median SM clock under load, the max clock, and the throttle
    reasons seen active in any sample (a run with a slowdown reason is re-measured)."""
    import bench
    c = bench.ClockSampler(0)
    c.rows = [["0", "1965", "1965", "700.1", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"],
              ["0", "1920", "1965", "990.0", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
              ["0", "1965", "1965", "800.5", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"]]
    s = c.summary()
    assert s == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    c.rows = [["0", "[N/A]", "1965", "1.0", "0x8", "Active", "Not Active", "Active", "Not Active"]]
    s = c.summary()
    assert s["sm_mhz"] is None and s["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]
    c.rows = []
    assert c.summary()["reasons"] == ["unsampled"]
