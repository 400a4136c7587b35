"""Host placement helper: the CPUs next to a GPU, read from a sysfs tree."""

import os

from reframework_b200.parallel.dist import _parse_cpulist, device_local_cpus


def test_parse_cpulist():
    assert _parse_cpulist("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11]
    assert _parse_cpulist("") == []


def test_device_local_cpus_reads_sysfs(tmp_path):
    d = tmp_path / "bus" / "pci" / "devices" / "0000:1b:00.0"
    d.mkdir(parents=True)
    (d / "local_cpulist").write_text("0-55,112-167\n")
    cpus = device_local_cpus(0, 0x1B, 0, sysfs=str(tmp_path))
    assert cpus[:2] == [0, 1] and len(cpus) == 112 and cpus[-1] == 167
    assert device_local_cpus(0, 0x1C, 0, sysfs=str(tmp_path)) is None  # unknown device
    (d / "local_cpulist").write_text("garbage")
    assert device_local_cpus(0, 0x1B, 0, sysfs=str(tmp_path)) is None
