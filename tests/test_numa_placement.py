"""CPU: placement of pinned host staging buffers near a GPU (dtorch_b200.multiprocess.near_device): the cpulist
parser, and that the calling thread runs on the device-local CPUs inside the block and gets its old CPU set back
afterwards (the device-local set is given here, as sysfs would report it)."""

import os

import pytest

from dtorch_b200.multiprocess import near_device, parse_cpulist


def test_parse_cpulist():
    assert parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert parse_cpulist("5") == {5}
    assert parse_cpulist("") == set()


def test_near_device_restricts_and_restores():
    old = os.sched_getaffinity(0)
    if len(old) < 2:
        pytest.skip("needs >= 2 allowed CPUs")
    local = set(sorted(old)[: len(old) // 2])
    with near_device(0, cpus=local) as used:
        assert used == local
        assert os.sched_getaffinity(0) == local
    assert os.sched_getaffinity(0) == old


def test_near_device_unchanged_when_nothing_applies():
    old = os.sched_getaffinity(0)
    with near_device(0, cpus=set()) as used:  # unknown locality
        assert used is None and os.sched_getaffinity(0) == old
    with near_device(0, cpus={max(old) + 4096}) as used:  # local CPUs not allowed to this process
        assert used is None and os.sched_getaffinity(0) == old
    assert os.sched_getaffinity(0) == old
