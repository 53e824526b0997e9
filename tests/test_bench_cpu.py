"""CPU: the bench's timing rules that need no GPU -- when the timed steps flush L2 (inputs that fit in it) and
when they run back to back (inputs larger than L2), and the nccl-tests bus-bandwidth factors every line uses."""

import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_l2_plan(bench):
    l2 = 126 << 20
    flush, got_l2, note = bench.l2_plan(128 << 20, None, l2_bytes=l2)  # C2 per rank at N > 1
    assert not flush and got_l2 == l2 and "larger than L2" in note and "no flush" in note
    flush, _, note = bench.l2_plan(1 << 30, None, l2_bytes=l2)  # C2 at N = 1: eight 128 MiB partials
    assert not flush
    flush, _, note = bench.l2_plan(8 << 20, None, l2_bytes=l2)  # C1 per rank at N = 8
    assert flush and "fit in L2" in note and "flushed" in note
    assert bench.l2_plan(l2, None, l2_bytes=l2)[0], "inputs exactly the size of L2 are flushed"


def test_bus_factors(bench):
    assert bench.bus_factor("all_reduce", 8) == pytest.approx(1.75)
    assert bench.bus_factor("all_gather", 8) == pytest.approx(0.875)
    assert bench.bus_factor("reduce_scatter", 2) == pytest.approx(0.5)
    assert bench.sweep_sizes(20, 22) == [1 << 20, 1 << 21, 1 << 22]
