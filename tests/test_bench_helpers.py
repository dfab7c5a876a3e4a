"""bench.py's host-side helpers (no GPU): the per-call statistic, the prefill
roofline object, the published-shape splitter and the rotating state buffers."""
import importlib.util

import pytest
import torch

from tests.conftest import REPO


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("gdn_bench_helpers", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_per_call_ms_is_the_mean_of_the_middle_80_percent(bench):
    # event times on a ~2 us grid: a median would snap to a grid value
    times = [0.00614] * 6 + [0.00819] * 4  # ms
    assert bench.per_call_ms(times) == pytest.approx((0.00614 * 5 + 0.00819 * 3) / 8)
    # one outlier at each end is dropped (10 % of 20 calls)
    times = [0.010] * 18 + [0.001, 1.0]
    assert bench.per_call_ms(times) == pytest.approx(0.010)
    # too few calls to trim: the plain mean
    assert bench.per_call_ms([0.002, 0.004]) == pytest.approx(0.003)


def test_prefill_roofline_picks_the_longer_floor(bench):
    peaks = {"hbm_gbs": 1000.0, "bf16_tflops": 1.0}
    # 1 GB at 1000 GB/s = 1 ms; 1 TFLOP at 1 TFLOP/s = 1000 ms: tensor-bound
    r = bench.prefill_roofline(1e9, 1e12, 2000.0, peaks)
    assert r["bound"] == "tensor"
    assert r["frac"] == pytest.approx(0.5, rel=1e-3)
    r = bench.prefill_roofline(1e12, 1e9, 2000.0, peaks)
    assert r["bound"] == "hbm" and r["frac"] == pytest.approx(0.5, rel=1e-3)


def test_split_total_is_seeded_and_exact(bench):
    a = bench.split_total(5709, 2, 5709)
    assert sum(a) == 5709 and len(a) == 2 and min(a) >= 1
    assert a == bench.split_total(5709, 2, 5709)
    b = bench.split_total(8192, 34, 8192)
    assert sum(b) == 8192 and len(b) == 34 and min(b) >= 1


def test_rotating_states_are_distinct_buffers(bench):
    s = torch.zeros(2, 8, 128, 128)
    st = bench.rotating_states(s)
    assert len(st) == 3 and st[0] is s
    assert st[1].data_ptr() != s.data_ptr() and st[2].data_ptr() != st[1].data_ptr()
    assert all(t.shape == s.shape and t.dtype == s.dtype for t in st)
