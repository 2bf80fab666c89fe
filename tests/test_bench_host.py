"""Host-side logic of bench.py (no GPU): clock-sample filtering, head maps,
traffic scaling and the visible-pair formulas the roofline divides by."""

from __future__ import annotations

import datetime
import importlib.util
import os
import sys
import time

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    sys.argv = ["bench.py"]
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


def _line(t: float, sm: int, power_cap: bool) -> str:
    ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    cap = "Active" if power_cap else "Not Active"
    return f"{ts}, 0, {sm}, 1965, 950.0, 0x0, Not Active, Not Active, Not Active, {cap}"


def test_clock_samples_filtered_by_their_own_timestamps(bench):
    cs = bench.ClockSampler(0)

    class _Proc:
        def terminate(self):
            pass

        def wait(self, timeout=None):
            pass

    cs.proc = _Proc()
    now = time.time()
    cs.lines = [_line(now - 5.0, 1965, False),   # idle, before the timed region
                _line(now + 0.10, 1700, True),
                _line(now + 0.15, 1800, True),
                _line(now + 0.20, 1750, False),
                _line(now + 9.0, 1965, False)]   # after it
    out = cs.stop(now, now + 1.0)
    assert out["samples"] == 3
    assert out["sm_mhz"] == 1750.0
    assert out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]
    assert cs.stop()["samples"] == 5  # no window: every sample


def test_head_maps(bench):
    for world in (1, 2, 4, 8):
        for kind in ("contiguous", "balanced"):
            m = bench.head_map_for(world, "mixed", 32, kind, 65536)
            assert len(m) == world
            assert sorted(h for hs in m for h in hs) == list(range(32))
            assert all(len(hs) == 32 // world for hs in m)
    # shard_groups lists each rank's heads grouped by pattern, cheapest first
    m = bench.head_map_for(4, "mixed", 32, "balanced", 65536)
    groups = bench.shard_groups(1, 4, "mixed", 32, m)
    assert sorted(h for _, hs in groups for h in hs) == m[1]
    order = [p for p, _ in groups]
    rank = {"stream_llm": 0, "block_sparse": 1, "vertical_and_slash": 2, "dense": 3}
    assert order == sorted(order, key=rank.get)


def test_stream_visible_pairs_brute_force(bench):
    S, n_init, n_local = 300, 16, 40
    i = np.arange(S)[:, None]
    j = np.arange(S)[None, :]
    mask = (j <= i) & ((j < n_init) | (j > i - n_local))
    assert bench.stream_visible_pairs(S, n_init, n_local) == int(mask.sum())


def test_traffic_scales_with_heads(bench):
    class _Layer:
        slices = [("stream_llm", slice(0, 1)), ("block_sparse", slice(1, 3)),
                  ("vertical_and_slash", slice(3, 6))]

    per = bench.ATTN_DRAM_BYTES_PER_HEAD_64K
    want = per["stream_llm"] + 2 * per["block_sparse"] + 3 * per["vertical_and_slash"]
    assert bench.attn_traffic_bytes(_Layer(), 65536) == pytest.approx(want)
    assert bench.attn_traffic_bytes(_Layer(), 32768) is None
