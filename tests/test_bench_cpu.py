"""Host-side measurement helpers of bench.py, on CPU: the whole-step
algorithmic bytes, the per-class algorithmic bytes, the traffic scaled from the
committed ncu capture, and the clock sampler's timed-region window."""
from __future__ import annotations

import datetime
import pathlib
import sys
import time

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def test_step_bytes_is_config3_per_step_work():
    # weights once, KV of positions 0..pos read + this position written, logits row
    want = 346206720 + 256 * (531 * 24576 + 24576 + 607744)
    assert bench.step_bytes_at(256, 530) == pytest.approx(want)
    assert bench.step_bytes_at(1, 0) == pytest.approx(346206720 + 24576 + 24576 + 607744)


def test_attention_bytes_grow_with_context_and_sequences():
    a = bench.class_bytes_at("attention", 256, 516)
    assert a == pytest.approx(2 * bench.class_bytes_at("attention", 128, 516))
    assert bench.class_bytes_at("attention", 256, 1000) > a
    assert bench.class_bytes_at("no-such-class", 256, 516) == 0.0
    # the matvec class streams the layer weights once per step whatever the batch
    assert bench.class_bytes_at("gemv", 1, 0) > 24 * 8.3e6


def test_timed_steps_cover_the_decode_range():
    t = bench.strata(5, 1021, 20)
    assert len(set(t)) == 20 and t == sorted(t)
    assert t[0] < 5 + 1017 / 20 and t[-1] > 1021 - 1017 / 20
    # evenly spaced: the mean position is the middle of the range
    assert abs(sum(t) / 20 - (5 + 1021) / 2) < 1.0
    with pytest.raises(ValueError):
        bench.strata(0, 3, 5)


def test_strong_scaling_partition_splits_the_batch():
    from promptboot_b200 import shard
    for world in (1, 2, 4, 8):
        blocks = [shard.partition(256, r, world) for r in range(world)]
        assert all(c == 256 // world for _, c in blocks)
        assert [f for f, _ in blocks] == [r * 256 // world for r in range(world)]
    blocks = [shard.partition(10, r, 4) for r in range(4)]
    assert blocks == [(0, 3), (3, 3), (6, 2), (8, 2)]
    with pytest.raises(ValueError):
        shard.partition(2, 0, 4)


def test_profiled_traffic_scales_the_committed_capture():
    per = bench.profiled_traffic("attention", 1, 1.0)
    assert per is not None and 1024 <= per <= 1200        # bytes per sequence-position
    assert bench.profiled_traffic("attention", 256, 530.0) == pytest.approx(per * 256 * 530)


def test_bench_defaults_are_the_driver_contract():
    a = bench.parse([])
    assert (a.gpus, a.seqs, a.prompt, a.decode) == (1, 256, 512, 1024)
    assert a.warmup >= 3 and a.steps >= 1


def _line(t: float, mhz: int, cap: str = "Not Active") -> str:
    ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return f"{ts}, 0, {mhz}, 1965, 600.5, 0x0, Not Active, Not Active, Not Active, {cap}"


def test_clock_summary_keeps_samples_inside_the_timed_region():
    c = bench.ClockSampler(0)
    now = time.time()
    c.path.write_text("\n".join([_line(now - 0.3, 1200), _line(now + 0.05, 1950, "Active"),
                                 _line(now + 0.10, 1965), _line(now + 0.6, 1100)]) + "\n")
    c.mark(now, now + 0.2)
    s = c.summary()
    assert s["samples"] == 2 and s["sm_max_mhz"] == 1965
    assert s["sm_mhz"] == pytest.approx((1950 + 1965) / 2) and s["reasons"] == ["sw_power_cap"]


def test_clock_summary_short_region_takes_the_next_sample():
    c = bench.ClockSampler(0)
    now = time.time()
    c.path.write_text("\n".join([_line(now - 0.1, 1500), _line(now + 0.04, 1965)]) + "\n")
    c.mark(now, now + 0.01)
    s = c.summary()
    assert s["samples"] == 1 and s["sm_mhz"] == 1965


def test_clock_summary_without_samples_says_so():
    c = bench.ClockSampler(0)
    c.path.write_text("")
    c.mark(time.time(), time.time() + 0.1)
    assert c.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"],
                           "samples": 0}
