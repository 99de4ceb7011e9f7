"""Known-answer tests of the bench telemetry, ported from the reference's
Tests/QwenFieldfareCore/QwenRuntimeTelemetryTests.swift:6-53 (same inputs,
same expected values), plus the per-layer counters of the cache planner."""
import numpy as np
import pytest

from qfmoe.telemetry import (BoundedLatencyAccumulator, LatencySummary, cache_hit_rate,
                             cache_requests)

RECORD = 1_769_472


def test_nearest_rank_percentiles_and_mean():
    s = LatencySummary.summarize([5, 1, 4, 2, 3, 100])
    assert s.sample_count == 6
    assert s.minimum_ms == 1
    assert s.maximum_ms == 100
    assert s.mean_ms == 19.166666666666668
    assert s.p50_ms == 3
    assert s.p95_ms == 100


def test_bounded_accumulator_drops_oldest_samples_and_resets():
    a = BoundedLatencyAccumulator(capacity=3)
    for v in (1, 2, 3, 4):
        a.record(v)
    assert a.summary.sample_count == 3
    assert a.summary.minimum_ms == 2
    assert a.summary.maximum_ms == 4
    a.reset()
    assert a.summary.sample_count == 0
    assert a.summary.p95_ms is None


def test_accumulator_ignores_non_finite_and_negative_samples():
    a = BoundedLatencyAccumulator()
    for v in (float("nan"), float("inf"), -1.0, 2.0):
        a.record(v)
    assert a.summary.sample_count == 1 and a.summary.p50_ms == 2.0


def test_cache_derived_metrics_use_demand_requests_only():
    m = dict(capacity=1024, occupancy=900, probationary_occupancy=200, protected_occupancy=700,
             hits=75, misses=25, evictions=4, fetched_bytes=25 * RECORD, prefetch_requests=12,
             useful_prefetch_hits=8, wasted_prefetches=2)
    assert cache_requests(m) == 100
    assert cache_hit_rate(m) == 0.75
    assert cache_hit_rate(dict(m, hits=0, misses=0)) is None


@pytest.mark.parametrize("policy", ["slru", "lru"])
def test_per_layer_counters_sum_to_the_run_counters(policy):
    """qf_cache_layer_metrics: per-layer demand hits / lookups whose sums are
    the run-level hits and hits + misses; cleared by reset_metrics."""
    from qfmoe.cache import ExpertCache
    rng = np.random.default_rng(3)
    c = ExpertCache(40 * 12, layer_count=40, policy=policy)
    try:
        p = 1.0 / np.arange(1, 257) ** 1.2
        p /= p.sum()
        for _ in range(30):
            for layer in range(40):
                c.acquire_slots_parallel(layer, rng.choice(256, 8, replace=False, p=p))
        m = c.metrics_snapshot()
        hits, req = c.layer_metrics()
        assert hits.sum() == m["hits"] and req.sum() == m["hits"] + m["misses"]
        assert (req == 30 * 8).all()
        rates = c.layer_hit_rates()
        assert len(rates) == 40 and all(0.0 <= r <= 100.0 for r in rates)
        assert rates[0] == pytest.approx(100.0 * hits[0] / req[0])
        c.reset_metrics()
        hits, req = c.layer_metrics()
        assert not hits.any() and not req.any()
    finally:
        c.close()
