"""Expert-slot cache planner (libqf_moe.so, host C++) on the CPU.

  - the reference's own known-answer tests
    (Tests/QwenFieldfareCore/Storage/Q4BoundedExpertCacheTests.swift and
    Tests/QwenFieldfareCore/QwenActiveStreamingMemoryConfigurationTests.swift),
    restated against the product planner and against the oracle port;
  - differential replay of seeded random traces, product vs the oracle port of
    Q4BoundedExpertCache (slots, miss positions, fetch lists, metrics);
  - the plain-LRU policy against the oracle's LRU restatement.
No GPU is touched: the planner is host code."""
import random

import numpy as np
import pytest

import oracle as O
from qfmoe.cache import ExpertCache, plan_slots
from qfmoe._lib import QfError


# ---------------------------------------------------------------- reference KATs
def test_kat_layer_partitions_prevent_cross_layer_eviction():
    # Q4BoundedExpertCacheTests.swift:8-28
    c = ExpertCache(16, layer_count=2)
    s0, _, _ = c.acquire_slots_parallel(0, range(0, 8))
    s1, _, _ = c.acquire_slots_parallel(1, range(16, 24))
    assert set(s0).isdisjoint(s1)
    c.acquire_slots_parallel(0, range(32, 40))
    c.reset_metrics()
    s1b, miss, fetch = c.acquire_slots_parallel(1, range(16, 24))
    assert s1b == s1
    m = c.metrics_snapshot()
    assert (m["hits"], m["misses"]) == (8, 0)
    assert miss == [] and fetch == []


def test_kat_parallel_miss_fetch_writes_assigned_slots():
    # Q4BoundedExpertCacheTests.swift:30-45: every miss is fetched into the
    # slot returned for its position
    c = ExpertCache(8, layer_count=1)
    experts = list(range(40, 48))
    slots, miss, fetch = c.acquire_slots_parallel(0, experts)
    assert dict(fetch) == dict(zip(experts, slots))
    assert miss == list(range(8))
    assert c.metrics_snapshot()["misses"] == 8


def test_kat_parallel_planning_reports_only_miss_positions():
    # Q4BoundedExpertCacheTests.swift:47-75
    c = ExpertCache(8, layer_count=1)
    c.acquire_slots_parallel(0, range(8))
    c.reset_metrics()
    slots, miss, fetch = c.acquire_slots_parallel(0, list(range(7)) + [8])
    assert miss == [7]
    assert [e for e, _ in fetch] == [8] and fetch[0][1] == slots[7]
    m = c.metrics_snapshot()
    assert (m["hits"], m["misses"]) == (7, 1)


def test_kat_slot_budgets_at_8k():
    # QwenActiveStreamingMemoryConfigurationTests.swift:6-10
    assert [plan_slots(g, 8192)["slots"] for g in (3, 4, 5)] == [969, 1576, 2183]
    assert [O.plan_slots(g, 8192)[0] for g in (3, 4, 5)] == [969, 1576, 2183]


def test_kat_every_plan_within_target_and_keeps_router_locks():
    # QwenActiveStreamingMemoryConfigurationTests.swift:12-26
    for g in (3, 4, 5):
        for ctx in (4096, 8192, 16384, 32768, 65536):
            ref = O.plan_slots(g, ctx)
            if not ref[3]:
                with pytest.raises(QfError):
                    plan_slots(g, ctx)
                continue
            p = plan_slots(g, ctx)
            assert (p["slots"], p["estimated_bytes"], p["target_bytes"]) == ref[:3]
            assert p["slots"] >= 320 and p["estimated_bytes"] <= p["target_bytes"]


def test_kat_rejects_budget_that_cannot_keep_layer_locks():
    # QwenActiveStreamingMemoryConfigurationTests.swift:28-33
    with pytest.raises(QfError):
        plan_slots(3, 65536)
    assert not O.plan_slots(3, 65536)[3]


def test_kat_more_context_never_more_slots():
    # QwenActiveStreamingMemoryConfigurationTests.swift:35-41
    assert plan_slots(5, 65536)["slots"] < plan_slots(5, 8192)["slots"]


def test_plan_arguments():
    for g, ctx in ((0, 8192), (5, 0), (5, -1)):
        with pytest.raises(QfError):
            plan_slots(g, ctx)
    # larger budgets than the reference's 3/4/5 GiB follow the same formula
    assert plan_slots(160, 8192)["slots"] == O.plan_slots(160, 8192)[0]


# ---------------------------------------------------------------- partitions
@pytest.mark.parametrize("capacity,layers", [(320, 40), (969, 40), (1576, 40), (2183, 40),
                                             (10240, 40), (319, 40), (16, 2), (100, 3),
                                             (64, 48), (7, 1)])
def test_layer_capacities_match_oracle(capacity, layers):
    c = ExpertCache(capacity, layer_count=layers)
    ref = O.OracleCache(capacity, 0.25, layers)
    assert c.layer_count == ref.layer_count
    assert c.layer_capacities == ref.layer_capacities()
    assert c.probationary_capacity == ref.probationary_capacity
    assert sum(c.layer_capacities) == capacity
    if c.layer_count == 40:
        assert min(c.layer_capacities) >= 8


def test_argument_errors():
    for args in ((0, 40, 0.25, "slru"), (16, 0, 0.25, "slru"), (16, 2, 1.5, "slru"),
                 (16, 2, -0.1, "slru")):
        with pytest.raises(QfError):
            ExpertCache(args[0], layer_count=args[1], probationary_ratio=args[2], policy=args[3])
    with pytest.raises(KeyError):
        ExpertCache(16, policy="fifo")


# ---------------------------------------------------------------- differential replay
def _zipf_trace(rng, n_tokens, layers, s=1.2, reuse=5, p_reuse=0.7):
    """Per-layer Zipf expert popularity with temporal locality (a token re-uses
    `reuse` of the previous token's experts with probability p_reuse)."""
    ranks = np.arange(1, 257, dtype=np.float64)
    p = ranks ** -s
    p /= p.sum()
    perms = [rng.permutation(256) for _ in range(layers)]
    prev = [None] * layers
    out = []
    for _ in range(n_tokens):
        tok = []
        for l in range(layers):
            chosen = []
            if prev[l] is not None and rng.random() < p_reuse:
                chosen = list(rng.choice(prev[l], reuse, replace=False))
            while len(chosen) < 8:
                e = int(perms[l][rng.choice(256, p=p)])
                if e not in chosen:
                    chosen.append(e)
            prev[l] = np.array(chosen)
            tok.append(chosen)
        out.append(tok)
    return out


@pytest.mark.parametrize("capacity,layers,ratio,seed", [
    (2183, 40, 0.25, 1), (969, 40, 0.25, 2), (320, 40, 0.25, 3), (400, 40, 0.5, 4),
    (96, 4, 0.25, 5), (40, 4, 0.1, 6), (64, 1, 0.25, 7), (24, 1, 0.0, 8), (8, 1, 1.0, 9)])
def test_differential_vs_oracle(capacity, layers, ratio, seed):
    rng = np.random.default_rng(seed)
    prod = ExpertCache(capacity, layer_count=layers, probationary_ratio=ratio)
    ref = O.OracleCache(capacity, ratio, layers)
    trace = _zipf_trace(rng, 40 if layers == 40 else 200, layers)
    pyrng = random.Random(seed)
    for t, tok in enumerate(trace):
        for l, experts in enumerate(tok):
            a = prod.acquire_slots_parallel(l, experts)
            b = ref.acquire(l, experts)
            assert a == b, (t, l)
            if pyrng.random() < 0.05:  # interleave speculative prefetches
                cands = [pyrng.randrange(256) for _ in range(4)]
                pf = prod.speculative_prefetch(l, cands)
                ref.prefetch(l, cands)
                lo, hi = prod.layer_ranges()[min(l, prod.layer_count - 1)]
                assert all(lo <= s < hi and e in cands for e, s in pf)
        if t == len(trace) // 2:
            prod.reset_metrics()
            ref.reset_metrics()
    assert prod.metrics_snapshot() == ref.metrics()


def test_short_topk_and_duplicates_vs_oracle():
    prod = ExpertCache(48, layer_count=2)
    ref = O.OracleCache(48, 0.25, 2)
    for experts in ([1, 2, 3], [1, 1, 2], list(range(10)), [5], [200, 201, 202, 203, 204, 205,
                                                                   206, 207, 208]):
        for l in (0, 1, 5):  # layer 5 clamps to the last partition
            assert prod.acquire_slots_parallel(l, experts) == ref.acquire(l, experts)
    assert prod.metrics_snapshot() == ref.metrics()
    prod.clear()
    ref.clear()
    assert prod.acquire_slots_parallel(0, [9]) == ref.acquire(0, [9])


# ---------------------------------------------------------------- plain LRU
@pytest.mark.parametrize("capacity,seed", [(2183, 1), (400, 2), (320, 3)])
def test_lru_policy_vs_oracle_lru(capacity, seed):
    rng = np.random.default_rng(seed)
    prod = ExpertCache(capacity, layer_count=40, policy="lru")
    ref = O.OracleLRU(capacity, 40)
    for tok in _zipf_trace(rng, 30, 40):
        for l, experts in enumerate(tok):
            slots, miss, fetch = prod.acquire_slots_parallel(l, experts)
            rs, rf = ref.acquire(l, experts)
            assert (slots, fetch) == (rs, rf)
    m = prod.metrics_snapshot()
    assert (m["hits"], m["misses"], m["evictions"]) == (ref.hits, ref.misses, ref.evictions)
    assert m["protected_occupancy"] == 0
