"""Run telemetry of the bench harness: per-token latency summaries with
nearest-rank percentiles and the cache's derived rates.

Restates the reference's telemetry types
(Sources/QwenFieldfareCore/Runtime/Telemetry/QwenRuntimeTelemetry.swift):
`QwenLatencySummary.summarize` (:3-30), `QwenBoundedLatencyAccumulator`
(:32-56) and the derived fields of `QwenExpertCacheMetrics` (:58-75), which
the reference bench prints (Sources/QwenFieldfareBench/main.swift:740-806).
"""
from __future__ import annotations

import math
from collections import deque
from dataclasses import dataclass


@dataclass(frozen=True)
class LatencySummary:
    """Count, min, max, mean and nearest-rank p50 / p95 of millisecond samples;
    every statistic is None for an empty sample."""

    sample_count: int
    minimum_ms: float | None
    maximum_ms: float | None
    mean_ms: float | None
    p50_ms: float | None
    p95_ms: float | None

    @classmethod
    def summarize(cls, samples) -> "LatencySummary":
        s = sorted(float(v) for v in samples)
        if not s:
            return cls(0, None, None, None, None, None)

        def nearest_rank(p: float) -> float:
            # rank = max(1, ceil(p * n)), clamped to the last sample (:16-19)
            rank = max(1, int(math.ceil(p * len(s))))
            return s[min(len(s) - 1, rank - 1)]

        mean = 0.0
        for v in s:  # sum in ascending order, as sorted.reduce(0, +)
            mean += v
        return cls(len(s), s[0], s[-1], mean / len(s), nearest_rank(0.50), nearest_rank(0.95))

    def as_dict(self) -> dict:
        return {"samples": self.sample_count, "min_ms": self.minimum_ms,
                "max_ms": self.maximum_ms, "mean_ms": self.mean_ms,
                "p50_ms": self.p50_ms, "p95_ms": self.p95_ms}


class BoundedLatencyAccumulator:
    """Keeps the last `capacity` finite, non-negative samples (the oldest is
    dropped when full)."""

    def __init__(self, capacity: int = 4096):
        self.capacity = max(1, int(capacity))
        self._s: deque[float] = deque()

    def record(self, milliseconds: float) -> None:
        ms = float(milliseconds)
        if not math.isfinite(ms) or ms < 0:
            return
        if len(self._s) == self.capacity:
            self._s.popleft()
        self._s.append(ms)

    def reset(self) -> None:
        self._s.clear()

    @property
    def summary(self) -> LatencySummary:
        return LatencySummary.summarize(self._s)


def cache_requests(metrics: dict) -> int:
    """Demand lookups: hits + misses (prefetches are counted separately)."""
    return int(metrics["hits"]) + int(metrics["misses"])


def cache_hit_rate(metrics: dict) -> float | None:
    """hits / demand lookups, None before the first lookup."""
    r = cache_requests(metrics)
    return None if r == 0 else int(metrics["hits"]) / r
