"""Expert-slot cache over the C ABI: the slot planner, the HBM slot arena with
its pinned-host tier, and the streaming decode step.

Reference behaviour this mirrors (tanishqpatil/qwen-fieldfare):
  - Q4BoundedExpertCache (Sources/QwenFieldfareCore/Storage/Q4BoundedExpertCache.swift):
    per-layer slot partitions, segmented LRU, acquireSlotsParallel,
    speculativePrefetch, metricsSnapshot, layerCapacities, hitRate.
  - QwenActiveStreamingMemoryConfiguration.make
    (Sources/QwenFieldfareCore/Runtime/Generation/QwenActiveStreamingMemoryConfiguration.swift:95-135).
  - the streaming MoE loop of QwenQ4ActiveExpertStreamingRunner.forwardToken
    (QwenQ4ActiveExpertStreamingRunner.swift:958-1381).
The planner is C++ inside libqf_moe.so; the arena is device memory of the
library; records move host -> HBM with one cudaMemcpyAsync each.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import CacheMetrics, MoELayerDesc, QfError, check, lib
from .moe import EXPERTS, RECORD_BYTES, TOPK, MoEContext, MoELayerWeights, StackPlan, _check_x, _ptr

POLICIES = {"slru": 0, "lru": 1}


def _np_ptr(a: np.ndarray):
    return C.c_void_p(a.ctypes.data)


def _ok(status: int, what: str):
    if status != 0:
        raise QfError(status, what)


class ExpertCache:
    """Slot planner of the expert-slot cache (host state only).

    `policy` "slru" is the reference's segmented LRU (default), "lru" one
    least-recently-used order per layer partition."""

    def __init__(self, capacity: int, layer_count: int = 40, probationary_ratio: float = 0.25,
                 policy: str = "slru"):
        h = C.c_void_p()
        _ok(lib().qf_cache_create(capacity, layer_count, probationary_ratio, POLICIES[policy],
                                  C.byref(h)), "qf_cache_create: bad capacity/layers/ratio/policy")
        self.h = h
        self.capacity = capacity
        lc, pc, tc = C.c_int32(), C.c_int32(), C.c_int32()
        _ok(lib().qf_cache_info(h, C.byref(lc), C.byref(pc), C.byref(tc)), "qf_cache_info")
        self.layer_count = lc.value
        self.probationary_capacity = pc.value
        self.protected_capacity = tc.value

    def close(self):
        if getattr(self, "h", None):
            lib().qf_cache_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def acquire_slots_parallel(self, layer: int, experts):
        """(slots, miss_positions, fetches): slots for min(len, 8) experts, the
        positions whose expert is fetched, and the (expert, slot) copies to make."""
        ex = np.ascontiguousarray(experts, np.uint32)
        if ex.size < 1:
            raise ValueError("at least one expert")
        slots = np.zeros(8, np.uint32)
        miss = np.zeros(8, np.uint32)
        fe = np.zeros(8, np.uint32)
        fs = np.zeros(8, np.uint32)
        nm, nf = C.c_int32(), C.c_int32()
        _ok(lib().qf_cache_acquire(self.h, layer, _np_ptr(ex), ex.size, _np_ptr(slots),
                                   _np_ptr(miss), C.byref(nm), _np_ptr(fe), _np_ptr(fs),
                                   C.byref(nf)), "qf_cache_acquire")
        n = min(ex.size, TOPK)
        return (slots[:n].tolist(), miss[:nm.value].tolist(),
                list(zip(fe[:nf.value].tolist(), fs[:nf.value].tolist())))

    def speculative_prefetch(self, layer: int, candidates):
        """(expert, slot) copies placed into free slots of the layer."""
        c = np.ascontiguousarray(candidates, np.uint32)
        fe = np.zeros(max(1, c.size), np.uint32)
        fs = np.zeros(max(1, c.size), np.uint32)
        nf = C.c_int32()
        _ok(lib().qf_cache_prefetch(self.h, layer, _np_ptr(c), c.size, _np_ptr(fe), _np_ptr(fs),
                                    C.byref(nf)), "qf_cache_prefetch")
        return list(zip(fe[:nf.value].tolist(), fs[:nf.value].tolist()))

    def clear(self):
        _ok(lib().qf_cache_clear(self.h), "qf_cache_clear")

    def reset_metrics(self):
        _ok(lib().qf_cache_reset_metrics(self.h), "qf_cache_reset_metrics")

    def metrics_snapshot(self) -> dict:
        m = CacheMetrics()
        _ok(lib().qf_cache_get_metrics(self.h, C.byref(m)), "qf_cache_get_metrics")
        return {name: getattr(m, name) for name, _ in CacheMetrics._fields_}

    @property
    def hit_rate(self) -> float:
        m = self.metrics_snapshot()
        req = m["hits"] + m["misses"]
        return m["hits"] / req if req else 0.0

    def layer_metrics(self):
        """(hits, requests) per layer since the last reset: the reference cache's
        layerHits / layerRequests (Q4BoundedExpertCache.swift:49-50)."""
        hits = np.zeros(self.layer_count, np.int64)
        req = np.zeros(self.layer_count, np.int64)
        _ok(lib().qf_cache_layer_metrics(self.h, _np_ptr(hits), _np_ptr(req)),
            "qf_cache_layer_metrics")
        return hits, req

    def layer_hit_rates(self):
        """Per-layer hit rate in percent, 0 for a layer without requests (the
        bench report's "Layer cache hit rates", main.swift:799-805)."""
        hits, req = self.layer_metrics()
        return [float(h) * 100.0 / float(r) if r > 0 else 0.0 for h, r in zip(hits, req)]

    def layer_ranges(self):
        first = np.zeros(self.layer_count, np.int32)
        count = np.zeros(self.layer_count, np.int32)
        _ok(lib().qf_cache_layer_slots(self.h, _np_ptr(first), _np_ptr(count)),
            "qf_cache_layer_slots")
        return [(int(f), int(f + n)) for f, n in zip(first, count)]

    @property
    def layer_capacities(self):
        return [b - a for a, b in self.layer_ranges()]


def plan_slots(budget_gib: int, context_length: int) -> dict:
    """Expert slots that fit in `budget_gib` GiB next to the rest of the
    streaming runtime at `context_length` tokens.  Raises (like the reference's
    insufficientBudget) when fewer than 40 * 8 slots fit."""
    s, est, tgt = C.c_int64(), C.c_uint64(), C.c_uint64()
    st = lib().qf_cache_plan_slots(budget_gib, context_length, C.byref(s), C.byref(est),
                                   C.byref(tgt))
    if st not in (0, -4):
        raise QfError(st, "qf_cache_plan_slots: bad budget or context length")
    if st == -4:
        raise QfError(st, f"budget of {budget_gib} GiB leaves {s.value} expert slots; 320 needed")
    return {"slots": s.value, "estimated_bytes": est.value, "target_bytes": tgt.value}


class HostTier:
    """HBM slot arena of `slots` records on `device`, filled from host records
    (a uint8 CPU tensor [n, >= RECORD_BYTES], pinned for asynchronous copies)."""

    def __init__(self, device: int, slots: int, host_records: torch.Tensor):
        if host_records.device.type != "cpu" or host_records.dtype != torch.uint8 or \
                host_records.dim() != 2 or host_records.shape[1] < RECORD_BYTES or \
                host_records.stride(1) != 1:
            raise ValueError("host_records must be a uint8 CPU tensor [n, >= 1769472]")
        self.host_records = host_records  # keeps the memory alive
        h = C.c_void_p()
        _ok(lib().qf_tier_create(device, slots, C.c_void_p(host_records.data_ptr()),
                                 host_records.shape[0], host_records.stride(0), C.byref(h)),
            "qf_tier_create")
        self.h = h
        self.slots = slots
        bank, stride = C.c_void_p(), C.c_uint64()
        _ok(lib().qf_tier_arena(h, C.byref(bank), C.byref(stride)), "qf_tier_arena")
        self.arena_ptr = bank.value
        self.arena_stride = stride.value

    def close(self):
        if getattr(self, "h", None):
            lib().qf_tier_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def fetch(self, host_index, slots, stream: torch.cuda.Stream | None = None):
        hi = np.ascontiguousarray(host_index, np.int64)
        sl = np.ascontiguousarray(slots, np.uint32)
        if hi.size != sl.size:
            raise ValueError("host_index and slots differ in length")
        st = C.c_void_p(stream.cuda_stream) if stream is not None else \
            C.c_void_p(torch.cuda.current_stream().cuda_stream)
        _ok(lib().qf_tier_fetch(self.h, _np_ptr(hi), _np_ptr(sl), hi.size, st), "qf_tier_fetch")

    def stats(self):
        n, b, f = C.c_int64(), C.c_int64(), C.c_int64()
        _ok(lib().qf_tier_stats(self.h, C.byref(n), C.byref(b)), "qf_tier_stats")
        _ok(lib().qf_tier_failed_copies(self.h, C.byref(f)), "qf_tier_failed_copies")
        return {"copies": n.value, "bytes": b.value, "failed": f.value}

    def inject_fault(self, skip: int, count: int):
        """After `skip` more record copies, treat the next `count` as short copies
        (host-side fault injection for failure-detection tests)."""
        _ok(lib().qf_tier_inject_fault(self.h, skip, count), "qf_tier_inject_fault")

    def synchronize(self):
        _ok(lib().qf_tier_synchronize(self.h), "qf_tier_synchronize")

    def bank_desc_fields(self):
        """(expert_bank pointer, record_stride, bank_records) of the arena."""
        return self.arena_ptr, self.arena_stride, self.slots


class ArenaLayer:
    """A layer whose routed records are read from a tier's slot arena (pass it
    to block_forward with record_of_pos = the cache's slots)."""

    def __init__(self, layer: MoELayerWeights, tier: HostTier):
        self.layer = layer
        self.tier = tier

    def desc(self) -> MoELayerDesc:
        d = self.layer.desc()
        d.expert_bank, d.record_stride, d.bank_records = self.tier.bank_desc_fields()
        return d


def stream_step(ctx: MoEContext, cache: ExpertCache, tier: HostTier, plan: StackPlan,
                host_idx: np.ndarray, host_w: np.ndarray, x: torch.Tensor,
                residual: torch.Tensor | None, out: torch.Tensor, eps: float = 1e-6,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """One batch-1 decode step through all layers of `plan` with routed experts
    read from the cache's slots.  host_idx / host_w: [n_layers, 8] host arrays."""
    _check_x(x)
    if x.shape[0] != 1:
        raise ValueError("the streaming step is batch-1")
    n = len(plan.layers)
    idx = np.ascontiguousarray(host_idx, np.int32).reshape(-1)
    w = np.ascontiguousarray(host_w, np.float32).reshape(-1)
    if idx.size != n * TOPK or w.size != n * TOPK:
        raise ValueError("host_idx / host_w must hold n_layers * 8 entries")
    ws = workspace if workspace is not None else ctx.workspace(1)
    ctx._bind_stream()
    check(lib().qf_moe_stream_step(ctx.h, cache.h, tier.h, plan.arr, n, _np_ptr(idx), _np_ptr(w),
                                   _ptr(x), _ptr(residual), _ptr(out), eps, _ptr(ws), ws.numel()),
          ctx.h)
    return out


__all__ = ["ArenaLayer", "ExpertCache", "HostTier", "plan_slots", "stream_step"]
