"""ctypes front end of the CPU oracle (oracle/qf_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the
checker, and by bench.py's cpu_baseline / ``--impl reference`` legs.  The
product package (qwen-fieldfare_b200/qfmoe) never imports this module.

The oracle restates the reference's Metal kernel arithmetic
(Sources/QwenFieldfareCore/Metal/LinearAttention/deltanet.metal) and its
expert-cache planner (Sources/QwenFieldfareCore/Storage/Q4BoundedExpertCache.swift)
in C; see qf_oracle.h for the line-by-line map.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "libqf_oracle.so")

HIDDEN, EXPERTS, TOPK, INTER = 2048, 256, 8, 512
RECORD_BYTES = 1_769_472
SHARED_EXPERT = 256

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


_p = C.c_void_p
_i = C.c_int
_u64 = C.c_uint64


def _declare(L):
    L.qfo_f16_to_f32.argtypes = [C.c_uint16]
    L.qfo_f16_to_f32.restype = C.c_float
    L.qfo_f32_to_f16.argtypes = [C.c_float]
    L.qfo_f32_to_f16.restype = C.c_uint16
    L.qfo_synth_expert_record.argtypes = [_u64, C.c_uint32, C.c_uint32, _i, _p]
    L.qfo_synth_router.argtypes = [_u64, C.c_uint32, _i, _p, _p, _p]
    L.qfo_synth_coef.argtypes = [_u64, C.c_uint32, _i, _p, _p, _p]
    L.qfo_synth_hidden.argtypes = [_u64, _u64, _i, _p]
    L.qfo_topk.argtypes = [_p, _p, _i, _i, _p, _p]
    L.qfo_router_logits.argtypes = [_p, _p, _p]
    L.qfo_coef.argtypes = [_p, _p]
    L.qfo_coef.restype = C.c_float
    L.qfo_block.argtypes = [_p, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i]
    L.qfo_rmsnorm_to_f16.argtypes = [_p, _i, C.c_float, _p]
    L.qfo_dispatch_plan.argtypes = [_p, _i, _i, _i, _p, _p, _p]
    L.qfo_cache_create.argtypes = [_i, C.c_double, _i, _i, _i]
    L.qfo_cache_create.restype = _p
    L.qfo_cache_destroy.argtypes = [_p]
    L.qfo_cache_acquire.argtypes = [_p, _i, _p, _i, _p, _p, _p, _p, _p, _p]
    L.qfo_cache_acquire.restype = _i
    L.qfo_cache_prefetch.argtypes = [_p, _i, _p, _i]
    L.qfo_cache_clear.argtypes = [_p]
    L.qfo_cache_reset_metrics.argtypes = [_p]
    L.qfo_cache_metrics.argtypes = [_p, _p]
    L.qfo_cache_layer_count.argtypes = [_p]
    L.qfo_cache_layer_count.restype = _i
    L.qfo_cache_layer_capacities.argtypes = [_p, _p]
    L.qfo_cache_probationary_capacity.argtypes = [_p]
    L.qfo_cache_probationary_capacity.restype = _i
    L.qfo_slru_replay.argtypes = [_p, C.c_int64, _i]
    L.qfo_slru_replay.restype = C.c_int64
    L.qfo_gate_up.argtypes = [_p, _i, _p, _p]
    L.qfo_down.argtypes = [_p, _i, _p, _p]
    L.qfo_combine.argtypes = [_p, _p, _p, C.c_float, _p, _p]
    L.qfo_lm_head.argtypes = [_p, _p, _p, _i, _p, _i, _p]
    L.qfo_post_norm_to_f16.argtypes = [_p, _p, _i, C.c_float, _p]


def _ptr(a):
    return None if a is None else a.ctypes.data


# ---------------------------------------------------------------- synthetic data
def synth_record(seed: int, layer: int, expert: int, bf16: bool = False) -> np.ndarray:
    rec = np.empty(RECORD_BYTES, np.uint8)
    lib().qfo_synth_expert_record(seed, layer, expert, int(bf16), _ptr(rec))
    return rec


def synth_router(seed: int, layer: int, bf16: bool = False):
    w = np.empty(EXPERTS * HIDDEN, np.uint8)
    s = np.empty(EXPERTS * 32, np.uint16)
    b = np.empty(EXPERTS * 32, np.uint16)
    lib().qfo_synth_router(seed, layer, int(bf16), _ptr(w), _ptr(s), _ptr(b))
    return w, s, b


def synth_coef(seed: int, layer: int, bf16: bool = False):
    w = np.empty(HIDDEN, np.uint8)
    s = np.empty(32, np.uint16)
    b = np.empty(32, np.uint16)
    lib().qfo_synth_coef(seed, layer, int(bf16), _ptr(w), _ptr(s), _ptr(b))
    return w, s, b


def synth_hidden(seed: int, tok0: int, T: int) -> np.ndarray:
    x = np.empty((T, HIDDEN), np.uint16)
    lib().qfo_synth_hidden(seed, tok0, T, _ptr(x))
    return x


# ---------------------------------------------------------------- layer + block
class QfoLayer(C.Structure):
    _fields_ = [
        ("router_w", _p), ("router_s", _p), ("router_b", _p),
        ("coef_w", _p), ("coef_s", _p), ("coef_b", _p),
        ("shared_record", _p), ("expert_records", _p), ("scale_bf16", _i),
    ]


class OracleLayer:
    """Host copy of one MoE layer's weights, in the product's byte layout."""

    def __init__(self, router, coef, shared_record, expert_records, bf16=False):
        self.router = [np.ascontiguousarray(a) for a in router]
        self.coef = [np.ascontiguousarray(a) for a in coef]
        self.shared = np.ascontiguousarray(shared_record)
        # expert_records: dict expert -> uint8[RECORD_BYTES] or a [256, RECORD_BYTES] array
        self._keep = []
        ptrs = (C.c_void_p * EXPERTS)()
        for e in range(EXPERTS):
            rec = expert_records.get(e) if isinstance(expert_records, dict) else expert_records[e]
            if rec is not None:
                rec = np.ascontiguousarray(rec)
                self._keep.append(rec)
                ptrs[e] = rec.ctypes.data
        self._ptrs = ptrs
        self.bf16 = bf16
        self.c = QfoLayer(
            _ptr(self.router[0]), _ptr(self.router[1]), _ptr(self.router[2]),
            _ptr(self.coef[0]), _ptr(self.coef[1]), _ptr(self.coef[2]),
            _ptr(self.shared), C.cast(ptrs, C.c_void_p), int(bf16),
        )

    @classmethod
    def synth(cls, seed, layer, experts=None, bf16=False):
        experts = range(EXPERTS) if experts is None else experts
        recs = {e: synth_record(seed, layer, e, bf16) for e in experts}
        return cls(synth_router(seed, layer, bf16), synth_coef(seed, layer, bf16),
                   synth_record(seed, layer, SHARED_EXPERT, bf16), recs, bf16)


def block(layer: OracleLayer, x16: np.ndarray, residual=None, bias=None, idx_in=None, w_in=None,
          threads: int = 0):
    """Returns dict(out, idx, w, logits, coef) for T tokens of fp16 bits x16 [T, 2048]."""
    x16 = np.ascontiguousarray(x16, np.uint16).reshape(-1, HIDDEN)
    T = x16.shape[0]
    out = np.empty((T, HIDDEN), np.float32)
    idx = np.empty((T, TOPK), np.int32)
    w = np.empty((T, TOPK), np.float32)
    logits = np.empty((T, EXPERTS), np.float32)
    coef = np.empty(T, np.float32)
    res = None if residual is None else np.ascontiguousarray(residual, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    ii = None if idx_in is None else np.ascontiguousarray(idx_in, np.int32)
    wi = None if w_in is None else np.ascontiguousarray(w_in, np.float32)
    lib().qfo_block(C.byref(layer.c), T, _ptr(x16), _ptr(res), _ptr(b), _ptr(ii), _ptr(wi),
                    _ptr(out), _ptr(idx), _ptr(w), _ptr(logits), _ptr(coef), threads)
    return {"out": out, "idx": idx, "w": w, "logits": logits, "coef": coef}


def router(layer: OracleLayer, x16: np.ndarray):
    """(logits [T, 256], coef [T]) of fp16 bits x16 [T, 2048]: the router rows in the
    reference lane order (qfo_router_logits) and the shared-gate chain (qfo_coef)."""
    x = np.ascontiguousarray(x16, np.uint16).reshape(-1, HIDDEN).view(np.float16).astype(np.float32)
    T = x.shape[0]
    logits = np.empty((T, EXPERTS), np.float32)
    coef = np.empty(T, np.float32)
    L = lib()
    for t in range(T):
        L.qfo_router_logits(C.byref(layer.c), _ptr(x[t]), _ptr(logits[t]))
        coef[t] = L.qfo_coef(C.byref(layer.c), _ptr(x[t]))
    return logits, coef


def topk(logits: np.ndarray, k: int = TOPK, bias=None):
    logits = np.ascontiguousarray(logits, np.float32).reshape(-1, logits.shape[-1])
    n = logits.shape[1]
    idx = np.empty((logits.shape[0], k), np.int32)
    w = np.empty((logits.shape[0], k), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    for t in range(logits.shape[0]):
        lib().qfo_topk(logits[t].ctypes.data, _ptr(b), n, k, idx[t].ctypes.data, w[t].ctypes.data)
    return idx, w


def expert_ffn(record: np.ndarray, x16: np.ndarray, bf16: bool = False) -> np.ndarray:
    """y = D . (SiLU(G x) * (U x)) of one expert record for one fp16 token row
    (qfo_gate_up then qfo_down, reference order)."""
    x = np.ascontiguousarray(x16, np.uint16).view(np.float16).astype(np.float32)
    act = np.empty(INTER, np.float32)
    y = np.empty(HIDDEN, np.float32)
    rec = np.ascontiguousarray(record, np.uint8)
    lib().qfo_gate_up(_ptr(rec), int(bf16), _ptr(x), _ptr(act))
    lib().qfo_down(_ptr(rec), int(bf16), _ptr(act), _ptr(y))
    return y


def combine(y8: np.ndarray, w8: np.ndarray, sh_y: np.ndarray, coef: float, residual=None):
    """One token's combine: (residual + sigmoid(coef) * sh_y) + sum_k w_k y_k in router order."""
    y8 = np.ascontiguousarray(y8, np.float32)
    w8 = np.ascontiguousarray(w8, np.float32)
    sh = np.ascontiguousarray(sh_y, np.float32)
    res = None if residual is None else np.ascontiguousarray(residual, np.float32)
    out = np.empty(HIDDEN, np.float32)
    lib().qfo_combine(_ptr(y8), _ptr(w8), _ptr(sh), float(coef), _ptr(res), _ptr(out))
    return out


def rmsnorm_to_f16(h: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    h = np.ascontiguousarray(h, np.float32).reshape(-1, HIDDEN)
    x = np.empty(h.shape, np.uint16)
    lib().qfo_rmsnorm_to_f16(_ptr(h), h.shape[0], eps, _ptr(x))
    return x


def dispatch_plan(idx: np.ndarray, n_experts: int = EXPERTS):
    idx = np.ascontiguousarray(idx, np.int32)
    T, k = idx.shape
    counts = np.empty(n_experts, np.int32)
    offsets = np.empty(n_experts + 1, np.int32)
    perm = np.empty(T * k, np.int32)
    lib().qfo_dispatch_plan(_ptr(idx), T, k, n_experts, _ptr(counts), _ptr(offsets), _ptr(perm))
    return counts, offsets, perm


def f16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(bits, np.uint16).view(np.float16).astype(np.float32)


# ---------------------------------------------------------------- expert cache port
class OracleCache:
    """Exact port of Q4BoundedExpertCache's planner (host state only; no arena)."""

    def __init__(self, capacity, probationary_ratio=0.25, layer_count=40, key_layers=64,
                 key_experts=512):
        self.h = lib().qfo_cache_create(capacity, probationary_ratio, layer_count, key_layers,
                                        key_experts)

    def __del__(self):
        if getattr(self, "h", None):
            lib().qfo_cache_destroy(self.h)
            self.h = None

    def acquire(self, layer, experts):
        ex = np.ascontiguousarray(experts, np.uint32)
        slots = np.zeros(8, np.uint32)
        miss = np.zeros(8, np.uint32)
        fe = np.zeros(8, np.uint32)
        fs = np.zeros(8, np.uint32)
        nm = C.c_int()
        nf = C.c_int()
        n = lib().qfo_cache_acquire(self.h, layer, _ptr(ex), len(ex), _ptr(slots), _ptr(miss),
                                    C.byref(nm), _ptr(fe), _ptr(fs), C.byref(nf))
        return (slots[:n].tolist(), miss[:nm.value].tolist(),
                list(zip(fe[:nf.value].tolist(), fs[:nf.value].tolist())))

    def prefetch(self, layer, cands):
        c = np.ascontiguousarray(cands, np.uint32)
        lib().qfo_cache_prefetch(self.h, layer, _ptr(c), len(c))

    def clear(self):
        lib().qfo_cache_clear(self.h)

    def reset_metrics(self):
        lib().qfo_cache_reset_metrics(self.h)

    def metrics(self):
        m = np.zeros(11, np.int64)
        lib().qfo_cache_metrics(self.h, _ptr(m))
        keys = ["capacity", "occupancy", "probationary_occupancy", "protected_occupancy", "hits",
                "misses", "evictions", "fetched_bytes", "prefetch_requests",
                "useful_prefetch_hits", "wasted_prefetches"]
        return dict(zip(keys, m.tolist()))

    @property
    def layer_count(self):
        return lib().qfo_cache_layer_count(self.h)

    def layer_capacities(self):
        out = np.zeros(self.layer_count, np.int32)
        lib().qfo_cache_layer_capacities(self.h, _ptr(out))
        return out.tolist()

    @property
    def probationary_capacity(self):
        return lib().qfo_cache_probationary_capacity(self.h)


def slru_replay(trace, capacity: int) -> int:
    t = np.ascontiguousarray(trace, np.uint16)
    return int(lib().qfo_slru_replay(_ptr(t), len(t), capacity))


# ---------------------------------------------------------------- plain-LRU policy
class OracleLRU:
    """Per-layer least-recently-used slot cache: the "LRU eviction" policy of
    the cached-decode benchmark configuration, restated with the partitioning
    and tie rules of Q4BoundedExpertCache (Storage/Q4BoundedExpertCache.swift:
    slot ranges :64-123, victim search :253-297 with the protected segment
    never used): a miss takes the lowest empty slot of the layer, else the
    unlocked slot with the oldest access tick (lowest slot on ties); slots
    returned earlier in the same acquire are locked.  Pure Python, small cases."""

    def __init__(self, capacity, layer_count=40):
        ref = OracleCache(capacity, 0.25, layer_count)
        caps = ref.layer_capacities()
        self.ranges = []
        start = 0
        for c in caps:
            self.ranges.append((start, start + c))
            start += c
        self.key = [None] * capacity
        self.tick_of = [0] * capacity
        self.where = {}
        self.tick = 0
        self.hits = self.misses = self.evictions = 0

    def acquire(self, layer, experts):
        lo, hi = self.ranges[min(max(layer, 0), len(self.ranges) - 1)]
        self.tick += 1
        locked = set()
        slots, fetches = [], []
        for e in list(experts)[:8]:
            k = (layer, int(e))
            s = self.where.get(k)
            if s is not None:
                self.hits += 1
                self.tick_of[s] = self.tick
            else:
                self.misses += 1
                free = [t for t in range(lo, hi) if self.key[t] is None and t not in locked]
                if free:
                    s = free[0]
                else:
                    cand = [(self.tick_of[t], t) for t in range(lo, hi) if t not in locked]
                    s = min(cand)[1] if cand else 0
                    del self.where[self.key[s]]
                    self.evictions += 1
                self.key[s] = k
                self.where[k] = s
                self.tick_of[s] = self.tick
                fetches.append((int(e), s))
            locked.add(s)
            slots.append(s)
        return slots, fetches


# ---------------------------------------------------------------- slot budget
GIB = 1_073_741_824


def plan_slots(budget_gib: int, context_length: int):
    """QwenActiveStreamingMemoryConfiguration.make
    (Runtime/Generation/QwenActiveStreamingMemoryConfiguration.swift:95-135,
    constants :56-93; DenseLayerArena.totalByteLength = 22,456,448 at
    QwenQ4ActiveExpertStreamingRunner.swift:9).  Returns (slots, estimated,
    target, ok) with ok False where the reference throws insufficientBudget."""
    layers, full, linear = 40, 10, 30
    dense = layers * 22_456_448
    recurrent = linear * (8192 * 4 * 4 + 32 * 128 * 128 * 4)
    constants = (2048 * 4 + layers * 2 * 2048 * 4
                 + linear * (8192 * 4 * 4 + 32 * 4 + 32 * 4 + 128 * 4) + full * 2 * 256 * 4)
    fixed = dense + recurrent + constants + 1_341_348 + 366_570_000
    kv = full * 2 * 2 * 256 * 2 * context_length
    scratch = 16 * 4 * context_length
    non_cache = fixed + kv + scratch
    target = budget_gib * GIB
    slots = max(0, target - non_cache) // RECORD_BYTES
    return slots, non_cache + slots * RECORD_BYTES, target, slots >= layers * 8


def lm_head(w: np.ndarray, s: np.ndarray, b: np.ndarray, x: np.ndarray, bf16: bool = False) -> np.ndarray:
    """Q4 LM-head logits of one fp32 token row (qfo_lm_head, reference order):
    w uint8 [rows, 1024], s/b uint16 bits [rows, 32], x float32 [2048]."""
    w = np.ascontiguousarray(w, np.uint8)
    s = np.ascontiguousarray(s, np.uint16)
    b = np.ascontiguousarray(b, np.uint16)
    x = np.ascontiguousarray(x, np.float32)
    rows = w.shape[0]
    assert w.shape == (rows, 1024) and s.shape == (rows, 32) and b.shape == (rows, 32) and x.shape == (2048,)
    out = np.empty(rows, np.float32)
    lib().qfo_lm_head(_ptr(w), _ptr(s), _ptr(b), rows, _ptr(x), int(bf16), _ptr(out))
    return out


def post_norm_f16(h: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """The post-attention RMSNorm of fp32 rows [T, 2048] with weight w [2048],
    in qwen_rmsnorm_f32's 64-thread order, as fp16 bits (qfo_post_norm_to_f16)."""
    h = np.ascontiguousarray(h, np.float32).reshape(-1, HIDDEN)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty(h.shape, np.uint16)
    lib().qfo_post_norm_to_f16(_ptr(h), _ptr(w), h.shape[0], float(eps), _ptr(out))
    return out
