// qf_cache.cu -- expert-slot cache: the host-side slot planner and the HBM
// slot arena with a pinned-host tier.
//
// Policy: Q4BoundedExpertCache (Sources/QwenFieldfareCore/Storage/
// Q4BoundedExpertCache.swift:52-365), a segmented LRU partitioned by layer so
// that one layer's misses never evict another layer's experts:
//   - slot ranges per layer: eight slots each plus the remainder split by the
//     measured per-layer weights when there are 40 layers (:70-112), evenly
//     otherwise (:113-123), one global range for caches smaller than 8 per
//     layer (:64-67);
//   - a hit refreshes the slot's tick and promotes a probationary slot to
//     protected, demoting the layer's least recently used unlocked protected
//     slot when the layer holds more than its protected share (:222-246);
//   - a miss takes the first empty unlocked slot of the layer, else the least
//     recently used probationary one, else the least recently used protected
//     one, else the first unlocked one (:253-297);
//   - acquire plans all eight positions before any fetch and reports the miss
//     positions (acquireSlotsParallel, :330-365).
// QF_CACHE_LRU replaces the segments by one least-recently-used order per
// layer (the "LRU eviction" of the streaming benchmark).
//
// Slot budget: QwenActiveStreamingMemoryConfiguration.make
// (Sources/QwenFieldfareCore/Runtime/Generation/
// QwenActiveStreamingMemoryConfiguration.swift:95-135).
//
// Tier: the slot arena lives in HBM; missing records are copied from pinned
// host memory with one cudaMemcpyAsync per record on the tier's own stream,
// and the consumer stream waits on an event recorded after the copies, in
// place of the reference's parallel pread of the packed expert store.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/qf_moe.h"
#include "qf_handle.h"
#include "qf_internal.h"

namespace {

constexpr int kTopKSlots = 8;  // router top-8: slots locked per layer
constexpr uint64_t kRecord = qf::kRecordBytes;

// per-layer excess weights for 40 layers (Q4BoundedExpertCache.swift:76-81)
constexpr int kLayerWeights40[40] = {86, 82, 78, 72, 64, 58, 54, 48, 35, 42, 58, 59, 45, 48,
                                     38, 43, 45, 41, 42, 38, 34, 37, 53, 55, 43, 45, 38, 41,
                                     46, 41, 43, 40, 48, 54, 55, 42, 45, 47, 51, 66};

enum Segment : uint8_t { kEmpty = 0, kProbationary = 1, kProtected = 2 };

uint64_t key_of(int32_t layer, uint32_t expert) {
  return (static_cast<uint64_t>(static_cast<uint32_t>(layer)) << 32) | expert;
}

}  // namespace

struct qf_cache {
  int capacity = 0;
  int layer_count = 1;
  int prob_capacity = 0;
  int prot_capacity = 0;
  int policy = QF_CACHE_SLRU;
  std::vector<int> range_first, range_count;
  // per slot
  std::vector<uint64_t> slot_key;
  std::vector<uint8_t> slot_seg;
  std::vector<uint64_t> slot_tick;
  std::vector<uint64_t> lock_gen;  // slot is locked while lock_gen == gen
  uint64_t gen = 0;
  std::unordered_map<uint64_t, int> key_slot;
  std::unordered_map<uint64_t, int> prefetched;  // key -> 1
  uint64_t tick = 0;
  qf_cache_metrics_t m{};
  // demand hits / lookups per layer partition (Q4BoundedExpertCache.layerHits /
  // layerRequests, Q4BoundedExpertCache.swift:49-50, 205, 216); reset with m
  std::vector<int64_t> layer_hits, layer_requests;
  std::string err;

  void build_ranges(int requested_layers) {
    const int want = std::max(1, requested_layers);
    layer_count = capacity >= want * kTopKSlots ? want : 1;
    range_first.assign(layer_count, 0);
    layer_hits.assign(layer_count, 0);
    layer_requests.assign(layer_count, 0);
    range_count.assign(layer_count, 0);
    if (layer_count == 40) {
      const int remaining = capacity - layer_count * kTopKSlots;
      int excess_total = 0;
      for (int w : kLayerWeights40) excess_total += w - kTopKSlots;
      int used = 0;
      std::vector<std::pair<int64_t, int>> rem(40);
      for (int l = 0; l < 40; l++) {
        const int64_t prod = static_cast<int64_t>(remaining) * (kLayerWeights40[l] - kTopKSlots);
        range_count[l] = kTopKSlots + static_cast<int>(prod / excess_total);
        used += range_count[l];
        rem[l] = {prod % excess_total, l};
      }
      // largest remainders first, ties to the lower layer
      std::stable_sort(rem.begin(), rem.end(),
                       [](const std::pair<int64_t, int>& a, const std::pair<int64_t, int>& b) {
                         return a.first > b.first;
                       });
      for (int i = 0; used < capacity; i++, used++) range_count[rem[i].second] += 1;
    } else if (layer_count > 1) {
      for (int l = 0; l < layer_count; l++)
        range_count[l] = capacity / layer_count + (l < capacity % layer_count ? 1 : 0);
    } else {
      range_count[0] = capacity;
    }
    int start = 0;
    for (int l = 0; l < layer_count; l++) {
      range_first[l] = start;
      start += range_count[l];
    }
  }

  int layer_of(int32_t layer) const { return std::min(std::max(0, layer), layer_count - 1); }

  void clear() {
    std::fill(slot_key.begin(), slot_key.end(), 0);
    std::fill(slot_seg.begin(), slot_seg.end(), kEmpty);
    std::fill(slot_tick.begin(), slot_tick.end(), 0);
    key_slot.clear();
    prefetched.clear();
    tick = 0;
  }

  bool locked(int s) const { return lock_gen[s] == gen; }

  // least recently used unlocked slot of segment seg in [a, b), or -1
  int lru_in(int a, int b, uint8_t seg) const {
    uint64_t best = UINT64_MAX;
    int victim = -1;
    for (int s = a; s < b; s++)
      if (slot_seg[s] == seg && !locked(s) && slot_tick[s] < best) {
        best = slot_tick[s];
        victim = s;
      }
    return victim;
  }

  // The occupant a miss displaced, kept so that a failed copy can give the slot
  // back: the slot's bytes are still that occupant's.
  struct Undo {
    int slot;
    uint64_t old_key, old_tick;
    uint8_t old_seg;
  };

  // A record copy into `u.slot` failed: the fetched expert is not resident; the
  // slot holds (and is mapped to) its previous occupant again, as before the
  // acquire; the miss stays counted (the lookup did miss), the eviction and the
  // fetched bytes are taken back.
  void undo_fetch(const Undo& u) {
    const int s = u.slot;
    if (slot_seg[s] != kEmpty) key_slot.erase(slot_key[s]);
    m.fetched_bytes -= static_cast<int64_t>(kRecord);
    slot_key[s] = u.old_key;
    slot_seg[s] = u.old_seg;
    slot_tick[s] = u.old_tick;
    if (u.old_seg != kEmpty) {
      key_slot[u.old_key] = s;
      m.evictions -= 1;
    }
  }

  int acquire(int32_t layer, const uint32_t* experts, int n, uint32_t* slots, uint32_t* miss_pos,
              int* n_miss, uint32_t* fetch_expert, uint32_t* fetch_slot, int* n_fetch,
              Undo* undo = nullptr) {
    const int np = std::min(n, kTopKSlots);
    const int L = layer_of(layer);
    const int a = range_first[L], b = a + range_count[L];
    const int layer_prot_cap = std::max(
        kTopKSlots, static_cast<int>(static_cast<double>(range_count[L]) * static_cast<double>(prot_capacity) /
                                     static_cast<double>(capacity)));
    tick += 1;
    gen += 1;
    int nf = 0;
    uint32_t fetched_experts[kTopKSlots];
    for (int p = 0; p < np; p++) {
      const uint64_t key = key_of(layer, experts[p]);
      auto pf = prefetched.find(key);
      if (pf != prefetched.end()) {
        m.useful_prefetch_hits += 1;
        prefetched.erase(pf);
      }
      auto it = key_slot.find(key);
      layer_requests[L] += 1;
      if (it != key_slot.end()) {
        const int s = it->second;
        m.hits += 1;
        layer_hits[L] += 1;
        slot_tick[s] = tick;
        lock_gen[s] = gen;
        slots[p] = static_cast<uint32_t>(s);
        if (policy == QF_CACHE_SLRU && slot_seg[s] == kProbationary) {
          slot_seg[s] = kProtected;
          int prot = 0;
          for (int q = a; q < b; q++) prot += slot_seg[q] == kProtected;
          if (prot > layer_prot_cap) {
            const int d = lru_in(a, b, kProtected);
            if (d >= 0) slot_seg[d] = kProbationary;
          }
        }
        continue;
      }
      m.misses += 1;
      int victim = -1;
      for (int s = a; s < b; s++)
        if (slot_seg[s] == kEmpty && !locked(s)) {
          victim = s;
          break;
        }
      if (victim < 0) {
        if (policy == QF_CACHE_SLRU) {
          victim = lru_in(a, b, kProbationary);
          if (victim < 0) victim = lru_in(a, b, kProtected);
        } else {
          victim = lru_in(a, b, kProbationary);
        }
      }
      if (victim < 0)
        for (int s = a; s < b; s++)
          if (!locked(s)) {
            victim = s;
            break;
          }
      if (victim < 0) victim = 0;
      if (undo) undo[nf] = Undo{victim, slot_key[victim], slot_tick[victim], slot_seg[victim]};
      if (slot_seg[victim] != kEmpty) {
        const uint64_t old = slot_key[victim];
        auto op = prefetched.find(old);
        if (op != prefetched.end()) {
          m.wasted_prefetches += 1;
          prefetched.erase(op);
        }
        key_slot.erase(old);
        m.evictions += 1;
      }
      m.fetched_bytes += static_cast<int64_t>(kRecord);
      key_slot[key] = victim;
      slot_key[victim] = key;
      slot_tick[victim] = tick;
      slot_seg[victim] = kProbationary;  // LRU policy: every occupied slot is "probationary"
      lock_gen[victim] = gen;
      slots[p] = static_cast<uint32_t>(victim);
      if (fetch_expert) fetch_expert[nf] = experts[p];
      if (fetch_slot) fetch_slot[nf] = static_cast<uint32_t>(victim);
      fetched_experts[nf] = experts[p];
      nf++;
    }
    int nm = 0;
    for (int p = 0; p < np; p++) {
      bool missed = false;
      for (int f = 0; f < nf; f++) missed = missed || fetched_experts[f] == experts[p];
      if (missed && miss_pos) miss_pos[nm] = static_cast<uint32_t>(p);
      nm += missed;
    }
    if (n_miss) *n_miss = nm;
    if (n_fetch) *n_fetch = nf;
    return np;
  }

  int prefetch(int32_t layer, const uint32_t* cands, int n, uint32_t* fetch_expert, uint32_t* fetch_slot) {
    const int L = layer_of(layer);
    const int a = range_first[L], b = a + range_count[L];
    bool any_free = false;
    for (int s = a; s < b; s++) any_free = any_free || slot_seg[s] == kEmpty;
    if (!any_free) return 0;
    int nf = 0;
    for (int c = 0; c < n; c++) {
      const uint64_t key = key_of(layer, cands[c]);
      if (key_slot.count(key)) continue;
      int free_slot = -1;
      for (int s = a; s < b; s++)
        if (slot_seg[s] == kEmpty) {
          free_slot = s;
          break;
        }
      if (free_slot < 0) break;
      m.fetched_bytes += static_cast<int64_t>(kRecord);
      key_slot[key] = free_slot;
      slot_key[free_slot] = key;
      slot_tick[free_slot] = tick;
      slot_seg[free_slot] = kProbationary;
      prefetched[key] = 1;
      m.prefetch_requests += 1;
      if (fetch_expert) fetch_expert[nf] = cands[c];
      if (fetch_slot) fetch_slot[nf] = static_cast<uint32_t>(free_slot);
      nf++;
    }
    return nf;
  }

  void snapshot(qf_cache_metrics_t* out) const {
    *out = m;
    out->capacity = capacity;
    out->occupancy = static_cast<int64_t>(key_slot.size());
    int64_t prob = 0, prot = 0;
    for (uint8_t s : slot_seg) {
      prob += s == kProbationary;
      prot += s == kProtected;
    }
    out->probationary_occupancy = prob;
    out->protected_occupancy = prot;
  }
};

// Steps of qf_moe_stream_step that may be in flight at once; the host waits for
// step n - kStepRing before it plans step n.
constexpr int kStepRing = 4;

struct qf_tier {
  int device = 0;
  int slots = 0;
  uint8_t* arena = nullptr;
  const uint8_t* host = nullptr;
  int64_t host_records = 0;
  uint64_t host_stride = 0;
  cudaStream_t side = nullptr;
  cudaEvent_t done = nullptr;
  int64_t copies = 0;
  int64_t bytes = 0;
  // host-side fault injection: after `inject_skip` more record copies, the next
  // `inject_count` are treated as short copies (not issued); failed_copies
  // counts every record copy that failed
  int64_t inject_skip = 0, inject_count = 0;
  int64_t failed_copies = 0;
  // streaming steps: the last step whose kernel reads each slot, an event
  // recorded after each step's kernel, and per-step routing staging
  std::vector<int64_t> slot_last_step;
  int64_t step = -1;
  cudaEvent_t step_done[kStepRing] = {};
  int stage_layers = 0;
  int32_t* stage_host[kStepRing] = {};  // pinned: idx | rec | w (as bits)
  int32_t* stage_dev[kStepRing] = {};
};

namespace {

struct TierDevice {
  int prev = -1;
  explicit TierDevice(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~TierDevice() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

constexpr uint64_t kGiB = 1073741824ull;

// QwenActiveStreamingMemoryConfiguration constants (:56-93)
constexpr uint64_t kLayers = 40, kFullAttn = 10, kLinearAttn = 30;
constexpr uint64_t kDenseResident = kLayers * 22456448ull;  // DenseLayerArena.totalByteLength
constexpr uint64_t kRecurrentState = kLinearAttn * ((8192 * 4 * 4) + (32 * 128 * 128 * 4));
constexpr uint64_t kDecodedConstants = 2048 * 4 + kLayers * 2 * 2048 * 4 +
                                       kLinearAttn * ((8192 * 4 * 4) + (32 * 4) + (32 * 4) + (128 * 4)) +
                                       kFullAttn * 2 * 256 * 4;
constexpr uint64_t kFixedScratch = 1341348;
constexpr uint64_t kMappedAndReserve = 366570000;
constexpr uint64_t kPerContextKV = kFullAttn * 2 * 2 * 256 * 2;
constexpr uint64_t kPerContextScratch = 16 * 4;

}  // namespace

extern "C" {

qf_status qf_cache_create(int32_t capacity, int32_t layer_count, double probationary_ratio, int32_t policy,
                          qf_cache** out) {
  if (!out) return QF_ERR_ARG;
  *out = nullptr;
  if (capacity < 1 || capacity > (1 << 24) || layer_count < 1 || layer_count > 4096 ||
      !(probationary_ratio >= 0.0 && probationary_ratio <= 1.0) ||
      (policy != QF_CACHE_SLRU && policy != QF_CACHE_LRU))
    return QF_ERR_ARG;
  qf_cache* c = new (std::nothrow) qf_cache();
  if (!c) return QF_ERR_OOM;
  c->capacity = capacity;
  c->policy = policy;
  c->build_ranges(layer_count);
  c->prob_capacity = std::max(16, static_cast<int>(static_cast<double>(capacity) * probationary_ratio));
  c->prot_capacity = capacity - c->prob_capacity;
  c->slot_key.assign(capacity, 0);
  c->slot_seg.assign(capacity, kEmpty);
  c->slot_tick.assign(capacity, 0);
  c->lock_gen.assign(capacity, 0);
  c->key_slot.reserve(static_cast<size_t>(capacity) * 2);
  *out = c;
  return QF_OK;
}

void qf_cache_destroy(qf_cache* c) { delete c; }

qf_status qf_cache_acquire(qf_cache* c, int32_t layer, const uint32_t* experts, int32_t n, uint32_t* slots,
                           uint32_t* miss_pos, int32_t* n_miss, uint32_t* fetch_expert, uint32_t* fetch_slot,
                           int32_t* n_fetch) {
  if (!c || !experts || !slots || n < 1) return QF_ERR_ARG;
  int nm = 0, nf = 0;
  c->acquire(layer, experts, n, slots, miss_pos, &nm, fetch_expert, fetch_slot, &nf);
  if (n_miss) *n_miss = nm;
  if (n_fetch) *n_fetch = nf;
  return QF_OK;
}

qf_status qf_cache_prefetch(qf_cache* c, int32_t layer, const uint32_t* candidates, int32_t n,
                            uint32_t* fetch_expert, uint32_t* fetch_slot, int32_t* n_fetch) {
  if (!c || (n > 0 && !candidates) || n < 0) return QF_ERR_ARG;
  const int nf = c->prefetch(layer, candidates, n, fetch_expert, fetch_slot);
  if (n_fetch) *n_fetch = nf;
  return QF_OK;
}

qf_status qf_cache_clear(qf_cache* c) {
  if (!c) return QF_ERR_ARG;
  c->clear();
  return QF_OK;
}

qf_status qf_cache_reset_metrics(qf_cache* c) {
  if (!c) return QF_ERR_ARG;
  c->m = qf_cache_metrics_t{};
  std::fill(c->layer_hits.begin(), c->layer_hits.end(), 0);
  std::fill(c->layer_requests.begin(), c->layer_requests.end(), 0);
  return QF_OK;
}

qf_status qf_cache_layer_metrics(const qf_cache* c, int64_t* hits, int64_t* requests) {
  if (!c || !hits || !requests) return QF_ERR_ARG;
  for (int l = 0; l < c->layer_count; l++) {
    hits[l] = c->layer_hits[l];
    requests[l] = c->layer_requests[l];
  }
  return QF_OK;
}

qf_status qf_cache_get_metrics(const qf_cache* c, qf_cache_metrics_t* out) {
  if (!c || !out) return QF_ERR_ARG;
  c->snapshot(out);
  return QF_OK;
}

qf_status qf_cache_info(const qf_cache* c, int32_t* layer_count, int32_t* probationary_capacity,
                        int32_t* protected_capacity) {
  if (!c) return QF_ERR_ARG;
  if (layer_count) *layer_count = c->layer_count;
  if (probationary_capacity) *probationary_capacity = c->prob_capacity;
  if (protected_capacity) *protected_capacity = c->prot_capacity;
  return QF_OK;
}

qf_status qf_cache_layer_slots(const qf_cache* c, int32_t* first, int32_t* count) {
  if (!c || !first || !count) return QF_ERR_ARG;
  for (int l = 0; l < c->layer_count; l++) {
    first[l] = c->range_first[l];
    count[l] = c->range_count[l];
  }
  return QF_OK;
}

qf_status qf_cache_plan_slots(int32_t budget_gib, int64_t context_length, int64_t* slots, uint64_t* estimated_bytes,
                              uint64_t* target_bytes) {
  if (!slots || context_length <= 0 || budget_gib < 1 || budget_gib > 1024) return QF_ERR_ARG;
  const uint64_t ctx = static_cast<uint64_t>(context_length);
  if (ctx > (UINT64_MAX / 2) / (kPerContextKV + kPerContextScratch)) return QF_ERR_ARG;
  const uint64_t fixed = kDenseResident + kRecurrentState + kDecodedConstants + kFixedScratch + kMappedAndReserve;
  const uint64_t non_cache = fixed + kPerContextKV * ctx + kPerContextScratch * ctx;
  const uint64_t target = static_cast<uint64_t>(budget_gib) * kGiB;
  const uint64_t remaining = target > non_cache ? target - non_cache : 0;
  const int64_t avail = static_cast<int64_t>(remaining / kRecord);
  if (target_bytes) *target_bytes = target;
  if (estimated_bytes) *estimated_bytes = non_cache + static_cast<uint64_t>(avail) * kRecord;
  *slots = avail;
  // at least eight locked slots per layer for the router's top-8
  return avail >= static_cast<int64_t>(kLayers * kTopKSlots) ? QF_OK : QF_ERR_OOM;
}

qf_status qf_tier_create(int32_t device, int32_t slots, const void* host_records, int64_t n_host_records,
                         uint64_t host_record_stride, qf_tier** out) {
  if (!out) return QF_ERR_ARG;
  *out = nullptr;
  if (slots < 1 || (n_host_records > 0 && !host_records) || n_host_records < 0 ||
      (n_host_records > 0 && host_record_stride < kRecord))
    return QF_ERR_ARG;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return QF_ERR_CUDA;
  TierDevice g(device);
  qf_tier* t = new (std::nothrow) qf_tier();
  if (!t) return QF_ERR_OOM;
  t->device = device;
  t->slots = slots;
  t->host = static_cast<const uint8_t*>(host_records);
  t->host_records = n_host_records;
  t->host_stride = host_record_stride;
  if (cudaMalloc(&t->arena, static_cast<size_t>(slots) * kRecord) != cudaSuccess) {
    delete t;
    cudaGetLastError();
    return QF_ERR_OOM;
  }
  bool ok = cudaStreamCreateWithFlags(&t->side, cudaStreamNonBlocking) == cudaSuccess &&
            cudaEventCreateWithFlags(&t->done, cudaEventDisableTiming) == cudaSuccess;
  for (int i = 0; ok && i < kStepRing; i++)
    ok = cudaEventCreateWithFlags(&t->step_done[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    qf_tier_destroy(t);
    return QF_ERR_CUDA;
  }
  t->slot_last_step.assign(slots, -1);
  *out = t;
  return QF_OK;
}

void qf_tier_destroy(qf_tier* t) {
  if (!t) return;
  TierDevice g(t->device);
  for (int i = 0; i < kStepRing; i++) {
    if (t->step_done[i]) {
      cudaEventSynchronize(t->step_done[i]);
      cudaEventDestroy(t->step_done[i]);
    }
    if (t->stage_host[i]) cudaFreeHost(t->stage_host[i]);
    if (t->stage_dev[i]) cudaFree(t->stage_dev[i]);
  }
  if (t->side) {
    cudaStreamSynchronize(t->side);
    cudaStreamDestroy(t->side);
  }
  if (t->done) cudaEventDestroy(t->done);
  cudaFree(t->arena);
  delete t;
}

qf_status qf_tier_arena(const qf_tier* t, void** bank, uint64_t* stride) {
  if (!t || !bank) return QF_ERR_ARG;
  *bank = t->arena;
  if (stride) *stride = kRecord;
  return QF_OK;
}

namespace {
// Issues the record copies on the tier's stream and makes the consumer wait
// for them.  ok[i] (optional) tells which records were copied; a record whose
// copy fails (an injected short copy, or a failed enqueue) is skipped and the
// result is QF_ERR_IO once the others are issued.
qf_status tier_fetch(qf_tier* t, const int64_t* host_index, const uint32_t* slot, int32_t n,
                     void* consumer_stream, uint8_t* ok) {
  TierDevice g(t->device);
  int failed = 0;
  for (int i = 0; i < n; i++) {
    bool good = true;
    if (t->inject_skip > 0) {
      t->inject_skip -= 1;
    } else if (t->inject_count > 0) {
      t->inject_count -= 1;
      good = false;  // simulated short copy: nothing issued
    }
    if (good && cudaMemcpyAsync(t->arena + static_cast<size_t>(slot[i]) * kRecord,
                                t->host + static_cast<size_t>(host_index[i]) * t->host_stride, kRecord,
                                cudaMemcpyHostToDevice, t->side) != cudaSuccess) {
      cudaGetLastError();
      good = false;
    }
    if (ok) ok[i] = good ? 1 : 0;
    if (good) {
      t->copies += 1;
      t->bytes += static_cast<int64_t>(kRecord);
    } else {
      failed += 1;
    }
  }
  t->failed_copies += failed;
  if (cudaEventRecord(t->done, t->side) != cudaSuccess) return QF_ERR_CUDA;
  if (cudaStreamWaitEvent(static_cast<cudaStream_t>(consumer_stream), t->done, 0) != cudaSuccess)
    return QF_ERR_CUDA;
  return failed ? QF_ERR_IO : QF_OK;
}
}  // namespace

qf_status qf_tier_fetch(qf_tier* t, const int64_t* host_index, const uint32_t* slot, int32_t n,
                        void* consumer_stream) {
  if (!t || n < 0 || (n > 0 && (!host_index || !slot))) return QF_ERR_ARG;
  for (int i = 0; i < n; i++)
    if (host_index[i] < 0 || host_index[i] >= t->host_records || slot[i] >= static_cast<uint32_t>(t->slots))
      return QF_ERR_ARG;
  return tier_fetch(t, host_index, slot, n, consumer_stream, nullptr);
}

qf_status qf_tier_inject_fault(qf_tier* t, int32_t skip, int32_t count) {
  if (!t || skip < 0 || count < 0) return QF_ERR_ARG;
  t->inject_skip = skip;
  t->inject_count = count;
  return QF_OK;
}

qf_status qf_tier_failed_copies(const qf_tier* t, int64_t* failed) {
  if (!t || !failed) return QF_ERR_ARG;
  *failed = t->failed_copies;
  return QF_OK;
}

qf_status qf_tier_stats(const qf_tier* t, int64_t* copies, int64_t* bytes) {
  if (!t) return QF_ERR_ARG;
  if (copies) *copies = t->copies;
  if (bytes) *bytes = t->bytes;
  return QF_OK;
}

qf_status qf_tier_synchronize(qf_tier* t) {
  if (!t) return QF_ERR_ARG;
  TierDevice g(t->device);
  return cudaStreamSynchronize(t->side) == cudaSuccess ? QF_OK : QF_ERR_CUDA;
}

qf_status qf_moe_stream_step(qf_moe* h, qf_cache* c, qf_tier* t, const qf_moe_layer* layers,
                             int32_t n_layers, const int32_t* host_idx, const float* host_w,
                             const uint16_t* x, const float* residual, float* out, float eps,
                             void* workspace, size_t workspace_bytes) {
  using qf::cuda_fail;
  using qf::fail;
  if (!h) return QF_ERR_ARG;
  if (!c || !t || !layers || n_layers < 1 || !host_idx || !host_w || !x || !out)
    return fail(h, QF_ERR_ARG, "stream step: cache, tier, layers, routing, x and out are required");
  if (t->device != h->device) return fail(h, QF_ERR_ARG, "stream step: tier and handle are on different devices");
  if (c->layer_count != n_layers)
    return fail(h, QF_ERR_ARG, "stream step: the cache must hold one slot partition per layer");
  if (c->capacity > t->slots) return fail(h, QF_ERR_ARG, "stream step: the tier has fewer slots than the cache");
  if (!(eps > 0.f)) return fail(h, QF_ERR_ARG, "eps must be > 0");
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) ||
      workspace_bytes < qf::fused_workspace_bytes(1))
    return fail(h, QF_ERR_ARG, "workspace too small or not 256-byte aligned");
  if (reinterpret_cast<uintptr_t>(x) & 15) return fail(h, QF_ERR_ARG, "x must be 16-byte aligned");
  const int P = qf::kTopK;
  for (int i = 0; i < n_layers * P; i++)
    if (host_idx[i] < 0 || host_idx[i] >= qf::kExperts)
      return fail(h, QF_ERR_ARG, "stream step: expert id out of range");
  if (static_cast<int64_t>(n_layers) * qf::kExperts > t->host_records)
    return fail(h, QF_ERR_ARG, "stream step: the host tier holds fewer than n_layers * 256 records");
  std::vector<qf::LayerW> lw(n_layers);
  for (int l = 0; l < n_layers; l++) {
    qf_moe_layer d = layers[l];
    d.expert_bank = t->arena;
    d.record_stride = kRecord;
    d.bank_records = static_cast<uint32_t>(t->slots);
    qf_status st = qf::layer_to_w(h, &d, &lw[l]);
    if (st != QF_OK) return st;
  }
  TierDevice g(h->device);
  cudaStream_t main = h->stream;
  const int64_t n = t->step + 1;
  const int ring = static_cast<int>(n % kStepRing);
  cudaError_t e = cudaSuccess;
  // step n - kStepRing owns this staging slot and event: wait for it
  if (n >= kStepRing && (e = cudaEventSynchronize(t->step_done[ring])) != cudaSuccess)
    return cuda_fail(h, e, "stream step: wait for an earlier step");
  if (t->stage_layers < n_layers) {
    for (int i = 0; i < kStepRing; i++) {
      if (t->stage_host[i]) cudaFreeHost(t->stage_host[i]);
      if (t->stage_dev[i]) cudaFree(t->stage_dev[i]);
      t->stage_host[i] = nullptr;
      t->stage_dev[i] = nullptr;
    }
    t->stage_layers = 0;
    const size_t bytes = static_cast<size_t>(n_layers) * P * 3 * sizeof(int32_t);
    for (int i = 0; i < kStepRing; i++) {
      if ((e = cudaMallocHost(&t->stage_host[i], bytes)) != cudaSuccess ||
          (e = cudaMalloc(&t->stage_dev[i], bytes)) != cudaSuccess)
        return cuda_fail(h, e, "stream step: staging buffers");
    }
    t->stage_layers = n_layers;
  }
  int32_t* sh = t->stage_host[ring];
  int32_t* sd = t->stage_dev[ring];
  const size_t NP = static_cast<size_t>(n_layers) * P;
  // plan every layer's slots (acquireSlotsParallel per layer), collect copies
  std::vector<int64_t> src;
  std::vector<uint32_t> dst;
  std::vector<qf_cache::Undo> undo;
  int64_t wait_step = -1;
  for (int l = 0; l < n_layers; l++) {
    uint32_t ex[8], slots[8], fe[8], fs[8];
    qf_cache::Undo un[8];
    for (int k = 0; k < P; k++) ex[k] = static_cast<uint32_t>(host_idx[l * P + k]);
    int nm = 0, nf = 0;
    c->acquire(l, ex, P, slots, nullptr, &nm, fe, fs, &nf, un);
    for (int f = 0; f < nf; f++) {
      wait_step = std::max(wait_step, t->slot_last_step[fs[f]]);
      src.push_back(static_cast<int64_t>(l) * qf::kExperts + fe[f]);
      dst.push_back(fs[f]);
      undo.push_back(un[f]);
    }
    for (int k = 0; k < P; k++) {
      sh[l * P + k] = host_idx[l * P + k];
      sh[NP + l * P + k] = static_cast<int32_t>(slots[k]);
      t->slot_last_step[slots[k]] = n;
    }
  }
  std::memcpy(sh + 2 * NP, host_w, NP * sizeof(float));
  // copies overwrite evicted slots: wait for the last step that read one of them
  // (steps up to n - kStepRing are already complete)
  if (!src.empty()) {
    if (wait_step > n - kStepRing && wait_step >= 0 &&
        (e = cudaStreamWaitEvent(t->side, t->step_done[wait_step % kStepRing], 0)) != cudaSuccess)
      return cuda_fail(h, e, "stream step: order copies after readers");
    std::vector<uint8_t> ok(src.size(), 0);
    qf_status st = tier_fetch(t, src.data(), dst.data(), static_cast<int32_t>(src.size()), main, ok.data());
    if (st == QF_ERR_IO) {
      // some records did not arrive: give their slots back to the experts they
      // held (latest first) and run nothing; the caller may retry the step
      for (size_t i = src.size(); i-- > 0;)
        if (!ok[i]) c->undo_fetch(undo[i]);
      return fail(h, st, "stream step: a host-tier record copy failed (step not run)");
    }
    if (st != QF_OK) return fail(h, st, "stream step: host-tier copy failed");
  }
  if ((e = cudaMemcpyAsync(sd, sh, NP * 3 * sizeof(int32_t), cudaMemcpyHostToDevice, main)) != cudaSuccess)
    return cuda_fail(h, e, "stream step: routing upload");
  qf::RoutingArgs r;
  r.bias = nullptr;
  r.idx_in = sd;
  r.rec_of_pos = sd + NP;
  r.w_in = reinterpret_cast<const float*>(sd + 2 * NP);
  e = qf::fused_stack(main, lw.data(), n_layers, h->dims.scale_dtype == QF_SCALE_BF16, 1, x, residual,
                      out, eps, r, nullptr, nullptr, workspace, h->d_status, &h->prof);
  if (e != cudaSuccess) return cuda_fail(h, e, "stream step: block stack");
  if ((e = cudaEventRecord(t->step_done[ring], main)) != cudaSuccess)
    return cuda_fail(h, e, "stream step: step event");
  t->step = n;
  return QF_OK;
}

}  // extern "C"
