/*
 * qf_moe.h -- C ABI of the B200 MoE-block library (libqf_moe.so).
 *
 * Drop-in boundary for the MoE step of QwenFieldfareCore.  In the reference
 * (tanishqpatil/qwen-fieldfare, Swift + Metal) the "operator API" of this path
 * is the Metal kernels' buffer-index ABI, encoded from Swift at
 *   Sources/QwenFieldfareCore/Runtime/Generation/QwenQ4ActiveExpertStreamingRunner.swift:1169-1381
 *   Sources/QwenFieldfareCore/Runtime/Generation/QwenQ4ChatRunner.swift:891-1000
 * plus the Swift class Q4BoundedExpertCache
 *   Sources/QwenFieldfareCore/Storage/Q4BoundedExpertCache.swift:14-419.
 * Each entry point below names the reference kernel(s) or method it replaces.
 *
 * Conventions
 *   - Plain C: pointers, sizes, no CUDA or torch types.  Streams are passed
 *     as `void*` (a cudaStream_t); NULL = the handle's stream.
 *   - Device pointers are caller-owned (the reference caller owns every
 *     MTLBuffer, kernels own nothing).  Calls are stream-ordered and
 *     asynchronous; results are valid after the stream reaches them.
 *   - Errors: every call returns qf_status; qf_last_error() returns the
 *     message of the last failure on that handle.  No exceptions cross the
 *     ABI.  A device-side status word (bounds/limit violations detected by
 *     the kernels) is read by qf_moe_check().
 *   - One handle per host thread (the reference runner is single-owner,
 *     docs/AGENT_RUNTIME_PLAN.md:33).
 *
 * Weight layout (byte-exact with the reference):
 *   expert record (1,769,472 B) = gate W | gate S | gate B | up W | up S | up B |
 *                                 down W | down S | down B
 *   at offsets 0, 524288, 557056, 589824, 1114112, 1146880, 1179648, 1703936,
 *   1736704 (QwenQ4ExpertStoreBuilder.swift:47-56; deltanet.metal:2155-2211).
 *   Q4 codes: element 2i is the low nibble of byte i; 64-column groups;
 *   w = q*scale + bias with 16-bit scale/bias (fp16 or bf16).
 *   Router: Q8 [256 x 2048] codes + [256 x 32] scales/biases; shared-expert
 *   gate coefficient: Q8 [1 x 2048] (QwenQ4ActiveExpertStreamingRunner.swift:36-50).
 */
#ifndef QF_MOE_H
#define QF_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QF_MOE_ABI_VERSION 1

typedef enum qf_status {
    QF_OK = 0,
    QF_ERR_ARG = -1,         /* invalid argument / unsupported geometry */
    QF_ERR_CUDA = -2,        /* CUDA runtime error */
    QF_ERR_NCCL = -3,        /* collective error */
    QF_ERR_OOM = -4,         /* allocation failed */
    QF_ERR_IO = -5,          /* host tier / copy failure */
    QF_ERR_TIMEOUT = -6,     /* a bounded device wait expired */
    QF_ERR_DEVICE = -7,      /* device status word reported a violation */
    QF_ERR_UNSUPPORTED = -8  /* feature not built for this configuration */
} qf_status;

typedef enum qf_scale_dtype { QF_SCALE_F16 = 0, QF_SCALE_BF16 = 1 } qf_scale_dtype;

/* Geometry.  This build is specialised for the Qwen3.6-35B-A3B MoE block:
 * hidden 2048, 256 experts, top-8, intermediate 512, group 64. */
typedef struct qf_moe_dims {
    int32_t hidden;
    int32_t experts;
    int32_t top_k;
    int32_t intermediate;
    int32_t group;
    int32_t scale_dtype; /* qf_scale_dtype */
} qf_moe_dims;

/* One layer's MoE weights (device pointers).  Replaces the DenseLayerArena
 * offsets routerW/S/B, shCoeffW/S/B, shGate..shDown
 * (QwenQ4ActiveExpertStreamingRunner.swift:36-50) and the expert arena /
 * cache buffer (Q4BoundedExpertCache.swift:23). */
typedef struct qf_moe_layer {
    const uint8_t *router_w;   /* [experts * hidden] Q8 codes (16-byte aligned) */
    const uint16_t *router_s;  /* [experts * hidden/64] (16-byte aligned) */
    const uint16_t *router_b;  /* (16-byte aligned) */
    const uint8_t *coef_w;     /* [hidden] Q8 codes of the shared-expert gate */
    const uint16_t *coef_s;    /* [hidden/64] */
    const uint16_t *coef_b;
    const uint8_t *shared_record; /* one expert record: the shared expert (32-byte aligned) */
    const uint8_t *expert_bank;   /* record 0 of the routed bank / slot arena (32-byte aligned) */
    uint64_t record_stride;       /* bytes between records (>= 1,769,472, multiple of 32) */
    uint32_t bank_records;        /* records in the bank (experts, or cache slots); a
                                     routed record index >= this is a device error */
    uint32_t reserved;            /* must be 0 */
} qf_moe_layer;

/* Routing controls.  All pointers are device pointers, may be NULL. */
typedef struct qf_routing {
    const float *logit_bias;       /* [experts] added to logits before top-k (harness) */
    const int32_t *topk_idx;       /* [T * top_k] supplied expert ids (skip selection) */
    const float *topk_w;           /* [T * top_k] supplied weights (with topk_idx) */
    const int32_t *record_of_pos;  /* [T * top_k] bank record per routed position
                                      (the cache's slot_indices); NULL: record = expert */
} qf_routing;

typedef struct qf_moe qf_moe;

/* ---- handle ---------------------------------------------------------- */
/* Replaces MetalContext (Infrastructure/Metal/MetalContext.swift:52-107). */
qf_status qf_moe_create(const qf_moe_dims *dims, int device, qf_moe **out);
void qf_moe_destroy(qf_moe *h);
qf_status qf_moe_set_stream(qf_moe *h, void *stream);
const char *qf_last_error(const qf_moe *h);
/* Synchronises the handle's stream and returns the device status word
 * (QF_OK, or QF_ERR_DEVICE/QF_ERR_TIMEOUT with the message set). */
qf_status qf_moe_check(qf_moe *h);
int qf_moe_abi_version(void);

/* ---- kernels --------------------------------------------------------- */
/* Router logits, Q8 affine.  Replaces qwen_router_q8_logits_simd_f32
 * (deltanet.metal:2262-2281, dispatched at
 * QwenQ4ActiveExpertStreamingRunner.swift:1178-1184).  Fixed reduction
 * order: the reference's lane decomposition + xor-butterfly simd_sum, so the
 * logits are bit-reproducible on the CPU.
 *   x: fp16 [T * hidden]; logits: fp32 [T * experts]; coef (optional): fp32 [T]
 *   (the shared-expert gate pre-activation, qwen_gemv_q8_affine rows=1,
 *   deltanet.metal:863-902 / runner :1192-1200). */
qf_status qf_router_logits_q8(qf_moe *h, const qf_moe_layer *layer, int32_t T,
                              const uint16_t *x, float *logits, float *coef);

/* Q4 LM head: logits[t][r] = row r of W (rows x 2048, MLX-affine Q4, group
 * 64) dotted with the fp32 row x[t] (the final RMSNorm output), for T token
 * rows.  Replaces deltanet.metal:1897-1919 qwen_gemv_q4_affine_simd_f32 as
 * dispatched for the 248,320-row LM head at
 * QwenQ4ActiveExpertStreamingRunner.swift:1393-1400, with the same per-lane
 * arithmetic order (bit-exact with the CPU oracle).  w [rows][1024] bytes,
 * scales / biases [rows][32] 16-bit in the handle's scale dtype, x [T][2048]
 * (w, scales, biases and x 16-B aligned), logits [T][rows]; the weights
 * stream once per token row. */
qf_status qf_lm_head_q4(qf_moe *h, const void *w, const void *scales, const void *biases, int32_t rows,
                        int32_t T, const float *x, float *logits);

/* Top-k by logit (ties to the lower expert index), softmax over all experts,
 * renormalised over the top-k.  Replaces qwen_router_top8_logits_f32
 * (deltanet.metal:2283-2329, dispatched at runner :1186-1190).
 *   logits: fp32 [T * experts]; bias: fp32 [experts] or NULL;
 *   idx: int32 [T * top_k]; w: fp32 [T * top_k]. */
qf_status qf_router_topk(qf_moe *h, const float *logits, const float *bias, int32_t T,
                         int32_t *idx, float *w);

/* Stable dispatch plan (absent in the reference, which is decode-only):
 * counts[experts], offsets[experts+1], perm[T*top_k] = position ids t*top_k+k
 * sorted by (expert, t, k).  T <= 32768.  workspace: device scratch of at
 * least qf_moe_dispatch_workspace_size bytes. */
qf_status qf_moe_dispatch_workspace_size(qf_moe *h, int32_t T, size_t *bytes);
qf_status qf_moe_dispatch_plan(qf_moe *h, const int32_t *idx, int32_t T, int32_t *counts,
                               int32_t *offsets, int32_t *perm, void *workspace,
                               size_t workspace_bytes);

/* ---- pieces of the streaming runner's MoE step -------------------------
 * The reference runs a token's MoE step in two command buffers so that the
 * experts already in the cache compute while the missing ones are read
 * (QwenQ4ActiveExpertStreamingRunner.swift:1227-1381): right after planning,
 * the shared expert and the HIT subset (:1246-1314); after the reads, the
 * MISS subset (:1339-1366) and the combine (:1368-1381).  These four entries
 * replace those dispatches one for one; device pointers, the handle's stream.
 *
 * Routed experts of a subset of ONE token's top-8 positions
 * (qwen_cached_moe_gate_up_subset_q4_simd_f32 + qwen_cached_moe_down_subset_q4_simd_f32,
 * deltanet.metal:2155-2211):
 *   layer->expert_bank   the slot arena (record = slot);
 *   slot_of_pos [8]      the slot of each top-8 position (activeSlotIndicesBuf);
 *   w [8]                the routing weights of the 8 positions (scoresBuf);
 *   positions [n]        the subset's positions, distinct, in [0, 8);  n in [0, 8];
 *   routed_out [2048]    sum over i < 8 of (i < n ? w[p_i] * D_{p_i}(SiLU(G x) * (U x)) : 0),
 *                        left to right, activations in fp32 (the reference's order).
 * workspace: qf_moe_workspace_size at T = 1 (256-byte aligned); a call uses it
 * until its kernels end, so two overlapping calls need two workspaces. */
qf_status qf_moe_routed_subset(qf_moe *h, const qf_moe_layer *layer, const uint16_t *x,
                               const int32_t *slot_of_pos, const float *w, const int32_t *positions,
                               int32_t n, float *routed_out, void *workspace, size_t workspace_bytes);
/* Shared expert of T <= 64 tokens with its gate:
 * out[t] = sigmoid(coef[t]) * D_sh(SiLU(G_sh x_t) * (U_sh x_t)), coef = the
 * shared-gate logits of qf_router_logits_q8 (qwen_shared_gate_up_silu_q4_simd_f32
 * + qwen_shared_down_gate_q4_simd_f32, deltanet.metal:2050-2122).  workspace:
 * qf_moe_workspace_size at T. */
qf_status qf_shared_expert(qf_moe *h, const qf_moe_layer *layer, int32_t T, const uint16_t *x,
                           const float *coef, float *out, void *workspace, size_t workspace_bytes);
/* out = ((residual + shared_out) + hit_out) + miss_out over T x 2048 fp32
 * values; residual, hit_out and miss_out may be NULL (a zero term, as a zero
 * hit or miss count in qwen_combine_cached_moe_subsets_f32, deltanet.metal:2213-2227). */
qf_status qf_moe_combine(qf_moe *h, int32_t T, const float *residual, const float *shared_out,
                         const float *hit_out, const float *miss_out, float *out);
/* The routed experts of T <= 32768 tokens as one grouped tcgen05 GEMM pair
 * (absent in the reference, which is decode-only): dispatch plan, row gather,
 * grouped gate/up and down over a resident bank of 256 experts;
 * y [T * 8][2048] fp32 (16-B aligned) = D_e(SiLU(G_e x_t) * (U_e x_t)) for
 * position t * 8 + k, e = idx[t * 8 + k] (unweighted; no shared expert, no
 * combine).  workspace: qf_moe_grouped_ffn_workspace_size. */
qf_status qf_moe_grouped_ffn_workspace_size(qf_moe *h, int32_t T, size_t *bytes);
qf_status qf_moe_grouped_ffn(qf_moe *h, const qf_moe_layer *layer, int32_t T, const uint16_t *x,
                             const int32_t *idx, float *y, void *workspace, size_t workspace_bytes);

/* Workspace bytes needed by qf_moe_block_forward / qf_moe_stack_forward at T tokens. */
qf_status qf_moe_workspace_size(qf_moe *h, int32_t T, size_t *bytes);

/* One MoE block: out = residual + shared(x) + sum_k w_k * expert_k(x).
 * Replaces the whole MoE step of forwardToken: router + top-8 + shared
 * coefficient + shared gate/up/down + hit/miss subset gate/up/down + combine
 * (deltanet.metal:2050-2227 as dispatched at
 * QwenQ4ActiveExpertStreamingRunner.swift:1169-1381; resident variant
 * deltanet.metal:1212-1411 at QwenQ4ChatRunner.swift:891-1000).
 *   x: fp16 [T * hidden] post-norm hidden; residual: fp32 [T * hidden] or NULL;
 *   out: fp32 [T * hidden]; idx_out/w_out: optional [T * top_k];
 *   routing: optional; workspace: >= qf_moe_workspace_size bytes (256-B aligned).
 * T = 1 runs the one-token persistent kernel (no grid barriers: vectors cross
 * CTAs as tagged words); T in [2, 8] a persistent kernel with grid barriers.
 * T in [9, 32768] runs the grouped tensor-core path when the bank holds all
 * 256 experts (bank_records >= 256) and there is no record_of_pos; otherwise
 * T in [9, 64] runs five kernels per block and T > 64 is rejected. */
qf_status qf_moe_block_forward(qf_moe *h, const qf_moe_layer *layer, int32_t T,
                               const uint16_t *x, const float *residual, float *out,
                               const qf_routing *routing, int32_t *idx_out, float *w_out,
                               void *workspace, size_t workspace_bytes);

/* The MoE block from the residual stream: x = post-attention RMSNorm of
 * `hidden` with weight `norm_w`, then qf_moe_block_forward(x, residual =
 * hidden).  Replaces the rmsnorm dispatch before the router
 * (deltanet.metal:18-53 at QwenQ4ActiveExpertStreamingRunner.swift:1169-1176)
 * together with the MoE step; the norm keeps the reference kernel's order
 * (64 threads, fma chains, lane butterfly) and rounds x to fp16 for the block.
 *   hidden: fp32 [T * 2048]; norm_w: fp32 [2048]; workspace: >=
 *   qf_moe_workspace_size rounded up to 256, plus T * 4096 bytes (x lives at
 *   its end).  At T = 1 the norm runs in the one-token kernel's prologue;
 *   otherwise as a 64-thread kernel before the block. */
qf_status qf_moe_block_forward_prenorm(qf_moe *h, const qf_moe_layer *layer, int32_t T, const float *hidden,
                                       const float *norm_w, float eps, float *out, const qf_routing *routing,
                                       int32_t *idx_out, float *w_out, void *workspace, size_t workspace_bytes);

/* n_layers stacked blocks (the decode loop over 40 layers of forwardToken,
 * runner :958).  Layer l reads x_l (fp16) and residual h_l; writes
 * h_{l+1} = out_l; x_{l+1} = fp16(RMSNorm(out_l)) with unit weight and `eps`
 * (qwen_rmsnorm_f32, deltanet.metal:18-53).  `layers` is a HOST array of
 * n_layers descriptors.  idx_out/w_out (optional): [n_layers * T * top_k].
 * T in [1, 8]: the whole stack is one persistent launch; T in [9, 64]: one
 * block at a time (grouped path for resident banks) with the RMSNorm between. */
qf_status qf_moe_stack_forward(qf_moe *h, const qf_moe_layer *layers, int32_t n_layers,
                               int32_t T, const uint16_t *x, const float *residual, float *out,
                               float eps, int32_t *idx_out, float *w_out, void *workspace,
                               size_t workspace_bytes);

/* Allocation-free variant of qf_moe_block_forward (no counterpart in the
 * reference, whose caller owns every buffer).  For callers that cannot call
 * cudaMalloc when they run the block (an engine whose device memory comes from
 * its own arena, a language binding with no device allocator, a step that must
 * not touch the allocator): it needs no handle and no workspace.  Its scratch
 * is a 1 MiB device array inside the library, held on every GPU that loads the
 * library until exit.
 *   - T in [1, 8]; larger T (or any bad argument) returns QF_ERR_ARG.
 *   - Runs on the calling thread's current device, on `stream` (NULL: legacy
 *     default stream).  The first call on a device resolves the array's device
 *     address and kernel attributes; make it before any stream capture.
 *   - All calls share the array: calls whose GPU work overlaps race.  Each
 *     call clears what must start at zero (the status word); out-of-range
 *     record ids are skipped on the device but not reported by this call.
 *   - It allocates nothing (no cudaMalloc/cudaFree, no allocating library). */
qf_status qf_moe_block_forward_static(int32_t scale_dtype, const qf_moe_layer *layer, int32_t T,
                                      const uint16_t *x, const float *residual, float *out,
                                      int32_t *idx_out, float *w_out, void *stream);

/* ---- expert-slot cache ----------------------------------------------- */
/* Host-side slot planner.  Replaces Q4BoundedExpertCache's planning state
 * (Storage/Q4BoundedExpertCache.swift:52-365): slots partitioned by layer
 * (eight per layer plus the measured per-layer weights for 40 layers,
 * :64-123), a segmented LRU per layer (probationary / protected, :222-297),
 * and acquireSlotsParallel's plan-then-fetch contract (:330-365).
 * QF_CACHE_LRU keeps one least-recently-used order per layer instead. */
typedef enum qf_cache_policy { QF_CACHE_SLRU = 0, QF_CACHE_LRU = 1 } qf_cache_policy;

/* QwenExpertCacheMetrics (Runtime/Telemetry/QwenRuntimeTelemetry.swift:58-69). */
typedef struct qf_cache_metrics_t {
    int64_t capacity;
    int64_t occupancy;
    int64_t probationary_occupancy;
    int64_t protected_occupancy;
    int64_t hits;
    int64_t misses;
    int64_t evictions;
    int64_t fetched_bytes;
    int64_t prefetch_requests;
    int64_t useful_prefetch_hits;
    int64_t wasted_prefetches;
} qf_cache_metrics_t;

typedef struct qf_cache qf_cache;

/* capacity >= 1 slot; layer_count: the model's layers (one partition per
 * layer when capacity >= 8 * layer_count, else one shared partition);
 * probationary_ratio in [0, 1] (reference default 0.25). */
qf_status qf_cache_create(int32_t capacity, int32_t layer_count, double probationary_ratio,
                          int32_t policy, qf_cache **out);
void qf_cache_destroy(qf_cache *c);
/* acquireSlotsParallel for one layer's top-k: slots[n'] (n' = min(n, 8)) are
 * the slots that hold (or will hold) experts[0..n'); miss_pos[*n_miss] lists the
 * positions whose expert is being fetched; fetch_expert/fetch_slot[*n_fetch]
 * (up to 8 each, optional) are the copies to issue, in order.  Host memory. */
qf_status qf_cache_acquire(qf_cache *c, int32_t layer, const uint32_t *experts, int32_t n,
                           uint32_t *slots, uint32_t *miss_pos, int32_t *n_miss,
                           uint32_t *fetch_expert, uint32_t *fetch_slot, int32_t *n_fetch);
/* prefetch (:367-400): candidates not resident go into free slots of the layer
 * while any is free; fetch lists as for acquire (each up to n entries). */
qf_status qf_cache_prefetch(qf_cache *c, int32_t layer, const uint32_t *candidates, int32_t n,
                            uint32_t *fetch_expert, uint32_t *fetch_slot, int32_t *n_fetch);
qf_status qf_cache_clear(qf_cache *c);
qf_status qf_cache_reset_metrics(qf_cache *c);
qf_status qf_cache_get_metrics(const qf_cache *c, qf_cache_metrics_t *out);
qf_status qf_cache_info(const qf_cache *c, int32_t *layer_count,
                        int32_t *probationary_capacity, int32_t *protected_capacity);
/* Per-layer demand counters since the last reset: hits[layer_count] and
 * requests[layer_count] (Q4BoundedExpertCache.layerHits / layerRequests,
 * Storage/Q4BoundedExpertCache.swift:49-50, 205, 216, printed by the bench at
 * Sources/QwenFieldfareBench/main.swift:799-805).  A layer outside
 * [0, layer_count) counts in the nearest partition, the one it is served from. */
qf_status qf_cache_layer_metrics(const qf_cache *c, int64_t *hits, int64_t *requests);
/* first[layer_count], count[layer_count]: each partition's slot range. */
qf_status qf_cache_layer_slots(const qf_cache *c, int32_t *first, int32_t *count);

/* Slot budget: QwenActiveStreamingMemoryConfiguration.make
 * (Runtime/Generation/QwenActiveStreamingMemoryConfiguration.swift:95-135).
 * Slots that fit in budget_gib GiB after the dense layers, recurrent state,
 * constants, scratch, reserve and the KV cache of context_length tokens;
 * QF_ERR_OOM (slots still written) when fewer than 40 * 8 fit. */
qf_status qf_cache_plan_slots(int32_t budget_gib, int64_t context_length, int64_t *slots,
                              uint64_t *estimated_bytes, uint64_t *target_bytes);

/* HBM slot arena + pinned-host tier.  Replaces the cache buffer
 * (Q4BoundedExpertCache.swift:23) and its parallel pread of packed records
 * (:330-365): the arena holds `slots` records of 1,769,472 bytes on `device`;
 * host_records (pinned, or any host memory) holds n_host_records records
 * `host_record_stride` bytes apart, indexed by layer * experts + expert or
 * however the caller numbers them. */
typedef struct qf_tier qf_tier;
qf_status qf_tier_create(int32_t device, int32_t slots, const void *host_records,
                         int64_t n_host_records, uint64_t host_record_stride, qf_tier **out);
void qf_tier_destroy(qf_tier *t);
/* The arena as a record bank for qf_moe_layer.expert_bank (stride 1,769,472). */
qf_status qf_tier_arena(const qf_tier *t, void **bank, uint64_t *stride);
/* Copies host record host_index[i] into arena slot slot[i] (one cudaMemcpyAsync
 * per record on the tier's stream), then makes consumer_stream (NULL: legacy
 * default stream) wait for the copies. */
qf_status qf_tier_fetch(qf_tier *t, const int64_t *host_index, const uint32_t *slot, int32_t n,
                        void *consumer_stream);
qf_status qf_tier_stats(const qf_tier *t, int64_t *copies, int64_t *bytes);
qf_status qf_tier_synchronize(qf_tier *t);
/* Host-side fault injection (failure-detection tests; the reference's fetch
 * falls back to a second source when a read fails,
 * QwenQ4ActiveExpertStreamingRunner.swift:839-866): after `skip` more record
 * copies, the next `count` are treated as short copies and not issued.  A
 * failed record copy makes qf_tier_fetch return QF_ERR_IO (the other records
 * are still copied) and qf_moe_stream_step return QF_ERR_IO without running the
 * step, with each failed record's slot given back to the expert it held before
 * (so the cache never maps an expert whose bytes did not arrive; the miss
 * stays counted, as the reference's telemetry counts it).  skip = count = 0
 * disarms it. */
qf_status qf_tier_inject_fault(qf_tier *t, int32_t skip, int32_t count);
/* Record copies that failed since the tier was created. */
qf_status qf_tier_failed_copies(const qf_tier *t, int64_t *failed);

/* ---- packed expert store, format v2 (host) ----------------------------- */
/* Reader of the reference's packed expert files, the source of the host
 * tier: <directory>/manifest.json plus layer_00.q4exp .. layer_39.q4exp, each
 * a 4,096-byte little-endian header followed by 256 records of 1,769,472
 * bytes in expert order -- the slot layout above, byte for byte
 * (Sources/QwenFieldfareCore/Storage/QwenQ4ExpertStore.swift:50-159, written
 * by QwenQ4ExpertStoreBuilder.swift:284-352).  Failures return QF_ERR_ARG
 * (invalid manifest, header or source index) or QF_ERR_IO (open, stat,
 * short read); qf_store_last_error() gives the message on the calling
 * thread.  The reader is thread-safe; counters are atomic. */
#define QF_STORE_HEADER_BYTES 4096
typedef struct qf_store_header {
    int32_t layer_index;
    int32_t experts_per_layer;
    int32_t expert_byte_length;
    uint64_t payload_byte_length;
    char payload_sha256[65];        /* 64 lowercase hex characters + NUL */
    char source_index_sha256[65];
} qf_store_header;
/* QwenQ4ExpertLayerHeader.encode (QwenQ4ExpertStore.swift:76-99): out gets
 * QF_STORE_HEADER_BYTES bytes; rejects digests that are not 64 lowercase hex
 * characters and negative or zero counts. */
qf_status qf_store_header_encode(const qf_store_header *h, uint8_t *out);
/* QwenQ4ExpertLayerHeader.decode (QwenQ4ExpertStore.swift:101-124): checks
 * length, magic "Q4EXP02\0", schema 2, header length and both digests. */
qf_status qf_store_header_decode(const uint8_t *bytes, size_t n, qf_store_header *out);
/* QwenQ4ExpertStore.validateManifest (QwenQ4ExpertStore.swift:322-342) on the
 * text of manifest.json: schema 2, a valid source digest, every layer 0..39
 * exactly once with its canonical file name and size and a valid digest. */
qf_status qf_store_validate_manifest(const char *json, size_t n);

typedef struct qf_store qf_store;
/* QwenQ4ExpertStore.init (QwenQ4ExpertStore.swift:213-282): validates the
 * manifest, opens the 40 layer files (regular files, no symlink followed),
 * checks each size and each header against the manifest.  With
 * source_index_path (the checkpoint's model.safetensors.index.json) its
 * SHA-256 must equal the manifest's; NULL skips that check. */
qf_status qf_store_open(const char *directory, const char *source_index_path, qf_store **out);
void qf_store_close(qf_store *s);
/* QwenQ4ExpertStore.readExpert (QwenQ4ExpertStore.swift:288-306): one
 * 1,769,472-byte record into dst (host memory). */
qf_status qf_store_read_expert(qf_store *s, int32_t layer, int32_t expert, void *dst);
/* Fills a host tier for qf_tier_create: record (layer - first_layer) * 256 +
 * expert at host_records + index * host_record_stride, for layers
 * [first_layer, first_layer + n_layers), read by `threads` threads (<= 0: 8).
 * Replaces the per-miss pread of the streaming runner
 * (QwenQ4ActiveExpertStreamingRunner.swift:839-888) with one load up front. */
qf_status qf_store_load_tier(qf_store *s, int32_t first_layer, int32_t n_layers, void *host_records,
                             uint64_t host_record_stride, int32_t threads);
typedef struct qf_store_metrics {
    int64_t packed_reads;       /* records read in full */
    int64_t pread_operations;   /* record reads issued */
    int64_t read_failures;      /* out-of-range requests and short reads */
} qf_store_metrics;
/* QwenQ4ExpertStore.metricsSnapshot (QwenQ4ExpertStore.swift:308-316),
 * kind "qwen-q4-packed-v2". */
qf_status qf_store_get_metrics(const qf_store *s, qf_store_metrics *out);
/* SHA-256 of one layer's payload against the manifest digest (the builder's
 * layer check, QwenQ4ExpertStoreBuilder.swift:354-370): *matches = 1 or 0. */
qf_status qf_store_verify_layer(qf_store *s, int32_t layer, int32_t *matches);
/* QwenQ4ExpertStoreBuilder.pack (QwenQ4ExpertStoreBuilder.swift:59-180):
 * builds the v2 store of the checkpoint in model_path (out_dir NULL:
 * <model_path>/qwen_q4_experts) from its switch_mlp tensors.  An existing
 * store is opened and validated, not rebuilt (layers_written 0).  Progress is
 * kept in pack.resume.json; a layer is written to <file>.partial, fsynced
 * and renamed.  A leftover checkpoint, completed or partial file makes the
 * call fail unless `resume` is set, in which case completed layers are
 * verified by their payload SHA-256 and the rest are packed.  Records that
 * read as all zeros stay holes of the pre-sized file (same bytes). */
typedef struct qf_store_pack_result {
    int32_t layers_written;
    uint64_t total_bytes;            /* 40 layer files */
    char source_index_sha256[65];
} qf_store_pack_result;
qf_status qf_store_pack(const char *model_path, const char *out_dir, int32_t resume, qf_store_pack_result *res);
/* QwenQ4ExpertStoreBuilder.verify (:182-199): opens the store against the
 * checkpoint's index and checks every layer's header and payload SHA-256. */
qf_status qf_store_verify(const char *model_path, const char *out_dir, int32_t *layers_verified);

/* ---- MLX checkpoint (safetensors) loader (host) ----------------------- */
/* The MoE tensors of one layer, read from the checkpoint the reference runs
 * (QwenQ4ActiveExpertStreamingRunner.swift:596-620, names resolved through
 * model.safetensors.index.json's weight_map, shard headers parsed as in
 * QwenQ4ExpertStoreBuilder.discoverSlices, :202-282), into the host-side
 * layout of qf_moe_layer:
 *   mlp.gate.{weight,scales,biases}               -> router_w / router_s / router_b
 *   mlp.shared_expert_gate.{weight,scales,biases} -> coef_w / coef_s / coef_b
 *   mlp.shared_expert.{gate,up,down}_proj.*       -> shared_record (one record)
 *   mlp.switch_mlp.{gate,up,down}_proj.*          -> expert_bank (256 records)
 * Tensor byte lengths are checked (as the builder does); scales and biases
 * must all be BF16 or all F16, reported through *scale_dtype.  Any dst
 * pointer may be NULL to skip that part.  Shard headers are parsed on first
 * use, so one qf_checkpoint is used by one thread at a time. */
typedef struct qf_checkpoint qf_checkpoint;
typedef struct qf_layer_host {
    void *router_w;       /* 524,288 bytes: Q8 codes [256][2048] */
    void *router_s;       /* 16,384 bytes: 16-bit [256][32] */
    void *router_b;
    void *coef_w;         /* 2,048 bytes */
    void *coef_s;         /* 64 bytes */
    void *coef_b;
    void *shared_record;  /* 1,769,472 bytes */
    void *expert_bank;    /* 256 records, record_stride bytes apart */
    uint64_t record_stride;
} qf_layer_host;
/* model_path: the directory holding model.safetensors.index.json and the shards. */
qf_status qf_checkpoint_open(const char *model_path, qf_checkpoint **out);
void qf_checkpoint_close(qf_checkpoint *c);
/* One layer's MoE weights (`threads` readers for the routed records, <= 0: 8). */
qf_status qf_checkpoint_load_layer(qf_checkpoint *c, int32_t layer, const qf_layer_host *dst,
                                   int32_t threads, int32_t *scale_dtype);
/* SHA-256 of n bytes as 64 lowercase hex characters + NUL (out: 65 bytes). */
qf_status qf_sha256_hex(const void *data, size_t n, char *out);
/* Message of the last failed qf_store_* / qf_checkpoint_* / qf_sha256_hex call
 * on this thread. */
const char *qf_store_last_error(void);

/* One batch-1 decode step through n_layers MoE blocks whose routed experts
 * stream through the cache: the active-streaming forwardToken MoE loop
 * (QwenQ4ActiveExpertStreamingRunner.swift:958-1381 with
 * Q4BoundedExpertCache.acquireSlotsParallel per layer).
 *   - Routing is supplied on the host: host_idx [n_layers * 8] expert ids and
 *     host_w [n_layers * 8] weights, layer-major.
 *   - The cache plans each layer's slots (it must have one partition per
 *     layer: layer_count == n_layers); misses are copied from host record
 *     layer * 256 + expert into their slots on the tier's stream, after the
 *     last earlier step that read an evicted slot, so copies for this step
 *     overlap the previous step's kernel.
 *   - The blocks then run as one persistent kernel on the handle's stream,
 *     reading routed records through the slot map (layers[l].expert_bank,
 *     record_stride and bank_records are replaced by the tier's arena).
 *   - x, residual, out: device, as for qf_moe_stack_forward at T = 1.
 *   - At most four steps are in flight; the fifth waits on the host. */
qf_status qf_moe_stream_step(qf_moe *h, qf_cache *c, qf_tier *t, const qf_moe_layer *layers,
                             int32_t n_layers, const int32_t *host_idx, const float *host_w,
                             const uint16_t *x, const float *residual, float *out, float eps,
                             void *workspace, size_t workspace_bytes);

/* ---- expert parallelism over NVLink ----------------------------------- */
/* No counterpart in the reference (single GPU).  The 256 routed experts are
 * split across `world` GPUs of one node, one process per GPU: rank r owns
 * experts [r * 256/world, (r+1) * 256/world) and each rank routes its own
 * tokens.  Every rank exports one device region (CUDA IPC); dispatch stores
 * routed token rows straight into the owners' regions over NVLink, the owners
 * run the grouped expert GEMMs on their own memory, and each rank pulls its
 * result rows back and combines them in router order (outputs bit-identical to
 * the single-GPU block).  All waits are bounded (QF_ERR_TIMEOUT via
 * qf_moe_check).  Setup, collective over the ranks:
 *   qf_ep_create -> qf_ep_ipc_handle -> (exchange the world handles on the
 *   host, rank order) -> qf_ep_connect.
 * Every rank must then make the same sequence of qf_moe_block_forward_ep
 * calls.  Before qf_ep_destroy, all ranks must have finished their last call
 * (a host barrier after synchronising the stream). */
#define QF_EP_HANDLE_BYTES 64
typedef struct qf_ep qf_ep;
/* world in {1, 2, 4, 8}; max_tokens: the most tokens any rank passes per call
 * (the same on every rank; it sizes the receive rows). */
qf_status qf_ep_create(qf_moe *h, int32_t rank, int32_t world, int32_t max_tokens, qf_ep **out);
qf_status qf_ep_ipc_handle(const qf_ep *ep, void *handle);
/* handles: world * QF_EP_HANDLE_BYTES bytes in rank order (this rank's entry is ignored). */
qf_status qf_ep_connect(qf_ep *ep, const void *handles);
void qf_ep_destroy(qf_ep *ep);
qf_status qf_ep_info(const qf_ep *ep, int32_t *experts_per_rank, int64_t *receive_rows,
                     uint64_t *region_bytes);
/* Deadline of each bounded wait of the EP kernels (a rank that never arrives),
 * 1 ms .. 60 s; default 2 s.  After a wait expired (QF_ERR_TIMEOUT from
 * qf_moe_check) the call's remaining kernels do no work and its output is
 * undefined; the EP group's counters no longer agree, so every rank destroys
 * its qf_ep and creates a new one.  The handle itself stays usable. */
qf_status qf_ep_set_timeout_ms(qf_ep *ep, uint32_t ms);
/* Down-at-home mode (enable 1; default 0, every rank the same): each owner
 * runs only the gate/up of its experts and returns the fp16 activation rows
 * (1 KB per routed row instead of 8 KB of fp32 results); every rank then runs
 * the down projection of its own tokens with all 256 experts.  Needs
 * layer->expert_bank to hold all 256 experts on every rank (the down
 * projections are replicated); outputs are bit-identical either way.  No
 * counterpart in the reference, which runs one GPU. */
qf_status qf_ep_set_down_at_home(qf_ep *ep, int32_t enable);
/* One MoE block over this rank's T tokens (T <= max_tokens), on the handle's
 * stream.  layer->expert_bank holds this rank's 256/world experts in order
 * (record i = expert rank * 256/world + i), or all 256 in down-at-home mode;
 * router, coefficient and shared expert are the full replicated weights.
 * routing: logit_bias, or a supplied top-k (topk_idx/topk_w, global expert
 * ids); record_of_pos is not supported. */
qf_status qf_moe_block_forward_ep(qf_ep *ep, const qf_moe_layer *layer, int32_t T,
                                  const uint16_t *x, const float *residual, float *out,
                                  const qf_routing *routing, int32_t *idx_out, float *w_out);

/* ---- kernel timing (bench harness) ----------------------------------- */
/* Records CUDA events around every launch of one kernel of the block
 * (0 router, 1 top-k/grouping, 2 gate/up, 3 down, 4 combine, 5 the persistent
 * decode kernel, 6 expert-parallel dispatch) issued on this
 * handle until qf_moe_profile_end, which synchronises and returns the summed
 * duration of the first min(launches, max_launches) recorded launches.
 * Launches captured into a CUDA graph report their most recent replay.
 * (Counterpart of the reference's GPU profile, gpuStartTime/gpuEndTime,
 * QwenQ4ActiveExpertStreamingRunner.swift:1486-1491.) */
qf_status qf_moe_profile_begin(qf_moe *h, int32_t kernel_id, int32_t max_launches);
qf_status qf_moe_profile_end(qf_moe *h, float *total_ms, int32_t *launches);

/* ---- seeded synthetic data (bench/test harness) ---------------------- */
/* Fills records for experts [expert0, expert0+count) of `layer` into
 * bank + (expert - expert0) * stride (device memory).  expert id 256 is the
 * shared expert.  Byte-identical to the CPU generator of the test oracle. */
qf_status qf_synth_records(qf_moe *h, uint64_t seed, uint32_t layer, uint32_t expert0,
                           uint32_t count, uint8_t *bank, uint64_t stride);
qf_status qf_synth_router(qf_moe *h, uint64_t seed, uint32_t layer, uint8_t *w, uint16_t *s,
                          uint16_t *b);
qf_status qf_synth_coef(qf_moe *h, uint64_t seed, uint32_t layer, uint8_t *w, uint16_t *s,
                        uint16_t *b);
/* host memory: fp16 bits [T * 2048], N(0,1) then RMS-normalised */
void qf_synth_hidden_host(uint64_t seed, uint64_t tok0, int32_t T, uint16_t *x);

#ifdef __cplusplus
}
#endif
#endif /* QF_MOE_H */
