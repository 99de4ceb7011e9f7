/*
 * qf_oracle.h -- CPU oracle for the QwenFieldfare MoE-block hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker, never the thing
 * measured or shipped: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * (libqf_moe.so) never links or calls it.
 *
 * What it restates (paths are inside the reference project
 * tanishqpatil/qwen-fieldfare):
 *   - Q4/Q8 MLX-affine dequant matvecs in the production SIMD lane order:
 *       Sources/QwenFieldfareCore/Metal/LinearAttention/deltanet.metal
 *       :1838-1895 (Q4 row), :1985-2048 (gate/up row), :2229-2260 (Q8 row)
 *   - router top-8 / softmax / renormalise            deltanet.metal:2283-2329
 *   - shared-expert gate coefficient (Q8, rows=1)      deltanet.metal:863-902
 *   - shared expert gate/up + down with sigmoid gate   deltanet.metal:2050-2122
 *   - routed subset gate/up + down, 8-way fixed sum    deltanet.metal:2155-2211
 *   - combine                                          deltanet.metal:2213-2227
 *   - RMSNorm (stack transition)                       deltanet.metal:18-53
 *   - expert-slot cache SLRU planner
 *       Sources/QwenFieldfareCore/Storage/Q4BoundedExpertCache.swift:52-400
 *   - bench SLRU replay   Sources/QwenFieldfareBench/main.swift:400-482
 * `simd_sum` has no specified order in Metal; the oracle (and the CUDA
 * kernels that must match it bit-exactly) use the xor butterfly 16,8,4,2,1.
 *
 * Parity status: the reference holds no numeric fixture for the matvec,
 * router or combine ("parity unpinned" for numerics); the cache planner,
 * slot planner and telemetry are pinned by the reference's own unit-test
 * known answers (tests/golden/).
 *
 * Build with -ffp-contract=off: every fused multiply-add below is an explicit
 * fmaf() so the arithmetic order is exactly the one written.
 */
#ifndef QF_ORACLE_H
#define QF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* geometry (Qwen3.6-35B-A3B MoE block) */
#define QFO_HIDDEN 2048
#define QFO_EXPERTS 256
#define QFO_TOPK 8
#define QFO_INTER 512
#define QFO_GROUP 64
#define QFO_RECORD_BYTES 1769472ull

/* byte offsets inside one expert record (QwenQ4ExpertStoreBuilder.swift:47-56) */
#define QFO_OFF_GATE_W 0u
#define QFO_OFF_GATE_S 524288u
#define QFO_OFF_GATE_B 557056u
#define QFO_OFF_UP_W 589824u
#define QFO_OFF_UP_S 1114112u
#define QFO_OFF_UP_B 1146880u
#define QFO_OFF_DOWN_W 1179648u
#define QFO_OFF_DOWN_S 1703936u
#define QFO_OFF_DOWN_B 1736704u

/* 16-bit float helpers (round-to-nearest-even) */
float qfo_f16_to_f32(uint16_t h);
uint16_t qfo_f32_to_f16(float f);
float qfo_bf16_to_f32(uint16_t h);
uint16_t qfo_f32_to_bf16(float f);

/* ---- seeded synthetic data (counter-based SplitMix64) ---- */
uint64_t qfo_stream_key(uint64_t seed, uint32_t layer, uint32_t tag, uint32_t index);
uint64_t qfo_draw(uint64_t key, uint64_t i);
/* one expert record (routed expert `expert`, or the shared expert when expert == 256) */
void qfo_synth_expert_record(uint64_t seed, uint32_t layer, uint32_t expert, int scale_bf16,
                             uint8_t *record);
/* router Q8 [256 x 2048] codes, scales, biases */
void qfo_synth_router(uint64_t seed, uint32_t layer, int scale_bf16, uint8_t *w, uint16_t *s,
                      uint16_t *b);
/* shared-expert gate coefficient Q8 [1 x 2048] */
void qfo_synth_coef(uint64_t seed, uint32_t layer, int scale_bf16, uint8_t *w, uint16_t *s,
                    uint16_t *b);
/* fp16 hidden states for global tokens [tok0, tok0+T): N(0,1) then RMS-normalised */
void qfo_synth_hidden(uint64_t seed, uint64_t tok0, int T, uint16_t *x);

/* ---- one MoE layer's weights as host pointers ---- */
typedef struct {
    const uint8_t *router_w;  /* [256*2048] */
    const uint16_t *router_s; /* [256*32] */
    const uint16_t *router_b;
    const uint8_t *coef_w; /* [2048] */
    const uint16_t *coef_s; /* [32] */
    const uint16_t *coef_b;
    const uint8_t *shared_record;        /* one record */
    const uint8_t *const *expert_records; /* [256] record pointers */
    int scale_bf16;                      /* 0: fp16 scales/biases, 1: bf16 */
} qfo_layer;

/* reference-order primitives */
float qfo_q4_row(const uint8_t *w_row, const uint16_t *s_row, const uint16_t *b_row,
                 const float *vec, int cols, int scale_bf16);
float qfo_q8_row(const uint8_t *w_row, const uint16_t *s_row, const uint16_t *b_row,
                 const float *vec, int scale_bf16);
void qfo_router_logits(const qfo_layer *L, const float *x, float *logits);
/* deltanet.metal:1897-1919 qwen_gemv_q4_affine_simd_f32 with cols 2048, the
 * LM head (QwenQ4ActiveExpertStreamingRunner.swift:1393-1400): out[r] =
 * qfo_q4_row of row r; w [rows][1024], s/b [rows][32] */
void qfo_lm_head(const uint8_t *w, const uint16_t *s, const uint16_t *b, int rows, const float *x,
                 int scale_bf16, float *out);
/* top-k by logit (ties -> lower index), softmax over all, renormalise over top-k */
void qfo_topk(const float *logits, const float *bias, int n, int k, int32_t *idx, float *w);
float qfo_coef(const qfo_layer *L, const float *x);
void qfo_gate_up(const uint8_t *record, int scale_bf16, const float *x, float *act);
void qfo_down(const uint8_t *record, int scale_bf16, const float *act, float *y);
/* combine of one token: y [8][2048] in router order, w [8], shared y [2048],
 * shared-gate pre-activation c, residual [2048] or NULL */
void qfo_combine(const float *y, const float *w, const float *sh_y, float c, const float *res,
                 float *out);

/*
 * One MoE block over T tokens.
 *   x          fp16 [T*2048] post-norm hidden (what router and experts read)
 *   residual   fp32 [T*2048] or NULL (0)
 *   bias       fp32 [256] router logit bias or NULL
 *   idx_in/w_in  supplied routing [T*8] or NULL (router decides)
 *   out        fp32 [T*2048]
 *   idx_out/w_out/logits_out/coef_out optional
 * threads: OpenMP threads over tokens (<=0: library default)
 */
void qfo_block(const qfo_layer *L, int T, const uint16_t *x, const float *residual,
               const float *bias, const int32_t *idx_in, const float *w_in, float *out,
               int32_t *idx_out, float *w_out, float *logits_out, float *coef_out, int threads);

/* RMSNorm of the stack transition (deltanet.metal:18-53) in a fixed order: 128 tiles of
 * 16 elements, fma chain per tile, tiles summed in order; out = fp16(in * inv) */
void qfo_rmsnorm_to_f16(const float *in, int T, float eps, uint16_t *x_out);
/* deltanet.metal:18-53 qwen_rmsnorm_f32 with 64 threads (the post-attention
 * norm, QwenQ4ActiveExpertStreamingRunner.swift:1169-1176), weighted, then fp16 */
void qfo_post_norm_to_f16(const float *in, const float *w, int T, float eps, uint16_t *x_out);

/* stable dispatch plan: counts[E], offsets[E+1], perm[T*k] sorted by (expert, token, k) */
void qfo_dispatch_plan(const int32_t *idx, int T, int k, int E, int32_t *counts,
                       int32_t *offsets, int32_t *perm);

/* ---- expert-slot cache: exact port of Q4BoundedExpertCache ---- */
typedef struct qfo_cache qfo_cache;
qfo_cache *qfo_cache_create(int capacity, double probationary_ratio, int requested_layers,
                            int key_layers, int key_experts);
void qfo_cache_destroy(qfo_cache *c);
/* acquireSlotsParallel: slots[n'] (n' = min(n,8)); miss_pos[] and *n_miss are the
 * positions whose expert missed; fetch_expert/fetch_slot (optional, size 8) list
 * the planned fetches in order; returns n' */
int qfo_cache_acquire(qfo_cache *c, int layer, const uint32_t *experts, int n, uint32_t *slots,
                      uint32_t *miss_pos, int *n_miss, uint32_t *fetch_expert,
                      uint32_t *fetch_slot, int *n_fetch);
void qfo_cache_prefetch(qfo_cache *c, int layer, const uint32_t *cands, int n);
void qfo_cache_clear(qfo_cache *c);
void qfo_cache_reset_metrics(qfo_cache *c);
/* metrics: capacity, occupancy, probationary, protected, hits, misses, evictions,
 * fetched_bytes, prefetch_requests, useful_prefetch_hits, wasted_prefetches */
void qfo_cache_metrics(const qfo_cache *c, int64_t out[11]);
int qfo_cache_layer_count(const qfo_cache *c);
void qfo_cache_layer_capacities(const qfo_cache *c, int32_t *out);
int qfo_cache_probationary_capacity(const qfo_cache *c);

/* bench replay: Sources/QwenFieldfareBench/main.swift:400-482 (returns misses) */
int64_t qfo_slru_replay(const uint16_t *trace, int64_t n, int capacity);

#ifdef __cplusplus
}
#endif
#endif
