// qf_fused1.cu -- persistent decode kernel for ONE token (T = 1) through a
// stack of MoE blocks: one cooperative launch, one CTA per SM (>= 128 SMs).
//
// A batch-1 block reads ~16.5 MB of weights, 2.6 us at HBM speed; what costs
// time is the dependency chain x -> router -> top-8 -> gate/up -> down ->
// combine -> RMSNorm -> next x.  This kernel shortens the time spent waiting
// on memory along that chain:
//   - weights that do not depend on the token (router rows, the shared-gate
//     row, the shared expert) are copied into shared memory one layer ahead,
//     into one of two per-layer buffers (layer parity);
//   - right after top-k every CTA issues ALL of its routed weight rows (its
//     gate/up tiles and the down rows of its output tile), ~110 KB per SM as
//     16-byte cp.async from all 512 threads (about 14 per thread), so the
//     routed set of the layer (~14 MB) is in flight at once; the down rows
//     land while gate/up computes;
//   - the 8 positions of the token are 8 records, no grouping (a record named
//     twice is fetched twice).
// Rows land at a padded pitch so that the mma.sync fragment reads are free of
// bank conflicts.
//
// Work of CTA b per layer:
//   R  b < 64: shared-expert gate/up row pairs [8b, 8b+8); 64 <= b < 96: router
//      rows [8(b-64), +8) in the reference lane order (deltanet.metal:2229-2281);
//      b == 96: the shared-gate coefficient row (deltanet.metal:863-902).
//   E  top-8 (every CTA, one warp; deltanet.metal:2283-2329) -> issue the routed
//      copies -> routed gate/up tiles i = b and b + G (< 256): position i / 32,
//      row pairs [16 (i % 32), +16) (deltanet.metal:2155-2179).
//   D  b < 128: output rows [16b, 16b + 16) of the 8 routed and the shared down
//      projections (deltanet.metal:2181-2211, 2099-2122), the router-order
//      combine (deltanet.metal:2213-2227) and the RMS partial of those rows for
//      the next block's RMSNorm (deltanet.metal:18-53).
// No grid barriers: every vector that crosses CTAs (logits + coefficient, the
// activations, the block output + RMS partials) is written as 8-byte words
// {32-bit value, layer tag}, single-copy atomic, and the consumers poll the
// words until every tag is the layer's (bounded).  Single buffers suffice:
// every CTA contributes gate/up tiles to every layer, so a writer of layer
// l + 1 has, through the chain of data it waited for, seen every CTA finish
// reading layer l's copy of the same buffer.
// Arithmetic: exact Q4 dequant on mma.sync with fp32 accumulation (see
// qf_persist.cuh), fixed reduction orders, so results are bit-reproducible run
// to run; router logits are bit-exact with the CPU oracle.
#include <math.h>

#include "qf_persist.cuh"

namespace qf {

namespace {

using namespace pk;

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxLayers = 64;

// ---- tile layouts in shared memory (bytes)
constexpr int kGuPitch = 1024 + 32;  // padded Q4 row, K = 2048
constexpr int kDnPitch = 256 + 32;   // padded Q4 row, K = 512
// MMA tile of a gate/up projection: rows 0..7 gate rows r..r+7, rows 8..15 up
// rows r..r+7; then s[16][32] and b[16][32] (16-bit) in the same row order.
constexpr int kGuTileBytes = 16 * kGuPitch + 2048;  // 18944
// Down tile: 16 rows of K = 512, then s[16][8], b[16][8].
constexpr int kDnTileBytes = 16 * kDnPitch + 512;  // 5120
constexpr int kRPart = kGuTileBytes;               // R task: >= 8 router rows + s/b (17408)
constexpr int kDiBytes = kRPart + kDnTileBytes;    // token-independent part of a CTA
static_assert(8 * 2048 + 2 * 512 <= kRPart, "R part");

constexpr int kNShGu = 64;                       // shared gate/up MMA tiles (8 row pairs)
constexpr int kNRouter = 32;                     // router tasks (8 rows)
constexpr int kNR = kNShGu + kNRouter + 1;       // + the coefficient row: 97 CTAs
constexpr int kNGu = kTopK * (kInter / 16);      // routed gate/up tiles of 16 row pairs: 256
constexpr int kNOut = kHidden / 16;              // output tiles: 128 CTAs
constexpr int kMaxGu = 2;                        // routed gate/up tiles per CTA (G >= 128)
constexpr int kMinGrid = kNGu / kMaxGu;          // 128
constexpr int kRoutedBytes = kMaxGu * 2 * kGuTileBytes + kTopK * kDnTileBytes;  // 116736
constexpr int kDnCols = kTopK + 1;               // down columns: 8 routed + shared
constexpr int kItemsD = kDnCols * 4;             // (column, K-quarter) items of phase D

struct Misc1 {
  int pred[kTopK];  // predicted (or known) records of the next layer
  int idx[kTopK];
  float w[kTopK];
  int rec[kTopK];
  float vs[kExperts];
  int cols[kDnCols][8];  // cols[e] = {e, -1, ...}: MMA column 0 <- fragment column e
  float res[16];         // residual of this CTA's output rows (layers > 0)
  float coef;            // shared-gate coefficient of the layer
  float inv;
  int fail;
};

constexpr int kOffDi = 0;
constexpr int kOffRouted = kOffDi + 2 * kDiBytes;
// The activations cross CTAs as fp16 pairs: 9 columns (8 routed positions,
// then the shared expert) of 512 values.
constexpr int kActWords = kDnCols * kInter / 2;  // 2304
constexpr int kPollWords = kActWords;            // staging area (u32 words)
static_assert(kPollWords >= kHidden + kHidden / 16 && kPollWords >= 2 * 8 * 4 * 32, "poll area");
constexpr int kOffPoll = kOffRouted + kRoutedBytes;   // u32 [kPollWords]
constexpr int kOffXh = kOffPoll + kPollWords * 4;
constexpr int kOffXfrag = kOffXh + kHidden * 2;        // [32 groups][1 col][4][32 B]
constexpr int kOffAfrag = kOffXfrag + 32 * 128;        // [8 groups][9 cols][4][32 B]
constexpr int kOffXS = kOffAfrag + 8 * kDnCols * 128;
constexpr int kOffXC = kOffXS + 32 * 4;
constexpr int kOffAS = kOffXC + 32 * 4;
constexpr int kOffAC = kOffAS + 8 * kDnCols * 4;
constexpr int kOffRed = kOffAC + 8 * kDnCols * 4;
constexpr int kRedFloats = kItemsD * 16 + 16;
constexpr int kOffMisc = (kOffRed + kRedFloats * 4 + 127) & ~127;
constexpr int kOffBar = (kOffMisc + (int)sizeof(Misc1) + 127) & ~127;
constexpr int kNBars = 6;  // dib[2] (token-independent, by layer parity), rgu[2], rdn, pred
// Speculative prefetch of the next layer's routed records.  The CTAs past the
// output tiles (b >= 128: no R task, no D phase, one routed gate/up tile)
// predict layer l + 1's top-8 by applying layer l + 1's router to x_l (the
// residual stream changes little from layer to layer: about 85% of the next
// layer's experts are predicted on the synthetic 40-layer stack), once their
// own gate/up tile of layer l is done, i.e. after the bulk of layer l's
// routed fetch; they then prefetch the 8 predicted records (14.2 MB) into L2,
// split among them, while HBM is otherwise idle (layer l's down phase, the
// next prologue, router and top-8).  Layer l + 1's routed copies then hit L2
// for the predicted experts.  With supplied routing (idx_in) the next layer's
// records are known and prefetched exactly.  Results are unaffected: only
// the prefetch is speculative.
constexpr int kPredMinCtas = 16;                  // predictor CTAs needed (rows per CTA <= 16)
constexpr int kPredMaxRows = kExperts / kPredMinCtas;
constexpr int kPredRowBytes = 2048 + 2 * 64;      // codes + scales + biases of a router row
constexpr int kOffPred = 2 * kGuTileBytes;        // inside the routed area: predictors use tile 0 only
constexpr int kPredChunk = 16384;                 // L2 prefetch granule
constexpr int kChunksPerRecord = static_cast<int>(kRecordBytes / kPredChunk);  // 108
static_assert(kRecordBytes % kPredChunk == 0, "record = whole prefetch chunks");
static_assert(kOffPred + kPredMaxRows * kPredRowBytes <= kRoutedBytes, "prediction rows fit");
constexpr int kSmemBytes = kOffBar + kNBars * 8;
static_assert(kSmemBytes <= 227 * 1024, "shared memory");
static_assert(kOffXfrag % 16 == 0 && kOffAfrag % 16 == 0 && kOffRouted % 128 == 0, "alignment");
static_assert(kGuTileBytes % 16 == 0 && kDnTileBytes % 16 == 0 && kDiBytes % 128 == 0, "alignment");

struct Fused1Args {
  int n_layers;      // layers in this launch
  int first_layer;   // global index of layer 0 of this launch
  int total_layers;  // layers of the whole stack
  const uint16_t* x0;
  const float* res0;
  // optional: x_0 = fp16(post-attention RMSNorm(pre_h) * pre_w) computed here
  // (deltanet.metal:18-53 order, 64 threads) instead of read from x0
  const float* pre_h;
  const float* pre_w;
  float pre_eps;
  float* out;
  float eps;
  RoutingArgs r;
  int* idx_out;
  float* w_out;
  // 8-byte words {value bits, tag = global layer index + 1}, cleared per call
  uint64_t* ll_logits;  // [257]: router logits, then the shared-gate coefficient
  uint64_t* ll_act;     // [9 * 256]: fp16 pairs; rows 0..7 routed positions, 8 the shared expert
  uint64_t* ll_h;       // [2048 + 128]: block output, then the RMS partials of its row tiles
  uint64_t* ll_pred;    // [256]: predicted logits of the next layer (tag = next layer + 1)
  int* status;
  LayerW layers[kMaxLayers];
};

template <bool BF16>
__device__ __forceinline__ float cvt16(uint16_t u) {
  if constexpr (BF16) {
    return __uint_as_float(static_cast<uint32_t>(u) << 16);
  } else {
    return __half2float(__ushort_as_half(u));
  }
}

// ---- copies: 16-byte cp.async spread over all threads of the CTA (a TMA bulk
// copy per row would cost ~40 ns of issue each, and rows must land at a padded
// pitch); completion: every thread arrives on the stage's mbarrier (count =
// kThreads) once its copies so far have landed.
//
// Chunks [0, rows << lg) of a block of rows (2^lg chunks of 16 B per row),
// dealt round-robin over the threads starting at thread t0; returns the next
// segment's t0 so that consecutive segments stay balanced.
__device__ __forceinline__ int copy_block(unsigned char* dst, int dst_pitch, const uint8_t* src,
                                          int src_pitch, int rows, int lg, int t0) {
  const int n = rows << lg;
  for (int c = (static_cast<int>(threadIdx.x) - t0) & (kThreads - 1); c < n; c += kThreads) {
    const int r = c >> lg, q = c & ((1 << lg) - 1);
    cp_async16(dst + r * dst_pitch + q * 16, src + static_cast<size_t>(r) * src_pitch + q * 16);
  }
  return (t0 + n) & (kThreads - 1);
}
// MMA gate/up tile of record `rec`, row pairs [r, r + 8): 8 gate + 8 up rows, then
// gate S, up S, gate B, up B (8 rows x 64 B each)
__device__ __forceinline__ int copy_gu(unsigned char* tile, const uint8_t* rec, int r, int t0) {
  t0 = copy_block(tile, kGuPitch, rec + kOffGateW + static_cast<size_t>(r) * 1024, 1024, 8, 6, t0);
  t0 = copy_block(tile + 8 * kGuPitch, kGuPitch, rec + kOffUpW + static_cast<size_t>(r) * 1024, 1024, 8, 6, t0);
  unsigned char* sb = tile + 16 * kGuPitch;
  t0 = copy_block(sb, 0, rec + kOffGateS + r * 64, 0, 1, 5, t0);
  t0 = copy_block(sb + 512, 0, rec + kOffUpS + r * 64, 0, 1, 5, t0);
  t0 = copy_block(sb + 1024, 0, rec + kOffGateB + r * 64, 0, 1, 5, t0);
  return copy_block(sb + 1536, 0, rec + kOffUpB + r * 64, 0, 1, 5, t0);
}
// down tile of output rows [16 j, 16 j + 16): 16 rows of 256 B, then S and B (256 B each)
__device__ __forceinline__ int copy_dn(unsigned char* tile, const uint8_t* rec, int j, int t0) {
  t0 = copy_block(tile, kDnPitch, rec + kOffDownW + static_cast<size_t>(j) * 4096, 256, 16, 4, t0);
  t0 = copy_block(tile + 16 * kDnPitch, 0, rec + kOffDownS + j * 256, 0, 1, 4, t0);
  return copy_block(tile + 16 * kDnPitch + 256, 0, rec + kOffDownB + j * 256, 0, 1, 4, t0);
}

// The token-independent rows CTA b needs for layer L (all threads): its R task
// and the shared expert's down tile of its output rows; completion on `bar`.
__device__ void issue_di(const LayerW& L, int b, unsigned char* buf, uint64_t* bar) {
  int t0 = 0;
  if (b < kNShGu) {
    t0 = copy_gu(buf, L.shared, 8 * b, t0);
  } else if (b < kNShGu + kNRouter) {
    const int r0 = 8 * (b - kNShGu);
    t0 = copy_block(buf, 2048, L.rw + static_cast<size_t>(r0) * 2048, 2048, 8, 7, t0);
    t0 = copy_block(buf + 8 * 2048, 0, reinterpret_cast<const uint8_t*>(L.rs + r0 * 32), 0, 1, 5, t0);
    t0 = copy_block(buf + 8 * 2048 + 512, 0, reinterpret_cast<const uint8_t*>(L.rb + r0 * 32), 0, 1, 5, t0);
  } else if (b < kNR) {
    t0 = copy_block(buf, 0, L.cw, 0, 1, 7, t0);
    t0 = copy_block(buf + 2048, 0, reinterpret_cast<const uint8_t*>(L.cs), 0, 1, 2, t0);
    t0 = copy_block(buf + 2048 + 64, 0, reinterpret_cast<const uint8_t*>(L.cb), 0, 1, 2, t0);
  }
  if (b < kNOut) copy_dn(buf + kRPart, L.shared, b, t0);
  cp_async_arrive(bar);
}

// Router rows from shared memory in the reference lane order
// (deltanet.metal:2229-2260): lane l of a row takes columns 8 l .. 8 l + 7 of
// each 256-column block; per block a dot of the 8 codes with x (fma chain) and
// the sum of the 8 x values (add chain), then acc = fma(s, dot, acc),
// acc = fma(b, sum, acc) block after block, and finally the xor-butterfly
// simd_sum.  Two warps share a row: one computes blocks 0..3, the other the
// dots and sums of blocks 4..7, which the first folds into its chain.
template <bool BF16>
__device__ __forceinline__ void router_blocks(const unsigned char* buf, int w, int h, const __half* xh, int lane,
                                              float (&dot)[4], float (&sum)[4]) {
  const uint8_t* wrow = buf + w * 2048;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int blk = 4 * h + i;
    const uint2 wv = *reinterpret_cast<const uint2*>(wrow + blk * 256 + lane * 8);
    const uint4 hv = *reinterpret_cast<const uint4*>(xh + blk * 256 + lane * 8);
    const float2 p0 = __half22float2(*reinterpret_cast<const __half2*>(&hv.x));
    const float2 p1 = __half22float2(*reinterpret_cast<const __half2*>(&hv.y));
    const float2 p2 = __half22float2(*reinterpret_cast<const __half2*>(&hv.z));
    const float2 p3 = __half22float2(*reinterpret_cast<const __half2*>(&hv.w));
    const float e[8] = {p0.x, p0.y, p1.x, p1.y, p2.x, p2.y, p3.x, p3.y};
    float d = 0.f;
#pragma unroll
    for (int k = 0; k < 4; k++) d = __fmaf_rn(byte_f(wv.x, k), e[k], d);
#pragma unroll
    for (int k = 0; k < 4; k++) d = __fmaf_rn(byte_f(wv.y, k), e[4 + k], d);
    float sm = e[0];
#pragma unroll
    for (int k = 1; k < 8; k++) sm = __fadd_rn(sm, e[k]);
    dot[i] = d;
    sum[i] = sm;
  }
}
template <bool BF16>
__device__ __forceinline__ float router_chain(const unsigned char* buf, int w, int h, int lane, const float (&dot)[4],
                                              const float (&sum)[4], float acc) {
  const uint16_t* srow = reinterpret_cast<const uint16_t*>(buf + 8 * 2048) + w * 32;
  const uint16_t* brow = reinterpret_cast<const uint16_t*>(buf + 8 * 2048 + 512) + w * 32;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int gq = (4 * h + i) * 4 + (lane >> 3);
    acc = __fmaf_rn(cvt16<BF16>(srow[gq]), dot[i], acc);
    acc = __fmaf_rn(cvt16<BF16>(brow[gq]), sum[i], acc);
  }
  return acc;
}

// The shared-gate coefficient (one warp; deltanet.metal:863-902 with rows = 1):
// lane l takes columns [64 l, 64 l + 64), dequantised element by element.
template <bool BF16>
__device__ __forceinline__ float coef_row(const unsigned char* buf, const __half* xh, int lane) {
  const float cs = cvt16<BF16>(reinterpret_cast<const uint16_t*>(buf + 2048)[lane]);
  const float cb = cvt16<BF16>(reinterpret_cast<const uint16_t*>(buf + 2048 + 64)[lane]);
  uint4 cwv[4];
#pragma unroll
  for (int q = 0; q < 4; q++) cwv[q] = reinterpret_cast<const uint4*>(buf + lane * 64)[q];
  float acc = 0.f;
#pragma unroll
  for (int q = 0; q < 4; q++) {
#pragma unroll
    for (int d = 0; d < 4; d++) {
      const uint32_t wd = word_of(cwv[q], d);
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float xe = __half2float(xh[lane * 64 + q * 16 + d * 4 + k]);
        acc = __fmaf_rn(__fmaf_rn(byte_f(wd, k), cs, cb), xe, acc);
      }
    }
  }
  return warp_sum(acc);
}

__device__ __forceinline__ uint32_t h2bits(__half lo, __half hi) {
  return static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}

// ---- 8-byte {value, tag} words
__device__ __forceinline__ void ll_put(uint64_t* p, uint32_t v, uint32_t tag) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"((static_cast<uint64_t>(tag) << 32) | v)
               : "memory");
}
__device__ __forceinline__ uint64_t ll_get(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// All threads: the values of words [0, n) once each carries `tag`, handed to
// sink(i, value).  Each round re-issues every word that still
// carries an older tag, so a round costs one memory round trip whatever the
// count.  Bounded: on expiry sets the status word and *fail, and returns with
// dst partly stale.
template <int U>
__device__ __forceinline__ bool ll_wait(const uint64_t* const (&src)[U], uint64_t (&v)[U], const bool (&use)[U],
                                        uint32_t tag, int* status, int* fail) {
  for (unsigned round = 0;; round++) {
    bool ready = true;
#pragma unroll
    for (int u = 0; u < U; u++) ready &= !use[u] || static_cast<uint32_t>(v[u] >> 32) == tag;
    if (ready) return true;
    if (round > kSpinLimit) {
      set_status(status, kStatusTimeout);
      *fail = 1;
      return false;
    }
    if (round > 32) __nanosleep(64);
#pragma unroll
    for (int u = 0; u < U; u++)
      if (use[u] && static_cast<uint32_t>(v[u] >> 32) != tag) v[u] = ll_get(src[u]);
  }
}
template <typename Sink>
__device__ __forceinline__ void ll_poll(const uint64_t* src, int n, uint32_t tag, Sink sink, int* status,
                                        int* fail) {
  constexpr int U = 5;  // one pass covers the largest vector (2304 words)
  for (int base = 0; base < n; base += U * kThreads) {
    const uint64_t* p[U];
    uint64_t v[U];
    bool use[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int i = base + u * kThreads + static_cast<int>(threadIdx.x);
      use[u] = i < n;
      p[u] = src + (use[u] ? i : 0);
      v[u] = use[u] ? ll_get(p[u]) : 0;
    }
    ll_wait<U>(p, v, use, tag, status, fail);
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int i = base + u * kThreads + static_cast<int>(threadIdx.x);
      if (use[u]) sink(i, static_cast<uint32_t>(v[u]));
    }
  }
}
// Warp 0 of every CTA: polls the 256 router logits (lane l takes experts
// 32 j + l) and the shared-gate coefficient straight into registers, then
// selects the top 8 in the order of the reference (descending logit, ties to
// the lower expert index; deltanet.metal:2283-2329): each lane sorts its 8
// candidates once (19-comparator network on (ordered value, -j) keys), then 8
// rounds take the largest lane head (warp max, then the lowest expert index
// among the lanes that hold it) and pop it.  Writes idx[k], the selected
// (biased) logits sel[k], the 256 biased logits vs[] and *coef.
__device__ __forceinline__ void topk_poll_select(const uint64_t* ll, uint32_t tag, const float* bias, int lane,
                                                 int* idx, float* sel, float* vs, float* coef, int* status,
                                                 int* fail) {
  const uint64_t* p[9];
  uint64_t w[9];
  bool use[9];
#pragma unroll
  for (int j = 0; j < 9; j++) {
    p[j] = j < 8 ? ll + j * 32 + lane : ll + kExperts;
    use[j] = true;
    w[j] = ll_get(p[j]);
  }
  ll_wait<9>(p, w, use, tag, status, fail);
  const uint64_t wc = w[8];
  if (lane == 0) *coef = __uint_as_float(static_cast<uint32_t>(wc));
  uint64_t c[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int e = j * 32 + lane;
    const float lg = __uint_as_float(static_cast<uint32_t>(w[j]));
    const float v = bias ? __fadd_rn(lg, __ldg(bias + e)) : lg;
    vs[e] = v;
    c[j] = (static_cast<uint64_t>(f2ord(v)) << 3) | static_cast<uint64_t>(7 - j);
  }
  // sort descending: larger value first, equal values by lower j
  auto cx = [&](int i0, int i1) {
    const uint64_t hi = c[i0] > c[i1] ? c[i0] : c[i1];
    const uint64_t lo = c[i0] > c[i1] ? c[i1] : c[i0];
    c[i0] = hi;
    c[i1] = lo;
  };
  cx(0, 1); cx(2, 3); cx(4, 5); cx(6, 7);
  cx(0, 2); cx(1, 3); cx(4, 6); cx(5, 7);
  cx(1, 2); cx(5, 6); cx(0, 4); cx(3, 7);
  cx(1, 5); cx(2, 6);
  cx(1, 4); cx(3, 6);
  cx(2, 4); cx(3, 5);
  cx(3, 4);
#pragma unroll 1
  for (int k = 0; k < kTopK; k++) {
    const uint32_t key = static_cast<uint32_t>(c[0] >> 3);
    const uint32_t mx = __reduce_max_sync(0xffffffffu, key);
    const uint32_t e = (7u - static_cast<uint32_t>(c[0] & 7u)) * 32u + static_cast<uint32_t>(lane);
    const uint32_t win = __reduce_min_sync(0xffffffffu, key == mx ? e : 0xffffffffu);
    if (static_cast<int>(win & 31u) == lane) {
#pragma unroll
      for (int j = 0; j < 7; j++) c[j] = c[j + 1];
      c[7] = 0;
    }
    if (lane == k) {
      idx[k] = static_cast<int>(win);
      sel[k] = ord2f(mx);
    }
  }
}

// Routing weights of the selected 8 (deltanet.metal:2283-2329): softmax over
// all 256 (biased) logits, renormalised over the 8; same operation order as
// pk::topk_weights, with lane k computing weight k.  w[k] holds the selected
// logit on entry and the weight on exit.
__device__ __forceinline__ void topk_weights1(const float* vs, int lane, float* w) {
  const float mxv = w[0];
  float den = 0.f;
#pragma unroll 1
  for (int j = 0; j < 8; j++) den = __fadd_rn(den, expf(__fsub_rn(vs[j * 32 + lane], mxv)));
  den = warp_sum(den);
  const float p = __fdiv_rn(expf(__fsub_rn(w[lane & 7], mxv)), den);
  float ps = __shfl_sync(0xffffffffu, p, 0);
#pragma unroll 1
  for (int k = 1; k < kTopK; k++) ps = __fadd_rn(ps, __shfl_sync(0xffffffffu, p, k));
  __syncwarp();
  if (lane < kTopK) w[lane] = __fdiv_rn(p, ps);
}

// fp16 vectors as MMA B fragments: pk::stage_block for fp16 sources with the
// pass loop rolled (this code runs once per layer; see the note on instruction
// fetch above k_fused1)
__device__ __forceinline__ void stage_f16(const __half* src, int nvec, int ngrp, int vec_stride, int ncols,
                                          __half* frag, float* S, float* C) {
  const int items = nvec * ngrp * 8;
#pragma unroll 1
  for (int base = 0; base < items; base += kThreads) {
    const int item = base + static_cast<int>(threadIdx.x);
    float s_part = 0.f, c_part = 0.f;
    int v = 0, g = 0;
    if (item < items) {
      v = item / (ngrp * 8);
      g = (item >> 3) % ngrp;
      const int q = item & 7;
      const uint4 hv = *reinterpret_cast<const uint4*>(src + v * vec_stride + g * 64 + q * 8);
      const __half* h8 = reinterpret_cast<const __half*>(&hv);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int e = q * 8 + j;
        const __half xh = h8[j];
        const __half fed = (e & 1) ? __float2half_rn(__half2float(xh) * 0.0625f) : xh;
        frag[(((size_t)g * ncols + v) * 4 + (e >> 4)) * 16 + frag_half(e)] = fed;
        s_part += __half2float(xh);
        c_part += __half2float(fed);
      }
    }
#pragma unroll
    for (int mm = 1; mm < 8; mm <<= 1) {
      s_part += __shfl_xor_sync(0xffffffffu, s_part, mm);
      c_part += __shfl_xor_sync(0xffffffffu, c_part, mm);
    }
    if (item < items && (item & 7) == 0) {
      S[g * ncols + v] = s_part;
      C[g * ncols + v] = 1024.f * c_part;
    }
  }
}

// Predictor p's router rows [r0, r0 + n) of a layer: codes row-major, then
// the scales, then the biases (64 bytes a row each); completion on `bar`.
__device__ void issue_pred_rows(const LayerW& L, int r0, int n, unsigned char* buf, uint64_t* bar) {
  int t0 = copy_block(buf, 2048, L.rw + static_cast<size_t>(r0) * 2048, 2048, n, 7, 0);
  t0 = copy_block(buf + n * 2048, 64, reinterpret_cast<const uint8_t*>(L.rs + r0 * 32), 64, n, 2, t0);
  copy_block(buf + n * 2048 + n * 64, 64, reinterpret_cast<const uint8_t*>(L.rb + r0 * 32), 64, n, 2, t0);
  cp_async_arrive(bar);
}

// One predicted logit per warp (rows w, w + 16, ...): the router row dotted
// with x (fp16) in the reference's per-lane order; only a prediction, so the
// order is not load-bearing.
template <bool BF16>
__device__ void predict_rows(const unsigned char* buf, int n, const __half* xh, int lane, int warp,
                             uint64_t* ll_pred, int r0, uint32_t tag) {
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(buf + n * 2048);
  const uint16_t* bi = sc + n * 32;
#pragma unroll 1
  for (int w = warp; w < n; w += kWarps) {
    float acc = 0.f;
#pragma unroll 1
    for (int blk = 0; blk < 8; blk++) {
      const uint2 wv = *reinterpret_cast<const uint2*>(buf + w * 2048 + blk * 256 + lane * 8);
      const uint4 hv = *reinterpret_cast<const uint4*>(xh + blk * 256 + lane * 8);
      const __half2* h2 = reinterpret_cast<const __half2*>(&hv);
      float d = 0.f, sm = 0.f;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float2 xf = __half22float2(h2[k]);
        const uint32_t wd = k < 2 ? wv.x : wv.y;
        d = __fmaf_rn(byte_f(wd, (2 * k) & 3), xf.x, d);
        d = __fmaf_rn(byte_f(wd, (2 * k + 1) & 3), xf.y, d);
        sm = __fadd_rn(__fadd_rn(sm, xf.x), xf.y);
      }
      const int g = blk * 4 + (lane >> 3);
      acc = __fmaf_rn(cvt16<BF16>(sc[w * 32 + g]), d, acc);
      acc = __fmaf_rn(cvt16<BF16>(bi[w * 32 + g]), sm, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) ll_put(ll_pred + r0 + w, __float_as_uint(acc), tag);
  }
}

// Warp 0 of a predictor: the 256 predicted logits (bounded wait; on expiry
// the prefetch is skipped, nothing is reported: it is only a prefetch), the
// top 8 of them (+ the harness bias), written to ex[8].  Returns false when
// the logits did not all arrive.
__device__ bool predict_top8(const uint64_t* ll_pred, uint32_t tag, const float* bias, int lane, int* ex) {
  uint64_t v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] = ll_get(ll_pred + j * 32 + lane);
#pragma unroll 1
  for (unsigned round = 0;; round++) {
    bool ready = true;
#pragma unroll
    for (int j = 0; j < 8; j++) ready &= static_cast<uint32_t>(v[j] >> 32) == tag;
    if (__all_sync(0xffffffffu, ready)) break;
    if (round > 4096) return false;  // a safety net only: the 256 words arrive within microseconds
    __nanosleep(64);
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (static_cast<uint32_t>(v[j] >> 32) != tag) v[j] = ll_get(ll_pred + j * 32 + lane);
  }
  uint32_t key[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    float lg = __uint_as_float(static_cast<uint32_t>(v[j]));
    if (bias) lg = __fadd_rn(lg, __ldg(bias + j * 32 + lane));
    key[j] = f2ord(lg);
  }
  uint32_t taken = 0;
#pragma unroll 1
  for (int k = 0; k < kTopK; k++) {
    uint32_t best = 0, bj = 0;
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (!((taken >> j) & 1u) && key[j] >= best) {
        best = key[j];
        bj = static_cast<uint32_t>(j);
      }
    const uint32_t mx = __reduce_max_sync(0xffffffffu, best);
    const uint32_t e = bj * 32u + static_cast<uint32_t>(lane);
    const uint32_t win = __reduce_min_sync(0xffffffffu, best == mx ? e : 0xffffffffu);
    if (static_cast<int>(win & 31u) == lane) taken |= 1u << (win >> 5);
    if (lane == 0) ex[k] = static_cast<int>(win);
  }
  return true;
}

// Predictor p of np: L2 prefetch of its share of the 8 records' 16 KB chunks.
__device__ void prefetch_records(const LayerW& L, const int* rec, int p, int np, int lane) {
  for (int c = p + np * lane; c < kTopK * kChunksPerRecord; c += np * 32) {
    const int k = c / kChunksPerRecord, q = c % kChunksPerRecord;
    const int r = rec[k];
    if (r < 0 || static_cast<uint32_t>(r) >= L.bank_records) continue;
    prefetch_l2(L.bank + static_cast<uint64_t>(r) * L.stride + static_cast<size_t>(q) * kPredChunk, kPredChunk);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1) k_fused1(const __grid_constant__ Fused1Args A) {
  extern __shared__ __align__(128) unsigned char sm[];
  unsigned char* const routed = sm + kOffRouted;
  uint32_t* const poll = reinterpret_cast<uint32_t*>(sm + kOffPoll);
  __half* const xh = reinterpret_cast<__half*>(sm + kOffXh);
  __half* const xfrag = reinterpret_cast<__half*>(sm + kOffXfrag);
  __half* const afrag = reinterpret_cast<__half*>(sm + kOffAfrag);
  float* const xS = reinterpret_cast<float*>(sm + kOffXS);
  float* const xC = reinterpret_cast<float*>(sm + kOffXC);
  float* const aS = reinterpret_cast<float*>(sm + kOffAS);
  float* const aC = reinterpret_cast<float*>(sm + kOffAC);
  float* const red = reinterpret_cast<float*>(sm + kOffRed);
  Misc1* const m = reinterpret_cast<Misc1*>(sm + kOffMisc);
  uint64_t* const bars = reinterpret_cast<uint64_t*>(sm + kOffBar);  // dib0, dib1, rgu0, rgu1, rdn

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.x, G = gridDim.x;
  const bool has_r = b < kNR, has_d = b < kNOut, has_di = has_r || has_d;
  const int n_gu = (b < kNGu ? 1 : 0) + (b + G < kNGu ? 1 : 0);
  // predictor CTAs (see kPredMinCtas): p of np, router rows [pr0, pr0 + pn)
  const int np = G - kNOut;
  const bool is_pred = np >= kPredMinCtas && b >= kNOut && n_gu == 1;
  const int pp = b - kNOut, prows = (kExperts + np - 1) / (np > 0 ? np : 1);
  const int pr0 = is_pred ? pp * prows : 0;
  const int pn = is_pred ? max(0, min(kExperts - pr0, prows)) : 0;
  unsigned char* const pbuf = sm + kOffRouted + kOffPred;
  // Per mbarrier: phases completed so far (wait parity) and whether a phase is
  // armed and not yet waited for.  Uniform across the CTA.
  uint32_t phase[kNBars] = {0, 0, 0, 0, 0, 0};
  uint32_t armed = 0;

  if (tid == 0) {
    for (int i = 0; i < kNBars; i++) mbar_init(&bars[i], kThreads);
    m->fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid < kDnCols * 8) m->cols[tid >> 3][tid & 7] = (tid & 7) == 0 ? (tid >> 3) : -1;
  __syncthreads();

  // bounded wait for barrier i's armed phase (no-op when nothing is armed)
  auto wait_bar = [&](int i) {
    if (!((armed >> i) & 1u)) return;
    if (!mbar_wait(&bars[i], phase[i] & 1u)) {
      set_status(A.status, kStatusTimeout);
      m->fail = 1;
    }
    phase[i]++;
    armed &= ~(1u << i);
  };
  // leave after a failure: first wait (bounded) for this CTA's copies in flight
  auto drain = [&]() {
    for (int i = 0; i < kNBars; i++)
      if ((armed >> i) & 1u) mbar_wait(&bars[i], phase[i] & 1u);
  };

  if (has_di) {
    issue_di(A.layers[0], b, sm + kOffDi, &bars[0]);
    armed |= 1u;
    if (A.n_layers > 1) {
      issue_di(A.layers[1], b, sm + kOffDi + kDiBytes, &bars[1]);
      armed |= 2u;
    }
  }

  if (is_pred && pn > 0 && !A.r.idx_in && A.n_layers > 1) {
    issue_pred_rows(A.layers[1], pr0, pn, pbuf, &bars[5]);
    armed |= 32u;
  }

  for (int li = 0; li < A.n_layers; li++) {
    const int l = A.first_layer + li;  // global layer index
    const uint32_t tag = static_cast<uint32_t>(l) + 1u;
    const int par = li & 1;
    const LayerW& L = A.layers[li];
    unsigned char* const di = sm + kOffDi + par * kDiBytes;
    const bool last = (l == A.total_layers - 1);

    // ---------------- prologue: x (fp16) and its MMA fragments
    // x_0 is the input; x_l = fp16(h_l / rms(h_l)), the RMS summed over 128 row
    // tiles of 16 rows (fma chain inside a tile, tiles summed in order).
    if (l == 0 && A.pre_h) {
      // every CTA computes the same norm: threads 0-63 are the reference
      // kernel's 64 threads (fma chain over i, i + 64, ...), one xor butterfly
      // per warp, the two partials added, 1 / sqrt correctly rounded
      float* part = reinterpret_cast<float*>(poll);
      if (tid < 64) {
        float acc = 0.f;
        for (int i = tid; i < kHidden; i += 64) {
          const float v = __ldg(A.pre_h + i);
          acc = __fmaf_rn(v, v, acc);
        }
#pragma unroll
        for (int mm = 16; mm >= 1; mm >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, mm));
        if ((tid & 31) == 0) part[tid >> 5] = acc;
      }
      __syncthreads();
      if (tid == 0)
        m->inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(__fadd_rn(part[0], part[1]), (float)kHidden),
                                                       A.pre_eps)));
      __syncthreads();
      const float iv = m->inv;
      const float4 h4 = __ldg(reinterpret_cast<const float4*>(A.pre_h) + tid);
      const float4 w4 = __ldg(reinterpret_cast<const float4*>(A.pre_w) + tid);
      reinterpret_cast<__half2*>(xh)[2 * tid] =
          __halves2half2(__float2half_rn(__fmul_rn(__fmul_rn(h4.x, iv), w4.x)),
                         __float2half_rn(__fmul_rn(__fmul_rn(h4.y, iv), w4.y)));
      reinterpret_cast<__half2*>(xh)[2 * tid + 1] =
          __halves2half2(__float2half_rn(__fmul_rn(__fmul_rn(h4.z, iv), w4.z)),
                         __float2half_rn(__fmul_rn(__fmul_rn(h4.w, iv), w4.w)));
    } else if (l == 0) {
      if (tid < kHidden / 8) reinterpret_cast<uint4*>(xh)[tid] = reinterpret_cast<const uint4*>(A.x0)[tid];
    } else {
      ll_poll(A.ll_h, kHidden + kNOut, tag - 1u, [&](int i, uint32_t v) { poll[i] = v; }, A.status, &m->fail);
      __syncthreads();
      const float* hv = reinterpret_cast<const float*>(poll);
      if (tid == 0) {
        float tot = 0.f;
        for (int c = 0; c < kNOut; c++) tot = __fadd_rn(tot, hv[kHidden + c]);
        const float mean = __fdiv_rn(tot, (float)kHidden);
        m->inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, A.eps)));
      }
      if (has_d && tid < 16) m->res[tid] = hv[16 * b + tid];
      __syncthreads();
      const float iv = m->inv;
      const float4 h4 = reinterpret_cast<const float4*>(hv)[tid];
      reinterpret_cast<__half2*>(xh)[2 * tid] =
          __halves2half2(__float2half_rn(__fmul_rn(h4.x, iv)), __float2half_rn(__fmul_rn(h4.y, iv)));
      reinterpret_cast<__half2*>(xh)[2 * tid + 1] =
          __halves2half2(__float2half_rn(__fmul_rn(h4.z, iv)), __float2half_rn(__fmul_rn(h4.w, iv)));
    }
    __syncthreads();
    stage_f16(xh, 1, 32, kHidden, 1, xfrag, xS, xC);
    __syncthreads();
    if (m->fail) {
      drain();
      return;
    }

    // ---------------- phase R
    if (has_r) {
      wait_bar(par);
      if (b < kNShGu) {
        // shared gate/up row pairs [8b, 8b+8): warp w takes groups 2w, 2w+1
        const uint16_t* s = reinterpret_cast<const uint16_t*>(di + 16 * kGuPitch);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        mma_tile_smem<BF16, 2>(di, kGuPitch, 2 * warp, s, s + 512, 32, xfrag, xS, xC, 1, m->cols[0], acc,
                               lane);
        if ((lane & 3) == 0) {
          red[warp * 16 + (lane >> 2)] = acc[0];
          red[warp * 16 + 8 + (lane >> 2)] = acc[2];
        }
        __syncthreads();
        if (tid < 8) {
          float gs = 0.f, us = 0.f;
#pragma unroll
          for (int q = 0; q < kWarps; q++) {
            gs = __fadd_rn(gs, red[q * 16 + tid]);
            us = __fadd_rn(us, red[q * 16 + 8 + tid]);
          }
          const __half a = __float2half_rn(silu_mul(gs, us));
          const __half a1 = __shfl_down_sync(0xffu, a, 1);
          if ((tid & 1) == 0)
            ll_put(A.ll_act + (kTopK * kInter + 8 * b + tid) / 2, h2bits(a, a1), tag);
        }
      } else if (b < kNShGu + kNRouter) {
        // warp w: row w % 8, blocks 4 (w / 8) .. +3; the upper halves travel
        // through shared memory ([row][block][lane][dot, sum])
        const int row = warp & 7, h = warp >> 3;
        float dot[4], sum[4];
        router_blocks<BF16>(di, row, h, xh, lane, dot, sum);
        float2* xchg = reinterpret_cast<float2*>(poll);
        float acc = 0.f;
        if (h == 1) {
#pragma unroll
          for (int i = 0; i < 4; i++) xchg[(row * 4 + i) * 32 + lane] = make_float2(dot[i], sum[i]);
        } else {
          acc = router_chain<BF16>(di, row, 0, lane, dot, sum, 0.f);
        }
        __syncthreads();
        if (h == 0) {
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const float2 ds = xchg[(row * 4 + i) * 32 + lane];
            dot[i] = ds.x;
            sum[i] = ds.y;
          }
          acc = warp_sum(router_chain<BF16>(di, row, 1, lane, dot, sum, acc));
          if (lane == 0) ll_put(A.ll_logits + 8 * (b - kNShGu) + row, __float_as_uint(acc), tag);
        }
      } else if (warp == 0) {
        const float v = coef_row<BF16>(di, xh, lane);
        if (lane == 0) ll_put(A.ll_logits + kExperts, __float_as_uint(v), tag);
      }
    }

    // ---------------- phase E: top-k, routed copies, routed gate/up
    if (A.r.idx_in) {
      if (warp == 0) {
        // only the coefficient is needed from the router words
        const uint64_t* pc = A.ll_logits + kExperts;
        uint64_t wc = ll_get(pc);
        unsigned spins = 0;
        while (static_cast<uint32_t>(wc >> 32) != tag) {
          if (++spins > kSpinLimit) {
            set_status(A.status, kStatusTimeout);
            m->fail = 1;
            break;
          }
          if (spins > 32) __nanosleep(64);
          wc = ll_get(pc);
        }
        if (lane == 0) m->coef = __uint_as_float(static_cast<uint32_t>(wc));
      }
      if (tid < kTopK) {
        m->idx[tid] = A.r.idx_in[(size_t)l * kTopK + tid];
        m->w[tid] = A.r.w_in[(size_t)l * kTopK + tid];
      }
    } else if (warp == 0) {
      topk_poll_select(A.ll_logits, tag, A.r.bias, lane, m->idx, m->w, m->vs, &m->coef, A.status, &m->fail);
    }
    __syncthreads();
    if (m->fail) {
      drain();
      return;
    }
    if (tid < kTopK) {
      int rec = A.r.rec_of_pos ? A.r.rec_of_pos[(size_t)l * kTopK + tid] : m->idx[tid];
      if (rec < 0 || (unsigned)rec >= L.bank_records) {
        set_status(A.status, kStatusDevice);
        rec = 0;
      }
      m->rec[tid] = rec;
    }
    __syncthreads();
    // routed copies: gate/up tile u (two MMA tiles) on rgu[u] now; the 8 down
    // tiles of this CTA's output rows (needed only after the activation
    // exchange) once the first gate/up tile has landed, so that they do not
    // share the memory system with the gate/up rows on the critical path
    for (int u = 0, t0 = 0; u < n_gu; u++) {
      const int i = b + u * G, k = i >> 5, j = i & 31;
      const uint8_t* rec = L.bank + static_cast<uint64_t>(m->rec[k]) * L.stride;
      t0 = copy_gu(routed + (u * 2) * kGuTileBytes, rec, 16 * j, t0);
      t0 = copy_gu(routed + (u * 2 + 1) * kGuTileBytes, rec, 16 * j + 8, t0);
      cp_async_arrive(&bars[2 + u]);
    }
    armed |= (n_gu > 0 ? 4u : 0u) | (n_gu > 1 ? 8u : 0u);
    auto issue_dn = [&]() {
      int t0 = 0;
      for (int k = 0; k < kTopK; k++)
        t0 = copy_dn(routed + kMaxGu * 2 * kGuTileBytes + k * kDnTileBytes,
                     L.bank + static_cast<uint64_t>(m->rec[k]) * L.stride, b, t0);
      cp_async_arrive(&bars[4]);
      armed |= 16u;
    };
    if (has_d && n_gu == 0) issue_dn();
    // the weights are only needed by the combine: computed while the copies fly
    if (!A.r.idx_in && warp == 1) topk_weights1(m->vs, lane, m->w);
    for (int u = 0; u < n_gu; u++) {
      wait_bar(2 + u);
      if (u == 0 && has_d) issue_dn();
      const int i = b + u * G, k = i >> 5, j = i & 31;
      // warp w: MMA tile w / 8 (row pairs +0 / +8), K-eighth w % 8 (4 groups)
      const unsigned char* tb = routed + (u * 2 + (warp >> 3)) * kGuTileBytes;
      const uint16_t* s = reinterpret_cast<const uint16_t*>(tb + 16 * kGuPitch);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      mma_tile_smem<BF16, 4>(tb, kGuPitch, (warp & 7) * 4, s, s + 512, 32, xfrag, xS, xC, 1, m->cols[0],
                             acc, lane);
      if ((lane & 3) == 0) {
        red[warp * 16 + (lane >> 2)] = acc[0];
        red[warp * 16 + 8 + (lane >> 2)] = acc[2];
      }
      __syncthreads();
      if (tid < 16) {
        const int mt = tid >> 3, r = tid & 7;
        float gs = 0.f, us = 0.f;
#pragma unroll
        for (int q = 0; q < 8; q++) {
          gs = __fadd_rn(gs, red[(mt * 8 + q) * 16 + r]);
          us = __fadd_rn(us, red[(mt * 8 + q) * 16 + 8 + r]);
        }
        const __half a = __float2half_rn(silu_mul(gs, us));
        const __half a1 = __shfl_down_sync(0xffffu, a, 1);
        if ((tid & 1) == 0)
          ll_put(A.ll_act + (k * kInter + 16 * j + tid) / 2, h2bits(a, a1), tag);
      }
      __syncthreads();
      if (m->fail) {
        drain();
        return;
      }
    }
    // ---------------- predictors: the next layer's records into L2
    if (is_pred && li + 1 < A.n_layers) {
      const LayerW& Ln = A.layers[li + 1];
      if (A.r.idx_in) {
        if (tid < kTopK)
          m->pred[tid] = A.r.rec_of_pos ? A.r.rec_of_pos[(size_t)(l + 1) * kTopK + tid]
                                        : A.r.idx_in[(size_t)(l + 1) * kTopK + tid];
        __syncthreads();
        if (warp == 0) prefetch_records(Ln, m->pred, pp, np, lane);
      } else {
        wait_bar(5);
        __syncthreads();
        if (m->fail) {
          drain();
          return;
        }
        if (pn > 0) predict_rows<BF16>(pbuf, pn, xh, lane, warp, A.ll_pred, pr0, tag + 1u);
        if (warp == 0 && predict_top8(A.ll_pred, tag + 1u, A.r.bias, lane, m->pred)) {
          __syncwarp();
          prefetch_records(Ln, m->pred, pp, np, lane);
        }
      }
    }
    if (b == 0 && tid < kTopK) {
      if (A.idx_out) A.idx_out[(size_t)l * kTopK + tid] = m->idx[tid];
      if (A.w_out) A.w_out[(size_t)l * kTopK + tid] = m->w[tid];
    }

    // ---------------- phase D: down projections, combine, RMS partials
    if (has_d) {
      float res_v = 0.f;
      if (tid < 16) res_v = (l == 0) ? (A.res0 ? __ldg(A.res0 + 16 * b + tid) : 0.f) : m->res[tid];
      ll_poll(A.ll_act, kActWords, tag, [&](int i, uint32_t v) { poll[i] = v; }, A.status, &m->fail);
      __syncthreads();
      stage_f16(reinterpret_cast<const __half*>(poll), kDnCols, 8, kInter, kDnCols, afrag, aS, aC);
      wait_bar(par);
      wait_bar(4);
      __syncthreads();
      if (m->fail) {
        drain();
        return;
      }
      for (int it = warp; it < kItemsD; it += kWarps) {
        const int e = it >> 2, q = it & 3;  // column e (8 = shared), groups 2q, 2q+1
        const unsigned char* tile =
            e < kTopK ? routed + kMaxGu * 2 * kGuTileBytes + e * kDnTileBytes : di + kRPart;
        const uint16_t* s = reinterpret_cast<const uint16_t*>(tile + 16 * kDnPitch);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        mma_tile_smem<BF16, 2>(tile, kDnPitch, 2 * q, s, s + 128, 8, afrag, aS, aC, kDnCols, m->cols[e],
                               acc, lane);
        if ((lane & 3) == 0) {
          red[it * 16 + (lane >> 2)] = acc[0];
          red[it * 16 + 8 + (lane >> 2)] = acc[2];
        }
      }
      __syncthreads();
      if (tid < 16) {
        const int r = 16 * b + tid;
        float y[kDnCols];
#pragma unroll
        for (int e = 0; e < kDnCols; e++) {
          float v = 0.f;
#pragma unroll
          for (int q = 0; q < 4; q++) v = __fadd_rn(v, red[(e * 4 + q) * 16 + tid]);
          y[e] = v;
        }
        const float coeff = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-m->coef)));
        const float sh = __fmul_rn(y[kTopK], coeff);
        float routed_sum = __fmul_rn(y[0], m->w[0]);
#pragma unroll
        for (int k = 1; k < kTopK; k++) routed_sum = __fadd_rn(routed_sum, __fmul_rn(y[k], m->w[k]));
        const float v = __fadd_rn(__fadd_rn(res_v, sh), routed_sum);
        // RMS partial of the 16 rows: fma chain in row order (lane 0 gathers)
        float ssq = 0.f;
#pragma unroll
        for (int row = 0; row < 16; row++) {
          const float vr = __shfl_sync(0xffffu, v, row);
          ssq = __fmaf_rn(vr, vr, ssq);
        }
        if (last) {
          A.out[r] = v;
        } else {
          ll_put(A.ll_h + r, __float_as_uint(v), tag);
          if (tid == 0) ll_put(A.ll_h + kHidden + b, __float_as_uint(ssq), tag);
        }
      }
    }
    // every read of this layer's buffers is done: refill the parity buffer
    // with layer li + 2's token-independent rows
    fence_proxy_async_smem();
    __syncthreads();
    if (m->fail) {
      drain();
      return;
    }
    if (has_di && li + 2 < A.n_layers) {
      issue_di(A.layers[li + 2], b, di, &bars[par]);
      armed |= 1u << par;
    }
    if (is_pred && pn > 0 && !A.r.idx_in && li + 2 < A.n_layers) {
      issue_pred_rows(A.layers[li + 2], pr0, pn, pbuf, &bars[5]);
      armed |= 32u;
    }
  }
}

int g_fused1_grid[64] = {};  // per device: CTAs of the launch, -1 = unsupported

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

size_t fused1_workspace_bytes() {
  auto a = [](size_t n) { return (n + 255) & ~(size_t)255; };
  return a(8 * (kExperts + 1)) + a(8 * kActWords) + a(8 * (kHidden + kNOut)) + a(8 * kExperts);
}

cudaError_t fused1_init_attributes() {
  cudaError_t e = cudaFuncSetAttribute(k_fused1<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_fused1<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
}

cudaError_t fused1_stack(cudaStream_t st, const LayerW* layers, int n_layers, bool bf16,
                         const uint16_t* x, const float* residual, float* out, float eps,
                         const RoutingArgs& r, int* idx_out, float* w_out, void* workspace,
                         int* status, Prof* prof, const float* pre_h, const float* pre_w, float pre_eps) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorNotSupported;
  if (g_fused1_grid[dev] == 0) {
    int sms = 0, per = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &per, bf16 ? (const void*)k_fused1<true> : (const void*)k_fused1<false>, kThreads, kSmemBytes);
    if (e != cudaSuccess) return e;
    // every CTA must own a routed gate/up tile (the ordering argument of the
    // tagged words relies on it): at most 256 CTAs
    const int grid = sms < kNGu ? sms : kNGu;
    g_fused1_grid[dev] = (per >= 1 && grid >= kMinGrid) ? grid : -1;
  }
  if (g_fused1_grid[dev] < 0) return cudaErrorNotSupported;
  // every bulk copy needs 16-byte aligned sources
  if (!aligned16(x) || !aligned16(pre_h) || !aligned16(pre_w)) return cudaErrorNotSupported;
  for (int i = 0; i < n_layers; i++) {
    const LayerW& L = layers[i];
    if (!aligned16(L.rw) || !aligned16(L.rs) || !aligned16(L.rb) || !aligned16(L.cw) || !aligned16(L.cs) ||
        !aligned16(L.cb) || !aligned16(L.shared) || !aligned16(L.bank) || (L.stride & 15u) != 0)
      return cudaErrorNotSupported;
  }
  char* p = static_cast<char*>(workspace);
  auto take = [&](size_t n) {
    char* q = p;
    p += (n + 255) & ~(size_t)255;
    return q;
  };
  Fused1Args A;  // layers by value: copied into the launch's parameter space
  A.total_layers = n_layers;
  A.x0 = x;
  A.res0 = residual;
  A.pre_h = pre_h;
  A.pre_w = pre_w;
  A.pre_eps = pre_eps;
  A.out = out;
  A.eps = eps;
  A.r = r;
  A.idx_out = idx_out;
  A.w_out = w_out;
  A.ll_logits = reinterpret_cast<uint64_t*>(take(8 * (kExperts + 1)));
  A.ll_act = reinterpret_cast<uint64_t*>(take(8 * kActWords));
  A.ll_h = reinterpret_cast<uint64_t*>(take(8 * (kHidden + kNOut)));
  A.ll_pred = reinterpret_cast<uint64_t*>(take(8 * kExperts));
  const size_t ll_bytes = static_cast<size_t>(p - reinterpret_cast<char*>(A.ll_logits));
  // tags restart at 1 every call: clear the words of the previous call
  e = cudaMemsetAsync(A.ll_logits, 0, ll_bytes, st);
  if (e != cudaSuccess) return e;
  A.status = status;
  for (int l0 = 0; l0 < n_layers; l0 += kMaxLayers) {
    const int n = n_layers - l0 < kMaxLayers ? n_layers - l0 : kMaxLayers;
    A.first_layer = l0;
    A.n_layers = n;
    for (int i = 0; i < n; i++) A.layers[i] = layers[l0 + i];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(g_fused1_grid[dev]);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // optional timing events around the launch (bench harness)
    int slot = -1;
    unsigned flags = cudaEventRecordDefault;
    if (prof && prof->kernel == kKFused && prof->n < prof->cap) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      cudaStreamIsCapturing(st, &cs);
      if (cs == cudaStreamCaptureStatusActive) flags = cudaEventRecordExternal;
      slot = prof->n++;
      cudaEventRecordWithFlags(prof->ev0[slot], st, flags);
    }
    if (bf16)
      e = cudaLaunchKernelEx(&cfg, k_fused1<true>, A);
    else
      e = cudaLaunchKernelEx(&cfg, k_fused1<false>, A);
    if (slot >= 0) cudaEventRecordWithFlags(prof->ev1[slot], st, flags);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace qf
