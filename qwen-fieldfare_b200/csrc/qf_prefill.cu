// qf_prefill.cu -- MoE block for many tokens (prefill, T > 64): grouped expert
// GEMMs on the 5th-generation tensor cores.
//
// Flow (one stream, all on the device):
//   k_router_prefill  router logits in the reference lane order (bit-exact)
//   k_topk            top-8 / softmax / renormalise (with the harness bias)
//   dispatch plan     counts, offsets, stable permutation by (expert, token, k)
//   k_gather_rows     token rows in expert order (+ all T tokens for the
//                     shared expert after them), K-permuted, fp16
//   k_tile_list       128-row tiles of every expert (+ shared), longest first
//   k_grouped<0>      gate/up: SiLU(G x) * (U x) -> fp16 act rows
//   k_grouped<1>      down: D act -> fp32 y rows
//   k_combine         residual + sigmoid(c) * y_shared + sum_k w_k y_k (router order)
//
// Row space shared by the gathered x, act and y buffers: rows [0, P) are the
// P = 8T routed positions sorted by (expert, token, k); rows [P, P + T) are
// the shared expert's tokens.  Expert e owns rows [offsets[e], offsets[e+1])
// with offsets[256] = P, so the shared expert is simply expert 256.
//
// k_grouped computes D[weight row][token] = W[row][:] . X[token][:] with the
// expert's weights as the MMA's A operand in TENSOR MEMORY and the token rows
// as the B operand in shared memory.  Dequantised weights never touch shared
// memory: producer threads turn Q4 codes (read straight into registers) into
// fp16 and write them to TMEM with tcgen05.st, so shared-memory bandwidth is
// spent only on the token rows, which arrive by TMA (one 2-D tile load per
// 64-column step).
//
// K order inside every 8-element group is permuted to (0,4,1,5,2,6,3,7) in
// BOTH operands (the dot product is unchanged): that is the order in which
// the nibble extraction produces fp16 pairs, so the dequant needs no byte
// permutes.  k_gather_rows permutes x; act rows are written permuted by the
// gate/up epilogue.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <algorithm>

#include "qf_internal.h"

namespace qf {

namespace {

constexpr unsigned kSpin = 1u << 22;  // bounded waits (a few seconds at most)

__device__ __forceinline__ uint32_t s_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// K-major, 128-byte swizzle, 8-row groups 1024 bytes apart
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = s_u32(bar);
  for (unsigned i = 0; i < kSpin; i++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_u32(bar)), "r"(bytes) : "memory");
}
// 2-D tiled TMA load (128-byte swizzle in the tensor map) completing on bar
__device__ __forceinline__ void tma_tile(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          s_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(s_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load3(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          s_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(s_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load4(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
          s_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(s_u32(bar))
      : "memory");
}
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(s_u32(bar))
               : "memory");
}
// D[tmem d] (+)= A[tmem a] . B[smem desc]^T
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(
          d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%"
      "20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 32 bytes of Q4 codes straight into registers (read once; no L1 allocation)
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

template <bool BF16>
__device__ __forceinline__ float h16_to_f32(uint16_t u) {
  if constexpr (BF16) {
    return __uint_as_float(static_cast<uint32_t>(u) << 16);
  } else {
    return __half2float(__ushort_as_half(u));
  }
}


// ------------------------------------------------------------------ router
// Logits in the reference lane order (deltanet.metal:2229-2260): lane l of a
// warp owns bytes blk*256 + l*8 .. +7 of each of the 8 blocks of 256 and
// accumulates dot = fma-chain of 8 products, acc = fma(s, dot, acc),
// acc = fma(b, xsum, acc); the lanes are then summed with the xor butterfly
// 16, 8, 4, 2, 1 (simd_sum), so the logits are bit-identical to the decode
// router and the oracle.  A CTA computes 32 router rows x 8 tokens (4 rows
// per warp).  The two chains of a token pair run together in Blackwell's
// packed fp32 FMA (fma.rn.f32x2: each half rounded as a scalar fma, so every
// logit is bit-identical to the scalar chain): x is staged once per CTA as
// fp32 pairs {x_t, x_t+1} laid out [pair][block][element][lane] (a warp's
// 8-byte reads of one element are 256 contiguous bytes), each code byte
// becomes an exact {q, q} pair (byte into the 2^23 mantissa, one packed
// subtract), and the element loop runs outermost so that 4 rows x 4 pairs of
// dot chains stay in registers.  One row of CTAs
// computes the shared-gate coefficient instead, one lane per token, as the
// reference's single sequential chain (qwen_gemv_q8_affine,
// deltanet.metal:863-902); that row is blockIdx.y == 0, so its long chains
// start in the first wave instead of trailing the grid.
constexpr int kRtTok = 8;
constexpr int kRtPairs = kRtTok / 2;
constexpr int kRtWarps = 8;
constexpr int kRtRowsPerWarp = 4;
constexpr int kRtRows = kRtWarps * kRtRowsPerWarp;  // 32 router rows per CTA
constexpr int kRtThreads = kRtWarps * 32;
constexpr int kRtRowBlocks = kExperts / kRtRows;  // + 1 row of coefficient CTAs
constexpr size_t kRtSmem = sizeof(uint64_t) * (kRtPairs * kHidden + kRtPairs * 256);

__device__ __forceinline__ uint64_t rt_pk(float a, float b) {
  return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}
__device__ __forceinline__ uint64_t rt_fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// {q, q} of byte k of w, exact: (2^23 + q) - 2^23 in both halves
__device__ __forceinline__ uint64_t rt_byte2(uint32_t w, int k) {
  const uint32_t u = 0x4B000000u | ((w >> (8 * k)) & 0xFFu);
  const uint64_t m = (uint64_t)u | ((uint64_t)u << 32);
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(m), "l"(0xCB000000CB000000ull));
  return d;
}

template <bool BF16>
__global__ void __launch_bounds__(kRtThreads, 2) k_router_prefill(LayerW L, int T,
                                                                  const uint16_t* __restrict__ x,
                                                                  float* __restrict__ logits,
                                                                  float* __restrict__ coef) {
  extern __shared__ float4 rsm4[];
  uint64_t* xs2 = reinterpret_cast<uint64_t*>(rsm4);  // [pair][8 blk][8 k][32 lanes]
  uint64_t* xsum2 = xs2 + kRtPairs * kHidden;         // [pair][8 blk][32 lanes]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * kRtTok;
  const int tn = min(kRtTok, T - t0);
  // item = (pair, 8-element group c = blk * 32 + lane): both tokens' 8 values;
  // every load of the thread's items is issued before the first is used
  constexpr int kItems = kRtPairs * (kHidden / 8) / kRtThreads;  // 4 per thread
  static_assert(kItems * kRtThreads == kRtPairs * (kHidden / 8), "items per thread");
  uint4 ld[kItems][2];
#pragma unroll
  for (int it = 0; it < kItems; it++) {
    const int i = tid + it * kRtThreads;
    const int tp = i / (kHidden / 8), c = i % (kHidden / 8);
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int t = 2 * tp + h;
      ld[it][h] = t < tn ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)(t0 + t) * kHidden) + c)
                         : make_uint4(0u, 0u, 0u, 0u);
    }
  }
#pragma unroll
  for (int it = 0; it < kItems; it++) {
    const int i = tid + it * kRtThreads;
    const int tp = i / (kHidden / 8), c = i % (kHidden / 8);
    float v[2][8];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint4 u = ld[it][h];
      const __half2* hh = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 f = __half22float2(hh[j]);
        v[h][2 * j] = f.x;
        v[h][2 * j + 1] = f.y;
      }
    }
    const int blk = c >> 5, ln = c & 31;
    uint64_t* d = xs2 + ((size_t)(tp * 8 + blk) * 8) * 32 + ln;
    float sm[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      float a = v[h][0];
#pragma unroll
      for (int k = 1; k < 8; k++) a = __fadd_rn(a, v[h][k]);
      sm[h] = a;
    }
#pragma unroll
    for (int k = 0; k < 8; k++) d[k * 32] = rt_pk(v[0][k], v[1][k]);
    xsum2[(tp * 8 + blk) * 32 + ln] = rt_pk(sm[0], sm[1]);
  }
  __syncthreads();
  if (blockIdx.y > 0) {
    constexpr int R = kRtRowsPerWarp;
    const int rbase = (blockIdx.y - 1) * kRtRows + warp * R;
    const uint8_t* wrow = L.rw + (size_t)rbase * kHidden + lane * 8;
    uint64_t acc[R][kRtPairs];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int p = 0; p < kRtPairs; p++) acc[r][p] = 0ull;
    uint2 wn[R];
    uint16_t sn[R], bn[R];
    auto fetch = [&](int blk) {
      const int g = blk * 4 + (lane >> 3);
#pragma unroll
      for (int r = 0; r < R; r++) {
        wn[r] = __ldg(reinterpret_cast<const uint2*>(wrow + (size_t)r * kHidden + blk * 256));
        sn[r] = __ldg(L.rs + (size_t)(rbase + r) * (kHidden / kGroup) + g);
        bn[r] = __ldg(L.rb + (size_t)(rbase + r) * (kHidden / kGroup) + g);
      }
    };
    fetch(0);
#pragma unroll 1
    for (int blk = 0; blk < 8; blk++) {
      uint2 w[R];
      uint64_t sc[R], bi[R];
#pragma unroll
      for (int r = 0; r < R; r++) {
        w[r] = wn[r];
        const float s1 = h16_to_f32<BF16>(sn[r]), b1 = h16_to_f32<BF16>(bn[r]);
        sc[r] = rt_pk(s1, s1);
        bi[r] = rt_pk(b1, b1);
      }
      if (blk + 1 < 8) fetch(blk + 1);
      uint64_t dot[R][kRtPairs];
#pragma unroll
      for (int r = 0; r < R; r++)
#pragma unroll
        for (int p = 0; p < kRtPairs; p++) dot[r][p] = 0ull;
#pragma unroll
      for (int k = 0; k < 8; k++) {
        uint64_t xv[kRtPairs];
#pragma unroll
        for (int p = 0; p < kRtPairs; p++) xv[p] = xs2[((size_t)(p * 8 + blk) * 8 + k) * 32 + lane];
#pragma unroll
        for (int r = 0; r < R; r++) {
          const uint64_t q2 = rt_byte2(k < 4 ? w[r].x : w[r].y, k & 3);
#pragma unroll
          for (int p = 0; p < kRtPairs; p++) dot[r][p] = rt_fma2(q2, xv[p], dot[r][p]);
        }
      }
#pragma unroll
      for (int p = 0; p < kRtPairs; p++) {
        const uint64_t xsm = xsum2[(p * 8 + blk) * 32 + lane];
#pragma unroll
        for (int r = 0; r < R; r++) acc[r][p] = rt_fma2(bi[r], xsm, rt_fma2(sc[r], dot[r][p], acc[r][p]));
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int p = 0; p < kRtPairs; p++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int t = 2 * p + h;
          const float v = warp_sum(__uint_as_float((uint32_t)(acc[r][p] >> (32 * h))));
          if (lane == ((r * kRtTok + t) & 31) && t < tn) logits[(size_t)(t0 + t) * kExperts + rbase + r] = v;
        }
  } else if (coef && warp == 0) {
    const int t = lane;
    if (t < tn) {
      const int tp = t >> 1, h = t & 1;
      // x_t[e], e = c * 8 + k, c = blk * 32 + ln
      auto xe = [&](int e) {
        const int c = e >> 3, k = e & 7;
        const uint64_t pr = xs2[((size_t)(tp * 8 + (c >> 5)) * 8 + k) * 32 + (c & 31)];
        return __uint_as_float((uint32_t)(pr >> (32 * h)));
      };
      float acc = 0.f;
      for (int g = 0; g < kHidden / kGroup; g++) {
        const float sc = ld16<BF16>(L.cs, g), bi = ld16<BF16>(L.cb, g);
#pragma unroll 4
        for (int u = 0; u < 16; u++) {
          const uint32_t wv = __ldg(reinterpret_cast<const uint32_t*>(L.cw + g * 64) + u);
          const int e = g * 64 + u * 4;
          acc = __fmaf_rn(__fmaf_rn(byte_f(wv, 0), sc, bi), xe(e), acc);
          acc = __fmaf_rn(__fmaf_rn(byte_f(wv, 1), sc, bi), xe(e + 1), acc);
          acc = __fmaf_rn(__fmaf_rn(byte_f(wv, 2), sc, bi), xe(e + 2), acc);
          acc = __fmaf_rn(__fmaf_rn(byte_f(wv, 3), sc, bi), xe(e + 3), acc);
        }
      }
      coef[t0 + t] = acc;
    }
  }
}

// ------------------------------------------------------------------ row gather
// xs[r] = permute8(x[perm[r] / 8]) for r < P, xs[P + t] = permute8(x[t]);
// one warp per row, 16-byte vectors.
__global__ void __launch_bounds__(256) k_gather_rows(const int* __restrict__ perm, int P, int T,
                                                     const uint4* __restrict__ x, uint4* __restrict__ xs) {
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= P + T) return;
  const int src = r < P ? (perm[r] >> 3) : r - P;
  const uint4* s = x + (size_t)src * (kHidden / 8);
  uint4* d = xs + (size_t)r * (kHidden / 8);
  uint4 v[kHidden / 8 / 32];
#pragma unroll
  for (int j = 0; j < kHidden / 8 / 32; j++) v[j] = __ldg(s + lane + 32 * j);
#pragma unroll
  for (int j = 0; j < kHidden / 8 / 32; j++) d[lane + 32 * j] = permute8(v[j]);
}

// ------------------------------------------------------------------ tile list
// tiles[i] = (expert, first row, rows, first row of the expert in the row
// space); expert 256 = the shared expert over all T tokens (rows P..P+T-1).  Full kTileRows-row tiles
// come first, then partial tiles by decreasing size (ties: lower expert
// first), so a round-robin over persistent CTAs hands the longest units out
// first.
constexpr int kTileRows = 128;
constexpr int kListThreads = 288;  // one thread per expert and the shared expert

// shared_base (device, optional): first shared row; default T * 8; negative: none.
__global__ void __launch_bounds__(kListThreads) k_tile_list(const int* __restrict__ counts,
                                                             const int* __restrict__ offsets, int T,
                                                             const int* __restrict__ shared_base,
                                                             int4* __restrict__ tiles, int* __restrict__ n_tiles) {
  __shared__ int s_rem[kListThreads];
  __shared__ int s_warp[kListThreads / 32];
  const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
  int cnt = 0, base = 0;
  if (e < kExperts) {
    cnt = counts[e];
    base = offsets[e];
  } else if (e == kExperts) {
    base = shared_base ? *shared_base : T * kTopK;
    cnt = base < 0 ? 0 : T;  // a negative shared base (an aborted EP call): no shared rows
  }
  const int full = cnt / kTileRows, rem = cnt % kTileRows;
  s_rem[e] = rem;
  int v = full;  // inclusive warp scan of the full-tile counts
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += o;
  }
  if (lane == 31) s_warp[warp] = v;
  __syncthreads();
  int before = 0, total_full = 0;
  for (int w = 0; w < kListThreads / 32; w++) {
    const int s = s_warp[w];
    if (w < warp) before += s;
    total_full += s;
  }
  const int first = before + v - full;
  for (int j = 0; j < full; j++) tiles[first + j] = make_int4(e, j * kTileRows, kTileRows, base);
  if (rem > 0) {
    int pos = 0;
    for (int o = 0; o < kListThreads; o++) {
      const int r2 = s_rem[o];
      pos += (r2 > rem || (r2 == rem && o < e)) ? 1 : 0;
    }
    tiles[total_full + pos] = make_int4(e, full * kTileRows, rem, base);
  }
  const int n_part = __syncthreads_count(rem > 0);
  if (e == 0) *n_tiles = total_full + n_part;
}

// ------------------------------------------------------------------ small-T plan
// T <= 64 (at most 512 routed positions) in ONE CTA: top-8 of every token
// (topk_token, one token per warp; logits == nullptr when idx / w already hold
// the routing), or the copy of the supplied routing, then the copies of the
// routing to idx_out / w_out, the per-expert counts and offsets, the stable
// permutation by (expert, position) and the tile list -- the same results as
// k_topk + dispatch_plan_ws + k_tile_list, whose logic it repeats for a single
// chunk, without five launches and two copies per block.
constexpr int kPlanSmallThreads = 1024;
constexpr int kPlanTopkMaxTokens = kPlanSmallThreads / 32;
__global__ void __launch_bounds__(kPlanSmallThreads) k_plan_small(
    const float* __restrict__ logits, const float* __restrict__ bias, const int* __restrict__ idx_in,
    const float* __restrict__ w_in, int* __restrict__ idx, float* __restrict__ w, int T,
    int* __restrict__ idx_out, float* __restrict__ w_out, int* __restrict__ counts, int* __restrict__ offsets,
    int* __restrict__ perm, int4* __restrict__ tiles, int* __restrict__ n_tiles, int* status) {
  __shared__ int h[kExperts];
  __shared__ int excl[kExperts + 1];
  __shared__ int wh[kPlanSmallThreads / 32][kExperts];  // per-warp counts, then prefix
  __shared__ int s_rem[kListThreads];
  __shared__ int s_warp[kListThreads / 32];
  __shared__ int s_scan[kExperts / 32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = T * kTopK;
  if (idx_in) {
    if (tid < n) {
      idx[tid] = idx_in[tid];
      w[tid] = w_in[tid];
    }
  } else if (logits) {
    if (warp < T) topk_token(warp, logits, bias, idx, w, lane);
  }
  __syncthreads();
  const int nw = (n + 31) >> 5;  // warps that hold positions
  for (int i = tid; i < kExperts; i += blockDim.x) h[i] = 0;
  for (int i = tid; i < nw * kExperts; i += blockDim.x) (&wh[0][0])[i] = 0;
  __syncthreads();
  int e = -1;
  if (tid < n) {
    e = idx[tid];
    if (idx_out) idx_out[tid] = e;
    if (w_out) w_out[tid] = w[tid];
    if (e >= 0 && e < kExperts) {
      atomicAdd(&h[e], 1);
    } else {
      set_status(status, kStatusDevice);
      e = -1;
    }
  }
  // rank among equal experts inside the warp, per-warp counts
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && (peers & ((1u << lane) - 1u)) == 0) wh[warp][e] = __popc(peers);
  __syncthreads();
  {
    int total = 0;
    const int ex = block_scan256(tid < kExperts ? h[tid] : 0, s_scan, &total);
    if (tid < kExperts) excl[tid] = ex;
    if (tid == 0) excl[kExperts] = total;
  }
  for (int x = tid; x < kExperts; x += blockDim.x) {
    int acc = 0;
    for (int q = 0; q < nw; q++) {
      const int c = wh[q][x];
      wh[q][x] = acc;
      acc += c;
    }
  }
  __syncthreads();
  for (int x = tid; x <= kExperts; x += blockDim.x) {
    if (x < kExperts) counts[x] = h[x];
    offsets[x] = excl[x];
  }
  if (e >= 0) perm[excl[e] + wh[warp][e] + rank] = tid;
  // tile list (k_tile_list): threads 0..287, expert 256 = the shared expert
  int cnt = 0, base = 0;
  if (tid < kExperts) {
    cnt = h[tid];
    base = excl[tid];
  } else if (tid == kExperts) {
    cnt = T;
    base = T * kTopK;
  }
  const int full = cnt / kTileRows, rem = cnt % kTileRows;
  if (tid < kListThreads) s_rem[tid] = rem;
  int v = full;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += o;
  }
  if (tid < kListThreads && lane == 31) s_warp[warp] = v;
  __syncthreads();
  int n_part = 0;
  if (tid < kListThreads) {
    int before = 0, total_full = 0;
    for (int q = 0; q < kListThreads / 32; q++) {
      const int sw = s_warp[q];
      if (q < warp) before += sw;
      total_full += sw;
    }
    const int first = before + v - full;
    for (int j = 0; j < full; j++) tiles[first + j] = make_int4(tid, j * kTileRows, kTileRows, base);
    if (rem > 0) {
      int pos = 0;
      for (int o = 0; o < kListThreads; o++) {
        const int r2 = s_rem[o];
        pos += (r2 > rem || (r2 == rem && o < tid)) ? 1 : 0;
      }
      tiles[total_full + pos] = make_int4(tid, full * kTileRows, rem, base);
    }
    n_part = total_full;  // carried for thread 0 below
  }
  const int parts = __syncthreads_count(tid < kListThreads && rem > 0);
  if (tid == 0) *n_tiles = n_part + parts;
}

// ------------------------------------------------------------------ grouped GEMM
// Work unit = (tile of <= 128 token rows of one expert, two 128-row weight
// blocks sharing that token tile): gate rows f0..f0+127 and up rows
// f0..f0+127 for gate/up, output rows f0..f0+255 for down.  Every token row
// brought on chip feeds 256 weight rows.  Each weight block has its own TMEM
// accumulator and its own MMA-issuing thread: one tcgen05.mma (M=128, N=tile
// rows rounded to 16, K=16) has a fixed issue cost, and two issuers keep the
// tensor pipe fed at N <= 128.
//
// Warp roles: 0-7 weight producers (warp w: block w >> 2, TMEM lanes
// 32 * (w & 3) ...), 8-15 epilogue, 16-17 MMA issue (one thread each; warp 16
// also allocates TMEM), 18 weight loads, 19 token loads (one thread each
// issues the TMAs: the weight stream is gated only by the producers, the token
// tiles only by the MMAs that free their stages).
//
// The weights reach shared memory by TMA too: per 64-column step one tiled
// load brings the Q4 codes of the unit's 2 x 128 weight rows (32 bytes a row,
// 8 KB) into a 6-stage ring, and per 8 steps one load each brings their
// scales and biases (8 groups a row); producers read them from shared memory,
// so the DRAM latency of the weights is covered by the ring, not by registers.
constexpr int kGemmWarps = 20;
constexpr int kGemmThreads = kGemmWarps * 32;
constexpr int kMmaWarp = 16;
constexpr int kLoadWarp = 18;  // weight codes, scales and biases
constexpr int kTokWarp = 19;   // token tiles
constexpr int kEpiThreads = 256;
constexpr int kTokStages = 8;
constexpr int kAStages = 4;           // TMEM A stages
constexpr int kTokStageBytes = kTileRows * 128;  // 128 rows x 64 fp16, 128-byte swizzle
// a tile of <= 16 rows (decode batches: 1-4 positions per expert) loads only
// its 16 rows: the MMA of N = 16 reads no further, and the 128-byte swizzle
// pattern repeats every 8 rows, so the stage layout is the same
constexpr int kSmallTileRows = 16;
constexpr int kCodeStages = 6;
constexpr int kCodeStageBytes = 2 * 128 * 32;    // 2 blocks x 128 rows x 64 Q4 codes
constexpr int kSbWin = 8;                        // steps per scale/bias window
constexpr int kSbBufs = 2;
constexpr int kSbHalf = 2 * 128 * kSbWin * 2;    // scales (or biases) of one window: 4 KB
constexpr int kRingBytes = kTokStages * kTokStageBytes + kCodeStages * kCodeStageBytes + kSbBufs * 2 * kSbHalf;
// TMEM columns: acc0 [0,128) | acc1 [128,256) | A stage s at 256 + 64 s (block 0 +0, block 1 +32).
// A unit of <= kSmallAcc token rows accumulates in one half of each block's
// 128 columns (half = unit index & 1), so consecutive small units are
// double-buffered: the MMAs of one run while the epilogue drains the other.
constexpr int kSmallAcc = 64;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA = 256;

struct GemmSync {
  uint64_t tok_full[kTokStages];
  uint64_t tok_empty[kTokStages];
  uint64_t a_full[kAStages];
  uint64_t a_empty[kAStages];
  uint64_t acc_full[2];   // per accumulator half (columns +0 / +64 of each block)
  uint64_t acc_empty[2];
  uint64_t code_full[kCodeStages];
  uint64_t code_empty[kCodeStages];
  uint64_t sb_full[kSbBufs];
  uint64_t sb_empty[kSbBufs];
  uint32_t tmem;
  int col_pos[2][kTileRows];        // down epilogue: output row of each column
  float* col_row[2][kTileRows];     // expert-parallel down epilogue: destination row (NULL: skipped)
};
constexpr int kGemmSmem = 1024 + kRingBytes + (int)sizeof(GemmSync);
static_assert(kGemmSmem <= 227 * 1024, "shared memory");
static_assert(kGemmSmem > 114 * 1024, "one CTA per SM: the kernel allocates all of TMEM");

struct GemmArgs {
  CUtensorMap map_rows;  // B operand rows: MODE 0 gathered x [P+T][2048], MODE 1 act [P+T][512]; box 64 x 128
  CUtensorMap map_rows_small;  // the same rows, box 64 x kSmallTileRows (tiles of <= 16 rows)
  // weights, [0] the bank, [1] the shared record: codes (box 32 bytes x 2 x 128
  // rows), scales and biases (box 8 groups x 2 x 128 rows)
  CUtensorMap map_code[2], map_s[2], map_b[2];
  LayerW L;
  const int* perm;  // routed row -> y row (position t*8+k); NULL: the row itself
  const int4* tiles;
  const int* n_tiles;
  __half* act;  // MODE 0 output: [P+T][512] (permuted K)
  float* y;     // MODE 1 output: unweighted [P+T][2048]; routed row = position t*8+k
  EpOut ep;     // MODE 1 with ep.ret: result rows go to the ranks named by ep.ret
  int* status;
};

template <bool BF16>
__device__ __forceinline__ uint32_t half_bits(uint16_t u) {
  if constexpr (BF16) {
    return __half_as_ushort(__float2half_rn(__uint_as_float((uint32_t)u << 16)));
  } else {
    return u;
  }
}

// 8 nibbles of one word -> 4 fp16 pairs (e0,e4) (e1,e5) (e2,e6) (e3,e7):
// q exact (1024 + q, or 1024 + 16 q scaled by 1/16), then q*s + b rounded once
__device__ __forceinline__ void dequant_word(uint32_t w, __half2 s2, __half2 b2, uint32_t* o) {
  const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  const __half2 k16inv = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));
  const __half2 km64 = __halves2half2(__ushort_as_half(0xD400), __ushort_as_half(0xD400));
  const uint32_t w8 = w >> 8;
  uint32_t p0 = (w & 0x000F000Fu) | 0x64006400u;
  uint32_t p1 = (w & 0x00F000F0u) | 0x64006400u;
  uint32_t p2 = (w8 & 0x000F000Fu) | 0x64006400u;
  uint32_t p3 = (w8 & 0x00F000F0u) | 0x64006400u;
  __half2 q0 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&p0), k1024), s2, b2);
  __half2 q1 = __hfma2(__hfma2(*reinterpret_cast<__half2*>(&p1), k16inv, km64), s2, b2);
  __half2 q2 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&p2), k1024), s2, b2);
  __half2 q3 = __hfma2(__hfma2(*reinterpret_cast<__half2*>(&p3), k16inv, km64), s2, b2);
  o[0] = *reinterpret_cast<uint32_t*>(&q0);
  o[1] = *reinterpret_cast<uint32_t*>(&q1);
  o[2] = *reinterpret_cast<uint32_t*>(&q2);
  o[3] = *reinterpret_cast<uint32_t*>(&q3);
}

template <int MODE>
struct Geo {
  static constexpr int K = MODE == 0 ? kHidden : kInter;
  static constexpr int KS = K / 64;
  static constexpr int PARTS = MODE == 0 ? kInter / 128 : kHidden / 256;
};

__device__ __forceinline__ float silu_mul_fast(float g, float u) {
  const float e = __expf(fminf(-g, 80.0f));
  return __fdividef(g, 1.0f + e) * u;
}

template <bool BF16, int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1) k_grouped(const __grid_constant__ GemmArgs a) {
  constexpr int KS = Geo<MODE>::KS;
  constexpr int PARTS = Geo<MODE>::PARTS;
  static_assert(KS % kAStages == 0, "producer unroll needs KS % kAStages == 0");
  extern __shared__ uint8_t gsm_raw[];
  uint8_t* ring =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* codes = ring + kTokStages * kTokStageBytes;
  uint8_t* sbring = codes + kCodeStages * kCodeStageBytes;
  GemmSync* sy = reinterpret_cast<GemmSync*>(ring + kRingBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_units = *a.n_tiles * PARTS;
  const int G = gridDim.x;
  if ((int)blockIdx.x >= n_units) return;
  const int my_units = (n_units - (int)blockIdx.x + G - 1) / G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTokStages; s++) {
      mbar_init(&sy->tok_full[s], 1);
      mbar_init(&sy->tok_empty[s], 2);
    }
    for (int s = 0; s < kAStages; s++) {
      mbar_init(&sy->a_full[s], 8);
      mbar_init(&sy->a_empty[s], 2);
    }
    for (int h = 0; h < 2; h++) {
      mbar_init(&sy->acc_full[h], 2);
      mbar_init(&sy->acc_empty[h], 8);
    }
    for (int s = 0; s < kCodeStages; s++) {
      mbar_init(&sy->code_full[s], 1);
      mbar_init(&sy->code_empty[s], 8);
    }
    for (int s = 0; s < kSbBufs; s++) {
      mbar_init(&sy->sb_full[s], 1);
      mbar_init(&sy->sb_empty[s], 8);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_u32(&sy->tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sy->tmem;
  bool ok = true;

  if (warp < 8) {
    // ---------------- weight producers: Q4 (shared memory) -> fp16 -> TMEM (A operand)
    const int q = warp & 3, blk = warp >> 2, r = q * 32 + lane;
    const int total = my_units * KS;
    const int row_off = blk * 128 + r;
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + kTmemA + blk * 32;
    for (int g = 0; g < total; g += kAStages) {
#pragma unroll
      for (int j = 0; j < kAStages; j++) {
        const int flat = g + j;
        const int ks = flat % KS, win = flat / kSbWin;  // windows never straddle units (KS % 8 == 0)
        const int cs = flat % kCodeStages, sbuf = win % kSbBufs;
        if (ks % kSbWin == 0 && !mbar_wait(&sy->sb_full[sbuf], (win / kSbBufs) & 1)) ok = false;
        if (!mbar_wait(&sy->code_full[cs], (flat / kCodeStages) & 1)) ok = false;
        const uint4* cp = reinterpret_cast<const uint4*>(codes + cs * kCodeStageBytes + row_off * 32);
        const uint4 c0 = cp[0], c1 = cp[1];
        const uint16_t* sbp = reinterpret_cast<const uint16_t*>(sbring + sbuf * 2 * kSbHalf);
        const uint16_t sv = sbp[row_off * kSbWin + ks % kSbWin];
        const uint16_t bv = sbp[kSbHalf / 2 + row_off * kSbWin + ks % kSbWin];
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sy->code_empty[cs]);
          if (ks % kSbWin == kSbWin - 1) mbar_arrive(&sy->sb_empty[sbuf]);
        }
        const uint32_t sbits = half_bits<BF16>(sv), bbits = half_bits<BF16>(bv);
        const __half2 s2 = __halves2half2(__ushort_as_half(sbits), __ushort_as_half(sbits));
        const __half2 b2 = __halves2half2(__ushort_as_half(bbits), __ushort_as_half(bbits));
        const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        uint32_t o[32];
#pragma unroll
        for (int wi = 0; wi < 8; wi++) dequant_word(cw[wi], s2, b2, o + 4 * wi);
        if (!mbar_wait(&sy->a_empty[j], ((flat / kAStages) & 1) ^ 1)) ok = false;
        tc_fence_after();
        tmem_st32(tbase + j * 64, o);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sy->a_full[j]);
      }
    }
  } else if (warp < 16) {
    // ---------------- epilogue: TMEM -> SiLU(g)*u fp16 act / weighted fp32 y
    const int eq = warp & 3, half = (warp - 8) >> 2, et = threadIdx.x - 256;
    const uint32_t lrow = (uint32_t)(eq * 32) << 16;
    uint32_t acc_use[2] = {0u, 0u};
    for (int i = 0; i < my_units; i++) {
      const int u = blockIdx.x + i * G;
      const int4 t = a.tiles[u / PARTS];
      const int part = u % PARTS;
      const bool shared = t.x == kExperts;
      const int n = t.z;
      const int pb = t.w + t.y;  // first row of the tile in the row space
      if (MODE == 1 || a.ep.ret) {
        for (int c = et; c < n; c += kEpiThreads) {
          if (!a.ep.ret) {
            sy->col_pos[i & 1][c] = (shared || !a.perm) ? pb + c : a.perm[pb + c];
            continue;
          }
          float* dst;
          {
            // (rank << 24) | row: the row of that rank's result (MODE 1) or
            // activation (MODE 0) area, stored over NVLink while the following
            // tiles run
            const int code = a.ep.ret[pb + c];
            const int dr = code >> 24, row = code & 0xFFFFFF;
            if (dr < 0 || dr >= a.ep.n_peers || row >= a.ep.rows_cap) {
              set_status(a.status, kStatusDevice);
              dst = nullptr;
            } else if (MODE == 0) {
              dst = reinterpret_cast<float*>(a.ep.peer[dr] + a.ep.act_off + (size_t)row * kInter * 2);
            } else {
              dst = reinterpret_cast<float*>(a.ep.peer[dr] + a.ep.y_off) + (size_t)row * kHidden;
            }
          }
          sy->col_row[i & 1][c] = dst;
        }
        named_sync(2, kEpiThreads);
      }
      // accumulator halves: a tile of <= 64 rows uses half i & 1 alone, a
      // larger one both (acc_use counts each half's earlier units)
      const bool small_u = n <= kSmallAcc;
      const bool use0 = !small_u || (i & 1) == 0, use1 = !small_u || (i & 1) == 1;
      if (use0 && !mbar_wait(&sy->acc_full[0], acc_use[0] & 1)) ok = false;
      if (use1 && !mbar_wait(&sy->acc_full[1], acc_use[1] & 1)) ok = false;
      tc_fence_after();
      const uint32_t hcol = small_u ? (uint32_t)(i & 1) * kSmallAcc : 0u;
      const int cbeg = half * (kTileRows / 2), cend = min(n, cbeg + kTileRows / 2);
      if (MODE == 0) {
        const int f = part * 128 + eq * 32 + lane;
        const int fp = (f & ~7) | ((f & 3) << 1) | ((f >> 2) & 1);
        __half* dst = a.act + (size_t)pb * kInter + fp;
        for (int c0 = cbeg; c0 < cend; c0 += 16) {
          uint32_t g[16], v[16];
          tmem_ld16(tmem + lrow + hcol + c0, g);
          tmem_ld16(tmem + lrow + 128 + hcol + c0, v);
          tmem_ld_wait();
          if (a.ep.ret) {
#pragma unroll
            for (int j = 0; j < 16; j++)
              if (c0 + j < cend) {
                __half* d = reinterpret_cast<__half*>(sy->col_row[i & 1][c0 + j]);
                if (d) d[fp] = __float2half_rn(silu_mul_fast(__uint_as_float(g[j]), __uint_as_float(v[j])));
              }
          } else {
#pragma unroll
            for (int j = 0; j < 16; j++)
              if (c0 + j < cend)
                dst[(size_t)(c0 + j) * kInter] =
                    __float2half_rn(silu_mul_fast(__uint_as_float(g[j]), __uint_as_float(v[j])));
          }
        }
      } else {
        const int f = part * 256 + eq * 32 + lane;
        for (int c0 = cbeg; c0 < cend; c0 += 32) {
          uint32_t v0[32], v1[32];
          tmem_ld32(tmem + lrow + hcol + c0, v0);
          tmem_ld32(tmem + lrow + 128 + hcol + c0, v1);
          tmem_ld_wait();
          if (a.ep.ret) {
#pragma unroll
            for (int j = 0; j < 32; j++)
              if (c0 + j < cend) {
                float* d = sy->col_row[i & 1][c0 + j];
                if (d) {
                  d[f] = __uint_as_float(v0[j]);
                  d[f + 128] = __uint_as_float(v1[j]);
                }
              }
          } else {
            float* base = a.y + f;
#pragma unroll
            for (int j = 0; j < 32; j++)
              if (c0 + j < cend) {
                float* d = base + (size_t)sy->col_pos[i & 1][c0 + j] * kHidden;
                d[0] = __uint_as_float(v0[j]);
                d[128] = __uint_as_float(v1[j]);
              }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (use0) mbar_arrive(&sy->acc_empty[0]);
        if (use1) mbar_arrive(&sy->acc_empty[1]);
      }
      acc_use[0] += use0 ? 1u : 0u;
      acc_use[1] += use1 ? 1u : 0u;
    }
    // peer stores are visible system-wide before the kernel that signals them runs
    if (a.ep.ret) __threadfence_system();
  } else if (warp < kLoadWarp) {
    // ---------------- MMA issue: warp 16 -> block 0 / acc0, warp 17 -> block 1 / acc1
    if (lane == 0) {
      const uint32_t blk = (uint32_t)(warp - kMmaWarp);
      int gs = 0;
      uint32_t acc_use[2] = {0u, 0u};
      for (int i = 0; i < my_units; i++) {
        const int u = blockIdx.x + i * G;
        const int rows = a.tiles[u / PARTS].z;
        const uint32_t N = (uint32_t)((rows + 15) & ~15);
        const uint32_t idesc = (1u << 4) | ((N >> 3) << 17) | ((128u >> 4) << 24);
        // the same half choice as the epilogue: a small tile takes half i & 1
        const bool small_u = rows <= kSmallAcc;
        const bool use0 = !small_u || (i & 1) == 0, use1 = !small_u || (i & 1) == 1;
        const uint32_t dacc = tmem + blk * 128 + (small_u ? (uint32_t)(i & 1) * kSmallAcc : 0u);
        if (use0 && !mbar_wait(&sy->acc_empty[0], (acc_use[0] & 1) ^ 1)) ok = false;
        if (use1 && !mbar_wait(&sy->acc_empty[1], (acc_use[1] & 1) ^ 1)) ok = false;
        tc_fence_after();
        for (int ks = 0; ks < KS; ks++, gs++) {
          const int ts = gs % kTokStages, as = gs % kAStages;
          if (!mbar_wait(&sy->tok_full[ts], (gs / kTokStages) & 1)) ok = false;
          if (!mbar_wait(&sy->a_full[as], (gs / kAStages) & 1)) ok = false;
          tc_fence_after();
          const uint32_t bb = s_u32(ring + ts * kTokStageBytes);
          const uint32_t ac = tmem + kTmemA + as * 64 + blk * 32;
#pragma unroll
          for (int kk = 0; kk < 4; kk++) mma_ts(dacc, ac + kk * 8, sdesc(bb + kk * 32), idesc, (ks | kk) ? 1u : 0u);
          tc_commit(&sy->tok_empty[ts]);
          tc_commit(&sy->a_empty[as]);
        }
        if (use0) tc_commit(&sy->acc_full[0]);
        if (use1) tc_commit(&sy->acc_full[1]);
        acc_use[0] += use0 ? 1u : 0u;
        acc_use[1] += use1 ? 1u : 0u;
      }
    }
  } else if (warp == kLoadWarp && lane == 0) {
    // ---------------- weight loads by TMA, per 64-column step: the unit's codes
    // (and every 8 steps their scales and biases); gated only by the producers,
    // so the weight stream runs as far ahead as the rings allow
    int gs = 0;
    for (int i = 0; i < my_units; i++) {
      const int u = blockIdx.x + i * G;
      const int4 t = a.tiles[u / PARTS];
      const int part = u % PARTS;
      const int src = t.x == kExperts ? 1 : 0;
      const int rec = src ? 0 : t.x;
      for (int ks = 0; ks < KS; ks++, gs++) {
        const int cs = gs % kCodeStages, win = gs / kSbWin, sbuf = win % kSbBufs;
        if (ks % kSbWin == 0) {
          if (!mbar_wait(&sy->sb_empty[sbuf], ((win / kSbBufs) & 1) ^ 1)) ok = false;
          uint8_t* sd = sbring + sbuf * 2 * kSbHalf;
          mbar_expect_tx(&sy->sb_full[sbuf], 2 * kSbHalf);
          if (MODE == 0) {
            tma_load4(sd, &a.map_s[src], ks, part * 128, 0, rec, &sy->sb_full[sbuf]);
            tma_load4(sd + kSbHalf, &a.map_b[src], ks, part * 128, 0, rec, &sy->sb_full[sbuf]);
          } else {
            tma_load3(sd, &a.map_s[src], ks, part * 256, rec, &sy->sb_full[sbuf]);
            tma_load3(sd + kSbHalf, &a.map_b[src], ks, part * 256, rec, &sy->sb_full[sbuf]);
          }
        }
        if (!mbar_wait(&sy->code_empty[cs], ((gs / kCodeStages) & 1) ^ 1)) ok = false;
        mbar_expect_tx(&sy->code_full[cs], kCodeStageBytes);
        if (MODE == 0)
          tma_load4(codes + cs * kCodeStageBytes, &a.map_code[src], ks * 32, part * 128, 0, rec, &sy->code_full[cs]);
        else
          tma_load3(codes + cs * kCodeStageBytes, &a.map_code[src], ks * 32, part * 256, rec, &sy->code_full[cs]);
      }
    }
  } else if (warp == kTokWarp && lane == 0) {
    // ---------------- token tiles by TMA (gated by the MMAs that free the stages)
    int gs = 0;
    for (int i = 0; i < my_units; i++) {
      const int u = blockIdx.x + i * G;
      const int4 t = a.tiles[u / PARTS];
      const int pb = t.w + t.y;
      const bool small = t.z <= kSmallTileRows;
      for (int ks = 0; ks < KS; ks++, gs++) {
        const int ts = gs % kTokStages;
        if (!mbar_wait(&sy->tok_empty[ts], ((gs / kTokStages) & 1) ^ 1)) ok = false;
        mbar_expect_tx(&sy->tok_full[ts], small ? kSmallTileRows * 128 : kTokStageBytes);
        tma_tile(ring + ts * kTokStageBytes, small ? &a.map_rows_small : &a.map_rows, ks * 64, pb, &sy->tok_full[ts]);
      }
    }
  }

  if (!ok) set_status(a.status, kStatusTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// out = (residual + sigmoid(c) * shared) + sum_k w_k * y_k, the products
// rounded and summed in router order (deltanet.metal:2213-2227)
// x16_next (optional): fp16 RMSNorm of the output row for a following block
// (deltanet.metal:18-53, unit weight): the mean of squares summed as 128 tiles
// of 16 rows (fma chain inside a tile, tiles summed in order), the order of the
// decode kernels and the oracle, so stacked blocks equal chained ones bit for bit
__global__ void __launch_bounds__(256) k_combine_weighted(int T, const float* __restrict__ residual,
                                                          const float* __restrict__ y_pos,
                                                          const float* __restrict__ w,
                                                          const float* __restrict__ y_sh,
                                                          const float* __restrict__ coef,
                                                          float* __restrict__ out, float eps,
                                                          uint16_t* __restrict__ x16_next) {
  __shared__ float vrow[kHidden];
  __shared__ float part[kHidden / 16];
  __shared__ float inv;
  const int t = blockIdx.x;
  const float c = coef[t];
  const float coeff = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-c)));
  float wk[kTopK];
#pragma unroll
  for (int k = 0; k < kTopK; k++) wk[k] = w[t * kTopK + k];
  const float4* y4 = reinterpret_cast<const float4*>(y_pos + (size_t)t * kTopK * kHidden);
  const float4* s4 = reinterpret_cast<const float4*>(y_sh + (size_t)t * kHidden);
  const float4* r4 = residual ? reinterpret_cast<const float4*>(residual + (size_t)t * kHidden) : nullptr;
  float4* o4 = reinterpret_cast<float4*>(out + (size_t)t * kHidden);
  for (int i = threadIdx.x; i < kHidden / 4; i += 256) {
    float4 y = y4[i];
    float4 acc = make_float4(__fmul_rn(y.x, wk[0]), __fmul_rn(y.y, wk[0]), __fmul_rn(y.z, wk[0]), __fmul_rn(y.w, wk[0]));
#pragma unroll
    for (int k = 1; k < kTopK; k++) {
      y = y4[k * (kHidden / 4) + i];
      acc.x = __fadd_rn(acc.x, __fmul_rn(y.x, wk[k]));
      acc.y = __fadd_rn(acc.y, __fmul_rn(y.y, wk[k]));
      acc.z = __fadd_rn(acc.z, __fmul_rn(y.z, wk[k]));
      acc.w = __fadd_rn(acc.w, __fmul_rn(y.w, wk[k]));
    }
    const float4 sh = s4[i];
    const float4 base = r4 ? r4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 v = make_float4(__fadd_rn(__fadd_rn(base.x, __fmul_rn(sh.x, coeff)), acc.x),
                                 __fadd_rn(__fadd_rn(base.y, __fmul_rn(sh.y, coeff)), acc.y),
                                 __fadd_rn(__fadd_rn(base.z, __fmul_rn(sh.z, coeff)), acc.z),
                                 __fadd_rn(__fadd_rn(base.w, __fmul_rn(sh.w, coeff)), acc.w));
    o4[i] = v;
    if (x16_next) reinterpret_cast<float4*>(vrow)[i] = v;
  }
  if (!x16_next) return;
  __syncthreads();
  if (threadIdx.x < kHidden / 16) {
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const float e = vrow[threadIdx.x * 16 + j];
      a = __fmaf_rn(e, e, a);
    }
    part[threadIdx.x] = a;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int c2 = 0; c2 < kHidden / 16; c2++) tot = __fadd_rn(tot, part[c2]);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)kHidden), eps)));
  }
  __syncthreads();
  __half* o = reinterpret_cast<__half*>(x16_next) + (size_t)t * kHidden;
  for (int i = threadIdx.x; i < kHidden; i += 256) o[i] = __float2half_rn(__fmul_rn(vrow[i], inv));
}

}  // namespace

// ------------------------------------------------------------------ host side
static size_t al256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

static size_t max_tiles_for(int T) {
  return static_cast<size_t>(T) * kTopK / kTileRows + kExperts + (T + kTileRows - 1) / kTileRows + 1;
}

size_t prefill_workspace_bytes(int T) {
  const size_t P = static_cast<size_t>(T) * kTopK;
  const size_t R = P + static_cast<size_t>(T);  // row space: routed positions + shared tokens
  size_t b = 0;
  b += al256(4 * (size_t)T * kExperts);          // logits
  b += al256(4 * (size_t)T);                     // coef
  b += al256(4 * P) * 2;                         // idx, w
  b += al256(4 * (kExperts + 1)) * 2;            // counts, offsets
  b += al256(4 * P);                             // perm
  b += al256(dispatch_workspace_bytes(T));       // plan scratch
  b += al256(16 * max_tiles_for(T)) + al256(16); // tiles, count
  b += al256(2 * R * kHidden);                   // gathered x (fp16, permuted K)
  b += al256(2 * R * kInter);                    // act (fp16, permuted K)
  b += al256(4 * R * kHidden);                   // y (fp32)
  return b;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
static PFN_cuTensorMapEncodeTiled encode_fn() {
  static PFN_cuTensorMapEncodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
  }
  return fn;
}

// fp16 matrix [rows][cols] (row-major), box = 64 columns (128 bytes) x box_rows,
// 128-byte swizzle: the K-major operand layout the MMA descriptors expect
static bool encode_rows(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// n-D tiled map without swizzle (weight codes, scales, biases)
static bool encode_nd(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
                      const cuuint64_t* strides, const cuuint32_t* box) {
  PFN_cuTensorMapEncodeTiled fn = encode_fn();
  if (!fn) return false;
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return fn(m, dt, rank, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Weight maps of one source (the bank, or the shared record as a bank of 1).
// gate/up: codes [record][matrix gate|up][512 rows][1024 bytes], scales and
// biases [record][matrix][512 rows][32 groups]; down: codes [record][2048
// rows][256 bytes], scales and biases [record][2048 rows][8 groups].
static bool encode_weights(GemmArgs* g, int src, int mode, const uint8_t* rec0, uint64_t n_rec, uint64_t stride) {
  if (mode == 0) {
    const cuuint64_t dc[4] = {1024, 512, 2, n_rec}, sc[3] = {1024, 589824, stride};
    const cuuint32_t bc[4] = {32, 128, 2, 1};
    const cuuint64_t ds[4] = {32, 512, 2, n_rec}, ss[3] = {64, 589824, stride};
    const cuuint32_t bs[4] = {8, 128, 2, 1};
    return encode_nd(&g->map_code[src], CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, rec0 + kOffGateW, dc, sc, bc) &&
           encode_nd(&g->map_s[src], CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, rec0 + kOffGateS, ds, ss, bs) &&
           encode_nd(&g->map_b[src], CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, rec0 + kOffGateB, ds, ss, bs);
  }
  const cuuint64_t dc[3] = {256, 2048, n_rec}, sc[2] = {256, stride};
  const cuuint32_t bc[3] = {32, 256, 1};
  const cuuint64_t ds[3] = {8, 2048, n_rec}, ss[2] = {16, stride};
  const cuuint32_t bs[3] = {8, 256, 1};
  return encode_nd(&g->map_code[src], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, rec0 + kOffDownW, dc, sc, bc) &&
         encode_nd(&g->map_s[src], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, rec0 + kOffDownS, ds, ss, bs) &&
         encode_nd(&g->map_b[src], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, rec0 + kOffDownB, ds, ss, bs);
}

cudaError_t prefill_init_attributes() {
  if (!encode_fn()) return cudaErrorNotSupported;
  cudaError_t e;
  e = cudaFuncSetAttribute(k_router_prefill<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRtSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_router_prefill<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRtSmem);
  if (e != cudaSuccess) return e;
  // three router CTAs per SM need the largest shared-memory carveout
  e = cudaFuncSetAttribute(k_router_prefill<false>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_router_prefill<true>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_grouped<false, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_grouped<false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_grouped<true, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_grouped<true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
}

cudaError_t router_logits_prefill(cudaStream_t st, const LayerW& L, bool bf16, int T,
                                  const uint16_t* x, float* logits, float* coef) {
  // blockIdx.y == 0: the coefficient CTAs (no work when coef is NULL)
  const dim3 grid((T + kRtTok - 1) / kRtTok, kRtRowBlocks + 1);
  if (bf16)
    k_router_prefill<true><<<grid, kRtThreads, kRtSmem, st>>>(L, T, x, logits, coef);
  else
    k_router_prefill<false><<<grid, kRtThreads, kRtSmem, st>>>(L, T, x, logits, coef);
  return cudaGetLastError();
}

size_t grouped_max_tiles(int T) { return max_tiles_for(T); }

cudaError_t tile_list(cudaStream_t st, const int* counts, const int* offsets, int T_shared,
                      const int* shared_base, int4* tiles, int* n_tiles) {
  k_tile_list<<<1, kListThreads, 0, st>>>(counts, offsets, T_shared, shared_base, tiles, n_tiles);
  return cudaGetLastError();
}

cudaError_t grouped_ffn_stages(cudaStream_t st, const LayerW& L, bool bf16, const uint16_t* rows, size_t R,
                               __half* act, float* y, const int* perm, const int4* tiles, const int* n_tiles,
                               size_t max_tiles, int sms, int* status, Prof* prof, int stages,
                               const EpOut* ep0, const EpOut* ep1) {
  GemmArgs g0, g1;
  if ((stages & 1) && (!encode_rows(&g0.map_rows, rows, R, kHidden, kTileRows) ||
                       !encode_rows(&g0.map_rows_small, rows, R, kHidden, kSmallTileRows) ||
                       !encode_weights(&g0, 0, 0, L.bank, L.bank_records, L.stride) ||
                       !encode_weights(&g0, 1, 0, L.shared, 1, L.stride)))
    return cudaErrorInvalidValue;
  if ((stages & 2) && (!encode_rows(&g1.map_rows, act, R, kInter, kTileRows) ||
                       !encode_rows(&g1.map_rows_small, act, R, kInter, kSmallTileRows) ||
                       !encode_weights(&g1, 0, 1, L.bank, L.bank_records, L.stride) ||
                       !encode_weights(&g1, 1, 1, L.shared, 1, L.stride)))
    return cudaErrorInvalidValue;
  g0.L = g1.L = L;
  g0.perm = g1.perm = perm;
  g0.tiles = g1.tiles = tiles;
  g0.n_tiles = g1.n_tiles = n_tiles;
  g0.act = g1.act = act;
  g0.y = g1.y = y;
  g0.status = g1.status = status;
  g0.ep = ep0 ? *ep0 : EpOut{};
  g1.ep = ep1 ? *ep1 : EpOut{};
  if (stages & 1) {
    const unsigned grid0 = (unsigned)std::min<size_t>((size_t)sms, max_tiles * Geo<0>::PARTS);
    ProfScope ps(prof, kKGateUp, st);
    if (bf16)
      k_grouped<true, 0><<<grid0, kGemmThreads, kGemmSmem, st>>>(g0);
    else
      k_grouped<false, 0><<<grid0, kGemmThreads, kGemmSmem, st>>>(g0);
  }
  if (stages & 2) {
    const unsigned grid1 = (unsigned)std::min<size_t>((size_t)sms, max_tiles * Geo<1>::PARTS);
    ProfScope ps(prof, kKDown, st);
    if (bf16)
      k_grouped<true, 1><<<grid1, kGemmThreads, kGemmSmem, st>>>(g1);
    else
      k_grouped<false, 1><<<grid1, kGemmThreads, kGemmSmem, st>>>(g1);
  }
  return cudaGetLastError();
}

cudaError_t grouped_ffn(cudaStream_t st, const LayerW& L, bool bf16, const uint16_t* rows, size_t R,
                        __half* act, float* y, const int* perm, const int4* tiles, const int* n_tiles,
                        size_t max_tiles, int sms, int* status, Prof* prof, const EpOut* ep) {
  return grouped_ffn_stages(st, L, bf16, rows, R, act, y, perm, tiles, n_tiles, max_tiles, sms, status, prof, 3,
                            nullptr, ep);
}

// The routed experts of T tokens without the shared expert or the combine:
// y[t * 8 + k] = D_e(SiLU(G_e x_t) * (U_e x_t)), e = idx[t * 8 + k], through
// the dispatch plan, the row gather and the grouped GEMMs of the block (the
// tile list gets a negative shared base, so it holds no shared-expert tiles).
// Workspace: prefill_workspace_bytes(T).
cudaError_t grouped_ffn_routed(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                               const int* idx, float* y, void* workspace, int* status, Prof* prof) {
  const size_t P = static_cast<size_t>(T) * kTopK;
  const size_t max_tiles = max_tiles_for(T);
  char* p = static_cast<char*>(workspace);
  auto take = [&](size_t n) {
    char* q = p;
    p += al256(n);
    return q;
  };
  int* counts = reinterpret_cast<int*>(take(4 * (kExperts + 1)));
  int* offsets = reinterpret_cast<int*>(take(4 * (kExperts + 1)));
  int* perm = reinterpret_cast<int*>(take(4 * P));
  int* plan_ws = reinterpret_cast<int*>(take(dispatch_workspace_bytes(T)));
  int4* tiles = reinterpret_cast<int4*>(take(16 * max_tiles));
  int* n_tiles = reinterpret_cast<int*>(take(16));
  int* no_shared = n_tiles + 1;
  uint16_t* xs = reinterpret_cast<uint16_t*>(take(2 * P * kHidden));
  __half* act = reinterpret_cast<__half*>(take(2 * P * kInter));
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaMemsetAsync(no_shared, 0xFF, sizeof(int), st);  // -1: no shared rows
  if (e == cudaSuccess) e = dispatch_plan_ws(st, idx, T, counts, offsets, perm, plan_ws, status);
  if (e != cudaSuccess) return e;
  k_tile_list<<<1, kListThreads, 0, st>>>(counts, offsets, T, no_shared, tiles, n_tiles);
  k_gather_rows<<<(unsigned)((P + 7) / 8), 256, 0, st>>>(perm, (int)P, 0, reinterpret_cast<const uint4*>(x),
                                                          reinterpret_cast<uint4*>(xs));
  return grouped_ffn(st, L, bf16, xs, P, act, y, perm, tiles, n_tiles, max_tiles, sms, status, prof, nullptr);
}

cudaError_t prefill_block(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                          const float* residual, float* out, const RoutingArgs& r, int* idx_out,
                          float* w_out, void* workspace, int* status, Prof* prof, uint16_t* x16_next,
                          float eps) {
  const size_t P = static_cast<size_t>(T) * kTopK;
  const size_t R = P + static_cast<size_t>(T);
  const size_t max_tiles = max_tiles_for(T);
  char* p = static_cast<char*>(workspace);
  auto take = [&](size_t n) {
    char* q = p;
    p += al256(n);
    return q;
  };
  float* logits = reinterpret_cast<float*>(take(4 * (size_t)T * kExperts));
  float* coef = reinterpret_cast<float*>(take(4 * (size_t)T));
  int* idx = reinterpret_cast<int*>(take(4 * P));
  float* w = reinterpret_cast<float*>(take(4 * P));
  int* counts = reinterpret_cast<int*>(take(4 * (kExperts + 1)));
  int* offsets = reinterpret_cast<int*>(take(4 * (kExperts + 1)));
  int* perm = reinterpret_cast<int*>(take(4 * P));
  int* plan_ws = reinterpret_cast<int*>(take(dispatch_workspace_bytes(T)));
  int4* tiles = reinterpret_cast<int4*>(take(16 * max_tiles));
  int* n_tiles = reinterpret_cast<int*>(take(16));
  uint16_t* xs = reinterpret_cast<uint16_t*>(take(2 * R * kHidden));
  __half* act = reinterpret_cast<__half*>(take(2 * R * kInter));
  float* y = reinterpret_cast<float*>(take(4 * R * kHidden));

  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;

  {
    // decode batches (T <= 64): the decode router spreads over row blocks x
    // token chunks; both are bit-exact in the reference lane order
    ProfScope ps(prof, kKRouter, st);
    e = T <= kDecodeMaxTokens ? router_logits(st, L, bf16, T, x, logits, coef, status)
                              : router_logits_prefill(st, L, bf16, T, x, logits, coef);
  }
  if (e != cudaSuccess) return e;
  if (T <= kDecodeMaxTokens) {
    // above one token per warp the plan CTA's top-k costs more than its own launch
    const bool own_topk = !r.idx_in && T > kPlanTopkMaxTokens;
    if (own_topk) {
      ProfScope ps(prof, kKTopk, st);
      e = router_topk(st, T, logits, r.bias, idx, w, status);
      if (e != cudaSuccess) return e;
    }
    // timed as the top-k kernel when it selects the top-8 itself
    ProfScope ps(prof, own_topk || r.idx_in ? -2 : kKTopk, st);  // -2: never timed
    k_plan_small<<<1, kPlanSmallThreads, 0, st>>>(own_topk ? nullptr : logits, r.bias, r.idx_in, r.w_in, idx,
                                                 w, T, idx_out, w_out, counts, offsets, perm, tiles, n_tiles,
                                                 status);
  } else {
    if (r.idx_in) {
      e = cudaMemcpyAsync(idx, r.idx_in, 4 * P, cudaMemcpyDeviceToDevice, st);
      if (e != cudaSuccess) return e;
      e = cudaMemcpyAsync(w, r.w_in, 4 * P, cudaMemcpyDeviceToDevice, st);
    } else {
      ProfScope ps(prof, kKTopk, st);
      e = router_topk(st, T, logits, r.bias, idx, w, status);
    }
    if (e != cudaSuccess) return e;
    if (idx_out) e = cudaMemcpyAsync(idx_out, idx, 4 * P, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess && w_out) e = cudaMemcpyAsync(w_out, w, 4 * P, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return e;
    e = dispatch_plan_ws(st, idx, T, counts, offsets, perm, plan_ws, status);
    if (e != cudaSuccess) return e;
    k_tile_list<<<1, kListThreads, 0, st>>>(counts, offsets, T, nullptr, tiles, n_tiles);
  }
  k_gather_rows<<<(unsigned)((R + 7) / 8), 256, 0, st>>>(perm, (int)P, T, reinterpret_cast<const uint4*>(x),
                                                          reinterpret_cast<uint4*>(xs));
  e = grouped_ffn(st, L, bf16, xs, R, act, y, perm, tiles, n_tiles, max_tiles, sms, status, prof, nullptr);
  if (e != cudaSuccess) return e;
  {
    ProfScope ps(prof, kKCombine, st);
    k_combine_weighted<<<T, 256, 0, st>>>(T, residual, y, w, y + P * kHidden, coef, out, eps, x16_next);
  }
  return cudaGetLastError();
}

}  // namespace qf
