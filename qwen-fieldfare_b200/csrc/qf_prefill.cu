// qf_prefill.cu -- MoE block for many tokens (prefill, T > 64): grouped expert
// GEMMs on the 5th-generation tensor cores.
//
// Flow (one stream, all on the device):
//   k_router_prefill  router logits in the reference lane order (bit-exact)
//   k_topk            top-8 / softmax / renormalise (with the harness bias)
//   dispatch plan     counts, offsets, stable permutation by (expert, token, k)
//   k_tile_map        one entry per 128-row tile of every expert (+ shared)
//   k_moe_gemm<0>     gate/up: X[perm rows] . [G;U]^T -> SiLU(g)*u (fp16 act)
//   k_moe_gemm<1>     down: act . D^T * routing weight -> per-position rows
//   k_combine         residual + sigmoid(c) * shared + sum_k in router order
//
// k_moe_gemm: one CTA per (128-row tile, N tile).  A (token rows, fp16) is
// gathered with 16-byte cp.async into the 128-byte-swizzled K-major layout;
// the expert's Q4 codes are copied the same way and dequantised to fp16
// (w = q*s + b, one rounding) into the B operand; one thread issues
// tcgen05.mma (M=128, N=256, K=16 x 4 per 64-column group) accumulating in
// TMEM; completions are tracked with tcgen05.commit on mbarriers so loads,
// dequant and MMA of consecutive K steps overlap.  The epilogue reads TMEM
// with tcgen05.ld.
#include <math.h>

#include "qf_internal.h"

namespace qf {

namespace {

constexpr unsigned kSpin = 1u << 22;  // bounded waits (a few seconds at most)
constexpr int kStatusTimeout = -6;

__device__ __forceinline__ uint32_t s_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t sw128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }
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
__device__ __forceinline__ void cp16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ bool mbar_wait_p(uint64_t* bar, uint32_t parity) {
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

// ------------------------------------------------------------------ router
// CTA = 16 tokens (fp32 x in shared memory) x all 256 router rows + the
// shared-gate coefficient; warp w owns rows w, w+16, ...  Same per-lane order
// as the decode router (deltanet.metal:2229-2260), xor-butterfly reduction.
constexpr int kRtTok = 16;
constexpr int kRtThreads = 512;
constexpr size_t kRtSmem = sizeof(float) * (kRtTok * kHidden + kRtTok * 256);

template <bool BF16>
__global__ void __launch_bounds__(kRtThreads) k_router_prefill(LayerW L, int T,
                                                               const uint16_t* __restrict__ x,
                                                               float* __restrict__ logits,
                                                               float* __restrict__ coef) {
  extern __shared__ __align__(16) float rsm[];
  float* xs = rsm;                       // [16][2048]
  float* xsum = rsm + kRtTok * kHidden;  // [16][8 blk][32 lane]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRtTok;
  const int tn = min(kRtTok, T - t0);
  for (int i = threadIdx.x; i < tn * (kHidden / 8); i += kRtThreads) {
    const int t = i / (kHidden / 8), c = i % (kHidden / 8);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + (size_t)(t0 + t) * kHidden) + c);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    float4* d = reinterpret_cast<float4*>(xs + t * kHidden + c * 8);
    const float2 a = __half22float2(h[0]), b = __half22float2(h[1]), cc = __half22float2(h[2]),
                 dd = __half22float2(h[3]);
    d[0] = make_float4(a.x, a.y, b.x, b.y);
    d[1] = make_float4(cc.x, cc.y, dd.x, dd.y);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < tn * 256; i += kRtThreads) {
    const float* e = xs + (i >> 8) * kHidden + ((i >> 5) & 7) * 256 + (i & 31) * 8;
    float s = e[0];
#pragma unroll
    for (int j = 1; j < 8; j++) s = __fadd_rn(s, e[j]);
    xsum[i] = s;
  }
  __syncthreads();
  for (int r = warp; r <= kExperts; r += kRtThreads / 32) {
    if (r < kExperts) {
      const uint8_t* wrow = L.rw + (size_t)r * kHidden;
      float q[8][8];
      float sc[8], bi[8];
#pragma unroll
      for (int blk = 0; blk < 8; blk++) {
        const uint2 w = __ldg(reinterpret_cast<const uint2*>(wrow + blk * 256 + lane * 8));
#pragma unroll
        for (int i = 0; i < 4; i++) {
          q[blk][i] = byte_f(w.x, i);
          q[blk][4 + i] = byte_f(w.y, i);
        }
        const int g = blk * 4 + (lane >> 3);
        sc[blk] = ld16<BF16>(L.rs + r * 32, g);
        bi[blk] = ld16<BF16>(L.rb + r * 32, g);
      }
      for (int t = 0; t < tn; t++) {
        float acc = 0.f;
#pragma unroll
        for (int blk = 0; blk < 8; blk++) {
          const float4* e4 = reinterpret_cast<const float4*>(xs + t * kHidden + blk * 256 + lane * 8);
          const float4 a = e4[0], b = e4[1];
          float dot = 0.f;
          dot = __fmaf_rn(q[blk][0], a.x, dot);
          dot = __fmaf_rn(q[blk][1], a.y, dot);
          dot = __fmaf_rn(q[blk][2], a.z, dot);
          dot = __fmaf_rn(q[blk][3], a.w, dot);
          dot = __fmaf_rn(q[blk][4], b.x, dot);
          dot = __fmaf_rn(q[blk][5], b.y, dot);
          dot = __fmaf_rn(q[blk][6], b.z, dot);
          dot = __fmaf_rn(q[blk][7], b.w, dot);
          acc = __fmaf_rn(sc[blk], dot, acc);
          acc = __fmaf_rn(bi[blk], xsum[t * 256 + blk * 32 + lane], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) logits[(size_t)(t0 + t) * kExperts + r] = acc;
      }
    } else if (coef) {
      const float cs = ld16<BF16>(L.cs, lane), cb = ld16<BF16>(L.cb, lane);
      uint4 cw[4];
#pragma unroll
      for (int qq = 0; qq < 4; qq++) cw[qq] = __ldg(reinterpret_cast<const uint4*>(L.cw + lane * 64) + qq);
      for (int t = 0; t < tn; t++) {
        const float* e = xs + t * kHidden + lane * 64;
        float acc = 0.f;
#pragma unroll
        for (int qq = 0; qq < 4; qq++)
#pragma unroll
          for (int d = 0; d < 4; d++)
#pragma unroll
            for (int k = 0; k < 4; k++)
              acc = __fmaf_rn(__fmaf_rn(byte_f(word_of(cw[qq], d), k), cs, cb), e[qq * 16 + d * 4 + k], acc);
        acc = warp_sum(acc);
        if (lane == 0) coef[t0 + t] = acc;
      }
    }
  }
}

// ------------------------------------------------------------------ tile map
// tiles[i] = (expert, first row); expert 256 = the shared expert (all T tokens).
__global__ void k_tile_map(const int* __restrict__ counts, int T, int2* __restrict__ tiles,
                           int* __restrict__ n_tiles) {
  if (threadIdx.x != 0) return;
  int n = 0;
  for (int e = 0; e <= kExperts; e++) {
    const int cnt = e < kExperts ? counts[e] : T;
    for (int m0 = 0; m0 < cnt; m0 += 128) tiles[n++] = make_int2(e, m0);
  }
  *n_tiles = n;
}

// ------------------------------------------------------------------ grouped GEMM
constexpr int kGThreads = 256;
constexpr int kStages = 4;  // A / code stages in flight
constexpr int kABytes = 128 * 128;   // 128 rows x 64 fp16
constexpr int kBBytes = 256 * 128;   // 256 rows x 64 fp16
constexpr int kCodeBytes = 256 * 32; // 256 rows x 64 nibbles
// shared memory: A[kStages] | B fp16 [2] | codes[kStages] | scales | biases | barriers
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStages * kABytes;
constexpr int kOffCode = kOffB + 2 * kBBytes;
constexpr int kOffScale = kOffCode + kStages * kCodeBytes;
constexpr int kScaleBytes = 256 * 64;  // up to 32 groups x 2 B per row
constexpr int kOffBias = kOffScale + kScaleBytes;
constexpr int kOffBar = kOffBias + kScaleBytes;
constexpr int kGemmSmem = kOffBar + 256 + 1024;  // + alignment slack

struct GemmArgs {
  LayerW L;
  int T;
  const __half* a_routed;   // MODE 0: x [T][2048]; MODE 1: routed act [T*8][512] (perm order)
  const __half* a_shared;   // MODE 0: x; MODE 1: shared act [T][512]
  const int* perm;
  const int* offsets;
  const int2* tiles;
  const int* n_tiles;
  __half* act_out;          // MODE 0: routed act [T*8][512]
  __half* act_sh_out;       // MODE 0: shared act [T][512]
  const float* w;           // MODE 1: routing weights [T*8]
  float* y_pos;             // MODE 1: [T*8][2048]
  float* y_sh;              // MODE 1: [T][2048]
  int* status;
};

// q*s + b for 8 nibbles of one word, written as 8 fp16 in element order
__device__ __forceinline__ uint4 dequant8(uint32_t w, __half2 s2, __half2 b2) {
  const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  const __half2 k16inv = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));  // 1/16
  const __half2 km64 = __halves2half2(__ushort_as_half(0xD400), __ushort_as_half(0xD400));    // -64
  const uint32_t w8 = w >> 8;
  uint32_t p0 = (w & 0x000F000Fu) | 0x64006400u;   // 1024 + (e0, e4)
  uint32_t p1 = (w & 0x00F000F0u) | 0x64006400u;   // 1024 + 16*(e1, e5)
  uint32_t p2 = (w8 & 0x000F000Fu) | 0x64006400u;  // 1024 + (e2, e6)
  uint32_t p3 = (w8 & 0x00F000F0u) | 0x64006400u;  // 1024 + 16*(e3, e7)
  __half2 q0 = __hsub2(*reinterpret_cast<__half2*>(&p0), k1024);
  __half2 q1 = __hfma2(*reinterpret_cast<__half2*>(&p1), k16inv, km64);
  __half2 q2 = __hsub2(*reinterpret_cast<__half2*>(&p2), k1024);
  __half2 q3 = __hfma2(*reinterpret_cast<__half2*>(&p3), k16inv, km64);
  q0 = __hfma2(q0, s2, b2);
  q1 = __hfma2(q1, s2, b2);
  q2 = __hfma2(q2, s2, b2);
  q3 = __hfma2(q3, s2, b2);
  const uint32_t r0 = *reinterpret_cast<uint32_t*>(&q0), r1 = *reinterpret_cast<uint32_t*>(&q1);
  const uint32_t r2 = *reinterpret_cast<uint32_t*>(&q2), r3 = *reinterpret_cast<uint32_t*>(&q3);
  uint4 o;
  o.x = __byte_perm(r0, r1, 0x5410);  // e0 e1
  o.y = __byte_perm(r2, r3, 0x5410);  // e2 e3
  o.z = __byte_perm(r0, r1, 0x7632);  // e4 e5
  o.w = __byte_perm(r2, r3, 0x7632);  // e6 e7
  return o;
}

template <bool BF16>
__device__ __forceinline__ __half to_half(uint16_t u) {
  if constexpr (BF16) {
    return __float2half_rn(__uint_as_float((uint32_t)u << 16));
  } else {
    return __ushort_as_half(u);
  }
}

template <bool BF16, int MODE>
__global__ void __launch_bounds__(kGThreads, 1) k_moe_gemm(const __grid_constant__ GemmArgs a) {
  constexpr int K = MODE == 0 ? kHidden : kInter;
  constexpr int KS = K / 64;                  // 64-column groups
  constexpr int NG = K / 64;                  // scale groups per B row
  extern __shared__ uint8_t gsm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* mma_done = reinterpret_cast<uint64_t*>(sm + kOffBar);  // [kStages]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffBar + 128);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if ((int)blockIdx.x >= *a.n_tiles) return;
  const int2 tile = a.tiles[blockIdx.x];
  const int e = tile.x, m0 = tile.y;
  const bool shared = (e == kExperts);
  const int row_base = shared ? 0 : a.offsets[e];
  const int n_e = shared ? a.T : (a.offsets[e + 1] - a.offsets[e]);
  const int nrows = min(128, n_e - m0);
  const uint8_t* rec = shared ? a.L.shared : a.L.bank + (uint64_t)e * a.L.stride;

  // B rows of this N tile: MODE 0 rows 0..127 gate features f0.., 128..255 up
  // features f0..; MODE 1 rows = output features n0..n0+255.
  const int f0 = MODE == 0 ? blockIdx.y * 128 : blockIdx.y * 256;

  // scales and biases of the 256 B rows, all groups (one copy per CTA)
  {
    uint8_t* ss = sm + kOffScale;
    uint8_t* bb = sm + kOffBias;
    constexpr int rowb = NG * 2;            // bytes per row
    constexpr int chunks = rowb / 16;       // 16-byte chunks per row
    for (int c = tid; c < 256 * chunks; c += kGThreads) {
      const int r = c / chunks, q = c % chunks;
      size_t so, bo;
      if (MODE == 0) {
        const int f = f0 + (r & 127);
        so = (r < 128 ? kOffGateS : kOffUpS) + (size_t)f * rowb;
        bo = (r < 128 ? kOffGateB : kOffUpB) + (size_t)f * rowb;
      } else {
        so = kOffDownS + (size_t)(f0 + r) * rowb;
        bo = kOffDownB + (size_t)(f0 + r) * rowb;
      }
      cp16(ss + r * rowb + q * 16, rec + so + q * 16, 16);
      cp16(bb + r * rowb + q * 16, rec + bo + q * 16, 16);
    }
    cp_commit();
  }

  // per-thread A-row sources for the gather: 4 chunks per thread per stage
  // (row = (tid >> 3) + 32 * j, chunk = tid & 7)
  const int a_chunk = tid & 7;
  const __half* a_src[4];
  uint32_t a_bytes[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int i = (tid >> 3) + 32 * j;
    if (i < nrows) {
      const int p = row_base + m0 + i;
      if (MODE == 0) {
        const int tok = shared ? p : (a.perm[p] >> 3);
        a_src[j] = a.a_routed + (size_t)tok * kHidden + a_chunk * 8;
      } else {
        a_src[j] = (shared ? a.a_shared : a.a_routed) + (size_t)p * kInter + a_chunk * 8;
      }
      a_bytes[j] = 16;
    } else {
      a_src[j] = MODE == 0 ? a.a_routed : (shared ? a.a_shared : a.a_routed);
      a_bytes[j] = 0;  // zero fill
    }
  }
  // code sources: 2 chunks per thread per stage (row = tid, halves 0/1 of its 32 bytes)
  const uint8_t* c_src;
  {
    const int r = tid;
    size_t off;
    if (MODE == 0) {
      const int f = f0 + (r & 127);
      off = (r < 128 ? kOffGateW : kOffUpW) + (size_t)f * (kHidden / 2);
    } else {
      off = kOffDownW + (size_t)(f0 + r) * (kInter / 2);
    }
    c_src = rec + off;
  }
  auto issue = [&](int ks) {
    const int st = ks % kStages;
    uint8_t* A = sm + kOffA + st * kABytes;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int i = (tid >> 3) + 32 * j;
      cp16(A + sw128(i, a_chunk), a_src[j] + ks * 64, a_bytes[j]);
    }
    uint8_t* Cd = sm + kOffCode + st * kCodeBytes;
    cp16(Cd + tid * 32, c_src + ks * 32, 16);
    cp16(Cd + tid * 32 + 16, c_src + ks * 32 + 16, 16);
    cp_commit();
  };

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(s_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; s++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s_u32(&mma_done[s])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int ks = 0; ks < kStages - 1 && ks < KS; ks++) issue(ks);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t idesc = (1u << 4) | ((256u >> 3) << 17) | ((128u >> 4) << 24);
  bool ok = true;

  for (int ks = 0; ks < KS; ks++) {
    // this thread's copies for step ks have landed (the group count allows the
    // later steps, plus the scale group on the first step, to stay in flight)
    if (ks + kStages - 1 <= KS) cp_wait<kStages - 2>(); else cp_wait<0>();
    __syncthreads();
    // dequant the codes of step ks into B[ks & 1]
    {
      const uint8_t* Cd = sm + kOffCode + (ks % kStages) * kCodeBytes;
      uint8_t* B = sm + kOffB + (ks & 1) * kBBytes;
      const uint16_t* ss = reinterpret_cast<const uint16_t*>(sm + kOffScale);
      const uint16_t* bb = reinterpret_cast<const uint16_t*>(sm + kOffBias);
      for (int wdx = tid; wdx < 256 * 8; wdx += kGThreads) {
        const int r = wdx >> 3, c = wdx & 7;
        const uint32_t w = *reinterpret_cast<const uint32_t*>(Cd + r * 32 + c * 4);
        const __half s = to_half<BF16>(ss[r * NG + ks]);
        const __half b = to_half<BF16>(bb[r * NG + ks]);
        *reinterpret_cast<uint4*>(B + sw128(r, c)) = dequant8(w, __halves2half2(s, s), __halves2half2(b, b));
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t abase = s_u32(sm + kOffA + (ks % kStages) * kABytes);
      const uint32_t bbase = s_u32(sm + kOffB + (ks & 1) * kBBytes);
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const uint64_t da = sdesc(abase + kk * 32);
        const uint64_t db = sdesc(bbase + kk * 32);
        const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(
                tmem),
            "l"(da), "l"(db), "r"(idesc), "r"(accum));
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       s_u32(&mma_done[ks % kStages]))
                   : "memory");
    }
    // MMA(ks-1) must be done before its A stage is refilled (with step
    // ks + kStages - 1) and before B[(ks+1) & 1] is overwritten
    if (ks >= 1) {
      const int pk = ks - 1;
      if (!mbar_wait_p(&mma_done[pk % kStages], (pk / kStages) & 1)) ok = false;
    }
    if (ks + kStages - 1 < KS) issue(ks + kStages - 1);
  }
  // all MMAs complete (in order) once the last one is
  if (!mbar_wait_p(&mma_done[(KS - 1) % kStages], ((KS - 1) / kStages) & 1)) ok = false;
  if (!ok) set_status(a.status, kStatusTimeout);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

  // ---- epilogue: TMEM lane = tile row; warps w and w+4 split the columns
  const int i = (warp & 3) * 32 + lane;
  const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  if (MODE == 0) {
    const int cbeg = (warp >> 2) * 64;
    __half* dst = nullptr;
    if (i < nrows) {
      const int p = row_base + m0 + i;
      dst = shared ? a.act_sh_out + (size_t)p * kInter : a.act_out + (size_t)p * kInter;
    }
    for (int c = cbeg; c < cbeg + 64; c += 16) {
      uint32_t g[16], u[16];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(g[0]), "=r"(g[1]), "=r"(g[2]), "=r"(g[3]), "=r"(g[4]), "=r"(g[5]), "=r"(g[6]), "=r"(g[7]),
            "=r"(g[8]), "=r"(g[9]), "=r"(g[10]), "=r"(g[11]), "=r"(g[12]), "=r"(g[13]), "=r"(g[14]), "=r"(g[15])
          : "r"(lane_addr + c));
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
            "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15])
          : "r"(lane_addr + 128 + c));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (dst) {
        uint32_t h[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float a0 = silu_mul(__uint_as_float(g[2 * j]), __uint_as_float(u[2 * j]));
          const float a1 = silu_mul(__uint_as_float(g[2 * j + 1]), __uint_as_float(u[2 * j + 1]));
          const __half2 hv = __floats2half2_rn(a0, a1);
          h[j] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        uint4* d4 = reinterpret_cast<uint4*>(dst + f0 + c);
        d4[0] = make_uint4(h[0], h[1], h[2], h[3]);
        d4[1] = make_uint4(h[4], h[5], h[6], h[7]);
      }
    }
  } else {
    const int cbeg = (warp >> 2) * 128;
    float* dst = nullptr;
    float wgt = 1.f;
    if (i < nrows) {
      const int p = row_base + m0 + i;
      if (shared) {
        dst = a.y_sh + (size_t)p * kHidden;
      } else {
        const int pos = a.perm[p];
        dst = a.y_pos + (size_t)pos * kHidden;
        wgt = a.w[pos];
      }
    }
    for (int c = cbeg; c < cbeg + 128; c += 16) {
      uint32_t v[16];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(lane_addr + c));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (dst) {
        float4* d4 = reinterpret_cast<float4*>(dst + f0 + c);
#pragma unroll
        for (int j = 0; j < 4; j++)
          d4[j] = make_float4(__fmul_rn(__uint_as_float(v[4 * j]), wgt), __fmul_rn(__uint_as_float(v[4 * j + 1]), wgt),
                              __fmul_rn(__uint_as_float(v[4 * j + 2]), wgt), __fmul_rn(__uint_as_float(v[4 * j + 3]), wgt));
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
}

// out = (residual + sigmoid(c) * shared) + sum_k y_k, the y rows already
// weighted by the routing weight (router order, deltanet.metal:2213-2227)
__global__ void __launch_bounds__(256) k_combine_weighted(int T, const float* __restrict__ residual,
                                                          const float* __restrict__ y_pos,
                                                          const float* __restrict__ y_sh,
                                                          const float* __restrict__ coef,
                                                          float* __restrict__ out) {
  const int t = blockIdx.x;
  const float c = coef[t];
  const float coeff = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-c)));
  for (int r = threadIdx.x; r < kHidden; r += 256) {
    const float sh = __fmul_rn(y_sh[(size_t)t * kHidden + r], coeff);
    float routed = y_pos[(size_t)(t * kTopK) * kHidden + r];
#pragma unroll
    for (int k = 1; k < kTopK; k++) routed = __fadd_rn(routed, y_pos[(size_t)(t * kTopK + k) * kHidden + r]);
    const float base = residual ? residual[(size_t)t * kHidden + r] : 0.f;
    out[(size_t)t * kHidden + r] = __fadd_rn(__fadd_rn(base, sh), routed);
  }
}

}  // namespace

// ------------------------------------------------------------------ host side
static size_t al256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

size_t prefill_workspace_bytes(int T) {
  const size_t P = static_cast<size_t>(T) * kTopK;
  const size_t max_tiles = P / 128 + kExperts + (T + 127) / 128 + 1;
  size_t b = 0;
  b += al256(4 * (size_t)T * kExperts);          // logits
  b += al256(4 * (size_t)T);                     // coef
  b += al256(4 * P) * 2;                         // idx, w
  b += al256(4 * (kExperts + 1)) * 2;            // counts, offsets
  b += al256(4 * P);                             // perm
  b += al256(dispatch_workspace_bytes(T));       // plan scratch
  b += al256(8 * max_tiles) + al256(16);         // tiles, count
  b += al256(2 * P * kInter);                    // routed act (fp16)
  b += al256(2 * (size_t)T * kInter);            // shared act (fp16)
  b += al256(4 * P * kHidden);                   // y per position
  b += al256(4 * (size_t)T * kHidden);           // shared y
  return b;
}

cudaError_t prefill_init_attributes() {
  cudaError_t e;
  e = cudaFuncSetAttribute(k_router_prefill<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRtSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_router_prefill<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRtSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_moe_gemm<false, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_moe_gemm<false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_moe_gemm<true, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_moe_gemm<true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
}

cudaError_t router_logits_prefill(cudaStream_t st, const LayerW& L, bool bf16, int T,
                                  const uint16_t* x, float* logits, float* coef) {
  const int grid = (T + kRtTok - 1) / kRtTok;
  if (bf16)
    k_router_prefill<true><<<grid, kRtThreads, kRtSmem, st>>>(L, T, x, logits, coef);
  else
    k_router_prefill<false><<<grid, kRtThreads, kRtSmem, st>>>(L, T, x, logits, coef);
  return cudaGetLastError();
}

cudaError_t prefill_block(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                          const float* residual, float* out, const RoutingArgs& r, int* idx_out,
                          float* w_out, void* workspace, int* status, Prof* prof) {
  (void)prof;
  const size_t P = static_cast<size_t>(T) * kTopK;
  const size_t max_tiles = P / 128 + kExperts + (T + 127) / 128 + 1;
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
  int2* tiles = reinterpret_cast<int2*>(take(8 * max_tiles));
  int* n_tiles = reinterpret_cast<int*>(take(16));
  __half* act = reinterpret_cast<__half*>(take(2 * P * kInter));
  __half* act_sh = reinterpret_cast<__half*>(take(2 * (size_t)T * kInter));
  float* y_pos = reinterpret_cast<float*>(take(4 * P * kHidden));
  float* y_sh = reinterpret_cast<float*>(take(4 * (size_t)T * kHidden));

  cudaError_t e = router_logits_prefill(st, L, bf16, T, x, logits, coef);
  if (e != cudaSuccess) return e;
  if (r.idx_in) {
    e = cudaMemcpyAsync(idx, r.idx_in, 4 * P, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return e;
    e = cudaMemcpyAsync(w, r.w_in, 4 * P, cudaMemcpyDeviceToDevice, st);
  } else {
    e = router_topk(st, T, logits, r.bias, idx, w, status);
  }
  if (e != cudaSuccess) return e;
  if (idx_out) e = cudaMemcpyAsync(idx_out, idx, 4 * P, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && w_out) e = cudaMemcpyAsync(w_out, w, 4 * P, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return e;
  e = dispatch_plan_ws(st, idx, T, counts, offsets, perm, plan_ws, status);
  if (e != cudaSuccess) return e;
  k_tile_map<<<1, 32, 0, st>>>(counts, T, tiles, n_tiles);

  GemmArgs ga;
  ga.L = L;
  ga.T = T;
  ga.a_routed = reinterpret_cast<const __half*>(x);
  ga.a_shared = reinterpret_cast<const __half*>(x);
  ga.perm = perm;
  ga.offsets = offsets;
  ga.tiles = tiles;
  ga.n_tiles = n_tiles;
  ga.act_out = act;
  ga.act_sh_out = act_sh;
  ga.w = w;
  ga.y_pos = y_pos;
  ga.y_sh = y_sh;
  ga.status = status;
  const dim3 g1((unsigned)max_tiles, kInter / 128);
  if (bf16)
    k_moe_gemm<true, 0><<<g1, kGThreads, kGemmSmem, st>>>(ga);
  else
    k_moe_gemm<false, 0><<<g1, kGThreads, kGemmSmem, st>>>(ga);
  ga.a_routed = act;
  ga.a_shared = act_sh;
  const dim3 g2((unsigned)max_tiles, kHidden / 256);
  if (bf16)
    k_moe_gemm<true, 1><<<g2, kGThreads, kGemmSmem, st>>>(ga);
  else
    k_moe_gemm<false, 1><<<g2, kGThreads, kGemmSmem, st>>>(ga);
  k_combine_weighted<<<T, 256, 0, st>>>(T, residual, y_pos, y_sh, coef, out);
  return cudaGetLastError();
}

}  // namespace qf
