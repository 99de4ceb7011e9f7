// qf_decode.cu -- decode-path MoE block (T = 1..64 tokens) on B200 CUDA cores.
//
// One block = five stream-ordered launches:
//   k_router      Q8 router logits in the reference's lane order + shared-gate
//                 coefficient       (deltanet.metal:2229-2281, :863-902)
//   k_topk_group  top-8 / softmax / renormalise per token (warp shuffles), then
//                 a deterministic grouping of the T*8 routed positions by bank
//                 record (bitonic sort in shared memory)   (deltanet.metal:2283-2329)
//   k_gate_up     SiLU(G x) * (U x) for every (record, 16-row block), weights
//                 read once per record and applied to all tokens routed to it;
//                 the shared expert is one more record with all T tokens
//                                   (deltanet.metal:1985-2076, :2155-2179)
//   k_down        D * act per (record, 64-row block)      (deltanet.metal:2099-2211)
//   k_combine     out = (residual + sigmoid(c) * shared) + sum_k w_k y_k in router
//                 order, optionally followed by the stack's RMSNorm -> fp16
//                                   (deltanet.metal:2213-2227, :18-53)
// Weights stream from HBM with 16-byte (gate/up) and 8-byte (down) vector loads,
// nibbles are unpacked in registers, accumulation is fp32.
#include <math.h>

#include "qf_internal.h"

namespace qf {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTokChunk = 4;  // tokens (positions) staged in shared memory at once

// ---------------------------------------------------------------- workspace
static size_t align256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

size_t decode_workspace_bytes(int T) {
  const size_t P = static_cast<size_t>(T) * kTopK;
  size_t b = 0;
  b += align256(sizeof(float) * T * kExperts);          // logits
  b += align256(sizeof(float) * T);                     // coef
  b += align256(sizeof(int) * P);                       // idx
  b += align256(sizeof(float) * P);                     // w
  b += align256(sizeof(int) * 8);                       // meta
  b += 4 * align256(sizeof(int) * kMaxPositions);       // groups + sorted positions
  b += align256(sizeof(float) * P * kInter);            // act
  b += align256(sizeof(float) * T * kInter);            // act_sh
  b += align256(sizeof(float) * P * kHidden);           // y_part
  b += align256(sizeof(float) * T * kHidden);           // y_sh
  b += 2 * align256(sizeof(float) * T * kHidden);       // h ping-pong
  b += 2 * align256(sizeof(uint16_t) * T * kHidden);    // x16 ping-pong
  return b;
}

void decode_carve(void* base, int T, DecodeWs* ws) {
  char* p = static_cast<char*>(base);
  const size_t P = static_cast<size_t>(T) * kTopK;
  auto take = [&](size_t n) {
    char* r = p;
    p += align256(n);
    return r;
  };
  ws->logits = reinterpret_cast<float*>(take(sizeof(float) * T * kExperts));
  ws->coef = reinterpret_cast<float*>(take(sizeof(float) * T));
  ws->idx = reinterpret_cast<int*>(take(sizeof(int) * P));
  ws->w = reinterpret_cast<float*>(take(sizeof(float) * P));
  ws->meta = reinterpret_cast<int*>(take(sizeof(int) * 8));
  ws->group_rec = reinterpret_cast<int*>(take(sizeof(int) * kMaxPositions));
  ws->group_start = reinterpret_cast<int*>(take(sizeof(int) * kMaxPositions));
  ws->group_cnt = reinterpret_cast<int*>(take(sizeof(int) * kMaxPositions));
  ws->sorted_pos = reinterpret_cast<int*>(take(sizeof(int) * kMaxPositions));
  ws->act = reinterpret_cast<float*>(take(sizeof(float) * P * kInter));
  ws->act_sh = reinterpret_cast<float*>(take(sizeof(float) * T * kInter));
  ws->y_part = reinterpret_cast<float*>(take(sizeof(float) * P * kHidden));
  ws->y_sh = reinterpret_cast<float*>(take(sizeof(float) * T * kHidden));
  ws->h[0] = reinterpret_cast<float*>(take(sizeof(float) * T * kHidden));
  ws->h[1] = reinterpret_cast<float*>(take(sizeof(float) * T * kHidden));
  ws->x16[0] = reinterpret_cast<uint16_t*>(take(sizeof(uint16_t) * T * kHidden));
  ws->x16[1] = reinterpret_cast<uint16_t*>(take(sizeof(uint16_t) * T * kHidden));
}

// ---------------------------------------------------------------- router
constexpr int kRouterRowsPerCta = kWarps;  // one warp per row
constexpr int kRouterRowBlocks = (kExperts + 1 + kRouterRowsPerCta - 1) / kRouterRowsPerCta;
constexpr size_t kRouterSmem =
    sizeof(float) * (static_cast<size_t>(kTokChunk) * kHidden + kTokChunk * 8 * 32);

__device__ __forceinline__ void cvt8(const uint4& v, float4& lo, float4& hi) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
  const float2 a = __half22float2(h[0]);
  const float2 b = __half22float2(h[1]);
  const float2 c = __half22float2(h[2]);
  const float2 d = __half22float2(h[3]);
  lo = make_float4(a.x, a.y, b.x, b.y);
  hi = make_float4(c.x, c.y, d.x, d.y);
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads) k_router(LayerW L, int T,
                                                     const uint16_t* __restrict__ x,
                                                     float* __restrict__ logits,
                                                     float* __restrict__ coef) {
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;                              // [8][2048] plain layout
  float* xsum = smem + kTokChunk * kHidden;      // [8][8 blk][32 lane]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tc = (T + kTokChunk - 1) / kTokChunk;
  const int n_items = kRouterRowBlocks * n_tc;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int rb = item % kRouterRowBlocks;
    const int tc = item / kRouterRowBlocks;
    const int t0 = tc * kTokChunk;
    const int tn = min(kTokChunk, T - t0);
    const int r = rb * kRouterRowsPerCta + warp;
    uint2 wv[8];
    float sc[8], bi[8];
    uint4 cwv[4];
    float cs = 0.f, cb = 0.f;
    if (r < kExperts) {
      const uint8_t* wrow = L.rw + static_cast<size_t>(r) * kHidden;
#pragma unroll
      for (int blk = 0; blk < 8; blk++)
        wv[blk] = __ldg(reinterpret_cast<const uint2*>(wrow + blk * 256 + lane * 8));
#pragma unroll
      for (int blk = 0; blk < 8; blk++) {
        const int g = blk * 4 + (lane >> 3);
        sc[blk] = ld16<BF16>(L.rs + r * 32, g);
        bi[blk] = ld16<BF16>(L.rb + r * 32, g);
      }
    } else if (r == kExperts && coef != nullptr) {
#pragma unroll
      for (int q = 0; q < 4; q++) cwv[q] = __ldg(reinterpret_cast<const uint4*>(L.cw + lane * 64) + q);
      cs = ld16<BF16>(L.cs, lane);
      cb = ld16<BF16>(L.cb, lane);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < tn * (kHidden / 8); i += kThreads) {
      const int t = i / (kHidden / 8), c = i % (kHidden / 8);
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(t0 + t) * kHidden) + c);
      float4 lo, hi;
      cvt8(v, lo, hi);
      float4* dst = reinterpret_cast<float4*>(xs + t * kHidden + c * 8);
      dst[0] = lo;
      dst[1] = hi;
    }
    __syncthreads();
    // sum of the 8 activations each lane sees per block (row independent)
    for (int i = threadIdx.x; i < tn * 256; i += kThreads) {
      const float* e = xs + (i >> 8) * kHidden + ((i >> 5) & 7) * 256 + (i & 31) * 8;
      float s = e[0];
#pragma unroll
      for (int j = 1; j < 8; j++) s = __fadd_rn(s, e[j]);
      xsum[i] = s;
    }
    __syncthreads();
    if (r < kExperts) {
      for (int t = 0; t < tn; t++) {
        float acc = 0.f;
#pragma unroll
        for (int blk = 0; blk < 8; blk++) {
          const float4* e4 = reinterpret_cast<const float4*>(xs + t * kHidden + blk * 256 + lane * 8);
          const float4 a = e4[0], b = e4[1];
          float dot = 0.f;
          dot = __fmaf_rn(byte_f(wv[blk].x, 0), a.x, dot);
          dot = __fmaf_rn(byte_f(wv[blk].x, 1), a.y, dot);
          dot = __fmaf_rn(byte_f(wv[blk].x, 2), a.z, dot);
          dot = __fmaf_rn(byte_f(wv[blk].x, 3), a.w, dot);
          dot = __fmaf_rn(byte_f(wv[blk].y, 0), b.x, dot);
          dot = __fmaf_rn(byte_f(wv[blk].y, 1), b.y, dot);
          dot = __fmaf_rn(byte_f(wv[blk].y, 2), b.z, dot);
          dot = __fmaf_rn(byte_f(wv[blk].y, 3), b.w, dot);
          acc = __fmaf_rn(sc[blk], dot, acc);
          acc = __fmaf_rn(bi[blk], xsum[t * 256 + blk * 32 + lane], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) logits[static_cast<size_t>(t0 + t) * kExperts + r] = acc;
      }
    } else if (r == kExperts && coef != nullptr) {
      // shared-expert gate coefficient: lane owns one 64-column group
      for (int t = 0; t < tn; t++) {
        const float* e = xs + t * kHidden + lane * 64;
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const uint32_t wd[4] = {cwv[q].x, cwv[q].y, cwv[q].z, cwv[q].w};
#pragma unroll
          for (int d = 0; d < 4; d++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const float wq = __fmaf_rn(byte_f(wd[d], k), cs, cb);
              acc = __fmaf_rn(wq, e[q * 16 + d * 4 + k], acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) coef[t0 + t] = acc;
      }
    }
  }
}

__global__ void __launch_bounds__(1024) k_topk(int T, const float* __restrict__ logits,
                                               const float* __restrict__ bias, int* idx, float* w) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp < T) topk_token(warp, logits, bias, idx, w, lane);
}

// top-k (or supplied routing) for all T tokens, then the grouping of the T*8
// positions by bank record: sorted_pos lists positions by (record, position),
// group g covers sorted_pos[group_start[g] .. +group_cnt[g]).
__global__ void __launch_bounds__(1024) k_topk_group(int T, const float* __restrict__ logits,
                                                     RoutingArgs r, uint32_t bank_records,
                                                     DecodeWs ws, int* idx_out, float* w_out,
                                                     int* status) {
  __shared__ uint32_t keys[kMaxPositions];
  __shared__ int warp_cnt[32];
  __shared__ int warp_off[32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = T * kTopK;
  if (r.idx_in) {
    for (int i = tid; i < n; i += blockDim.x) {
      ws.idx[i] = r.idx_in[i];
      ws.w[i] = r.w_in[i];
    }
  } else {
    for (int t = warp; t < T; t += blockDim.x / 32) topk_token(t, logits, r.bias, ws.idx, ws.w, lane);
  }
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    if (idx_out) idx_out[i] = ws.idx[i];
    if (w_out) w_out[i] = ws.w[i];
  }
  if (tid < kMaxPositions) {
    uint32_t key = 0xFFFFFFFFu;
    if (tid < n) {
      int rec = r.rec_of_pos ? r.rec_of_pos[tid] : ws.idx[tid];
      if (rec < 0 || static_cast<uint32_t>(rec) >= bank_records) {
        set_status(status, kStatusDevice);
        rec = 0;
      }
      key = (static_cast<uint32_t>(rec) << 9) | static_cast<uint32_t>(tid);
    }
    keys[tid] = key;
  }
  for (int k = 2; k <= kMaxPositions; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      __syncthreads();
      if (tid < kMaxPositions) {
        const int ixj = tid ^ j;
        if (ixj > tid) {
          const bool up = (tid & k) == 0;
          const uint32_t a = keys[tid], b = keys[ixj];
          if ((a > b) == up) {
            keys[tid] = b;
            keys[ixj] = a;
          }
        }
      }
    }
  }
  __syncthreads();
  bool start = false;
  if (tid < n) start = (tid == 0) || ((keys[tid] >> 9) != (keys[tid - 1] >> 9));
  const unsigned mask = __ballot_sync(0xffffffffu, start);
  if (lane == 0) warp_cnt[warp] = __popc(mask);
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int i = 0; i < 32; i++) {
      warp_off[i] = acc;
      acc += warp_cnt[i];
    }
    ws.meta[0] = acc;
  }
  __syncthreads();
  if (tid < n) {
    ws.sorted_pos[tid] = static_cast<int>(keys[tid] & 511u);
    if (start) {
      const int gid = warp_off[warp] + __popc(mask & ((1u << lane) - 1u));
      ws.group_rec[gid] = static_cast<int>(keys[tid] >> 9);
      ws.group_start[gid] = tid;
    }
  }
  __syncthreads();
  const int ng = warp_off[31] + warp_cnt[31];
  if (tid < ng) ws.group_cnt[tid] = (tid + 1 < ng ? ws.group_start[tid + 1] : n) - ws.group_start[tid];
}

// ---------------------------------------------------------------- gate/up
// Warp = 2 rows of G and the same 2 rows of U ("row-matrices"); lane = 2 x 16
// bytes of each row (64 columns).  Nibbles are unpacked once per 4 columns and
// applied to every token of the staged chunk (up to 8), so a record's weights
// are read and unpacked once however many tokens are routed to it.
constexpr int kGuRowsPerWarp = 2;
constexpr int kGuRowsPerCta = kWarps * kGuRowsPerWarp;  // 16
constexpr int kGuRowBlocks = kInter / kGuRowsPerCta;     // 32
constexpr size_t kGuSmem = sizeof(float) * kTokChunk * kHidden;

// 16-byte chunk q of a 2048-float row -> swizzled chunk so that lane l reading
// chunks l*8 + j (j fixed) hits distinct banks.
__device__ __forceinline__ int swz2048(int q) {
  const int L = q >> 3, j = q & 7;
  return (L << 3) | (j ^ (L & 7));
}
// 16-byte chunk q of a 512-float row; lane l reads chunks 4l + j.
__device__ __forceinline__ int swz512(int q) {
  const int l = q >> 2, j = q & 3;
  return (l << 2) | (j ^ ((l >> 1) & 3));
}

struct GroupRef {
  const uint8_t* base;
  int npos;
  const int* plist;
  bool shared;
};

__device__ __forceinline__ GroupRef group_ref(const LayerW& L, const DecodeWs& ws, int g, int ng,
                                              int T) {
  GroupRef r;
  r.shared = (g == ng);
  if (!r.shared) {
    r.base = L.bank + static_cast<uint64_t>(ws.group_rec[g]) * L.stride;
    r.npos = ws.group_cnt[g];
    r.plist = ws.sorted_pos + ws.group_start[g];
  } else {
    r.base = L.shared;
    r.npos = T;
    r.plist = nullptr;
  }
  return r;
}

template <int RM, int PN>
__device__ __forceinline__ void gu_chunk(const uint4 (&wv)[RM][2], const float (&sc)[RM][2],
                                         const float (&bi)[RM][2], const float4* xs4, int lane,
                                         const int c, float (&acc)[PN][RM]) {
  float dot[PN][RM];
  float xsum[PN];
#pragma unroll
  for (int p = 0; p < PN; p++) {
    xsum[p] = 0.f;
#pragma unroll
    for (int m = 0; m < RM; m++) dot[p][m] = 0.f;
  }
  uint4 w[RM];
#pragma unroll
  for (int m = 0; m < RM; m++) w[m] = c ? wv[m][1] : wv[m][0];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    float q[RM][4];
#pragma unroll
    for (int m = 0; m < RM; m++) {
      const uint32_t wd = word_of(w[m], j >> 1);
#pragma unroll
      for (int e = 0; e < 4; e++) q[m][e] = nib(wd, (j & 1) * 4 + e);
    }
#pragma unroll
    for (int p = 0; p < PN; p++) {
      const float4 xv = xs4[p * 512 + swz2048((c * 32 + lane) * 8 + j)];
      xsum[p] = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(xsum[p], xv.x), xv.y), xv.z), xv.w);
#pragma unroll
      for (int m = 0; m < RM; m++) {
        dot[p][m] = __fmaf_rn(q[m][0], xv.x, dot[p][m]);
        dot[p][m] = __fmaf_rn(q[m][1], xv.y, dot[p][m]);
        dot[p][m] = __fmaf_rn(q[m][2], xv.z, dot[p][m]);
        dot[p][m] = __fmaf_rn(q[m][3], xv.w, dot[p][m]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < RM; m++) {
    const float s = c ? sc[m][1] : sc[m][0];
    const float b = c ? bi[m][1] : bi[m][0];
#pragma unroll
    for (int p = 0; p < PN; p++) {
      acc[p][m] = __fmaf_rn(s, dot[p][m], acc[p][m]);
      acc[p][m] = __fmaf_rn(b, xsum[p], acc[p][m]);
    }
  }
}

template <int RM, int PN>
__device__ __forceinline__ void gu_tokens(const uint4 (&wv)[RM][2], const float (&sc)[RM][2],
                                          const float (&bi)[RM][2], const float4* xs4, int lane,
                                          int pn, int pc, const GroupRef& G, const DecodeWs& ws,
                                          int r0) {
  float acc[PN][RM];
#pragma unroll
  for (int p = 0; p < PN; p++)
#pragma unroll
    for (int m = 0; m < RM; m++) acc[p][m] = 0.f;
  gu_chunk<RM, PN>(wv, sc, bi, xs4, lane, 0, acc);
  gu_chunk<RM, PN>(wv, sc, bi, xs4, lane, 1, acc);
  constexpr int R = RM / 2;
#pragma unroll
  for (int p = 0; p < PN; p++) {
    if (p < pn) {
      float* dst = G.shared ? ws.act_sh + (pc + p) * kInter : ws.act + G.plist[pc + p] * kInter;
#pragma unroll
      for (int rr = 0; rr < R; rr++) {
        const float gsum = warp_sum(acc[p][rr]);
        const float usum = warp_sum(acc[p][R + rr]);
        if (lane == 0) dst[r0 + rr] = silu_mul(gsum, usum);
      }
    }
  }
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads) k_gate_up(LayerW L, int T,
                                                      const uint16_t* __restrict__ x,
                                                      DecodeWs ws, int with_shared) {
  extern __shared__ __align__(16) float smem[];
  float4* xs4 = reinterpret_cast<float4*>(smem);  // [8 tok][512 chunks] swizzled
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int RM = 2 * kGuRowsPerWarp;  // row-matrices per warp: g0, g1, u0, u1
  const int ng = ws.meta[0];
  const int n_items = (ng + with_shared) * kGuRowBlocks;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const GroupRef G = group_ref(L, ws, item / kGuRowBlocks, ng, T);
    const int rb = item % kGuRowBlocks;
    const int r0 = rb * kGuRowsPerCta + warp * kGuRowsPerWarp;
    uint4 wv[RM][2];
    float sc[RM][2], bi[RM][2];
#pragma unroll
    for (int m = 0; m < RM; m++) {
      const int r = r0 + (m % kGuRowsPerWarp);
      const uint32_t offw = m < kGuRowsPerWarp ? kOffGateW : kOffUpW;
#pragma unroll
      for (int c = 0; c < 2; c++)
        wv[m][c] = __ldg(reinterpret_cast<const uint4*>(G.base + offw + r * 1024 + c * 512 + lane * 16));
    }
#pragma unroll
    for (int m = 0; m < RM; m++) {
      const int r = r0 + (m % kGuRowsPerWarp);
      const uint16_t* sp = reinterpret_cast<const uint16_t*>(G.base + (m < kGuRowsPerWarp ? kOffGateS : kOffUpS));
      const uint16_t* bp = reinterpret_cast<const uint16_t*>(G.base + (m < kGuRowsPerWarp ? kOffGateB : kOffUpB));
#pragma unroll
      for (int c = 0; c < 2; c++) {
        const int grp = c * 16 + (lane >> 1);
        sc[m][c] = ld16<BF16>(sp + r * 32, grp);
        bi[m][c] = ld16<BF16>(bp + r * 32, grp);
      }
    }
    for (int pc = 0; pc < G.npos; pc += kTokChunk) {
      const int pn = min(kTokChunk, G.npos - pc);
      __syncthreads();
      for (int i = threadIdx.x; i < pn * (kHidden / 8); i += kThreads) {
        const int p = i / (kHidden / 8), c = i % (kHidden / 8);
        const int tok = G.shared ? (pc + p) : (G.plist[pc + p] / kTopK);
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(tok) * kHidden) + c);
        float4 lo, hi;
        cvt8(v, lo, hi);
        xs4[p * 512 + swz2048(2 * c)] = lo;
        xs4[p * 512 + swz2048(2 * c + 1)] = hi;
      }
      {
        const int pw = pn <= 2 ? pn : kTokChunk;  // width of the specialised body
        for (int i = pn * 512 + threadIdx.x; i < pw * 512; i += kThreads)
          xs4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      __syncthreads();
      if (pn == 1)
        gu_tokens<RM, 1>(wv, sc, bi, xs4, lane, pn, pc, G, ws, r0);
      else if (pn == 2)
        gu_tokens<RM, 2>(wv, sc, bi, xs4, lane, pn, pc, G, ws, r0);
      else
        gu_tokens<RM, 4>(wv, sc, bi, xs4, lane, pn, pc, G, ws, r0);
    }
  }
}

// ---------------------------------------------------------------- down
// Warp = 8 rows of D (K = 512); lane = 8 bytes of each row (16 columns).
constexpr int kDnRowsPerWarp = 8;
constexpr int kDnRowsPerCta = kWarps * kDnRowsPerWarp;  // 64
constexpr int kDnRowBlocks = kHidden / kDnRowsPerCta;    // 32
constexpr size_t kDnSmem = sizeof(float) * kTokChunk * kInter;

template <int PN>
__device__ __forceinline__ void dn_tokens(const uint2 (&dw)[kDnRowsPerWarp],
                                          const float (&ds)[kDnRowsPerWarp],
                                          const float (&db)[kDnRowsPerWarp], const float4* as4,
                                          int lane, int pn, int pc, const GroupRef& G,
                                          const DecodeWs& ws, int r0) {
  float d[PN][kDnRowsPerWarp];
  float xsum[PN];
#pragma unroll
  for (int p = 0; p < PN; p++) {
    xsum[p] = 0.f;
#pragma unroll
    for (int rr = 0; rr < kDnRowsPerWarp; rr++) d[p][rr] = 0.f;
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
    float q[kDnRowsPerWarp][4];
#pragma unroll
    for (int rr = 0; rr < kDnRowsPerWarp; rr++) {
      const uint32_t wd = (j >> 1) ? dw[rr].y : dw[rr].x;
#pragma unroll
      for (int e = 0; e < 4; e++) q[rr][e] = nib(wd, (j & 1) * 4 + e);
    }
#pragma unroll
    for (int p = 0; p < PN; p++) {
      const float4 av = as4[p * 128 + swz512(lane * 4 + j)];
      xsum[p] = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(xsum[p], av.x), av.y), av.z), av.w);
#pragma unroll
      for (int rr = 0; rr < kDnRowsPerWarp; rr++) {
        d[p][rr] = __fmaf_rn(q[rr][0], av.x, d[p][rr]);
        d[p][rr] = __fmaf_rn(q[rr][1], av.y, d[p][rr]);
        d[p][rr] = __fmaf_rn(q[rr][2], av.z, d[p][rr]);
        d[p][rr] = __fmaf_rn(q[rr][3], av.w, d[p][rr]);
      }
    }
  }
#pragma unroll
  for (int p = 0; p < PN; p++) {
    if (p < pn) {
      float* dst = G.shared ? ws.y_sh + (pc + p) * kHidden : ws.y_part + G.plist[pc + p] * kHidden;
#pragma unroll
      for (int rr = 0; rr < kDnRowsPerWarp; rr++) {
        float a = __fmul_rn(ds[rr], d[p][rr]);
        a = __fmaf_rn(db[rr], xsum[p], a);
        a = warp_sum(a);
        if (lane == 0) dst[r0 + rr] = a;
      }
    }
  }
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads) k_down(LayerW L, int T, DecodeWs ws, int with_shared) {
  extern __shared__ __align__(16) float smem[];
  float4* as4 = reinterpret_cast<float4*>(smem);  // [8 pos][128 chunks] swizzled
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = ws.meta[0];
  const int n_items = (ng + with_shared) * kDnRowBlocks;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const GroupRef G = group_ref(L, ws, item / kDnRowBlocks, ng, T);
    const int rb = item % kDnRowBlocks;
    const int r0 = rb * kDnRowsPerCta + warp * kDnRowsPerWarp;
    uint2 dw[kDnRowsPerWarp];
    float ds[kDnRowsPerWarp], db[kDnRowsPerWarp];
#pragma unroll
    for (int rr = 0; rr < kDnRowsPerWarp; rr++)
      dw[rr] = __ldg(reinterpret_cast<const uint2*>(G.base + kOffDownW + (r0 + rr) * 256 + lane * 8));
#pragma unroll
    for (int rr = 0; rr < kDnRowsPerWarp; rr++) {
      ds[rr] = ld16<BF16>(reinterpret_cast<const uint16_t*>(G.base + kOffDownS) + (r0 + rr) * 8, lane >> 2);
      db[rr] = ld16<BF16>(reinterpret_cast<const uint16_t*>(G.base + kOffDownB) + (r0 + rr) * 8, lane >> 2);
    }
    for (int pc = 0; pc < G.npos; pc += kTokChunk) {
      const int pn = min(kTokChunk, G.npos - pc);
      __syncthreads();
      for (int i = threadIdx.x; i < pn * (kInter / 4); i += kThreads) {
        const int p = i / (kInter / 4), q = i % (kInter / 4);
        const float* src = G.shared ? ws.act_sh + (pc + p) * kInter : ws.act + G.plist[pc + p] * kInter;
        as4[p * 128 + swz512(q)] = reinterpret_cast<const float4*>(src)[q];
      }
      {
        const int pw = pn <= 2 ? pn : kTokChunk;
        for (int i = pn * 128 + threadIdx.x; i < pw * 128; i += kThreads)
          as4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      __syncthreads();
      if (pn == 1)
        dn_tokens<1>(dw, ds, db, as4, lane, pn, pc, G, ws, r0);
      else if (pn == 2)
        dn_tokens<2>(dw, ds, db, as4, lane, pn, pc, G, ws, r0);
      else
        dn_tokens<4>(dw, ds, db, as4, lane, pn, pc, G, ws, r0);
    }
  }
}

// ---------------------------------------------------------------- combine (+ RMSNorm)
__global__ void __launch_bounds__(kThreads) k_combine(int T, const float* __restrict__ residual,
                                                      DecodeWs ws, float* __restrict__ out,
                                                      uint16_t* __restrict__ x_next, float eps) {
  __shared__ float o[kHidden];
    const int t = blockIdx.x;
  const float c = ws.coef[t];
  const float coeff = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-c)));
  float w[kTopK];
#pragma unroll
  for (int k = 0; k < kTopK; k++) w[k] = ws.w[t * kTopK + k];
  for (int r = threadIdx.x; r < kHidden; r += kThreads) {
    const float sh = __fmul_rn(ws.y_sh[static_cast<size_t>(t) * kHidden + r], coeff);
    float routed = __fmul_rn(ws.y_part[static_cast<size_t>(t * kTopK) * kHidden + r], w[0]);
#pragma unroll
    for (int k = 1; k < kTopK; k++)
      routed = __fadd_rn(routed, __fmul_rn(ws.y_part[static_cast<size_t>(t * kTopK + k) * kHidden + r], w[k]));
    const float base = residual ? residual[static_cast<size_t>(t) * kHidden + r] : 0.f;
    const float v = __fadd_rn(__fadd_rn(base, sh), routed);
    out[static_cast<size_t>(t) * kHidden + r] = v;
    o[r] = v;
  }
  if (x_next == nullptr) return;
  __syncthreads();
  // RMS over 128 tiles of 16 rows: fma chain inside a tile, tiles summed in order
  __shared__ float tile_ss[kHidden / 16];
  __shared__ float inv_s;
  if (threadIdx.x < kHidden / 16) {
    float acc = 0.f;
    for (int j = 0; j < 16; j++) {
      const float v = o[threadIdx.x * 16 + j];
      acc = __fmaf_rn(v, v, acc);
    }
    tile_ss[threadIdx.x] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.f;
    for (int c = 0; c < kHidden / 16; c++) total = __fadd_rn(total, tile_ss[c]);
    const float mean = __fdiv_rn(total, static_cast<float>(kHidden));
    inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  }
  __syncthreads();
  const float inv = inv_s;
  for (int r = threadIdx.x; r < kHidden; r += kThreads)
    x_next[static_cast<size_t>(t) * kHidden + r] = __half_as_ushort(__float2half_rn(__fmul_rn(o[r], inv)));
}

// ---------------------------------------------------------------- host side
cudaError_t decode_init_attributes() {
  cudaError_t e;
  e = cudaFuncSetAttribute(k_router<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRouterSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_router<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRouterSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_gate_up<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGuSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_gate_up<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGuSmem);
  return e;
}

cudaError_t router_logits(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                          float* logits, float* coef, int* status) {
  (void)status;
  const int items = kRouterRowBlocks * ((T + kTokChunk - 1) / kTokChunk);
  if (bf16)
    k_router<true><<<items, kThreads, kRouterSmem, st>>>(L, T, x, logits, coef);
  else
    k_router<false><<<items, kThreads, kRouterSmem, st>>>(L, T, x, logits, coef);
  return cudaGetLastError();
}

cudaError_t router_topk(cudaStream_t st, int T, const float* logits, const float* bias, int* idx,
                        float* w, int* status) {
  (void)status;
  const int blocks = (T + 31) / 32;
  k_topk<<<blocks, 1024, 0, st>>>(T, logits, bias, idx, w);
  return cudaGetLastError();
}

namespace {
}  // namespace

cudaError_t decode_block(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                         const float* residual, float* out, const RoutingArgs& r, int* idx_out,
                         float* w_out, const DecodeWs& ws, uint16_t* x16_next, float eps,
                         int* status, Prof* prof) {
  cudaError_t e;
  {
    ProfScope ps(prof, kKRouter, st);
    e = router_logits(st, L, bf16, T, x, ws.logits, ws.coef, status);
  }
  if (e != cudaSuccess) return e;
  {
    ProfScope ps(prof, kKTopk, st);
    k_topk_group<<<1, 1024, 0, st>>>(T, ws.logits, r, L.bank_records, ws, idx_out, w_out, status);
  }
  const int max_groups = T * kTopK < kExperts ? T * kTopK : kExperts;
  const int gu_items = (max_groups + 1) * kGuRowBlocks;
  const int dn_items = (max_groups + 1) * kDnRowBlocks;
  const int gu_grid = gu_items < 148 * 3 ? gu_items : 148 * 3;
  const int dn_grid = dn_items < 148 * 4 ? dn_items : 148 * 4;
  {
    ProfScope ps(prof, kKGateUp, st);
    if (bf16)
      k_gate_up<true><<<gu_grid, kThreads, kGuSmem, st>>>(L, T, x, ws, 1);
    else
      k_gate_up<false><<<gu_grid, kThreads, kGuSmem, st>>>(L, T, x, ws, 1);
  }
  {
    ProfScope ps(prof, kKDown, st);
    if (bf16)
      k_down<true><<<dn_grid, kThreads, kDnSmem, st>>>(L, T, ws, 1);
    else
      k_down<false><<<dn_grid, kThreads, kDnSmem, st>>>(L, T, ws, 1);
  }
  {
    ProfScope ps(prof, kKCombine, st);
    k_combine<<<T, kThreads, 0, st>>>(T, residual, ws, out, x16_next, eps);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- subsets
// The streaming runner's split of one token's routed experts into the
// positions whose records are resident (hits) and those still being fetched
// (misses): qwen_cached_moe_gate_up_subset_q4_simd_f32 and
// qwen_cached_moe_down_subset_q4_simd_f32 (deltanet.metal:2155-2211), the
// shared expert with its gate (:2050-2122) and the subset combine (:2213-2227).
// The gate/up and down arithmetic is k_gate_up / k_down's (one group per
// position: the 8 positions of a token name 8 distinct records).

// Plan of a subset of token 0's top-8: group i = positions[i] alone, record
// slot_of_pos[positions[i]].  A position outside [0, 8) or a record outside
// the bank is reported (QF_ERR_DEVICE) and served by record 0.
__global__ void k_subset_plan(const int* __restrict__ slot_of_pos, const int* __restrict__ positions, int n,
                              uint32_t bank_records, DecodeWs ws, int* status) {
  const int i = threadIdx.x;
  if (i == 0) ws.meta[0] = n;
  if (i >= n) return;
  int pos = positions[i];
  if (pos < 0 || pos >= kTopK) {
    set_status(status, kStatusDevice);
    pos = 0;
  }
  int rec = slot_of_pos[pos];
  if (rec < 0 || static_cast<uint32_t>(rec) >= bank_records) {
    set_status(status, kStatusDevice);
    rec = 0;
  }
  ws.group_rec[i] = rec;
  ws.group_start[i] = i;
  ws.group_cnt[i] = 1;
  ws.sorted_pos[i] = pos;
}

// routed_out[r] = sum over i < 8 of (i < n ? y[positions[i]][r] * w[positions[i]] : 0),
// left to right (the reference's eight simdgroup partials, :2197-2210).
__global__ void __launch_bounds__(kThreads) k_subset_sum(const int* __restrict__ positions, int n,
                                                         const float* __restrict__ w, DecodeWs ws,
                                                         float* __restrict__ routed_out) {
  const int r = blockIdx.x * kThreads + threadIdx.x;
  if (r >= kHidden) return;
  float part[kTopK];
#pragma unroll
  for (int i = 0; i < kTopK; i++) {
    part[i] = 0.f;
    if (i < n) {
      const int pos = min(max(positions[i], 0), kTopK - 1);
      part[i] = __fmul_rn(ws.y_part[static_cast<size_t>(pos) * kHidden + r], w[pos]);
    }
  }
  float acc = part[0];
#pragma unroll
  for (int i = 1; i < kTopK; i++) acc = __fadd_rn(acc, part[i]);
  routed_out[r] = acc;
}

// shared_out[t][r] = y_sh[t][r] * (1 / (1 + exp(-coef[t])))   (:2117-2120)
__global__ void __launch_bounds__(kThreads) k_shared_gate(int T, const float* __restrict__ coef, DecodeWs ws,
                                                          float* __restrict__ out) {
  const int t = blockIdx.y, r = blockIdx.x * kThreads + threadIdx.x;
  if (r >= kHidden) return;
  const float coeff = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-coef[t])));
  out[static_cast<size_t>(t) * kHidden + r] = __fmul_rn(ws.y_sh[static_cast<size_t>(t) * kHidden + r], coeff);
}

// out = ((residual + shared) + hit) + miss; a NULL term is 0 (:2213-2227)
__global__ void __launch_bounds__(kThreads) k_combine_subsets(int n, const float* __restrict__ residual,
                                                              const float* __restrict__ shared_out,
                                                              const float* __restrict__ hit,
                                                              const float* __restrict__ miss,
                                                              float* __restrict__ out) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= n) return;
  const float res = residual ? residual[i] : 0.f;
  const float h = hit ? hit[i] : 0.f;
  const float m = miss ? miss[i] : 0.f;
  out[i] = __fadd_rn(__fadd_rn(__fadd_rn(res, shared_out[i]), h), m);
}

cudaError_t routed_subset(cudaStream_t st, const LayerW& L, bool bf16, const uint16_t* x,
                          const int* slot_of_pos, const float* w, const int* positions, int n,
                          float* routed_out, const DecodeWs& ws, int* status) {
  k_subset_plan<<<1, 32, 0, st>>>(slot_of_pos, positions, n, L.bank_records, ws, status);
  if (n > 0) {
    if (bf16) {
      k_gate_up<true><<<n * kGuRowBlocks, kThreads, kGuSmem, st>>>(L, 1, x, ws, 0);
      k_down<true><<<n * kDnRowBlocks, kThreads, kDnSmem, st>>>(L, 1, ws, 0);
    } else {
      k_gate_up<false><<<n * kGuRowBlocks, kThreads, kGuSmem, st>>>(L, 1, x, ws, 0);
      k_down<false><<<n * kDnRowBlocks, kThreads, kDnSmem, st>>>(L, 1, ws, 0);
    }
  }
  k_subset_sum<<<kHidden / kThreads, kThreads, 0, st>>>(positions, n, w, ws, routed_out);
  return cudaGetLastError();
}

cudaError_t shared_expert(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                          const float* coef, float* out, const DecodeWs& ws) {
  // no routed groups: k_gate_up / k_down run only the shared expert's items
  cudaError_t e = cudaMemsetAsync(ws.meta, 0, sizeof(int), st);
  if (e != cudaSuccess) return e;
  if (bf16) {
    k_gate_up<true><<<kGuRowBlocks, kThreads, kGuSmem, st>>>(L, T, x, ws, 1);
    k_down<true><<<kDnRowBlocks, kThreads, kDnSmem, st>>>(L, T, ws, 1);
  } else {
    k_gate_up<false><<<kGuRowBlocks, kThreads, kGuSmem, st>>>(L, T, x, ws, 1);
    k_down<false><<<kDnRowBlocks, kThreads, kDnSmem, st>>>(L, T, ws, 1);
  }
  k_shared_gate<<<dim3(kHidden / kThreads, T), kThreads, 0, st>>>(T, coef, ws, out);
  return cudaGetLastError();
}

cudaError_t combine_subsets(cudaStream_t st, int T, const float* residual, const float* shared_out,
                            const float* hit, const float* miss, float* out) {
  const int n = T * kHidden;
  k_combine_subsets<<<(n + kThreads - 1) / kThreads, kThreads, 0, st>>>(n, residual, shared_out, hit, miss, out);
  return cudaGetLastError();
}

// Post-attention RMSNorm of the residual stream into the block's fp16 input:
// deltanet.metal:18-53 qwen_rmsnorm_f32 as dispatched before the router
// (QwenQ4ActiveExpertStreamingRunner.swift:1169-1176, 64 threads): thread i
// sums v*v over elements i, i+64, ... with an fma chain, the two 32-lane
// groups reduce by xor butterfly, the two partials add, mean = sum / 2048,
// inv = 1 / sqrt(mean + eps) (correctly rounded), x = (h * inv) * w, then fp16.
// One CTA of 64 threads per token.
__global__ void __launch_bounds__(64) k_prenorm_f16(const float* __restrict__ h, const float* __restrict__ w,
                                                    float eps, uint16_t* __restrict__ x16) {
  __shared__ float partial[2];
  __shared__ float inv_s;
  const float* v = h + (size_t)blockIdx.x * kHidden;
  const int lid = threadIdx.x, lane = lid & 31;
  float acc = 0.f;
  for (int i = lid; i < kHidden; i += 64) acc = __fmaf_rn(v[i], v[i], acc);
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
  if (lane == 0) partial[lid >> 5] = acc;
  __syncthreads();
  if (lid == 0) {
    const float s = __fadd_rn(partial[0], partial[1]);
    inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)kHidden), eps)));
  }
  __syncthreads();
  const float inv = inv_s;
  __half* o = reinterpret_cast<__half*>(x16) + (size_t)blockIdx.x * kHidden;
  for (int i = lid; i < kHidden; i += 64) o[i] = __float2half_rn(__fmul_rn(__fmul_rn(v[i], inv), w[i]));
}

cudaError_t prenorm_f16(cudaStream_t st, int T, const float* h, const float* w, float eps, uint16_t* x16) {
  k_prenorm_f16<<<T, 64, 0, st>>>(h, w, eps, x16);
  return cudaGetLastError();
}

}  // namespace qf
