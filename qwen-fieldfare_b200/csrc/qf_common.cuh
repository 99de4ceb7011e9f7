// qf_common.cuh -- geometry, record layout and small device helpers shared by
// the MoE-block kernels.  Geometry is the Qwen3.6-35B-A3B MoE block used by
// tanishqpatil/qwen-fieldfare (hidden 2048, 256 experts, top-8, intermediate
// 512, Q4/Q8 MLX affine with 64-column groups).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace qf {

constexpr int kHidden = 2048;
constexpr int kExperts = 256;
constexpr int kTopK = 8;
constexpr int kInter = 512;
constexpr int kGroup = 64;
constexpr int kSharedExpert = 256;  // expert id of the shared expert in generators
constexpr uint64_t kRecordBytes = 1769472ull;

// Byte offsets inside one expert record: the slot layout of the reference's
// expert arena (QwenQ4ExpertStoreBuilder.swift:47-56, deltanet.metal:2155-2211).
constexpr uint32_t kOffGateW = 0u;
constexpr uint32_t kOffGateS = 524288u;
constexpr uint32_t kOffGateB = 557056u;
constexpr uint32_t kOffUpW = 589824u;
constexpr uint32_t kOffUpS = 1114112u;
constexpr uint32_t kOffUpB = 1146880u;
constexpr uint32_t kOffDownW = 1179648u;
constexpr uint32_t kOffDownS = 1703936u;
constexpr uint32_t kOffDownB = 1736704u;

// Decode path limits: T tokens, T*8 routed positions.
constexpr int kDecodeMaxTokens = 64;
constexpr int kMaxPositions = kDecodeMaxTokens * kTopK;  // 512

// Device status word values (mirrors qf_status).
constexpr int kStatusOk = 0;
constexpr int kStatusDevice = -7;
constexpr int kStatusTimeout = -6;

struct LayerW {
  const uint8_t* rw;
  const uint16_t* rs;
  const uint16_t* rb;
  const uint8_t* cw;
  const uint16_t* cs;
  const uint16_t* cb;
  const uint8_t* shared;
  const uint8_t* bank;
  uint64_t stride;
  uint32_t bank_records;
};

template <bool BF16>
__device__ __forceinline__ float ld16(const uint16_t* p, int i) {
  const uint16_t u = __ldg(p + i);
  if constexpr (BF16) {
    return __uint_as_float(static_cast<uint32_t>(u) << 16);
  } else {
    return __half2float(__ushort_as_half(u));
  }
}

// xor-butterfly simd_sum (16, 8, 4, 2, 1): every lane ends with the same value,
// and the order is the one the CPU oracle reproduces.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// q (0..15) of nibble k of a packed word, as an exact float.
__device__ __forceinline__ float nib(uint32_t w, int k) {
  return __uint_as_float(0x4B000000u | ((w >> (4 * k)) & 0xFu)) - 8388608.0f;
}
// byte k of a packed word, as an exact float.
__device__ __forceinline__ float byte_f(uint32_t w, int k) {
  return __uint_as_float(0x4B000000u | ((w >> (8 * k)) & 0xFFu)) - 8388608.0f;
}

// word d (compile-time after unrolling) of a 16-byte vector, without taking
// the vector's address (which would force it into local memory).
__device__ __forceinline__ uint32_t word_of(const uint4& v, int d) {
  return d == 0 ? v.x : (d == 1 ? v.y : (d == 2 ? v.z : v.w));
}

// fp16 (x0..x7) -> (x0,x4,x1,x5,x2,x6,x3,x7): the K order of the grouped GEMM
// operands (the Q4 dequant then needs no byte permutes)
__device__ __forceinline__ uint4 permute8(uint4 v) {
  return make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.x, v.z, 0x7632), __byte_perm(v.y, v.w, 0x5410),
                    __byte_perm(v.y, v.w, 0x7632));
}

__device__ __forceinline__ void set_status(int* status, int code) {
  if (status) atomicCAS(status, kStatusOk, code);
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  // SiLU(g) * u as in deltanet.metal:4-6 (x / (1 + e^-x)); expf is CUDA's.
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// ---------------------------------------------------------------- top-k
// Warp-parallel selection of the top-8 logits of one token: 8 rounds of a
// (value desc, index asc) warp argmax, which orders ties exactly like the
// reference's strict-> insertion scan.
__device__ __forceinline__ void topk_token(int t, const float* __restrict__ logits,
                                           const float* __restrict__ bias, int* __restrict__ idx,
                                           float* __restrict__ w, int lane) {
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int e = j * 32 + lane;
    const float l = logits[static_cast<size_t>(t) * kExperts + e];
    v[j] = bias ? __fadd_rn(l, bias[e]) : l;
  }
  unsigned taken = 0;
  float selv[kTopK];
  int seli[kTopK];
#pragma unroll
  for (int k = 0; k < kTopK; k++) {
    float bv = -INFINITY;
    int bix = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int e = j * 32 + lane;
      if (!((taken >> j) & 1u) && (v[j] > bv || (v[j] == bv && e < bix))) {
        bv = v[j];
        bix = e;
      }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bix, m);
      if (ov > bv || (ov == bv && oi < bix)) {
        bv = ov;
        bix = oi;
      }
    }
    selv[k] = bv;
    seli[k] = bix;
    if ((bix & 31) == lane) taken |= 1u << (bix >> 5);
  }
  const float mx = selv[0];
  float den = 0.f;
#pragma unroll
  for (int j = 0; j < 8; j++) den = __fadd_rn(den, expf(__fsub_rn(v[j], mx)));
  den = warp_sum(den);
  float p[kTopK];
  float ps = 0.f;
#pragma unroll
  for (int k = 0; k < kTopK; k++) {
    p[k] = __fdiv_rn(expf(__fsub_rn(selv[k], mx)), den);
    ps = __fadd_rn(ps, p[k]);
  }
#pragma unroll
  for (int k = 0; k < kTopK; k++) {
    if (lane == k) {
      idx[t * kTopK + k] = seli[k];
      w[t * kTopK + k] = __fdiv_rn(p[k], ps);
    }
  }
}

// Exclusive prefix sum of v over threads 0..255 of the block (threads past 255
// pass 0 and get their own running prefix, which callers ignore); *total is
// the sum over the 256.  Every thread of the block calls it (it contains a
// barrier); s_warp: 8 ints of shared memory, free again after the next
// barrier.
__device__ __forceinline__ int block_scan256(int v, int* s_warp, int* total) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int incl = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += o;
  }
  if (tid < 256 && lane == 31) s_warp[warp] = incl;
  __syncthreads();
  int before = 0, tot = 0;
#pragma unroll
  for (int q = 0; q < 8; q++) {
    const int sw = s_warp[q];
    if (q < warp) before += sw;
    tot += sw;
  }
  *total = tot;
  return before + incl - v;
}

}  // namespace qf
