// qf_lmhead.cu -- Q4 LM-head GEMV: logits of the 248,320-row vocabulary for
// one fp32 token row, bit for bit in the reference's order.
//
// Reference: deltanet.metal:1897-1919 qwen_gemv_q4_affine_simd_f32 over
// qwen_q4_row_simd_f32 (:1838-1895), dispatched for the LM head at
// QwenQ4ActiveExpertStreamingRunner.swift:1393-1400.  A row is 2,048 Q4
// codes (1,024 bytes) + 32 scales + 32 biases (16-bit); one 32-lane group per
// row; lane l takes bytes [blk*128 + 4l, +4) of the 8 blocks of 128 bytes,
// i.e. elements blk*256 + 8l .. +7 of group blk*4 + l/8; per block
// dot = fma chain over the 8 products, sum = e0 + .. + e7 (left to right),
// acc = fma(scale, dot, acc), acc = fma(bias, sum, acc); then the 32 lane
// accumulators are summed (xor butterfly 16, 8, 4, 2, 1, the order the CPU
// oracle restates simd_sum in).
//
// B200 mapping.  HBM-bound: 1,152 bytes per row (286 MB per token).
//   - x is row-independent: each lane holds its 64 activations in registers
//     (the odd element of each byte pre-divided by 16, see below) and the 8
//     block sums, computed once per warp.
//   - Nibble -> float, exactly, without conversion instructions: one PRMT
//     builds the float 2^23 + byte, one LOP3 clears the high nibble
//     (2^23 + lo); (2^23 + lo) - 2^23 = lo and (2^23 + byte) - (2^23 + lo) =
//     16 hi, both exact.  16 hi times x/16 is exactly hi times x, so the fma
//     chain rounds as the reference's.
//   - Blackwell's packed fp32 instructions (fma.rn.f32x2 / add.rn.f32x2, each
//     half rounded as a scalar fma/add) run two independent dot chains at
//     once: blocks 2p and 2p+1 of the same row.
//   - Rows stream through a per-warp shared-memory ring of 4 stages filled
//     by cp.async (16-byte pieces, no registers held): 4 rows in flight per
//     warp; each lane then reads its code words from the stage without bank
//     conflicts (word blk*32 + lane).  A warp reduces two rows per iteration
//     (8 independent chains), 128 registers, 4 blocks of 4 warps per SM.

#include <cuda_fp16.h>
#include <stdint.h>

#include "qf_internal.h"

namespace qf {
namespace {

constexpr int kLmThreads = 128;
constexpr int kLmBlocksPerSm = 4;

__device__ __forceinline__ uint64_t pk(float a, float b) {
  return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}
__device__ __forceinline__ float lo32(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi32(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <bool BF16>
__device__ __forceinline__ float s16(uint16_t u) {
  if constexpr (BF16) {
    return __uint_as_float((uint32_t)u << 16);
  } else {
    return __half2float(__ushort_as_half(u));
  }
}

constexpr int kLmStages = 4;                  // rows in flight per warp
constexpr int kLmStageBytes = 1024 + 64 + 64;  // codes | scales | biases of one row
constexpr int kLmWarps = kLmThreads / 32;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// one row into a stage: 1,024 bytes of codes (two 16-byte pieces per lane),
// scales and biases (lanes 0-7); an empty group when the row is past the end
__device__ __forceinline__ void issue_row(uint8_t* stage, const uint8_t* __restrict__ w,
                                          const uint8_t* __restrict__ s, const uint8_t* __restrict__ b, int r,
                                          int rows, int lane) {
  if (r < rows) {
    const uint8_t* wr = w + (size_t)r * 1024;
    cp_async16(stage + 16 * lane, wr + 16 * lane);
    cp_async16(stage + 512 + 16 * lane, wr + 512 + 16 * lane);
    if (lane < 4) cp_async16(stage + 1024 + 16 * lane, s + (size_t)r * 64 + 16 * lane);
    else if (lane < 8) cp_async16(stage + 1088 + 16 * (lane - 4), b + (size_t)r * 64 + 16 * (lane - 4));
  }
  cp_commit();
}

template <bool BF16>
__global__ void __launch_bounds__(kLmThreads) k_lm_head(const uint8_t* __restrict__ w,
                                                        const uint8_t* __restrict__ s,
                                                        const uint8_t* __restrict__ b, int rows,
                                                        const float* __restrict__ x, float* __restrict__ out) {
  __shared__ __align__(16) uint8_t ring[kLmWarps][kLmStages][kLmStageBytes];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int nwarps = gridDim.x * kLmWarps;
  const int r0 = blockIdx.x * kLmWarps + wib;
  // rows r0 + i * nwarps, i = 0, 1, ...: the first kLmStages are requested
  // before the activations are read
#pragma unroll
  for (int i = 0; i < kLmStages; i++) issue_row(ring[wib][i], w, s, b, r0 + i * nwarps, rows, lane);
  // activations of this lane, block pairs (2p, 2p+1) packed: ev[p][j] =
  // (x of byte j's low nibble in block 2p, the same in block 2p+1), od[p][j]
  // the high nibbles' x / 16
  uint64_t ev[4][4], od[4][4];
  float esum[8];
#pragma unroll
  for (int p = 0; p < 4; p++) {
    float v[2][8];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const float4* xp = reinterpret_cast<const float4*>(x + (2 * p + h) * 256 + 8 * lane);
      const float4 a = __ldg(xp), c = __ldg(xp + 1);
      v[h][0] = a.x, v[h][1] = a.y, v[h][2] = a.z, v[h][3] = a.w;
      v[h][4] = c.x, v[h][5] = c.y, v[h][6] = c.z, v[h][7] = c.w;
      float sum = v[h][0];
#pragma unroll
      for (int i = 1; i < 8; i++) sum = __fadd_rn(sum, v[h][i]);
      esum[2 * p + h] = sum;
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
      ev[p][j] = pk(v[0][2 * j], v[1][2 * j]);
      od[p][j] = pk(__fmul_rn(v[0][2 * j + 1], 0.0625f), __fmul_rn(v[1][2 * j + 1], 0.0625f));
    }
  }
  const uint64_t neg_magic = pk(-8388608.0f, -8388608.0f);
  const uint64_t minus1 = pk(-1.0f, -1.0f);
  // two rows per iteration (stages 2k and 2k+1 of the ring): twice the
  // independent chains per warp
  int stage = 0;
  for (int r = r0; r < rows; r += 2 * nwarps) {
    const int r2 = r + nwarps;
    cp_wait<kLmStages - 2>();
    __syncwarp();
    uint32_t c[2][8];
    float sl[2], bl[2];
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const uint8_t* st = ring[wib][stage + q];
      const uint32_t* cw = reinterpret_cast<const uint32_t*>(st);
#pragma unroll
      for (int blk = 0; blk < 8; blk++) c[q][blk] = cw[blk * 32 + lane];
      sl[q] = s16<BF16>(reinterpret_cast<const uint16_t*>(st + 1024)[lane]);
      bl[q] = s16<BF16>(reinterpret_cast<const uint16_t*>(st + 1088)[lane]);
    }
    __syncwarp();
    issue_row(ring[wib][stage], w, s, b, r + kLmStages * nwarps, rows, lane);
    issue_row(ring[wib][stage + 1], w, s, b, r2 + kLmStages * nwarps, rows, lane);
    stage = stage + 2 == kLmStages ? 0 : stage + 2;
    float acc[2] = {0.0f, 0.0f};
#pragma unroll
    for (int p = 0; p < 4; p++) {
      uint64_t dot[2] = {0, 0};  // (+0, +0)
#pragma unroll
      for (int j = 0; j < 4; j++) {
#pragma unroll
        for (int q = 0; q < 2; q++) {
          const uint32_t a0 = __byte_perm(c[q][2 * p], 0x4B000000u, 0x7540u | j);
          const uint32_t a1 = __byte_perm(c[q][2 * p + 1], 0x4B000000u, 0x7540u | j);
          const uint64_t A = (uint64_t)a0 | ((uint64_t)a1 << 32);
          const uint64_t L = A & 0xFFFFFF0FFFFFFF0Full;
          const uint64_t lo = add2(L, neg_magic);
          const uint64_t hi16 = fma2(L, minus1, A);
          dot[q] = fma2(lo, ev[p][j], dot[q]);
          dot[q] = fma2(hi16, od[p][j], dot[q]);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int blk = 2 * p + h;
        const int g = blk * 4 + (lane >> 3);
#pragma unroll
        for (int q = 0; q < 2; q++) {
          const float sc = __shfl_sync(0xffffffffu, sl[q], g);
          const float bi = __shfl_sync(0xffffffffu, bl[q], g);
          acc[q] = __fmaf_rn(sc, h ? hi32(dot[q]) : lo32(dot[q]), acc[q]);
          acc[q] = __fmaf_rn(bi, esum[blk], acc[q]);
        }
      }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      acc[0] = __fadd_rn(acc[0], __shfl_xor_sync(0xffffffffu, acc[0], m));
      acc[1] = __fadd_rn(acc[1], __shfl_xor_sync(0xffffffffu, acc[1], m));
    }
    if (lane == 0) {
      out[r] = acc[0];
      if (r2 < rows) out[r2] = acc[1];
    }
  }
  cp_wait<0>();  // no copy in flight when the warp exits
}

}  // namespace

cudaError_t lm_head_q4(cudaStream_t st, bool bf16, const void* w, const void* s, const void* b, int rows,
                       const float* x, float* out, int sms) {
  const unsigned grid = (unsigned)(sms * kLmBlocksPerSm);
  if (bf16)
    k_lm_head<true><<<grid, kLmThreads, 0, st>>>(static_cast<const uint8_t*>(w), static_cast<const uint8_t*>(s),
                                                 static_cast<const uint8_t*>(b), rows, x, out);
  else
    k_lm_head<false><<<grid, kLmThreads, 0, st>>>(static_cast<const uint8_t*>(w), static_cast<const uint8_t*>(s),
                                                  static_cast<const uint8_t*>(b), rows, x, out);
  return cudaGetLastError();
}

}  // namespace qf
