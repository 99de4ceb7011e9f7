// qf_persist.cuh -- device helpers shared by the persistent decode kernels
// (qf_fused.cu: T = 2..8 tokens; qf_fused1.cu: one token): mbarrier and copy
// PTX, the bounded grid barrier, the exact-Q4 mma.sync tile and the warp top-k.
#pragma once

#include <math.h>

#include "qf_internal.h"

namespace qf {
namespace pk {

constexpr unsigned kSpinLimit = 1u << 22;  // bounded waits: a few seconds at most

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// bounded wait for the phase with the given parity to complete
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  for (unsigned spins = 0; spins < kSpinLimit; spins++) {
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
// 16-byte async copy global -> shared (L2 only), and the arrive that fires on
// `bar` once every cp.async issued so far by this thread has landed.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bulk L2 prefetch; needs a 16-byte aligned address and a multiple-of-16 size.
__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes) {
  if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0 || (bytes & 15u) != 0) return;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
// Orders this thread's earlier shared-memory accesses before the asynchronous
// copies it issues next into the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier: one monotonically increasing arrival counter (zeroed before the
// launch); arrival is a release reduction, the wait an acquire poll.  Bounded:
// on expiry the status word gets QF_ERR_TIMEOUT and the CTA leaves the kernel
// (the others then expire too).
__device__ __forceinline__ bool grid_sync(unsigned* count, unsigned& epoch, int* status, int* fail) {
  __syncthreads();
  if (threadIdx.x == 0) {
    epoch++;
    red_release_add(count, 1u);
    const unsigned target = gridDim.x * epoch;
    unsigned spins = 0;
    while (ld_acquire(count) < target) {
      if (++spins > kSpinLimit) {
        set_status(status, kStatusTimeout);
        *fail = 1;
        break;
      }
      if (spins > 64) __nanosleep(20);
    }
  }
  __syncthreads();
  return *fail == 0;
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// two nibbles of a word as fp16 halves 1024+q (j even) or 1024+16q (j odd)
__device__ __forceinline__ uint32_t pairsel(uint32_t w, int j) {
  const uint32_t v = (j >= 2) ? (w >> 8) : w;
  const uint32_t mask = (j & 1) ? 0x00F000F0u : 0x000F000Fu;
  return (v & mask) | 0x64006400u;
}

// Half index of element e (0..63 of a 64-column group) inside the 32-byte
// fragment chunk of its thread-slot t = e/16.
__device__ __forceinline__ int frag_half(int e) {
  const int w2 = (e & 15) >> 3, k = e & 7, j = k & 3, hi = k >> 2;
  return (j * 2 + w2) * 2 + hi;
}

// Stage nvec activation vectors (ngrp groups of 64 values each) as MMA B
// fragments: item = (vector, group, eighth); each thread handles 8 values
// (two float4 loads, all issued before any use), 8 consecutive lanes reduce S
// and C for their group.  Vector v goes to fragment column v.
template <bool kHalfSrc, int NT>
__device__ __forceinline__ void stage_block(const void* src, int nvec, int ngrp, size_t vec_stride,
                                            int ncols, __half* frag, float* S, float* C) {
  const int items = nvec * ngrp * 8;
  for (int base = 0; base < items; base += 2 * NT) {
    float vals[2][8];
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int item = base + u * NT + threadIdx.x;
      if (item < items) {
        const int v = item / (ngrp * 8), g = (item >> 3) % ngrp, q = item & 7;
        const size_t off = v * vec_stride + g * 64 + q * 8;
        if constexpr (kHalfSrc) {
          const uint4 hv = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(src) + off);
          const __half2* h2 = reinterpret_cast<const __half2*>(&hv);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const float2 f = __half22float2(h2[j]);
            vals[u][2 * j] = f.x;
            vals[u][2 * j + 1] = f.y;
          }
        } else {
          const float4 a = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + off));
          const float4 b = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + off + 4));
          vals[u][0] = a.x; vals[u][1] = a.y; vals[u][2] = a.z; vals[u][3] = a.w;
          vals[u][4] = b.x; vals[u][5] = b.y; vals[u][6] = b.z; vals[u][7] = b.w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int item0 = base + u * NT;
      if (item0 >= items) break;  // uniform across the CTA
      const int item = item0 + threadIdx.x;
      float s_part = 0.f, c_part = 0.f;
      int v = 0, g = 0;
      if (item < items) {
        v = item / (ngrp * 8);
        g = (item >> 3) % ngrp;
        const int q = item & 7;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const int e = q * 8 + j;
          const __half xh = __float2half_rn(vals[u][j]);
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
}

// One warp: a 16-row tile x NG groups (starting at grp0) of a Q4 matrix held in
// shared memory (rows at `pitch` bytes; scales/biases s, b as [16][sgroups]
// halves), against up to 8 activation columns (cols[s] = fragment column of
// slot s, or -1).  acc: rows (g, g+8) x slots (2t, 2t+1).
template <bool BF16, int NG>
__device__ __forceinline__ void mma_tile_smem(const uint8_t* rows, int pitch, int grp0,
                                              const uint16_t* s, const uint16_t* b, int sgroups,
                                              const __half* frag, const float* S, const float* C,
                                              int ncols, const int* cols, float (&acc)[4],
                                              int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int colb = cols[g];
  const int c0 = cols[2 * t], c1 = cols[2 * t + 1];
#pragma unroll
  for (int i = 0; i < NG; i++) {
    const int grp = grp0 + i;
    const uint2 wa = *reinterpret_cast<const uint2*>(rows + g * pitch + grp * 32 + 8 * t);
    const uint2 wb = *reinterpret_cast<const uint2*>(rows + (g + 8) * pitch + grp * 32 + 8 * t);
    float sa, ba, sb, bb;
    if constexpr (BF16) {
      sa = __uint_as_float((uint32_t)s[g * sgroups + grp] << 16);
      ba = __uint_as_float((uint32_t)b[g * sgroups + grp] << 16);
      sb = __uint_as_float((uint32_t)s[(g + 8) * sgroups + grp] << 16);
      bb = __uint_as_float((uint32_t)b[(g + 8) * sgroups + grp] << 16);
    } else {
      sa = __half2float(__ushort_as_half(s[g * sgroups + grp]));
      ba = __half2float(__ushort_as_half(b[g * sgroups + grp]));
      sb = __half2float(__ushort_as_half(s[(g + 8) * sgroups + grp]));
      bb = __half2float(__ushort_as_half(b[(g + 8) * sgroups + grp]));
    }
    uint4 bf0 = make_uint4(0, 0, 0, 0), bf1 = make_uint4(0, 0, 0, 0);
    if (colb >= 0) {
      const uint4* p = reinterpret_cast<const uint4*>(frag + (((size_t)grp * ncols + colb) * 4 + t) * 16);
      bf0 = p[0];
      bf1 = p[1];
    }
    const uint32_t bw[8] = {bf0.x, bf0.y, bf0.z, bf0.w, bf1.x, bf1.y, bf1.z, bf1.w};
    float tmp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      uint32_t a[4];
      a[0] = pairsel(wa.x, j);
      a[1] = pairsel(wb.x, j);
      a[2] = pairsel(wa.y, j);
      a[3] = pairsel(wb.y, j);
      mma16816(tmp, a, bw[2 * j], bw[2 * j + 1]);
    }
    const float S0 = c0 >= 0 ? S[grp * ncols + c0] : 0.f;
    const float C0 = c0 >= 0 ? C[grp * ncols + c0] : 0.f;
    const float S1 = c1 >= 0 ? S[grp * ncols + c1] : 0.f;
    const float C1 = c1 >= 0 ? C[grp * ncols + c1] : 0.f;
    acc[0] = __fmaf_rn(sa, tmp[0] - C0, __fmaf_rn(ba, S0, acc[0]));
    acc[1] = __fmaf_rn(sa, tmp[1] - C1, __fmaf_rn(ba, S1, acc[1]));
    acc[2] = __fmaf_rn(sb, tmp[2] - C0, __fmaf_rn(bb, S0, acc[2]));
    acc[3] = __fmaf_rn(sb, tmp[3] - C1, __fmaf_rn(bb, S1, acc[3]));
  }
}


// top-k of token `t` by one warp: 8 rounds of (max value, then min index among
// the lanes holding it) with warp reductions; orders ties like the reference's
// strict-> insertion scan (deltanet.metal:2283-2329).  Split in two halves so
// that the weights (needed only by the combine) are computed off the critical
// path.
__device__ __forceinline__ uint32_t f2ord(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}
// Selection half: idx_out[t*8+k] and the selected (biased) logits sel_out[t*8+k];
// the 256 biased logits go to vs[256] for the weights half.
__device__ __forceinline__ void topk_select(const float* logits, const float* bias, int t, int lane, int* idx_out,
                            float* sel_out, float* vs) {
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int e = j * 32 + lane;
    const float lg = __ldcg(logits + t * kExperts + e);
    v[j] = bias ? __fadd_rn(lg, __ldg(bias + e)) : lg;
    vs[e] = v[j];
  }
  unsigned taken = 0;
  float selv[kTopK];
  int seli[kTopK];
#pragma unroll
  for (int k = 0; k < kTopK; k++) {
    uint32_t best = 0;
    int bj = 0;
#pragma unroll
    for (int j = 7; j >= 0; j--) {  // ties within a lane: lower j (lower expert id) wins
      const uint32_t o = ((taken >> j) & 1u) ? 0u : f2ord(v[j]);
      if (o >= best) {
        best = o;
        bj = j;
      }
    }
    const uint32_t mx = __reduce_max_sync(0xffffffffu, best);
    const uint32_t cand = (best == mx) ? (uint32_t)(bj * 32 + lane) : 0xffffffffu;
    const uint32_t win = __reduce_min_sync(0xffffffffu, cand);
    if ((int)(win & 31) == lane) taken |= 1u << (win >> 5);
    selv[k] = ord2f(mx);
    seli[k] = (int)win;
  }
#pragma unroll
  for (int k = 0; k < kTopK; k++)
    if (lane == k) {
      idx_out[t * kTopK + k] = seli[k];
      sel_out[t * kTopK + k] = selv[k];
    }
}

// Weights half: softmax over all 256 (biased) logits, renormalised over the
// selected 8 (deltanet.metal:2283-2329); w[t*8+k] holds the selected logit on
// entry and the weight on exit.
__device__ __forceinline__ void topk_weights(const float* vs, int t, int lane, float* w) {
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] = vs[j * 32 + lane];
  float selv[kTopK];
#pragma unroll
  for (int k = 0; k < kTopK; k++) selv[k] = w[t * kTopK + k];
  __syncwarp();
  const float mxv = selv[0];
  float den = 0.f;
#pragma unroll
  for (int j = 0; j < 8; j++) den = __fadd_rn(den, expf(__fsub_rn(v[j], mxv)));
  den = warp_sum(den);
  float p[kTopK];
  float ps = 0.f;
#pragma unroll
  for (int k = 0; k < kTopK; k++) {
    p[k] = __fdiv_rn(expf(__fsub_rn(selv[k], mxv)), den);
    ps = __fadd_rn(ps, p[k]);
  }
#pragma unroll
  for (int k = 0; k < kTopK; k++)
    if (lane == k) w[t * kTopK + k] = __fdiv_rn(p[k], ps);
}


}  // namespace pk
}  // namespace qf
