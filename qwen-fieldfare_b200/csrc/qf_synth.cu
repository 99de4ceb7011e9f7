// qf_synth.cu -- seeded synthetic MoE weights generated directly in HBM.
//
// Counter-based SplitMix64 streams keyed by (seed, layer, tensor tag, index),
// so any record can be produced by any thread without sequential state.
// Codes are raw random bytes (Q4: uniform nibbles, packed 8 per uint32, low
// nibble first; Q8: uniform bytes).  Scales are |N(0,1)|*0.01 + 1e-3 with the
// normal drawn as Irwin-Hall(12) of 16-bit uniforms: every step is integer or
// a single correctly rounded fp32 operation, so the CPU generator of the test
// oracle produces the same bytes.  Biases are -8*scale (Q4) / -128*scale (Q8);
// Q8 scales are additionally multiplied by 1/16 so router logits stay O(1).
#include <math.h>
#include <string.h>

#include "qf_common.cuh"
#include "qf_internal.h"

namespace qf {

enum : uint32_t {
  TAG_GATE_W = 1,
  TAG_GATE_S = 2,
  TAG_UP_W = 3,
  TAG_UP_S = 4,
  TAG_DOWN_W = 5,
  TAG_DOWN_S = 6,
  TAG_ROUTER_W = 7,
  TAG_ROUTER_S = 8,
  TAG_COEF_W = 9,
  TAG_COEF_S = 10,
  TAG_HIDDEN = 11
};
constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint32_t layer,
                                                        uint32_t tag, uint32_t index) {
  uint64_t k = mix64(seed + kGamma);
  k = mix64(k ^ ((static_cast<uint64_t>(layer) + 1ull) * kGamma));
  k = mix64(k ^ ((static_cast<uint64_t>(tag) << 32) | index));
  return k;
}
__host__ __device__ __forceinline__ uint64_t draw(uint64_t key, uint64_t i) {
  return mix64(key + (i + 1ull) * kGamma);
}
__host__ __device__ __forceinline__ int32_t irwin_hall_sum(uint64_t key, uint64_t g) {
  int32_t s = 0;
  for (int d = 0; d < 3; d++) {
    const uint64_t r = draw(key, 3ull * g + static_cast<uint64_t>(d));
    for (int j = 0; j < 4; j++) s += static_cast<int32_t>((r >> (16 * j)) & 0xFFFFu);
  }
  return s - 393210;
}

// One thread per 8 code bytes.
__global__ void k_synth_codes(uint64_t key_base_seed, uint32_t layer, uint32_t tag,
                              uint32_t expert0, uint32_t count, uint8_t* dst0, uint64_t stride,
                              uint32_t tensor_bytes) {
  const uint32_t words = tensor_bytes / 8u;
  const uint64_t total = static_cast<uint64_t>(words) * count;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t e = static_cast<uint32_t>(i / words);
    const uint32_t j = static_cast<uint32_t>(i % words);
    const uint64_t key = stream_key(key_base_seed, layer, tag, expert0 + e);
    const uint64_t r = draw(key, j);
    *reinterpret_cast<uint64_t*>(dst0 + e * stride + static_cast<uint64_t>(j) * 8u) = r;
  }
}

template <bool BF16>
__device__ __forceinline__ uint16_t round16(float f) {
  if constexpr (BF16) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  } else {
    return __half_as_ushort(__float2half_rn(f));
  }
}
template <bool BF16>
__device__ __forceinline__ float widen16(uint16_t u) {
  if constexpr (BF16) {
    return __uint_as_float(static_cast<uint32_t>(u) << 16);
  } else {
    return __half2float(__ushort_as_half(u));
  }
}

// One thread per 64-column group: scale and bias.
template <bool BF16>
__global__ void k_synth_scales(uint64_t seed, uint32_t layer, uint32_t tag, uint32_t expert0,
                               uint32_t count, uint8_t* s0, uint8_t* b0, uint64_t stride,
                               uint32_t ngroups, float mult, float bias_mult) {
  const uint64_t total = static_cast<uint64_t>(ngroups) * count;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t e = static_cast<uint32_t>(i / ngroups);
    const uint32_t g = static_cast<uint32_t>(i % ngroups);
    const uint64_t key = stream_key(seed, layer, tag, expert0 + e);
    const float z = static_cast<float>(irwin_hall_sum(key, g)) * (1.0f / 65536.0f);
    const float a = fabsf(z);
    const float m = __fmul_rn(a, 0.01f);
    const float v = __fmul_rn(__fadd_rn(m, 0.001f), mult);
    const uint16_t sb = round16<BF16>(v);
    const uint16_t bb = round16<BF16>(__fmul_rn(bias_mult, widen16<BF16>(sb)));
    reinterpret_cast<uint16_t*>(s0 + e * stride)[g] = sb;
    reinterpret_cast<uint16_t*>(b0 + e * stride)[g] = bb;
  }
}

static int grid_for(uint64_t n) {
  uint64_t g = (n + 255) / 256;
  return static_cast<int>(g > 148ull * 16ull ? 148ull * 16ull : (g == 0 ? 1 : g));
}

cudaError_t synth_records(cudaStream_t st, uint64_t seed, uint32_t layer, uint32_t expert0,
                          uint32_t count, uint8_t* bank, uint64_t stride, bool bf16) {
  static const uint32_t wtag[3] = {TAG_GATE_W, TAG_UP_W, TAG_DOWN_W};
  static const uint32_t stag[3] = {TAG_GATE_S, TAG_UP_S, TAG_DOWN_S};
  static const uint32_t woff[3] = {kOffGateW, kOffUpW, kOffDownW};
  static const uint32_t soff[3] = {kOffGateS, kOffUpS, kOffDownS};
  static const uint32_t boff[3] = {kOffGateB, kOffUpB, kOffDownB};
  for (int p = 0; p < 3; p++) {
    k_synth_codes<<<grid_for(65536ull * count), 256, 0, st>>>(seed, layer, wtag[p], expert0,
                                                              count, bank + woff[p], stride,
                                                              524288u);
    if (bf16)
      k_synth_scales<true><<<grid_for(16384ull * count), 256, 0, st>>>(
          seed, layer, stag[p], expert0, count, bank + soff[p], bank + boff[p], stride, 16384u,
          1.0f, -8.0f);
    else
      k_synth_scales<false><<<grid_for(16384ull * count), 256, 0, st>>>(
          seed, layer, stag[p], expert0, count, bank + soff[p], bank + boff[p], stride, 16384u,
          1.0f, -8.0f);
  }
  return cudaGetLastError();
}

cudaError_t synth_q8(cudaStream_t st, uint64_t seed, uint32_t layer, bool router, uint8_t* w,
                     uint16_t* s, uint16_t* b, bool bf16) {
  const uint32_t rows = router ? 256u : 1u;
  const uint32_t wt = router ? TAG_ROUTER_W : TAG_COEF_W;
  const uint32_t stg = router ? TAG_ROUTER_S : TAG_COEF_S;
  k_synth_codes<<<grid_for(rows * 256ull), 256, 0, st>>>(seed, layer, wt, 0, 1, w, 0,
                                                         rows * 2048u);
  if (bf16)
    k_synth_scales<true><<<grid_for(rows * 32ull), 256, 0, st>>>(
        seed, layer, stg, 0, 1, reinterpret_cast<uint8_t*>(s), reinterpret_cast<uint8_t*>(b), 0,
        rows * 32u, 0.0625f, -128.0f);
  else
    k_synth_scales<false><<<grid_for(rows * 32ull), 256, 0, st>>>(
        seed, layer, stg, 0, 1, reinterpret_cast<uint8_t*>(s), reinterpret_cast<uint8_t*>(b), 0,
        rows * 32u, 0.0625f, -128.0f);
  return cudaGetLastError();
}

// Host-side fp32 -> fp16 (round to nearest even).
static uint16_t host_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return static_cast<uint16_t>(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
  if (ax < 0x38800000u) {
    if (ax < 0x33000000u) return static_cast<uint16_t>(sign);
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    const uint32_t sh = 126u - e;
    uint32_t q = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u);
    const uint32_t half = 1u << (sh - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return static_cast<uint16_t>(sign | q);
  }
  uint32_t r = ax - 0x38000000u;
  r += 0xFFFu + ((r >> 13) & 1u);
  if (r >= 0x0F800000u) return static_cast<uint16_t>(sign | 0x7C00u);
  return static_cast<uint16_t>(sign | (r >> 13));
}

void synth_hidden_host(uint64_t seed, uint64_t tok0, int T, uint16_t* x) {
  float z[kHidden];
  for (int t = 0; t < T; t++) {
    const uint64_t key = stream_key(seed, 0, TAG_HIDDEN,
                                    static_cast<uint32_t>(tok0 + static_cast<uint64_t>(t)));
    double ss = 0.0;
    for (int i = 0; i < kHidden; i++) {
      z[i] = static_cast<float>(irwin_hall_sum(key, static_cast<uint64_t>(i))) *
             (1.0f / 65536.0f);
      ss += static_cast<double>(z[i]) * static_cast<double>(z[i]);
    }
    const double inv = 1.0 / sqrt(ss / kHidden + 1e-6);
    for (int i = 0; i < kHidden; i++)
      x[static_cast<size_t>(t) * kHidden + i] =
          host_f32_to_f16(static_cast<float>(static_cast<double>(z[i]) * inv));
  }
}

}  // namespace qf
