// SHA-256 compression with the x86 SHA extensions (host code, g++ with -msha):
// the published instruction sequence for these instructions -- two rounds
// per sha256rnds2 on the (ABEF, CDGH) state halves, the message schedule by
// sha256msg1 / alignr / sha256msg2 -- used by the packed-store reader to hash
// layer payloads (453 MB each).  The caller checks sha256_ni_available()
// first; the scalar FIPS 180-4 code in qf_store.cu is the fallback.

#include <cpuid.h>
#include <immintrin.h>
#include <stddef.h>
#include <stdint.h>

namespace qf {

bool sha256_ni_available() {
  unsigned a = 0, b = 0, c = 0, d = 0;
  if (!__get_cpuid_count(7, 0, &a, &b, &c, &d)) return false;
  const bool sha = (b >> 29) & 1u;
  unsigned a1 = 0, b1 = 0, c1 = 0, d1 = 0;
  if (!__get_cpuid(1, &a1, &b1, &c1, &d1)) return false;
  const bool ssse3 = (c1 >> 9) & 1u, sse41 = (c1 >> 19) & 1u;
  return sha && ssse3 && sse41;
}

// state: h0..h7; p: n blocks of 64 bytes
void sha256_ni_blocks(uint32_t* state, const uint8_t* p, size_t n) {
  alignas(16) static const uint32_t K[64] = {
      0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
      0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
      0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
      0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
      0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
      0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
      0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
      0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
  // big-endian message words
  const __m128i bswap = _mm_set_epi64x(0x0c0d0e0f08090a0bLL, 0x0405060700010203LL);
  // (h0 h1 h2 h3), (h4 h5 h6 h7) -> ABEF, CDGH
  __m128i t = _mm_loadu_si128(reinterpret_cast<const __m128i*>(state));
  __m128i s1 = _mm_loadu_si128(reinterpret_cast<const __m128i*>(state + 4));
  t = _mm_shuffle_epi32(t, 0xB1);
  s1 = _mm_shuffle_epi32(s1, 0x1B);
  __m128i s0 = _mm_alignr_epi8(t, s1, 8);
  s1 = _mm_blend_epi16(s1, t, 0xF0);
  for (; n; n--, p += 64) {
    const __m128i save0 = s0, save1 = s1;
    __m128i w[4];
    for (int i = 0; i < 4; i++)
      w[i] = _mm_shuffle_epi8(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p + 16 * i)), bswap);
    for (int g = 0; g < 16; g++) {
      __m128i m = _mm_add_epi32(w[g & 3], _mm_load_si128(reinterpret_cast<const __m128i*>(K + 4 * g)));
      s1 = _mm_sha256rnds2_epu32(s1, s0, m);
      m = _mm_shuffle_epi32(m, 0x0E);
      s0 = _mm_sha256rnds2_epu32(s0, s1, m);
      if (g < 12) {
        // W[g+4] = sigma1(W[g+3]..) + W[g+3 .. g+2 tail] + sigma0(W[g+1]) + W[g]
        __m128i x = _mm_sha256msg1_epu32(w[g & 3], w[(g + 1) & 3]);
        x = _mm_add_epi32(x, _mm_alignr_epi8(w[(g + 3) & 3], w[(g + 2) & 3], 4));
        w[g & 3] = _mm_sha256msg2_epu32(x, w[(g + 3) & 3]);
      }
    }
    s0 = _mm_add_epi32(s0, save0);
    s1 = _mm_add_epi32(s1, save1);
  }
  // ABEF, CDGH -> (h0 h1 h2 h3), (h4 h5 h6 h7)
  t = _mm_shuffle_epi32(s0, 0x1B);
  s1 = _mm_shuffle_epi32(s1, 0xB1);
  s0 = _mm_blend_epi16(t, s1, 0xF0);
  s1 = _mm_alignr_epi8(s1, t, 8);
  _mm_storeu_si128(reinterpret_cast<__m128i*>(state), s0);
  _mm_storeu_si128(reinterpret_cast<__m128i*>(state + 4), s1);
}

}  // namespace qf
