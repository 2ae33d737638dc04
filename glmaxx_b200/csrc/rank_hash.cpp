// SHA-256 (FIPS 180-4) and CRC32C (Castagnoli, reflected 0x82f63b78,
// crates/glm-format/src/crc32c.rs) for the rank-file reader.
//
// SHA-256 runs on the x86 SHA extensions when the CPU has them (two rounds
// per sha256rnds2, message schedule with sha256msg1/msg2) and on portable
// rounds otherwise; CRC32C uses the SSE4.2 crc32 instruction, which computes
// exactly this polynomial, or a byte table.
#include "rank_hash.h"

#include <cpuid.h>
#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cstring>

#include "glmaxx_rank_file.h"

namespace glmaxx::rankfile {
namespace {

alignas(16) constexpr uint32_t kRound[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

constexpr uint32_t kInitial[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                                  0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void compress_portable(uint32_t* h, const uint8_t* p, size_t blocks) {
  for (; blocks; --blocks, p += 64) {
    uint32_t w[64];
    for (int t = 0; t < 16; ++t)
      w[t] = uint32_t(p[4 * t]) << 24 | uint32_t(p[4 * t + 1]) << 16 |
             uint32_t(p[4 * t + 2]) << 8 | uint32_t(p[4 * t + 3]);
    for (int t = 16; t < 64; ++t) {
      const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
      const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
      w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], k = h[7];
    for (int t = 0; t < 64; ++t) {
      const uint32_t t1 = k + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) +
                          kRound[t] + w[t];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      k = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h[0] += a;
    h[1] += b;
    h[2] += c;
    h[3] += d;
    h[4] += e;
    h[5] += f;
    h[6] += g;
    h[7] += k;
  }
}

// The SHA extensions keep the state as two vectors, (A,B,E,F) and (C,D,G,H)
// with A and C in the top lanes; sha256rnds2(cdgh, abef, wk) runs the two
// rounds whose message+constant sums sit in wk's low lanes and returns the new
// (A,B,E,F), the old one becoming (C,D,G,H).
__attribute__((target("sha,sse4.1,ssse3"))) void compress_sha_ni(uint32_t* h, const uint8_t* p,
                                                                  size_t blocks) {
  const __m128i bswap = _mm_set_epi64x(0x0c0d0e0f08090a0bLL, 0x0405060700010203LL);
  __m128i dcba = _mm_loadu_si128(reinterpret_cast<const __m128i*>(h));      // lanes A B C D
  __m128i hgfe = _mm_loadu_si128(reinterpret_cast<const __m128i*>(h + 4));  // lanes E F G H
  const __m128i badc = _mm_shuffle_epi32(dcba, 0xB1);                       // B A D C
  const __m128i efgh = _mm_shuffle_epi32(hgfe, 0x1B);                       // H G F E
  __m128i abef = _mm_alignr_epi8(badc, efgh, 8);                            // F E B A
  __m128i cdgh = _mm_blend_epi16(efgh, badc, 0xF0);                         // H G D C
  for (; blocks; --blocks, p += 64) {
    const __m128i abef0 = abef, cdgh0 = cdgh;
    __m128i w[4];
    for (int i = 0; i < 4; ++i)
      w[i] = _mm_shuffle_epi8(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p + 16 * i)), bswap);
    for (int g = 0; g < 16; ++g) {
      const __m128i cur = w[g & 3];
      const __m128i wk =
          _mm_add_epi32(cur, _mm_load_si128(reinterpret_cast<const __m128i*>(kRound + 4 * g)));
      cdgh = _mm_sha256rnds2_epu32(cdgh, abef, wk);
      abef = _mm_sha256rnds2_epu32(abef, cdgh, _mm_shuffle_epi32(wk, 0x0E));
      if (g < 12) {
        // W[g+4] = msg2(msg1(W[g], W[g+1]) + alignr(W[g+3], W[g+2], 4), W[g+3])
        const __m128i w1 = w[(g + 1) & 3], w2 = w[(g + 2) & 3], w3 = w[(g + 3) & 3];
        __m128i next = _mm_sha256msg1_epu32(cur, w1);
        next = _mm_add_epi32(next, _mm_alignr_epi8(w3, w2, 4));
        w[g & 3] = _mm_sha256msg2_epu32(next, w3);
      }
    }
    abef = _mm_add_epi32(abef, abef0);
    cdgh = _mm_add_epi32(cdgh, cdgh0);
  }
  const __m128i feba = _mm_shuffle_epi32(abef, 0x1B);  // A B E F
  const __m128i dchg = _mm_shuffle_epi32(cdgh, 0xB1);  // G H C D
  dcba = _mm_blend_epi16(feba, dchg, 0xF0);            // A B C D
  hgfe = _mm_alignr_epi8(dchg, feba, 8);               // E F G H
  _mm_storeu_si128(reinterpret_cast<__m128i*>(h), dcba);
  _mm_storeu_si128(reinterpret_cast<__m128i*>(h + 4), hgfe);
}

bool cpu_has_sha() {
  unsigned a, b, c, d;
  if (!__get_cpuid(1, &a, &b, &c, &d)) return false;
  const bool ssse3 = c & (1u << 9), sse41 = c & (1u << 19);
  if (!__get_cpuid_count(7, 0, &a, &b, &c, &d)) return false;
  return ssse3 && sse41 && (b & (1u << 29));
}

bool cpu_has_sse42() {
  unsigned a, b, c, d;
  return __get_cpuid(1, &a, &b, &c, &d) && (c & (1u << 20));
}

const bool g_sha_ni = cpu_has_sha();
const bool g_sse42 = cpu_has_sse42();
std::atomic<bool> g_force_portable{false};

__attribute__((target("sse4.2"))) uint32_t crc32c_hw(uint32_t crc, const uint8_t* p, size_t n) {
  uint64_t c = crc;
  for (; n >= 8; n -= 8, p += 8) {
    uint64_t v;
    std::memcpy(&v, p, 8);
    c = _mm_crc32_u64(c, v);
  }
  uint32_t c32 = uint32_t(c);
  for (; n; --n, ++p) c32 = _mm_crc32_u8(c32, *p);
  return c32;
}

struct CrcTable {
  uint32_t t[256];
  CrcTable() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int b = 0; b < 8; ++b) c = (c >> 1) ^ (0x82f63b78u & (0u - (c & 1u)));
      t[i] = c;
    }
  }
};

uint32_t crc32c_table(uint32_t crc, const uint8_t* p, size_t n) {
  static const CrcTable table;
  for (; n; --n, ++p) crc = (crc >> 8) ^ table.t[(crc ^ *p) & 0xffu];
  return crc;
}

}  // namespace

void Sha256::reset() {
  std::memcpy(h_, kInitial, sizeof(h_));
  fill_ = 0;
  total_ = 0;
}

void Sha256::blocks(const uint8_t* p, size_t n) {
  if (g_sha_ni && !g_force_portable.load(std::memory_order_relaxed))
    compress_sha_ni(h_, p, n);
  else
    compress_portable(h_, p, n);
}

void Sha256::update(const void* data, size_t length) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  total_ += length;
  if (fill_) {
    const size_t take = std::min(length, size_t(64) - fill_);
    std::memcpy(buf_ + fill_, p, take);
    fill_ += take;
    p += take;
    length -= take;
    if (fill_ < 64) return;
    blocks(buf_, 1);
    fill_ = 0;
  }
  if (length >= 64) {
    blocks(p, length / 64);
    p += length / 64 * 64;
    length %= 64;
  }
  std::memcpy(buf_, p, length);
  fill_ = length;
}

void Sha256::finish(uint8_t out[32]) {
  const uint64_t bits = total_ * 8;
  uint8_t pad[72] = {0x80};
  const size_t pad_len = (fill_ < 56 ? 56 : 120) - fill_;
  for (int i = 0; i < 8; ++i) pad[pad_len + i] = uint8_t(bits >> (56 - 8 * i));
  update(pad, pad_len + 8);
  for (int i = 0; i < 8; ++i)
    for (int j = 0; j < 4; ++j) out[4 * i + j] = uint8_t(h_[i] >> (24 - 8 * j));
}

void sha256(const void* data, size_t length, uint8_t out[32]) {
  Sha256 s;
  s.update(data, length);
  s.finish(out);
}

uint32_t crc32c(const void* data, size_t length) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  const uint32_t c = g_sse42 ? crc32c_hw(~0u, p, length) : crc32c_table(~0u, p, length);
  return ~c;
}

}  // namespace glmaxx::rankfile

extern "C" {

void glmaxx_sha256(const void* data, uint64_t length, uint8_t digest[32]) {
  glmaxx::rankfile::sha256(data, size_t(length), digest);
}

uint32_t glmaxx_crc32c(const void* data, uint64_t length) {
  return glmaxx::rankfile::crc32c(data, size_t(length));
}

int32_t glmaxx_sha256_accelerated(void) {
  return glmaxx::rankfile::g_sha_ni && !glmaxx::rankfile::g_force_portable.load() ? 1 : 0;
}

void glmaxx_sha256_force_portable(int32_t on) { glmaxx::rankfile::g_force_portable.store(on != 0); }

}  // extern "C"
