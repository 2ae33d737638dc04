// EXL3 3-bit trellis decode helpers shared by the decode-fused GEMV (exl3.cu)
// and the tensor-core path (exl3_gemm.cu).  Reference: crates/glm-format/src/
// exl3.rs:471-513 (3INST decode, bitstream windows, tile layout).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace glmaxx {

constexpr uint32_t kExl3Bits = 3;
constexpr uint32_t kExl3TileHalves = 16 * kExl3Bits;  // 48 halves = 24 words per 16x16 tile

// Bit position (MSB-first stream order) of lane `lane`'s first window inside
// the tile's 768-bit circular stream: weight i of the tile uses the 16 bits
// ending at bit (i + 257) * 3 (exl3.rs:490-513), and lane l owns i = 8l .. 8l+7,
// so its 8 windows lie in 37 consecutive bits starting at (8l + 257) * 3 - 16.
struct Exl3LaneWindow {
  uint32_t word0;  // first 32-bit word (mod 24) holding the span
  uint32_t off;    // bit offset of the span inside that word (0 = MSB)
};
__device__ __forceinline__ Exl3LaneWindow exl3_lane_window(uint32_t lane) {
  const uint32_t start = (lane * 8 + 257) * kExl3Bits - 16;
  return {start / 32, start % 32};
}

// The three words of a tile that hold lane's span (halves base[0..47] are
// words (h0 | h1 << 16), the stream wraps after 24 words).
__device__ __forceinline__ void exl3_load_span(const uint16_t* __restrict__ base,
                                               Exl3LaneWindow lw, uint32_t (&wd)[3]) {
  constexpr uint32_t kTileWords = 8 * kExl3Bits;
  const uint32_t* base32 = reinterpret_cast<const uint32_t*>(base);
#pragma unroll
  for (int j = 0; j < 3; ++j) wd[j] = __ldg(base32 + (lw.word0 + j) % kTileWords);
}

// 3INST decode of the 8 windows in the span: value = window * 0xCBAC1FED,
// (value & 0x8FFF8FFF) ^ 0x3B603B60 read as two fp16 halves, summed.  Both halves
// have exponent fields 12..15, so their exact sum fits fp32 and the fp16 add
// rounds it once, exactly as fp16(f32(lo) + f32(hi)) of the reference.  The 8
// weights come out as 4 packed pairs (weight 2j in the low half of p[j], 2j + 1
// in the high half): the layout both consumers store.  The
// span is assembled with funnel shifts (no special case for a zero offset); for
// each pair the two masked products are regrouped into (low halves) and (high
// halves) by two byte permutes, and one fp16x2 add gives both sums -- each half
// of that add rounds once, exactly as the single add per weight above.
__device__ __forceinline__ void exl3_decode_span_pairs(const uint32_t (&wd)[3], uint32_t off,
                                                       uint32_t (&p)[4]) {
  const uint32_t hi = __funnelshift_l(wd[1], wd[0], off);  // span bits 63..32
  const uint32_t lo = __funnelshift_l(wd[2], wd[1], off);  // span bits 31..0
  uint32_t win[8];
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const int sh = 48 - 3 * w;  // the window is span bits sh + 15 .. sh
    win[w] = (sh >= 32 ? hi >> (sh - 32) : __funnelshift_r(lo, hi, sh)) & 0xffffu;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t q0 = ((win[2 * j] * 0xCBAC1FEDu) & 0x8FFF8FFFu) ^ 0x3B603B60u;
    const uint32_t q1 = ((win[2 * j + 1] * 0xCBAC1FEDu) & 0x8FFF8FFFu) ^ 0x3B603B60u;
    const uint32_t los = __byte_perm(q0, q1, 0x5410);  // (q0 low half, q1 low half)
    const uint32_t his = __byte_perm(q0, q1, 0x7632);  // (q0 high half, q1 high half)
    const __half2 sum = __hadd2(*reinterpret_cast<const __half2*>(&los),
                                *reinterpret_cast<const __half2*>(&his));
    p[j] = *reinterpret_cast<const uint32_t*>(&sum);
  }
}

}  // namespace glmaxx
