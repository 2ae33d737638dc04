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
// rounds it once, exactly as fp16(f32(lo) + f32(hi)) of the reference.
__device__ __forceinline__ void exl3_decode_span(const uint32_t (&wd)[3], uint32_t off,
                                                 uint16_t (&w16)[8]) {
  const uint64_t v = (uint64_t(wd[0]) << 32) | wd[1];
  const uint64_t span = off ? ((v << off) | (wd[2] >> (32 - off))) : v;  // bit 63 = span start
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t window = uint32_t(span >> (48 - 3 * w)) & 0xffffu;
    const uint32_t packed = ((window * 0xCBAC1FEDu) & 0x8FFF8FFFu) ^ 0x3B603B60u;
    const __half2 h = *reinterpret_cast<const __half2*>(&packed);
    w16[w] = __half_as_ushort(__hadd(__low2half(h), __high2half(h)));
  }
}

}  // namespace glmaxx
