// Native rank-file (.g5n) reader with a direct-to-HBM sink.
//
// Format rules follow spec/format-v0.md sections 4-19 and the reference's
// Rust reader: NativeRankReader::open (crates/glm-format/src/native_reader.rs:
// 119-335), validate_descriptors (:724-858), verify_and_stream (:378-537),
// validate_rank_set (:543-588); TensorDescriptor::decode (container.rs:150-
// 213); Nvfp4Metadata::decode/validate and Nvfp4PlaneValidator (nvfp4.rs:
// 84-160, 309-464); Exl3Metadata::decode/validate and
// Exl3Trellis::from_container_planes/validate (exl3.rs:72-157, 229-340).
// Checks run in the reference's order so that a file with one defect reports
// the same error kind.
//
// verify_and_stream reads the payload region once in 8 MiB chunks into a ring
// of staging slots (pinned once anything goes to the device, and kept with the
// file handle between loads).  One thread
// hashes the whole payload in order; P plane workers each own the tensors
// t = w (mod P) and, for their tensors, check padding, hash the planes, run
// the codec validators and issue the device copies; the calling thread reads.
// A slot is reused after every consumer has released it and the copies from
// it have completed (a CUDA event recorded by the last consumer).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "glmaxx_rank_file.h"
#include "rank_hash.h"

static_assert(sizeof(glmaxx_rank_file_info) == 328, "glmaxx_rank_file_info layout");
static_assert(sizeof(glmaxx_rank_tensor_info) == 136, "glmaxx_rank_tensor_info layout");
static_assert(sizeof(glmaxx_rank_placement) == 56, "glmaxx_rank_placement layout");
static_assert(sizeof(glmaxx_rank_payload_proof) == 88, "glmaxx_rank_payload_proof layout");
static_assert(sizeof(glmaxx_rank_sink) == 40, "glmaxx_rank_sink layout");

namespace glmaxx::rankfile {
namespace {

constexpr uint64_t kHeaderBytes = 4096;
constexpr uint64_t kDescriptorBytes = 256;
constexpr uint64_t kAlignment = 4096;
constexpr uint64_t kPayloadAlignment = 256;
constexpr uint64_t kControlRegionMax = 1ull << 30;
constexpr uint64_t kControlTotalMax = 512ull << 20;
constexpr uint64_t kChunkBytes = 8ull << 20;
constexpr int kSlots = 8;
constexpr uint16_t kValueLayout = 0x1201;
constexpr uint16_t kScaleLayout = 0x1201;
constexpr uint32_t kMcgMultiplier = 0xCBAC1FEDu;
constexpr uint8_t kDescriptorAuxRequired = 1u << 7;

// Pinned layout and quantisation-policy identities of NVFP4 metadata version
// 0.1 (nvfp4.rs:7-14); a record must carry exactly these.
constexpr uint8_t kLayoutSourceSha256[32] = {
    0x59, 0x8e, 0x05, 0x4b, 0xef, 0x21, 0xed, 0xf9, 0x4b, 0x1f, 0xd6, 0xbb, 0x14, 0x47, 0xcf, 0xa9,
    0xcf, 0xcf, 0x5a, 0x59, 0x07, 0xab, 0x37, 0x01, 0x28, 0x10, 0x24, 0x48, 0xdb, 0xb6, 0xd5, 0x30};
constexpr uint8_t kQuantPolicySha256[32] = {
    0xcd, 0x90, 0x95, 0x79, 0x33, 0x44, 0x05, 0xec, 0xd4, 0xcd, 0x8d, 0x9a, 0x6c, 0x2d, 0xfc, 0xba,
    0x7f, 0x01, 0x24, 0xc4, 0xc4, 0xba, 0x92, 0xbc, 0x40, 0xc9, 0x76, 0xd5, 0x74, 0xbe, 0x05, 0xa3};

struct Fail {
  int32_t code;
};
[[noreturn]] void fail(int32_t code) { throw Fail{code}; }

uint16_t get_u16(const uint8_t* p, size_t o) {
  uint16_t v;
  std::memcpy(&v, p + o, 2);
  return v;
}
int16_t get_i16(const uint8_t* p, size_t o) { return int16_t(get_u16(p, o)); }
uint32_t get_u32(const uint8_t* p, size_t o) {
  uint32_t v;
  std::memcpy(&v, p + o, 4);
  return v;
}
uint64_t get_u64(const uint8_t* p, size_t o) {
  uint64_t v;
  std::memcpy(&v, p + o, 8);
  return v;
}
float get_f32(const uint8_t* p, size_t o) {
  float v;
  std::memcpy(&v, p + o, 4);
  return v;
}
bool all_zero(const uint8_t* p, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (p[i]) return false;
  return true;
}
uint64_t add(uint64_t a, uint64_t b) {
  if (a > UINT64_MAX - b) fail(GLMAXX_RANK_ERR_OVERFLOW);
  return a + b;
}
uint64_t mul(uint64_t a, uint64_t b) {
  if (a && b > UINT64_MAX / a) fail(GLMAXX_RANK_ERR_OVERFLOW);
  return a * b;
}
uint64_t align_up(uint64_t v, uint64_t a) { return add(v, a - 1) / a * a; }

struct Region {
  uint64_t start = 0, end = 0;
  uint64_t len() const { return end - start; }
};

// ------------------------------------------------------------ descriptors
struct Descriptor {
  uint32_t tensor_id, name_offset;
  uint16_t name_bytes, role_id;
  int16_t layer_id, expert_id;
  uint16_t codec_id, logical_dtype, stored_dtype;
  int8_t tp_shard_axis;
  uint8_t ndim, flags;
  uint32_t logical_shape[4], padded_shape[4];
  uint64_t payload_offset, payload_bytes, aux_offset, aux_bytes, codec_metadata_offset,
      codec_metadata_bytes;
  uint32_t payload_alignment, quant_group_elements;
  uint8_t payload_sha256[32], aux_sha256[32], codec_metadata_sha256[32];
};

// shape_elements (container.rs:945-959)
uint64_t shape_elements(const uint32_t* shape, uint8_t ndim) {
  if (ndim < 1 || ndim > 4) fail(GLMAXX_RANK_ERR_DESCRIPTOR);
  uint64_t product = 1;
  for (int i = 0; i < ndim; ++i) {
    if (shape[i] == 0) fail(GLMAXX_RANK_ERR_DESCRIPTOR);
    product = mul(product, shape[i]);
  }
  return product;
}

// TensorDescriptor::decode (container.rs:150-213)
Descriptor decode_descriptor(const uint8_t* b) {
  const uint32_t alignment = get_u32(b, 120);
  if (!all_zero(b + 25, 3) || !all_zero(b + 224, 32) || b[23] == 0 || b[23] > 4 ||
      __builtin_popcount(b[24] & 0x7u) > 1 || alignment < kPayloadAlignment ||
      (alignment & (alignment - 1)) != 0)
    fail(GLMAXX_RANK_ERR_DESCRIPTOR);
  Descriptor d{};
  d.ndim = b[23];
  for (int i = 0; i < 4; ++i) {
    d.logical_shape[i] = get_u32(b, 28 + 4 * i);
    d.padded_shape[i] = get_u32(b, 44 + 4 * i);
  }
  const uint64_t logical_elements = shape_elements(d.logical_shape, d.ndim);
  for (int i = d.ndim; i < 4; ++i)
    if (d.logical_shape[i] != 1 || d.padded_shape[i] != 1) fail(GLMAXX_RANK_ERR_DESCRIPTOR);
  if (get_u64(b, 64) != logical_elements) fail(GLMAXX_RANK_ERR_DESCRIPTOR);
  d.tensor_id = get_u32(b, 0);
  d.name_offset = get_u32(b, 4);
  d.name_bytes = get_u16(b, 8);
  d.role_id = get_u16(b, 10);
  d.layer_id = get_i16(b, 12);
  d.expert_id = get_i16(b, 14);
  d.codec_id = get_u16(b, 16);
  d.logical_dtype = get_u16(b, 18);
  d.stored_dtype = get_u16(b, 20);
  d.tp_shard_axis = int8_t(b[22]);
  d.flags = b[24];
  d.payload_offset = get_u64(b, 72);
  d.payload_bytes = get_u64(b, 80);
  d.aux_offset = get_u64(b, 88);
  d.aux_bytes = get_u64(b, 96);
  d.codec_metadata_offset = get_u64(b, 104);
  d.codec_metadata_bytes = get_u64(b, 112);
  d.payload_alignment = alignment;
  d.quant_group_elements = get_u32(b, 124);
  std::memcpy(d.payload_sha256, b + 128, 32);
  std::memcpy(d.aux_sha256, b + 160, 32);
  std::memcpy(d.codec_metadata_sha256, b + 192, 32);
  return d;
}

bool is_plain(uint16_t codec) {
  return codec == GLMAXX_CODEC_BF16 || codec == GLMAXX_CODEC_FP16 || codec == GLMAXX_CODEC_FP32;
}
bool is_nvfp4(uint16_t codec) {
  return codec == GLMAXX_CODEC_NVFP4_1D || codec == GLMAXX_CODEC_NVFP4_2D;
}
uint64_t plain_element_bytes(uint16_t codec) { return codec == GLMAXX_CODEC_FP32 ? 4 : 2; }

// validate_plain_geometry (container.rs:846-877)
void validate_plain_geometry(uint16_t codec, const Descriptor& d, uint64_t payload_bytes) {
  if (d.ndim < 1 || d.ndim > 4) fail(GLMAXX_RANK_ERR_DESCRIPTOR);
  for (int i = 0; i < d.ndim; ++i)
    if (d.logical_shape[i] == 0 || d.logical_shape[i] > d.padded_shape[i])
      fail(GLMAXX_RANK_ERR_DESCRIPTOR);
  for (int i = d.ndim; i < 4; ++i)
    if (d.logical_shape[i] != 1 || d.padded_shape[i] != 1) fail(GLMAXX_RANK_ERR_DESCRIPTOR);
  if (mul(shape_elements(d.padded_shape, d.ndim), plain_element_bytes(codec)) != payload_bytes)
    fail(GLMAXX_RANK_ERR_DESCRIPTOR);
}

bool plain_padded(const Descriptor& d) {
  return std::memcmp(d.logical_shape, d.padded_shape, sizeof(d.logical_shape)) != 0;
}

// validate_plain_padding_chunk (container.rs:899-943): every element whose
// coordinate lies outside the logical shape is zero.
void validate_plain_padding_chunk(const Descriptor& d, const uint8_t* p, uint64_t len,
                                  uint64_t plane_offset) {
  if (!is_plain(d.codec_id) || !plain_padded(d)) return;
  const uint64_t eb = plain_element_bytes(d.codec_id);
  const uint64_t total = mul(shape_elements(d.padded_shape, d.ndim), eb);
  const uint64_t end = add(plane_offset, len);
  if (plane_offset % eb || len % eb || end > total) fail(GLMAXX_RANK_ERR_DESCRIPTOR);
  const uint64_t first = plane_offset / eb;
  for (uint64_t e = 0; e < len / eb; ++e) {
    uint64_t rem = first + e;
    bool padding = false;
    for (int axis = d.ndim - 1; axis >= 0; --axis) {
      const uint64_t extent = d.padded_shape[axis];
      padding |= rem % extent >= d.logical_shape[axis];
      rem /= extent;
    }
    if (padding && !all_zero(p + e * eb, eb)) fail(GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT);
  }
}

// ------------------------------------------------------------ codec metadata
struct Nvfp4Meta {
  bool two_d = false;
  uint32_t logical_n = 0, logical_k = 0, padded_n = 0, padded_k = 0;
  float global_scale = 0, global_amax = 0;
  uint32_t value_bytes = 0, scale_bytes = 0;
};

// Nvfp4Metadata::validate (nvfp4.rs:128-160)
void nvfp4_validate(const Nvfp4Meta& m) {
  if (m.logical_n == 0 || m.logical_k == 0 || m.padded_n < m.logical_n ||
      m.padded_k < m.logical_k || m.padded_n % 128 || m.padded_k % 64 ||
      !std::isfinite(m.global_scale) || m.global_scale <= 0.0f || !std::isfinite(m.global_amax) ||
      std::signbit(m.global_amax))
    fail(GLMAXX_RANK_ERR_NVFP4_INVALID_SHAPE_OR_SCALE);
  volatile float amax = m.global_amax;  // one IEEE f32 division, as the format defines
  const float expected = amax == 0.0f ? 1.0f : amax / 2688.0f;
  uint32_t a, b;
  std::memcpy(&a, &m.global_scale, 4);
  std::memcpy(&b, &expected, 4);
  if (a != b) fail(GLMAXX_RANK_ERR_NVFP4_INVALID_SHAPE_OR_SCALE);
  const uint64_t elements = uint64_t(m.padded_n) * m.padded_k;
  if (m.value_bytes != elements / 2 || m.scale_bytes != elements / 16)
    fail(GLMAXX_RANK_ERR_NVFP4_BYTE_ACCOUNTING);
}

// Nvfp4Metadata::decode (nvfp4.rs:84-126)
Nvfp4Meta nvfp4_decode(const uint8_t* b, uint64_t length) {
  if (length != 128) fail(GLMAXX_RANK_ERR_NVFP4_METADATA_LENGTH);
  uint8_t checked[128];
  std::memcpy(checked, b, 128);
  std::memset(checked + 120, 0, 4);
  if (crc32c(checked, 128) != get_u32(b, 120)) fail(GLMAXX_RANK_ERR_NVFP4_METADATA_CRC);
  if (get_u16(b, 0) != 0 || get_u16(b, 2) != 1 || b[7] != 1 || get_u16(b, 24) != 16 ||
      get_u16(b, 28) != kValueLayout || get_u16(b, 30) != kScaleLayout || b[32] != 1 ||
      b[33] != 1 || b[34] != 1 || b[35] != 1 || !all_zero(b + 52, 4) ||
      std::memcmp(b + 56, kLayoutSourceSha256, 32) || std::memcmp(b + 88, kQuantPolicySha256, 32) ||
      !all_zero(b + 124, 4))
    fail(GLMAXX_RANK_ERR_NVFP4_UNSUPPORTED_METADATA);
  Nvfp4Meta m;
  const uint16_t codec = get_u16(b, 4);
  if (codec == GLMAXX_CODEC_NVFP4_1D && b[6] == 1 && get_u16(b, 26) == 1)
    m.two_d = false;
  else if (codec == GLMAXX_CODEC_NVFP4_2D && b[6] == 2 && get_u16(b, 26) == 16)
    m.two_d = true;
  else
    fail(GLMAXX_RANK_ERR_NVFP4_UNSUPPORTED_METADATA);
  m.logical_n = get_u32(b, 8);
  m.logical_k = get_u32(b, 12);
  m.padded_n = get_u32(b, 16);
  m.padded_k = get_u32(b, 20);
  m.global_scale = get_f32(b, 36);
  m.global_amax = get_f32(b, 40);
  m.value_bytes = get_u32(b, 44);
  m.scale_bytes = get_u32(b, 48);
  nvfp4_validate(m);
  return m;
}

struct Exl3Meta {
  uint8_t projection = 0, bits = 0, rank = 0;
  uint16_t layer = 0, expert = 0;
  uint32_t logical_k = 0, logical_n = 0;
  uint64_t trellis_words = 0, rotation_words = 0;
};

// trellis_word_count (exl3.rs:461-469)
uint64_t trellis_word_count(uint32_t k, uint32_t n, uint8_t bits) {
  if (k == 0 || n == 0 || k % 16 || n % 16 || bits == 0)
    fail(GLMAXX_RANK_ERR_EXL3_UNSUPPORTED_CONTRACT);
  const uint64_t tiles = uint64_t(k / 16) * (n / 16);
  if (tiles > UINT64_MAX / (16u * bits)) fail(GLMAXX_RANK_ERR_EXL3_OVERFLOW);
  return tiles * 16u * bits;
}

// Exl3Metadata::validate (exl3.rs:72-102)
void exl3_validate(const Exl3Meta& m) {
  if (m.layer < 3 || m.layer > 78 || m.expert >= 256 || m.rank >= 4 || m.bits != 3 ||
      m.logical_k == 0 || m.logical_n == 0 || m.logical_k % 128 || m.logical_n % 128)
    fail(GLMAXX_RANK_ERR_EXL3_UNSUPPORTED_CONTRACT);
  if (m.trellis_words != trellis_word_count(m.logical_k, m.logical_n, m.bits) ||
      m.rotation_words != uint64_t(m.logical_k) + m.logical_n)
    fail(GLMAXX_RANK_ERR_EXL3_BYTE_ACCOUNTING);
  const bool gate_up = m.projection == 1 || m.projection == 2;
  const uint32_t ek = gate_up ? 6144 : 512, en = gate_up ? 512 : 6144;
  if (m.layer <= 77 && (m.logical_k != ek || m.logical_n != en))
    fail(GLMAXX_RANK_ERR_EXL3_UNSUPPORTED_CONTRACT);
}

// Exl3Metadata::decode (exl3.rs:124-157)
Exl3Meta exl3_decode(const uint8_t* b, uint64_t length) {
  static const uint8_t kMagic[8] = {'G', 'L', 'X', '3', 'T', 'R', '3', 0};
  if (length != 96) fail(GLMAXX_RANK_ERR_EXL3_METADATA_LENGTH);
  uint8_t checked[96];
  std::memcpy(checked, b, 96);
  std::memset(checked + 88, 0, 4);
  if (crc32c(checked, 96) != get_u32(b, 88)) fail(GLMAXX_RANK_ERR_EXL3_METADATA_CRC);
  if (std::memcmp(b, kMagic, 8) || get_u16(b, 8) != 1 || get_u16(b, 10) != 1 ||
      get_u32(b, 28) != kMcgMultiplier || b[15] != 0 || !all_zero(b + 48, 40) ||
      !all_zero(b + 92, 4))
    fail(GLMAXX_RANK_ERR_EXL3_UNSUPPORTED_CONTRACT);
  if (b[12] < 1 || b[12] > 3) fail(GLMAXX_RANK_ERR_EXL3_UNSUPPORTED_CONTRACT);
  Exl3Meta m;
  m.projection = b[12];
  m.bits = b[13];
  m.rank = b[14];
  m.layer = get_u16(b, 16);
  m.expert = get_u16(b, 18);
  m.logical_k = get_u32(b, 20);
  m.logical_n = get_u32(b, 24);
  m.trellis_words = get_u64(b, 32);
  m.rotation_words = get_u64(b, 40);
  exl3_validate(m);
  return m;
}

// scale_offset (nvfp4.rs:493-521), the 128x4 atom swizzle
inline uint64_t scale_offset(uint64_t n, uint64_t g, uint64_t k_blocks) {
  return 512 * ((n >> 7) * k_blocks + (g >> 2)) + 16 * (n & 31) + 4 * ((n & 127) >> 5) + (g & 3);
}

// Nvfp4PlaneValidator (nvfp4.rs:325-464) over streamed planes.
struct Nvfp4Check {
  const Nvfp4Meta* m = nullptr;
  std::vector<uint8_t> nonzero;  // one bit per scale: the block has a nonzero code
  std::vector<uint8_t> scales;
  uint64_t value_seen = 0, scale_seen = 0;

  void begin(const Nvfp4Meta& meta) {
    nvfp4_validate(meta);
    m = &meta;
    try {
      nonzero.assign((uint64_t(meta.scale_bytes) + 7) / 8, 0);
      scales.assign(meta.scale_bytes, 0);
    } catch (const std::bad_alloc&) {
      fail(GLMAXX_RANK_ERR_NVFP4_ALLOCATION);
    }
    value_seen = scale_seen = 0;
  }
  uint64_t scratch() const { return nonzero.capacity() + scales.capacity(); }

  void value_chunk(const uint8_t* p, uint64_t len, uint64_t off) {
    const uint64_t end = off + len;
    if (off != value_seen || end > m->value_bytes || off % 8 || len % 8)
      fail(GLMAXX_RANK_ERR_NVFP4_BYTE_ACCOUNTING);
    const uint64_t gk = m->padded_k / 16, kb = m->padded_k / 64;
    const bool padded = m->logical_n != m->padded_n || m->logical_k != m->padded_k;
    uint64_t row = (off / 8) / gk, grp = (off / 8) % gk;
    for (uint64_t i = 0; i < len; i += 8) {
      uint64_t v;
      std::memcpy(&v, p + i, 8);
      if (row >= m->padded_n) fail(GLMAXX_RANK_ERR_NVFP4_BYTE_ACCOUNTING);
      if (padded) {
        const uint64_t start = grp * 16;
        if (row >= m->logical_n || start >= m->logical_k) {
          if (v) fail(GLMAXX_RANK_ERR_NVFP4_NON_CANONICAL_PADDING);
        } else {
          const uint64_t lanes = std::min<uint64_t>(m->logical_k - start, 16);
          if (lanes < 16 && (v >> (4 * lanes)) != 0)
            fail(GLMAXX_RANK_ERR_NVFP4_NON_CANONICAL_PADDING);
        }
      }
      if (v) {
        const uint64_t s = scale_offset(row, grp, kb);
        nonzero[s >> 3] |= uint8_t(1u << (s & 7));
      }
      if (++grp == gk) {
        grp = 0;
        ++row;
      }
    }
    value_seen = end;
  }

  void scale_chunk(const uint8_t* p, uint64_t len, uint64_t off) {
    if (off != scale_seen || off + len > m->scale_bytes)
      fail(GLMAXX_RANK_ERR_NVFP4_BYTE_ACCOUNTING);
    for (uint64_t i = 0; i < len; ++i)  // validate_scale_plane: sign clear, E4M3 finite
      if ((p[i] & 0x80) || p[i] == 0x7f) fail(GLMAXX_RANK_ERR_NVFP4_SCALE_ENCODING);
    std::memcpy(scales.data() + off, p, len);
    scale_seen = off + len;
  }

  void finish() {
    if (value_seen != m->value_bytes || scale_seen != m->scale_bytes)
      fail(GLMAXX_RANK_ERR_NVFP4_BYTE_ACCOUNTING);
    const uint64_t kb = m->padded_k / 64, gk = m->padded_k / 16;
    if (!m->two_d && m->logical_n == m->padded_n && m->logical_k == m->padded_k) {
      // no padding domain and no sharing: only the zero-scale rule can fail
      for (uint64_t o = 0; o < scales.size(); ++o)
        if (scales[o] == 0 && (nonzero[o >> 3] >> (o & 7) & 1))
          fail(GLMAXX_RANK_ERR_NVFP4_ZERO_SCALE_VALUE);
      return;
    }
    for (uint64_t row = 0; row < m->padded_n; ++row)
      for (uint64_t g = 0; g < gk; ++g) {
        const uint64_t o = scale_offset(row, g, kb);
        const uint8_t s = scales[o];
        if (s == 0 && (nonzero[o >> 3] >> (o & 7) & 1)) fail(GLMAXX_RANK_ERR_NVFP4_ZERO_SCALE_VALUE);
        const bool domain = g * 16 < m->logical_k &&
                            (m->two_d ? (row / 16) * 16 < m->logical_n : row < m->logical_n);
        if (!domain && s != 0) fail(GLMAXX_RANK_ERR_NVFP4_NON_CANONICAL_PADDING);
        if (m->two_d && s != scales[scale_offset((row / 16) * 16, g, kb)])
          fail(GLMAXX_RANK_ERR_NVFP4_SCALE_SHARING);
      }
  }
};

// ------------------------------------------------------------ file identity
struct Fingerprint {
  uint64_t dev = 0, ino = 0, size = 0;
  int64_t mtime = 0, mtime_ns = 0, ctime = 0, ctime_ns = 0;
  static Fingerprint of(const struct stat& s) {
    Fingerprint f;
    f.dev = s.st_dev;
    f.ino = s.st_ino;
    f.size = uint64_t(s.st_size);
    f.mtime = s.st_mtim.tv_sec;
    f.mtime_ns = s.st_mtim.tv_nsec;
    f.ctime = s.st_ctim.tv_sec;
    f.ctime_ns = s.st_ctim.tv_nsec;
    return f;
  }
  bool operator==(const Fingerprint& o) const {
    return dev == o.dev && ino == o.ino && size == o.size && mtime == o.mtime &&
           mtime_ns == o.mtime_ns && ctime == o.ctime && ctime_ns == o.ctime_ns;
  }
};

void read_exact_at(int fd, uint8_t* out, uint64_t len, uint64_t off) {
  while (len) {
    const ssize_t r = ::pread(fd, out, len, off_t(off));
    if (r < 0) {
      if (errno == EINTR) continue;
      fail(GLMAXX_RANK_ERR_IO);
    }
    if (r == 0) fail(GLMAXX_RANK_ERR_IO);  // unexpected end of file
    out += r;
    off += uint64_t(r);
    len -= uint64_t(r);
  }
}

// Strict UTF-8 (no overlong forms, surrogates or code points above U+10FFFF).
bool valid_utf8(const uint8_t* p, size_t n) {
  size_t i = 0;
  while (i < n) {
    const uint8_t c = p[i];
    if (c < 0x80) {
      ++i;
      continue;
    }
    size_t len;
    uint32_t cp, min;
    if ((c & 0xE0) == 0xC0) {
      len = 2, cp = c & 0x1F, min = 0x80;
    } else if ((c & 0xF0) == 0xE0) {
      len = 3, cp = c & 0x0F, min = 0x800;
    } else if ((c & 0xF8) == 0xF0) {
      len = 4, cp = c & 0x07, min = 0x10000;
    } else {
      return false;
    }
    if (i + len > n) return false;
    for (size_t j = 1; j < len; ++j) {
      if ((p[i + j] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (p[i + j] & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += len;
  }
  return true;
}

// Stream staging kept with the file handle between loads: kSlots chunk
// buffers (pinned once a device load has run), their copy-done events and the
// pinned NVFP4 global-scale words.  Loads on one handle take its mutex.
struct Staging {
  std::mutex mu;
  bool pinned = false;
  int device = -1;  // device of the events (pinned staging only)
  uint8_t* slot[kSlots] = {};
  cudaEvent_t done[kSlots] = {};
  float* scales = nullptr;
  size_t scales_n = 0;

  ~Staging() { release(); }
  void release() {
    for (int i = 0; i < kSlots; ++i) {
      if (done[i]) cudaEventDestroy(done[i]);
      if (slot[i]) {
        if (pinned)
          cudaFreeHost(slot[i]);
        else
          std::free(slot[i]);
      }
      done[i] = nullptr;
      slot[i] = nullptr;
    }
    if (scales) cudaFreeHost(scales);
    scales = nullptr;
    scales_n = 0;
    pinned = false;
    device = -1;
  }
  // Chunk buffers for a load; pinned ones (and events, scale words) when the
  // load copies to device dev.  Events belong to one device, so staging made
  // for another device is rebuilt.
  void ensure(bool to_device, int dev, size_t tensors) {
    if (to_device && (!pinned || device != dev)) release();
    for (int i = 0; i < kSlots; ++i) {
      if (slot[i]) continue;
      if (to_device) {
        if (const cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&slot[i]), kChunkBytes,
                                                cudaHostAllocDefault))
          fail(int32_t(e));
        if (const cudaError_t e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming))
          fail(int32_t(e));
      } else {
        slot[i] = static_cast<uint8_t*>(std::aligned_alloc(4096, kChunkBytes));
        if (!slot[i]) fail(GLMAXX_RANK_ERR_NVFP4_ALLOCATION);
      }
    }
    if (to_device) {
      pinned = true;
      device = dev;
    }
    if (to_device && scales_n < tensors) {
      if (scales) cudaFreeHost(scales);
      scales = nullptr;
      if (const cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&scales),
                                              tensors * sizeof(float), cudaHostAllocDefault))
        fail(int32_t(e));
      scales_n = tensors;
    }
  }
};

}  // namespace
}  // namespace glmaxx::rankfile

using namespace glmaxx::rankfile;

struct glmaxx_rank_file {
  std::string path;
  int fd = -1;
  Fingerprint fingerprint;
  uint8_t header[kHeaderBytes];
  uint32_t rank = 0, header_flags = 0;
  uint64_t file_bytes = 0;
  Region manifest, descriptor, strings, metadata, payload;
  std::vector<Descriptor> d;
  std::vector<std::string> names;
  std::vector<uint8_t> metadata_bytes;
  std::vector<uint8_t> manifest_bytes;
  std::vector<Nvfp4Meta> nv;
  std::vector<Exl3Meta> ex;
  mutable Staging staging;

  ~glmaxx_rank_file() {
    if (fd >= 0) ::close(fd);
  }

  const uint8_t* codec_metadata(size_t i) const {
    return metadata_bytes.data() + (d[i].codec_metadata_offset - metadata.start);
  }

  // ensure_unchanged (native_reader.rs:590-604)
  void ensure_unchanged() const {
    struct stat open_stat, path_stat;
    if (::fstat(fd, &open_stat) != 0 || ::lstat(path.c_str(), &path_stat) != 0)
      fail(GLMAXX_RANK_ERR_IO);
    if (S_ISLNK(path_stat.st_mode) || !S_ISREG(path_stat.st_mode) || path_stat.st_nlink != 1 ||
        !(Fingerprint::of(open_stat) == fingerprint) || !(Fingerprint::of(path_stat) == fingerprint))
      fail(GLMAXX_RANK_ERR_CHANGED);
  }

  Region header_region(size_t offset_field, size_t length_field) const {
    const uint64_t start = get_u64(header, offset_field), bytes = get_u64(header, length_field);
    const uint64_t end = add(start, bytes);
    if (start % kAlignment || start > end || end > file_bytes) fail(GLMAXX_RANK_ERR_REGION);
    return Region{start, end};
  }

  std::vector<uint8_t> read_control(Region r) const {
    if (r.len() > kControlRegionMax) fail(GLMAXX_RANK_ERR_REGION);
    std::vector<uint8_t> bytes(r.len());
    read_exact_at(fd, bytes.data(), bytes.size(), r.start);
    return bytes;
  }

  void verify_zero_gap(uint64_t start, uint64_t end) const {
    if (start > end || end - start >= kAlignment) fail(GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT);
    uint8_t gap[kAlignment];
    read_exact_at(fd, gap, end - start, start);
    if (!all_zero(gap, end - start)) fail(GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT);
  }

  // checked_subregion (native_reader.rs:1061-1072)
  static Region subregion(uint64_t start, uint64_t bytes, Region parent, uint64_t file_bytes) {
    const uint64_t end = add(start, bytes);
    if (end > file_bytes || start < parent.start || end > parent.end) fail(GLMAXX_RANK_ERR_REGION);
    return Region{start, end};
  }

  void open(const char* p);
  void validate_descriptors();
};

// NativeRankReader::open (native_reader.rs:119-335)
void glmaxx_rank_file::open(const char* p) {
  path = p;
  struct stat path_stat, open_stat;
  if (::lstat(p, &path_stat) != 0) fail(GLMAXX_RANK_ERR_IO);
  if (!S_ISREG(path_stat.st_mode) || S_ISLNK(path_stat.st_mode) || path_stat.st_nlink != 1)
    fail(GLMAXX_RANK_ERR_UNSAFE_FILE);
  fd = ::open(p, O_RDONLY | O_CLOEXEC | O_NOFOLLOW);
  if (fd < 0) fail(GLMAXX_RANK_ERR_IO);
  if (::fstat(fd, &open_stat) != 0) fail(GLMAXX_RANK_ERR_IO);
  if (!S_ISREG(open_stat.st_mode) || open_stat.st_nlink != 1) fail(GLMAXX_RANK_ERR_UNSAFE_FILE);
  fingerprint = Fingerprint::of(open_stat);
  if (!(fingerprint == Fingerprint::of(path_stat))) fail(GLMAXX_RANK_ERR_CHANGED);
  file_bytes = uint64_t(open_stat.st_size);
  if (file_bytes < kHeaderBytes) fail(GLMAXX_RANK_ERR_TRUNCATED);

  read_exact_at(fd, header, kHeaderBytes, 0);
  header_flags = get_u32(header, 20);
  if (std::memcmp(header, "GLM5NAT0", 8) || get_u16(header, 8) != 0 || get_u16(header, 10) != 2 ||
      get_u32(header, 12) != kHeaderBytes || get_u32(header, 16) != 0x01020304u ||
      (header_flags & ~0x1Fu) || get_u32(header, 28) != 4 || !all_zero(header + 36, 4) ||
      get_u64(header, 408) != 0 || !all_zero(header + 484, kHeaderBytes - 484))
    fail(GLMAXX_RANK_ERR_HEADER);
  uint8_t checked[kHeaderBytes];
  std::memcpy(checked, header, kHeaderBytes);
  std::memset(checked + 416, 0, 4);
  if (crc32c(checked, kHeaderBytes) != get_u32(header, 416)) fail(GLMAXX_RANK_ERR_HEADER_CRC);
  rank = get_u32(header, 24);
  if (rank > 3) fail(GLMAXX_RANK_ERR_RANK);
  const uint32_t tensor_count = get_u32(header, 32);
  if (tensor_count == 0) fail(GLMAXX_RANK_ERR_TENSOR_COUNT);

  manifest = header_region(40, 48);
  descriptor = header_region(56, 64);
  strings = header_region(72, 80);
  metadata = header_region(88, 96);
  payload = header_region(104, 112);
  const uint64_t control =
      add(add(add(manifest.len(), descriptor.len()), strings.len()), metadata.len());
  const uint64_t expected_descriptor_bytes = mul(tensor_count, kDescriptorBytes);
  if (descriptor.len() != expected_descriptor_bytes || control > kControlTotalMax ||
      manifest.start != kAlignment || descriptor.start != align_up(manifest.end, kAlignment) ||
      strings.start != align_up(descriptor.end, kAlignment) ||
      metadata.start != align_up(strings.end, kAlignment) ||
      payload.start != align_up(metadata.end, kAlignment) || payload.end != file_bytes)
    fail(GLMAXX_RANK_ERR_REGION);

  manifest_bytes = read_control(manifest);
  const std::vector<uint8_t> descriptor_bytes = read_control(descriptor);
  const std::vector<uint8_t> string_bytes = read_control(strings);
  metadata_bytes = read_control(metadata);
  verify_zero_gap(manifest.end, descriptor.start);
  verify_zero_gap(descriptor.end, strings.start);
  verify_zero_gap(strings.end, metadata.start);
  verify_zero_gap(metadata.end, payload.start);

  uint8_t h[32];
  bool ok = true;
  sha256(manifest_bytes.data(), manifest_bytes.size(), h);
  ok &= !std::memcmp(h, header + 280, 32);
  sha256(descriptor_bytes.data(), descriptor_bytes.size(), h);
  ok &= !std::memcmp(h, header + 312, 32);
  sha256(string_bytes.data(), string_bytes.size(), h);
  ok &= !std::memcmp(h, header + 420, 32);
  sha256(metadata_bytes.data(), metadata_bytes.size(), h);
  ok &= !std::memcmp(h, header + 452, 32);
  if (!ok) fail(GLMAXX_RANK_ERR_STRONG_HASH);

  d.reserve(tensor_count);
  names.reserve(tensor_count);
  uint64_t name_cursor = 0;
  for (uint32_t i = 0; i < tensor_count; ++i) {
    const Descriptor dd = decode_descriptor(descriptor_bytes.data() + uint64_t(i) * kDescriptorBytes);
    if (dd.tensor_id != i || dd.name_bytes == 0 || dd.name_offset != name_cursor)
      fail(GLMAXX_RANK_ERR_TENSOR_ID);
    const uint64_t name_end = name_cursor + dd.name_bytes;
    if (name_end > string_bytes.size()) fail(GLMAXX_RANK_ERR_STRING_TABLE);
    const uint8_t* name = string_bytes.data() + name_cursor;
    if (!valid_utf8(name, dd.name_bytes)) fail(GLMAXX_RANK_ERR_STRING_TABLE);
    for (uint16_t j = 0; j < dd.name_bytes; ++j)
      if (name[j] < 0x20 || name[j] == 0x7f) fail(GLMAXX_RANK_ERR_STRING_TABLE);
    names.emplace_back(reinterpret_cast<const char*>(name), dd.name_bytes);
    name_cursor = name_end;
    d.push_back(dd);
  }
  if (name_cursor != string_bytes.size()) fail(GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT);

  validate_descriptors();

  // derive_header_flags (container.rs:816-844)
  bool saw_plain = false, saw_nvfp4 = false, saw_exl3 = false;
  for (const Descriptor& dd : d) {
    saw_plain |= is_plain(dd.codec_id);
    saw_nvfp4 |= is_nvfp4(dd.codec_id);
    saw_exl3 |= dd.codec_id == GLMAXX_CODEC_EXL3_SOURCE;
  }
  uint32_t flags = 0;
  if ((saw_plain || saw_nvfp4) && !saw_exl3) flags |= GLMAXX_RANK_FLAG_DIRECT_KERNEL;
  if (saw_nvfp4) flags |= GLMAXX_RANK_FLAG_NVFP4;
  if (saw_exl3) flags |= GLMAXX_RANK_FLAG_EXL3;
  if (saw_nvfp4 && saw_exl3) flags |= GLMAXX_RANK_FLAG_HYBRID;
  if (flags != header_flags) fail(GLMAXX_RANK_ERR_HEADER_FLAGS);

  // file_uuid = SHA256("g5n-file-v0\0" || conversion_uuid || rank || manifest, descriptor,
  // payload digests)[:16] (format-v0.md section 5.1)
  Sha256 s;
  s.update("g5n-file-v0", 12);
  s.update(header + 392, 16);
  const uint32_t rank_le = rank;
  s.update(&rank_le, 4);
  s.update(header + 280, 32);
  s.update(header + 312, 32);
  s.update(header + 344, 32);
  s.finish(h);
  if (std::memcmp(h, header + 376, 16)) fail(GLMAXX_RANK_ERR_FILE_UUID);
  ensure_unchanged();
}

// validate_descriptors (native_reader.rs:724-858)
void glmaxx_rank_file::validate_descriptors() {
  uint64_t metadata_cursor = metadata.start, payload_cursor = payload.start;
  nv.assign(d.size(), Nvfp4Meta{});
  ex.assign(d.size(), Exl3Meta{});
  for (size_t i = 0; i < d.size(); ++i) {
    const Descriptor& dd = d[i];
    const Region meta =
        subregion(dd.codec_metadata_offset, dd.codec_metadata_bytes, metadata, file_bytes);
    if (meta.start != metadata_cursor) fail(GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT);
    metadata_cursor = meta.end;
    const uint8_t* cm = metadata_bytes.data() + (meta.start - metadata.start);
    uint8_t h[32];
    sha256(cm, meta.len(), h);
    if (std::memcmp(h, dd.codec_metadata_sha256, 32)) fail(GLMAXX_RANK_ERR_TENSOR_REGION);

    const Region primary = subregion(dd.payload_offset, dd.payload_bytes, payload, file_bytes);
    const uint64_t expected_primary = align_up(payload_cursor, kPayloadAlignment);
    const Region aux = subregion(dd.aux_offset, dd.aux_bytes, payload, file_bytes);
    const uint64_t expected_aux = align_up(primary.end, kPayloadAlignment);
    if (primary.start != expected_primary || aux.start != expected_aux)
      fail(GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT);
    payload_cursor = aux.end;

    if (is_plain(dd.codec_id)) {
      const uint16_t dtype = dd.codec_id;  // dtype ids 1/2/3 equal the codec ids
      if (dd.logical_dtype != dtype || dd.stored_dtype != dtype ||
          (dd.flags & kDescriptorAuxRequired) || dd.quant_group_elements != 0 ||
          dd.aux_bytes != 0 || dd.codec_metadata_bytes != 0)
        fail(GLMAXX_RANK_ERR_DESCRIPTOR);
      validate_plain_geometry(dd.codec_id, dd, dd.payload_bytes);
    } else if (is_nvfp4(dd.codec_id)) {
      const Nvfp4Meta m = nvfp4_decode(cm, meta.len());
      if (dd.logical_dtype != 1 || dd.stored_dtype != 6 || dd.ndim != 2 ||
          !(dd.flags & kDescriptorAuxRequired) || dd.payload_alignment != kPayloadAlignment ||
          dd.quant_group_elements != 16 || m.logical_n != dd.logical_shape[0] ||
          m.logical_k != dd.logical_shape[1] || m.padded_n != dd.padded_shape[0] ||
          m.padded_k != dd.padded_shape[1] ||
          (m.two_d ? GLMAXX_CODEC_NVFP4_2D : GLMAXX_CODEC_NVFP4_1D) != dd.codec_id ||
          m.value_bytes != dd.payload_bytes || m.scale_bytes != dd.aux_bytes)
        fail(GLMAXX_RANK_ERR_DESCRIPTOR);
      nv[i] = m;
    } else if (dd.codec_id == GLMAXX_CODEC_EXL3_SOURCE) {
      const Exl3Meta m = exl3_decode(cm, meta.len());
      if (dd.layer_id < 0 || dd.expert_id < 0) fail(GLMAXX_RANK_ERR_DESCRIPTOR);
      if (m.trellis_words > UINT64_MAX / 2 || m.rotation_words > (UINT64_MAX - 4) / 2)
        fail(GLMAXX_RANK_ERR_OVERFLOW);
      if (dd.logical_dtype != 2 || dd.stored_dtype != 10 || dd.ndim != 2 ||
          !(dd.flags & kDescriptorAuxRequired) || dd.payload_alignment != kPayloadAlignment ||
          dd.quant_group_elements != 0 || m.rank != rank || m.layer != uint16_t(dd.layer_id) ||
          m.expert != uint16_t(dd.expert_id) || m.logical_n != dd.logical_shape[0] ||
          m.logical_k != dd.logical_shape[1] ||
          std::memcmp(dd.logical_shape, dd.padded_shape, sizeof(dd.logical_shape)) ||
          dd.payload_bytes != m.trellis_words * 2 || dd.aux_bytes != m.rotation_words * 2 + 4)
        fail(GLMAXX_RANK_ERR_DESCRIPTOR);
      ex[i] = m;
    } else {
      fail(GLMAXX_RANK_ERR_UNSUPPORTED_CODEC);
    }
  }
  if (metadata_cursor != metadata.end || payload_cursor != payload.end)
    fail(GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT);
}

// ============================================================ streaming
namespace {

void fill_tensor_info(const glmaxx_rank_file& f, size_t index, glmaxx_rank_tensor_info* out) {
  const Descriptor& d = f.d[index];
  std::memset(out, 0, sizeof(*out));
  out->tensor_id = d.tensor_id;
  out->role_id = d.role_id;
  out->layer_id = d.layer_id;
  out->expert_id = d.expert_id;
  out->codec_id = d.codec_id;
  out->logical_dtype = d.logical_dtype;
  out->stored_dtype = d.stored_dtype;
  out->tp_shard_axis = d.tp_shard_axis;
  out->ndim = d.ndim;
  out->flags = d.flags;
  out->exl3_projection = d.codec_id == GLMAXX_CODEC_EXL3_SOURCE ? f.ex[index].projection : 0;
  std::memcpy(out->logical_shape, d.logical_shape, sizeof(d.logical_shape));
  std::memcpy(out->padded_shape, d.padded_shape, sizeof(d.padded_shape));
  out->payload_offset = d.payload_offset;
  out->payload_bytes = d.payload_bytes;
  out->aux_offset = d.aux_offset;
  out->aux_bytes = d.aux_bytes;
  out->codec_metadata_offset = d.codec_metadata_offset;
  out->codec_metadata_bytes = d.codec_metadata_bytes;
  out->payload_alignment = d.payload_alignment;
  out->quant_group_elements = d.quant_group_elements;
  if (is_nvfp4(d.codec_id)) {
    out->global_scale = f.nv[index].global_scale;
    out->global_amax = f.nv[index].global_amax;
  }
  out->name = f.names[index].data();
  out->name_bytes = uint32_t(f.names[index].size());
}

int32_t cuda_code(cudaError_t e) { return e == cudaSuccess ? 0 : int32_t(e); }

struct Slot {
  uint8_t* data = nullptr;
  uint64_t start = 0, len = 0;  // file range held
  int pending = 0;              // consumers still to release the slot
  bool copies = false;          // device copies issued from this slot
  cudaEvent_t done = nullptr;
};

// One tensor's streaming state, owned by the plane worker t % P.
struct TensorWork {
  uint64_t begin = 0;  // extent start: end of the previous tensor's aux plane
  bool started = false;
  Sha256 primary_hash, aux_hash;
  Nvfp4Check nvfp4;
  bool exl3_marker_ok = true, exl3_finite = true;
  int stage = 0;  // 0 gap before, 1 primary, 2 gap between, 3 aux, 4 done
};

class Loader {
 public:
  Loader(const glmaxx_rank_file& f, const glmaxx_rank_placement* placements, uint32_t count,
         uint32_t flags, cudaStream_t stream, const glmaxx_rank_sink* sink = nullptr)
      : f_(f), stream_(stream), host_(flags & GLMAXX_RANK_LOAD_HOST_DESTINATIONS), sink_(sink) {
    const size_t n = f.d.size();
    place_.assign(n, nullptr);
    for (uint32_t i = 0; i < count; ++i) {
      const glmaxx_rank_placement& p = placements[i];
      if (p.tensor_index >= n || place_[p.tensor_index]) fail(GLMAXX_RANK_ERR_ARGUMENT);
      const uint16_t codec = f.d[p.tensor_index].codec_id;
      if (codec == GLMAXX_CODEC_EXL3_SOURCE && !(flags & GLMAXX_RANK_LOAD_EXL3_SOURCE) &&
          (p.dst[0] || p.dst[1] || p.dst[2]))
        fail(GLMAXX_RANK_ERR_ARGUMENT);
      if (is_plain(codec) && (p.dst[1] || p.dst[2])) fail(GLMAXX_RANK_ERR_ARGUMENT);
      // every destination holds its whole plane
      const Descriptor& d = f.d[p.tensor_index];
      uint64_t need[3] = {d.payload_bytes, 0, 0};
      if (is_nvfp4(codec)) {
        need[1] = d.aux_bytes;
        need[2] = 4;
      } else if (codec == GLMAXX_CODEC_EXL3_SOURCE) {
        need[1] = 2ull * f.ex[p.tensor_index].logical_k;
        need[2] = 2ull * f.ex[p.tensor_index].logical_n;
      }
      for (int j = 0; j < 3; ++j)
        if (p.dst[j] && p.dst_bytes[j] < need[j]) fail(GLMAXX_RANK_ERR_ARGUMENT);
      place_[p.tensor_index] = &p;
      device_ |= !host_ && (p.dst[0] || p.dst[1] || p.dst[2]);
    }
    work_.resize(n);
    uint64_t cursor = f.payload.start;
    for (size_t t = 0; t < n; ++t) {
      work_[t].begin = cursor;
      cursor = f.d[t].aux_offset + f.d[t].aux_bytes;
    }
    error_tensor_.store(n);
    tensor_error_.assign(n, 0);
  }

  ~Loader() = default;

  void run(glmaxx_rank_payload_proof* proof);

 private:
  void copy(uint64_t dst, const uint8_t* src, uint64_t len) {
    if (!dst || !len) return;
    if (host_) {
      std::memcpy(reinterpret_cast<void*>(dst), src, len);
    } else {
      const int32_t e = cuda_code(
          cudaMemcpyAsync(reinterpret_cast<void*>(dst), src, len, cudaMemcpyHostToDevice, stream_));
      if (e) fail(e);
    }
    device_bytes_.fetch_add(len, std::memory_order_relaxed);
  }

  void process(size_t t, const uint8_t* chunk, uint64_t c0, uint64_t c1, bool* copied);
  void finish_tensor(size_t t);
  void whole_worker();
  void plane_worker(int w);
  void release(Slot& s, bool copied);

  const glmaxx_rank_file& f_;
  cudaStream_t stream_;
  bool host_;
  const glmaxx_rank_sink* sink_;
  bool device_ = false;
  int device_id_ = 0;
  std::vector<const glmaxx_rank_placement*> place_;
  std::vector<TensorWork> work_;
  std::vector<int32_t> tensor_error_;
  std::atomic<size_t> error_tensor_{0};
  std::atomic<int32_t> fatal_{0};  // I/O or CUDA failure: stop everything
  std::atomic<uint64_t> device_bytes_{0};
  float* scales_host_ = nullptr;

  Slot slots_[kSlots];
  std::mutex mu_;
  std::condition_variable cv_;
  uint64_t published_ = 0;  // chunks made available
  bool eof_ = false;
  int consumers_ = 0;
  int workers_ = 1;
  Sha256 whole_;
  std::vector<uint64_t> scratch_;
};

void Loader::process(size_t t, const uint8_t* chunk, uint64_t c0, uint64_t c1, bool* copied) {
  const Descriptor& d = f_.d[t];
  TensorWork& w = work_[t];
  const glmaxx_rank_placement* p = place_[t];
  const uint64_t pe = d.payload_offset + d.payload_bytes, ae = d.aux_offset + d.aux_bytes;
  const uint64_t bounds[5] = {w.begin, d.payload_offset, pe, d.aux_offset, ae};
  while (w.stage < 4) {
    const uint64_t s0 = bounds[w.stage], s1 = bounds[w.stage + 1];
    const uint64_t a = std::max(s0, c0), b = std::min(s1, c1);
    if (a < b) {
      const uint8_t* q = chunk + (a - c0);
      const uint64_t len = b - a;
      switch (w.stage) {
        case 0:
        case 2:  // stream_padding (native_reader.rs:1011-1038)
          if (!all_zero(q, len)) fail(GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT);
          break;
        case 1: {
          const uint64_t off = a - d.payload_offset;
          validate_plain_padding_chunk(d, q, len, off);
          if (is_nvfp4(d.codec_id)) w.nvfp4.value_chunk(q, len, off);
          w.primary_hash.update(q, len);
          if (sink_ && sink_->primary_chunk && sink_->primary_chunk(sink_->user, q, len))
            fail(GLMAXX_RANK_ERR_SINK);
          if (p && p->dst[0]) {
            copy(p->dst[0] + off, q, len);
            *copied = true;
          }
          break;
        }
        case 3: {
          const uint64_t off = a - d.aux_offset;
          if (is_nvfp4(d.codec_id)) {
            w.nvfp4.scale_chunk(q, len, off);
            if (p && p->dst[1]) {
              copy(p->dst[1] + off, q, len);
              *copied = true;
            }
          } else if (d.codec_id == GLMAXX_CODEC_EXL3_SOURCE) {
            // aux plane = mcg marker u32 || suh[K] || svh[N] (exl3.rs:229-281)
            const Exl3Meta& m = f_.ex[t];
            uint64_t i = 0;
            if (off == 0) {
              w.exl3_marker_ok = get_u32(q, 0) == kMcgMultiplier;
              i = 4;
            }
            for (; i + 1 < len; i += 2)
              if ((get_u16(q, i) & 0x7c00) == 0x7c00) w.exl3_finite = false;
            if (p) {
              const uint64_t suh0 = 4, suh1 = 4 + 2ull * m.logical_k, svh1 = suh1 + 2ull * m.logical_n;
              const uint64_t x0 = std::max(off, suh0), x1 = std::min(off + len, suh1);
              if (x0 < x1 && p->dst[1]) copy(p->dst[1] + (x0 - suh0), q + (x0 - off), x1 - x0);
              const uint64_t y0 = std::max(off, suh1), y1 = std::min(off + len, svh1);
              if (y0 < y1 && p->dst[2]) copy(p->dst[2] + (y0 - suh1), q + (y0 - off), y1 - y0);
              *copied |= (x0 < x1 && p->dst[1]) || (y0 < y1 && p->dst[2]);
            }
          }
          w.aux_hash.update(q, len);
          if (sink_ && sink_->aux_chunk && sink_->aux_chunk(sink_->user, q, len))
            fail(GLMAXX_RANK_ERR_SINK);
          break;
        }
      }
    }
    if (c1 < s1) return;  // the stage continues in the next chunk
    // the stage is complete
    uint8_t h[32];
    if (w.stage == 1) {
      w.primary_hash.finish(h);
      if (std::memcmp(h, d.payload_sha256, 32)) fail(GLMAXX_RANK_ERR_TENSOR_REGION);
    } else if (w.stage == 3) {
      w.aux_hash.finish(h);
      if (std::memcmp(h, d.aux_sha256, 32)) fail(GLMAXX_RANK_ERR_TENSOR_REGION);
      finish_tensor(t);
      if (sink_ && sink_->finish_tensor && sink_->finish_tensor(sink_->user))
        fail(GLMAXX_RANK_ERR_SINK);
    }
    ++w.stage;
  }
}

void Loader::finish_tensor(size_t t) {
  const Descriptor& d = f_.d[t];
  TensorWork& w = work_[t];
  if (d.codec_id == GLMAXX_CODEC_EXL3_SOURCE) {
    exl3_validate(f_.ex[t]);
    if (!w.exl3_marker_ok) fail(GLMAXX_RANK_ERR_EXL3_CODEBOOK_MARKER);
    if (!w.exl3_finite) fail(GLMAXX_RANK_ERR_EXL3_NON_FINITE_ROTATION);
  } else if (is_nvfp4(d.codec_id)) {
    w.nvfp4.finish();
    std::vector<uint8_t>().swap(w.nvfp4.nonzero);
    std::vector<uint8_t>().swap(w.nvfp4.scales);
  }
}

void Loader::release(Slot& s, bool copied) {
  std::unique_lock<std::mutex> lock(mu_);
  s.copies |= copied && !host_;  // host destinations are complete when memcpy returns
  if (--s.pending == 0) {
    if (s.copies && !host_) {
      const cudaError_t e = cudaEventRecord(s.done, stream_);
      if (e != cudaSuccess) fatal_.store(int32_t(e));
    }
    cv_.notify_all();
  }
}

void Loader::whole_worker() {
  // it may be a chunk's last consumer, which records the copy event: same device
  if (device_)
    if (const cudaError_t e = cudaSetDevice(device_id_)) fatal_.store(int32_t(e));
  for (uint64_t k = 0;; ++k) {
    Slot* s;
    {
      std::unique_lock<std::mutex> lock(mu_);
      cv_.wait(lock, [&] { return published_ > k || eof_; });
      if (published_ <= k) return;
      s = &slots_[k % kSlots];
    }
    whole_.update(s->data, s->len);
    release(*s, false);
  }
}

void Loader::plane_worker(int wi) {
  if (device_)
    if (const cudaError_t e = cudaSetDevice(device_id_)) fatal_.store(int32_t(e));
  const size_t n = f_.d.size();
  size_t next = size_t(wi);  // this worker's next unfinished tensor
  uint64_t peak = 0;
  for (uint64_t k = 0;; ++k) {
    Slot* s;
    {
      std::unique_lock<std::mutex> lock(mu_);
      cv_.wait(lock, [&] { return published_ > k || eof_; });
      if (published_ <= k) break;
      s = &slots_[k % kSlots];
    }
    bool copied = false;
    const uint64_t c0 = s->start, c1 = s->start + s->len;
    for (size_t t = next; t < n && fatal_.load() == 0; t += size_t(workers_)) {
      const uint64_t end = f_.d[t].aux_offset + f_.d[t].aux_bytes;
      if (work_[t].begin >= c1) break;
      if (tensor_error_[t] == 0 && t < error_tensor_.load()) {
        try {
          if (!work_[t].started) {  // the first chunk of this tensor's extent
            work_[t].started = true;
            if (is_nvfp4(f_.d[t].codec_id)) {
              work_[t].nvfp4.begin(f_.nv[t]);
              peak = std::max(peak, work_[t].nvfp4.scratch());
            }
            if (sink_ && sink_->begin_tensor) {
              glmaxx_rank_tensor_info info;
              fill_tensor_info(f_, t, &info);
              if (sink_->begin_tensor(sink_->user, f_.rank, uint32_t(t), &info))
                fail(GLMAXX_RANK_ERR_SINK);
            }
          }
          process(t, s->data, c0, c1, &copied);
        } catch (const std::bad_alloc&) {
          fatal_.store(GLMAXX_RANK_ERR_NVFP4_ALLOCATION);
        } catch (const Fail& e) {
          if (e.code > 0) {
            fatal_.store(e.code);
          } else {
            tensor_error_[t] = e.code;
            size_t cur = error_tensor_.load();
            while (t < cur && !error_tensor_.compare_exchange_weak(cur, t)) {
            }
          }
        }
      }
      if (end <= c1) next = t + size_t(workers_);
      else break;
    }
    release(*s, copied);
  }
  std::lock_guard<std::mutex> lock(mu_);
  scratch_.push_back(peak);
}

void Loader::run(glmaxx_rank_payload_proof* proof) {
  using clock = std::chrono::steady_clock;
  const auto t_start = clock::now();
  f_.ensure_unchanged();
  const size_t n = f_.d.size();
  std::unique_lock<std::mutex> staging_lock(f_.staging.mu);
  if (device_) {
    if (const int32_t e = cuda_code(cudaGetDevice(&device_id_))) fail(e);
  }
  f_.staging.ensure(device_, device_id_, n);
  for (int i = 0; i < kSlots; ++i) {
    slots_[i].data = f_.staging.slot[i];
    slots_[i].done = f_.staging.done[i];
  }
  scales_host_ = f_.staging.scales;
  // NVFP4 global scales first: kernel-consumed control values (format-v0.md section 15)
  for (size_t t = 0; t < n; ++t)
    if (place_[t] && is_nvfp4(f_.d[t].codec_id) && place_[t]->dst[2]) {
      if (host_) {
        copy(place_[t]->dst[2], reinterpret_cast<const uint8_t*>(&f_.nv[t].global_scale), 4);
      } else {
        scales_host_[t] = f_.nv[t].global_scale;
        copy(place_[t]->dst[2], reinterpret_cast<const uint8_t*>(scales_host_ + t), 4);
      }
    }

  const unsigned hw = std::max(2u, std::thread::hardware_concurrency());
  // a caller sink sees one tensor at a time, in order: one plane worker
  workers_ = sink_ ? 1 : int(std::min<size_t>(std::max<size_t>(1, std::min<unsigned>(hw - 2, 8)), n));
  consumers_ = workers_ + 1;
  std::vector<std::thread> threads;
  threads.emplace_back([this] { whole_worker(); });
  for (int w = 0; w < workers_; ++w) threads.emplace_back([this, w] { plane_worker(w); });

  uint64_t read_ns = 0, chunks = 0;
  int32_t read_error = 0;
  uint64_t stop_at = f_.payload.end;
  for (uint64_t pos = f_.payload.start, k = 0; pos < stop_at; pos += kChunkBytes, ++k) {
    Slot& s = slots_[k % kSlots];
    {
      std::unique_lock<std::mutex> lock(mu_);
      cv_.wait(lock, [&] { return s.pending == 0; });
    }
    if (s.copies) {
      const cudaError_t e = cudaEventSynchronize(s.done);
      if (e != cudaSuccess) {
        read_error = int32_t(e);
        break;
      }
      s.copies = false;
    }
    if (fatal_.load()) break;
    const size_t et = error_tensor_.load();
    if (et < n && pos >= f_.d[et].aux_offset + f_.d[et].aux_bytes) break;  // earliest error known
    const uint64_t len = std::min(kChunkBytes, f_.payload.end - pos);
    const auto r0 = clock::now();
    try {
      read_exact_at(f_.fd, s.data, len, pos);
    } catch (const Fail& e) {
      read_error = e.code;
      break;
    }
    read_ns += uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(clock::now() - r0).count());
    {
      std::lock_guard<std::mutex> lock(mu_);
      s.start = pos;
      s.len = len;
      s.pending = consumers_;
      ++published_;
      ++chunks;
    }
    cv_.notify_all();
  }
  {
    std::lock_guard<std::mutex> lock(mu_);
    eof_ = true;
  }
  cv_.notify_all();
  for (std::thread& th : threads) th.join();
  if (device_) {
    const cudaError_t e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess && !read_error) read_error = int32_t(e);
  }
  if (read_error) fail(read_error);
  if (const int32_t e = fatal_.load()) fail(e);
  const size_t et = error_tensor_.load();
  if (et < n) fail(tensor_error_[et]);
  for (size_t t = 0; t < n; ++t)
    if (work_[t].stage != 4) fail(GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT);
  uint8_t digest[32];
  whole_.finish(digest);
  if (std::memcmp(digest, f_.header + 344, 32)) fail(GLMAXX_RANK_ERR_STRONG_HASH);
  f_.ensure_unchanged();
  if (proof) {
    std::memset(proof, 0, sizeof(*proof));
    proof->rank = f_.rank;
    proof->tensor_count = uint32_t(n);
    proof->payload_bytes = f_.payload.len();
    std::memcpy(proof->payload_sha256, digest, 32);
    proof->stream_chunks = chunks;
    uint64_t scratch = kSlots * kChunkBytes;
    for (uint64_t s : scratch_) scratch += s;
    proof->maximum_reader_scratch_bytes = scratch;
    proof->storage_read_nanoseconds = read_ns;
    proof->device_bytes = device_bytes_.load();
    proof->elapsed_nanoseconds =
        uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(clock::now() - t_start).count());
  }
}

template <typename F>
int32_t guarded(F&& f) {
  try {
    f();
    return GLMAXX_RANK_OK;
  } catch (const Fail& e) {
    return e.code;
  } catch (const std::bad_alloc&) {
    return GLMAXX_RANK_ERR_NVFP4_ALLOCATION;
  }
}

}  // namespace

extern "C" {

int32_t glmaxx_rank_file_open(const char* path, glmaxx_rank_file** out) {
  if (!path || !out) return GLMAXX_RANK_ERR_NULL;
  *out = nullptr;
  std::unique_ptr<glmaxx_rank_file> f(new glmaxx_rank_file());
  const int32_t r = guarded([&] { f->open(path); });
  if (r == GLMAXX_RANK_OK) *out = f.release();
  return r;
}

void glmaxx_rank_file_close(glmaxx_rank_file* file) { delete file; }

int32_t glmaxx_rank_file_info_get(const glmaxx_rank_file* f, glmaxx_rank_file_info* out) {
  if (!f || !out) return GLMAXX_RANK_ERR_NULL;
  std::memset(out, 0, sizeof(*out));
  out->rank = f->rank;
  out->tensor_count = uint32_t(f->d.size());
  out->header_flags = f->header_flags;
  out->file_bytes = f->file_bytes;
  out->payload_offset = f->payload.start;
  out->payload_bytes = f->payload.len();
  std::memcpy(out->conversion_uuid, f->header + 392, 16);
  std::memcpy(out->file_uuid, f->header + 376, 16);
  std::memcpy(out->model_config_sha256, f->header + 120, 32);
  std::memcpy(out->tokenizer_bundle_sha256, f->header + 152, 32);
  std::memcpy(out->chat_template_sha256, f->header + 184, 32);
  std::memcpy(out->weight_policy_sha256, f->header + 216, 32);
  std::memcpy(out->kernel_abi_sha256, f->header + 248, 32);
  std::memcpy(out->manifest_sha256, f->header + 280, 32);
  std::memcpy(out->descriptor_sha256, f->header + 312, 32);
  std::memcpy(out->payload_sha256, f->header + 344, 32);
  return GLMAXX_RANK_OK;
}

int32_t glmaxx_rank_file_tensor(const glmaxx_rank_file* f, uint32_t index,
                                glmaxx_rank_tensor_info* out) {
  if (!f || !out) return GLMAXX_RANK_ERR_NULL;
  if (index >= f->d.size()) return GLMAXX_RANK_ERR_TENSOR_ID;
  fill_tensor_info(*f, index, out);
  return GLMAXX_RANK_OK;
}

int32_t glmaxx_rank_file_codec_metadata(const glmaxx_rank_file* f, uint32_t index,
                                        const uint8_t** bytes, uint64_t* length) {
  if (!f || !bytes || !length) return GLMAXX_RANK_ERR_NULL;
  if (index >= f->d.size()) return GLMAXX_RANK_ERR_TENSOR_ID;
  *bytes = f->codec_metadata(index);
  *length = f->d[index].codec_metadata_bytes;
  return GLMAXX_RANK_OK;
}

int32_t glmaxx_rank_file_manifest(const glmaxx_rank_file* f, const uint8_t** bytes,
                                  uint64_t* length) {
  if (!f || !bytes || !length) return GLMAXX_RANK_ERR_NULL;
  *bytes = f->manifest_bytes.data();
  *length = f->manifest_bytes.size();
  return GLMAXX_RANK_OK;
}

int32_t glmaxx_rank_file_verify_and_stream(const glmaxx_rank_file* f,
                                           const glmaxx_rank_placement* placements, uint32_t count,
                                           uint32_t flags, void* stream,
                                           glmaxx_rank_payload_proof* proof) {
  if (!f || (count && !placements)) return GLMAXX_RANK_ERR_NULL;
  if (flags & ~uint32_t(GLMAXX_RANK_LOAD_EXL3_SOURCE | GLMAXX_RANK_LOAD_HOST_DESTINATIONS))
    return GLMAXX_RANK_ERR_ARGUMENT;
  return guarded([&] {
    Loader loader(*f, placements, count, flags, static_cast<cudaStream_t>(stream));
    loader.run(proof);
  });
}

int32_t glmaxx_rank_file_verify_and_stream_sink(const glmaxx_rank_file* f,
                                                const glmaxx_rank_sink* sink,
                                                glmaxx_rank_payload_proof* proof) {
  if (!f || !sink) return GLMAXX_RANK_ERR_NULL;
  return guarded([&] {
    Loader loader(*f, nullptr, 0, 0, nullptr, sink);
    loader.run(proof);
  });
}

// validate_rank_set (native_reader.rs:543-588)
int32_t glmaxx_rank_file_validate_set(const glmaxx_rank_file* const files[4]) {
  if (!files) return GLMAXX_RANK_ERR_NULL;
  for (int r = 0; r < 4; ++r)
    if (!files[r]) return GLMAXX_RANK_ERR_NULL;
  return guarded([&] {
    const glmaxx_rank_file& f0 = *files[0];
    Sha256 s;
    s.update("g5n-conversion-v0", 18);
    for (uint32_t r = 0; r < 4; ++r) {
      const glmaxx_rank_file& f = *files[r];
      f.ensure_unchanged();
      // conversion uuid, the five input identities, flags and tensor count agree
      if (f.rank != r || std::memcmp(f.header + 392, f0.header + 392, 16) ||
          std::memcmp(f.header + 120, f0.header + 120, 160) || f.header_flags != f0.header_flags ||
          f.d.size() != f0.d.size())
        fail(GLMAXX_RANK_ERR_RANK_SET);
      for (size_t i = 0; i < f0.d.size(); ++i) {
        const Descriptor &a = f.d[i], &b = f0.d[i];
        // descriptor_semantics_match (:860-878), names, codec_semantics_match (:902-937)
        const bool same = a.tensor_id == b.tensor_id && a.role_id == b.role_id &&
                          a.layer_id == b.layer_id && a.expert_id == b.expert_id &&
                          a.codec_id == b.codec_id && a.logical_dtype == b.logical_dtype &&
                          a.stored_dtype == b.stored_dtype && a.tp_shard_axis == b.tp_shard_axis &&
                          a.ndim == b.ndim && a.flags == b.flags &&
                          !std::memcmp(a.logical_shape, b.logical_shape, 16) &&
                          !std::memcmp(a.padded_shape, b.padded_shape, 16) &&
                          a.payload_bytes == b.payload_bytes && a.aux_bytes == b.aux_bytes &&
                          a.codec_metadata_bytes == b.codec_metadata_bytes &&
                          a.payload_alignment == b.payload_alignment &&
                          a.quant_group_elements == b.quant_group_elements;
        if (!same || f.names[i] != f0.names[i]) fail(GLMAXX_RANK_ERR_RANK_SET);
        if (is_nvfp4(a.codec_id)) {
          const Nvfp4Meta &x = f.nv[i], &y = f0.nv[i];
          if (x.two_d != y.two_d || x.logical_n != y.logical_n || x.logical_k != y.logical_k ||
              x.padded_n != y.padded_n || x.padded_k != y.padded_k ||
              x.value_bytes != y.value_bytes || x.scale_bytes != y.scale_bytes)
            fail(GLMAXX_RANK_ERR_RANK_SET);
        } else if (a.codec_id == GLMAXX_CODEC_EXL3_SOURCE) {
          const Exl3Meta &x = f.ex[i], &y = f0.ex[i];
          if (x.projection != y.projection || x.bits != y.bits || x.layer != y.layer ||
              x.expert != y.expert || x.logical_k != y.logical_k || x.logical_n != y.logical_n ||
              x.trellis_words != y.trellis_words || x.rotation_words != y.rotation_words)
            fail(GLMAXX_RANK_ERR_RANK_SET);
        }
      }
      s.update(f.header + 280, 32);
      s.update(f.header + 312, 32);
      s.update(f.header + 344, 32);
    }
    uint8_t h[32];
    s.finish(h);
    if (std::memcmp(h, f0.header + 392, 16)) fail(GLMAXX_RANK_ERR_RANK_SET);
  });
}

int32_t glmaxx_rank_nvfp4_validate(const uint8_t* metadata, uint64_t metadata_bytes,
                                   const uint8_t* values, uint64_t value_bytes,
                                   const uint8_t* scales, uint64_t scale_bytes) {
  if (!metadata || (value_bytes && !values) || (scale_bytes && !scales)) return GLMAXX_RANK_ERR_NULL;
  return guarded([&] {
    const Nvfp4Meta m = nvfp4_decode(metadata, metadata_bytes);
    if (value_bytes != m.value_bytes || scale_bytes != m.scale_bytes)
      fail(GLMAXX_RANK_ERR_NVFP4_BYTE_ACCOUNTING);
    Nvfp4Check check;
    check.begin(m);
    check.value_chunk(values, value_bytes, 0);
    check.scale_chunk(scales, scale_bytes, 0);
    check.finish();
  });
}

const char* glmaxx_rank_file_error_name(int32_t code) {
  switch (code) {
    case GLMAXX_RANK_OK: return "Ok";
    case GLMAXX_RANK_ERR_NULL: return "Null";
    case GLMAXX_RANK_ERR_ARGUMENT: return "Argument";
    case GLMAXX_RANK_ERR_IO: return "Io";
    case GLMAXX_RANK_ERR_UNSAFE_FILE: return "UnsafeFile";
    case GLMAXX_RANK_ERR_CHANGED: return "Changed";
    case GLMAXX_RANK_ERR_SINK: return "Sink";
    case GLMAXX_RANK_ERR_TRUNCATED: return "Truncated";
    case GLMAXX_RANK_ERR_HEADER: return "Header";
    case GLMAXX_RANK_ERR_HEADER_FLAGS: return "HeaderFlags";
    case GLMAXX_RANK_ERR_HEADER_CRC: return "HeaderCrc";
    case GLMAXX_RANK_ERR_RANK: return "Rank";
    case GLMAXX_RANK_ERR_TENSOR_COUNT: return "TensorCount";
    case GLMAXX_RANK_ERR_TENSOR_ID: return "TensorId";
    case GLMAXX_RANK_ERR_DESCRIPTOR: return "Descriptor";
    case GLMAXX_RANK_ERR_REGION: return "Region";
    case GLMAXX_RANK_ERR_TENSOR_REGION: return "TensorRegion";
    case GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT: return "NonCanonicalLayout";
    case GLMAXX_RANK_ERR_STRING_TABLE: return "StringTable";
    case GLMAXX_RANK_ERR_STRONG_HASH: return "StrongHash";
    case GLMAXX_RANK_ERR_FILE_UUID: return "FileUuid";
    case GLMAXX_RANK_ERR_RANK_SET: return "RankSet";
    case GLMAXX_RANK_ERR_OVERFLOW: return "Overflow";
    case GLMAXX_RANK_ERR_UNSUPPORTED_CODEC: return "UnsupportedCodec";
    case GLMAXX_RANK_ERR_CODEC_MISMATCH: return "CodecMismatch";
    case GLMAXX_RANK_ERR_NVFP4_OVERFLOW: return "Nvfp4(Overflow)";
    case GLMAXX_RANK_ERR_NVFP4_INVALID_SHAPE_OR_SCALE: return "Nvfp4(InvalidShapeOrScale)";
    case GLMAXX_RANK_ERR_NVFP4_BYTE_ACCOUNTING: return "Nvfp4(ByteAccounting)";
    case GLMAXX_RANK_ERR_NVFP4_METADATA_LENGTH: return "Nvfp4(MetadataLength)";
    case GLMAXX_RANK_ERR_NVFP4_METADATA_CRC: return "Nvfp4(MetadataCrc)";
    case GLMAXX_RANK_ERR_NVFP4_UNSUPPORTED_METADATA: return "Nvfp4(UnsupportedMetadata)";
    case GLMAXX_RANK_ERR_NVFP4_SCALE_ENCODING: return "Nvfp4(ScaleEncoding)";
    case GLMAXX_RANK_ERR_NVFP4_ZERO_SCALE_VALUE: return "Nvfp4(ZeroScaleValue)";
    case GLMAXX_RANK_ERR_NVFP4_NON_CANONICAL_PADDING: return "Nvfp4(NonCanonicalPadding)";
    case GLMAXX_RANK_ERR_NVFP4_SCALE_SHARING: return "Nvfp4(ScaleSharing)";
    case GLMAXX_RANK_ERR_NVFP4_ALLOCATION: return "Nvfp4(Allocation)";
    case GLMAXX_RANK_ERR_EXL3_METADATA_LENGTH: return "Exl3(MetadataLength)";
    case GLMAXX_RANK_ERR_EXL3_METADATA_CRC: return "Exl3(MetadataCrc)";
    case GLMAXX_RANK_ERR_EXL3_UNSUPPORTED_CONTRACT: return "Exl3(UnsupportedContract)";
    case GLMAXX_RANK_ERR_EXL3_CODEBOOK_MARKER: return "Exl3(CodebookMarker)";
    case GLMAXX_RANK_ERR_EXL3_BYTE_ACCOUNTING: return "Exl3(ByteAccounting)";
    case GLMAXX_RANK_ERR_EXL3_NON_FINITE_ROTATION: return "Exl3(NonFiniteRotation)";
    case GLMAXX_RANK_ERR_EXL3_OVERFLOW: return "Exl3(Overflow)";
    default: return code > 0 ? "Cuda" : "Unknown";
  }
}

}  // extern "C"
