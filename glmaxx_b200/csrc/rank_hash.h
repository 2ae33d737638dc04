// SHA-256 and CRC32C used by the rank-file reader (rank_hash.cpp).
#pragma once

#include <cstddef>
#include <cstdint>

namespace glmaxx::rankfile {

class Sha256 {
 public:
  Sha256() { reset(); }
  void reset();
  void update(const void* data, size_t length);
  void finish(uint8_t out[32]);

 private:
  void blocks(const uint8_t* p, size_t n);
  uint32_t h_[8];
  uint8_t buf_[64];
  size_t fill_;
  uint64_t total_;
};

void sha256(const void* data, size_t length, uint8_t out[32]);
uint32_t crc32c(const void* data, size_t length);

}  // namespace glmaxx::rankfile
