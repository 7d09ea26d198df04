// SHA-256 (FIPS 180-4), written from the published specification; used for the
// prefix-cache block hashes that external routers share.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <array>
#include <string>

namespace zs {

class Sha256 {
 public:
  Sha256();
  void update(const void* data, size_t n);
  std::array<uint8_t, 32> digest();

 private:
  void block(const uint8_t* p);
  uint32_t h_[8];
  uint8_t buf_[64];
  size_t buf_len_ = 0;
  uint64_t total_ = 0;
};

std::array<uint8_t, 32> sha256(const void* data, size_t n);

}  // namespace zs
