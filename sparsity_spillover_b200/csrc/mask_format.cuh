// Persisted form of the 16x64 tile bitmap (host code only).
//
// A bitmap made by spmlp_up_gate / spmlp_tile_bits_from_h / spmlp_gate can be
// copied to the host, encoded into a self-describing byte string, stored or sent,
// and decoded back into the exact word layout the down projection and the joint
// consumer read, so a later call (a cached prefill, another process) can reuse
// the skip decisions without recomputing h.
//
// Layout (little-endian), 64-byte header then payload:
//   0  "SPMB"            4  u16 version (1)      6  u16 encoding
//   8  u16 tile rows (16) 10 u16 tile cols (64)   12 u32 F (features)
//   16 u64 T (tokens)     24 u32 words per 16-row group
//   28 u32 CRC-32 of the payload                  32 u64 payload bytes
//   40 u64 live tiles     48 16 reserved bytes (zero)
// Payload, encoding 0 (raw): ceil(T/16) * words u32, the bitmap itself.
// Payload, encoding 1 (row runs): u32 run count, then per run of identical 16-row
//   groups a u32 length and the group's `words` u32; lossless.  Element-random
//   masks (every group alike) shrink to one run, token-blocked masks by their
//   block height.
#pragma once

#include <stdint.h>

#include <array>
#include <cstring>

namespace spmlp {
namespace mask {

constexpr uint32_t kMagic = 0x424D5053u;  // "SPMB"
constexpr uint16_t kVersion = 1;
constexpr int64_t kHeaderBytes = 64;

// CRC-32 (IEEE 802.3 polynomial, reflected), bytewise with a 256-entry table.
inline uint32_t crc32(const uint8_t* data, size_t n) {
  static const std::array<uint32_t, 256> table = [] {
    std::array<uint32_t, 256> t{};
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1u) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
      t[i] = c;
    }
    return t;
  }();
  uint32_t c = 0xFFFFFFFFu;
  for (size_t i = 0; i < n; ++i) c = table[(c ^ data[i]) & 0xFFu] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

template <class T>
inline void put(uint8_t* p, T v) {
  std::memcpy(p, &v, sizeof(T));  // the supported hosts are little-endian
}
template <class T>
inline T get(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof(T));
  return v;
}

inline int64_t groups_of(int64_t T) { return (T + 15) / 16; }

inline int64_t popcount_all(const uint32_t* bits, int64_t n) {
  int64_t c = 0;
  for (int64_t i = 0; i < n; ++i) c += __builtin_popcount(bits[i]);
  return c;
}

inline bool same_group(const uint32_t* bits, int words, int64_t a, int64_t b) {
  return std::memcmp(bits + a * words, bits + b * words, static_cast<size_t>(words) * 4) == 0;
}

inline int64_t run_count(const uint32_t* bits, int64_t groups, int words) {
  int64_t runs = groups > 0 ? 1 : 0;
  for (int64_t r = 1; r < groups; ++r) runs += same_group(bits, words, r, r - 1) ? 0 : 1;
  return runs;
}

// Payload bytes of a bitmap in an encoding (the run encoding depends on the bits).
inline int64_t payload_bytes(const uint32_t* bits, int64_t T, int words, int encoding) {
  const int64_t g = groups_of(T);
  if (encoding == 0) return g * words * 4;
  return 4 + run_count(bits, g, words) * (1 + words) * 4;
}

inline void write_payload(const uint32_t* bits, int64_t T, int words, int encoding, uint8_t* out) {
  const int64_t g = groups_of(T);
  if (encoding == 0) {
    std::memcpy(out, bits, static_cast<size_t>(g * words * 4));
    return;
  }
  uint8_t* o = out + 4;
  uint32_t runs = 0;
  for (int64_t r = 0; r < g;) {
    int64_t e = r + 1;
    while (e < g && same_group(bits, words, e, r)) ++e;
    put<uint32_t>(o, static_cast<uint32_t>(e - r));
    std::memcpy(o + 4, bits + r * words, static_cast<size_t>(words) * 4);
    o += (1 + words) * 4;
    ++runs;
    r = e;
  }
  put<uint32_t>(out, runs);
}

}  // namespace mask
}  // namespace spmlp
