#include "common/hash.h"

#include <cstring>

namespace lakeb {
namespace {

// SHA-256 round constants: first 32 bits of the fractional parts of the cube
// roots of the first 64 primes (FIPS 180-4, section 4.2.2).
constexpr uint32_t kK[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

struct Sha256 {
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  uint8_t buf[64];
  size_t fill = 0;
  uint64_t total = 0;

  void block(const uint8_t* p) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t(p[4 * i]) << 24) | (uint32_t(p[4 * i + 1]) << 16) | (uint32_t(p[4 * i + 2]) << 8) | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      uint32_t ch = (e & f) ^ (~e & g);
      uint32_t t1 = hh + S1 + ch + kK[i] + w[i];
      uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
      uint32_t t2 = S0 + mj;
      hh = g;
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
    h[7] += hh;
  }

  void update(const uint8_t* p, size_t n) {
    total += n;
    while (n) {
      size_t take = 64 - fill;
      if (take > n) take = n;
      std::memcpy(buf + fill, p, take);
      fill += take;
      p += take;
      n -= take;
      if (fill == 64) {
        block(buf);
        fill = 0;
      }
    }
  }

  std::array<uint8_t, 32> finish() {
    uint64_t bits = total * 8;
    uint8_t pad = 0x80;
    update(&pad, 1);
    uint8_t zero = 0;
    while (fill != 56) update(&zero, 1);
    uint8_t len[8];
    for (int i = 0; i < 8; ++i) len[i] = uint8_t(bits >> (56 - 8 * i));
    update(len, 8);
    std::array<uint8_t, 32> out;
    for (int i = 0; i < 8; ++i)
      for (int j = 0; j < 4; ++j) out[4 * i + j] = uint8_t(h[i] >> (24 - 8 * j));
    return out;
  }
};

}  // namespace

std::array<uint8_t, 32> sha256(const uint8_t* data, size_t n) {
  Sha256 s;
  s.update(data, n);
  return s.finish();
}

std::string chain_hash(const std::string& parent, const uint32_t* tokens, size_t n) {
  Sha256 s;
  s.update(reinterpret_cast<const uint8_t*>(parent.data()), parent.size());
  for (size_t i = 0; i < n; ++i) {
    uint8_t le[4] = {uint8_t(tokens[i]), uint8_t(tokens[i] >> 8), uint8_t(tokens[i] >> 16), uint8_t(tokens[i] >> 24)};
    s.update(le, 4);
  }
  auto d = s.finish();
  return std::string(reinterpret_cast<const char*>(d.data()), d.size());
}

std::vector<std::string> chain_block_hashes(const std::vector<uint32_t>& tokens, size_t block_size, bool full_only,
                                            const std::string& parent) {
  std::vector<std::string> out;
  if (block_size == 0) return out;
  size_t n = tokens.size();
  size_t end = full_only ? n - n % block_size : n;
  std::string p = parent;
  for (size_t i = 0; i < end; i += block_size) {
    size_t take = std::min(block_size, end - i);
    p = chain_hash(p, tokens.data() + i, take);
    out.push_back(p);
  }
  return out;
}

uint64_t hrw_score(const std::string& key, const std::string& node) {
  uint64_t len = key.size();
  uint8_t le[8];
  for (int i = 0; i < 8; ++i) le[i] = uint8_t(len >> (8 * i));
  uint64_t h = fnv1a64_update(kFnvOffset, le, 8);
  h = fnv1a64_update(h, key.data(), key.size());
  return fnv1a64_update(h, node.data(), node.size());
}

uint64_t mix64(uint64_t x) {
  // splitmix64 finaliser (Steele, Lea, Flood 2014)
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

uint64_t hash64(const void* data, size_t n, uint64_t seed) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  uint64_t h = mix64(seed ^ (0x9e3779b97f4a7c15ull * (n + 1)));
  size_t i = 0;
  for (; i + 8 <= n; i += 8) {
    uint64_t w;
    std::memcpy(&w, p + i, 8);
    h = mix64(h ^ w) + 0x9e3779b97f4a7c15ull;
  }
  uint64_t tail = 0;
  for (size_t j = 0; i + j < n; ++j) tail |= uint64_t(p[i + j]) << (8 * j);
  return mix64(h ^ tail ^ (uint64_t(n) << 56));
}

std::string to_hex(const std::string& bytes) {
  static const char* d = "0123456789abcdef";
  std::string s;
  s.reserve(bytes.size() * 2);
  for (unsigned char c : bytes) {
    s.push_back(d[c >> 4]);
    s.push_back(d[c & 15]);
  }
  return s;
}

}  // namespace lakeb
