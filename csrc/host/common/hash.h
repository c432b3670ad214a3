// Hash primitives shared by the host components.
//   sha256      FIPS 180-4, used for the block chain hash sha256(parent || u32-LE tokens)
//   fnv1a64     64-bit FNV-1a (rendezvous / HRW scores; byte layout shared with the router)
//   hash64      fast 64-bit mixing hash for in-process indices (ring vnodes, lineage)
#pragma once
#include <array>
#include <cstdint>
#include <string>
#include <vector>

namespace lakeb {

std::array<uint8_t, 32> sha256(const uint8_t* data, size_t n);

// Chain hash of one block: sha256(parent || tokens as u32 little-endian).
std::string chain_hash(const std::string& parent, const uint32_t* tokens, size_t n);

// Per-block chain hashes of a token sequence (trailing partial block included
// unless full_only).
std::vector<std::string> chain_block_hashes(const std::vector<uint32_t>& tokens, size_t block_size,
                                            bool full_only = false, const std::string& parent = std::string());

constexpr uint64_t kFnvOffset = 14695981039346656037ull;
constexpr uint64_t kFnvPrime = 1099511628211ull;

inline uint64_t fnv1a64_update(uint64_t h, const void* data, size_t n) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= kFnvPrime;
  }
  return h;
}

// Rendezvous score fnv1a64(u64-LE len(key) || key || node).
uint64_t hrw_score(const std::string& key, const std::string& node);

uint64_t hash64(const void* data, size_t n, uint64_t seed = 0);
inline uint64_t hash64(const std::string& s, uint64_t seed = 0) { return hash64(s.data(), s.size(), seed); }
uint64_t mix64(uint64_t x);

std::string to_hex(const std::string& bytes);

}  // namespace lakeb
