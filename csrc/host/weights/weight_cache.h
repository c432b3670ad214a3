// Pinned host cache of model weights, keyed by (model, revision, tensor name).
//
// A worker that starts (or restarts) on a node where the weights were seen
// before streams them host -> device at link speed instead of re-reading and
// re-converting files: `put` stages a tensor's bytes into one pinned slab
// (from host or device memory), `load_to` issues one cudaMemcpyAsync from the
// slab into a device pointer on the caller's stream. Entries are evicted least
// recently used when the slab is full; an entry is never evicted while a copy
// from it may be in flight on a stream the caller has not synchronised
// (callers pin entries they are loading and unpin after their stream syncs).
//
// Reference parity: rust/weight-cache/src/lib.rs is an empty crate and
// python/lake/engine/model_runner.py:157-158 only records weight state; the
// cache contract here is the one those hooks name.
#pragma once

#include <cstdint>
#include <list>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>

namespace lakeb::weights {

class WeightCache {
 public:
  explicit WeightCache(uint64_t capacity_bytes, bool pinned = true);
  ~WeightCache();
  WeightCache(const WeightCache&) = delete;
  WeightCache& operator=(const WeightCache&) = delete;

  static std::string key(const std::string& model, const std::string& revision, const std::string& name);
  // Stage `bytes` bytes from `src` (host or device pointer; device = true copies D2H synchronously).
  bool put(const std::string& key, uintptr_t src, uint64_t bytes, bool device);
  bool contains(const std::string& key) const;
  uint64_t size_of(const std::string& key) const;
  // One cudaMemcpyAsync slab -> dst on `stream` (a cudaStream_t as an integer). False if absent.
  bool load_to(const std::string& key, uintptr_t dst, uint64_t stream);
  // Copy the entry to host memory (tests, repacking).
  bool read(const std::string& key, uintptr_t dst, uint64_t bytes) const;
  void pin(const std::string& key);
  void unpin(const std::string& key);
  bool erase(const std::string& key);

  uint64_t capacity() const { return cap_; }
  uint64_t used() const;
  size_t entries() const;
  uint64_t hits() const { return hits_; }
  uint64_t misses() const { return misses_; }
  uint64_t evictions() const { return evictions_; }

 private:
  struct Entry {
    uint64_t off = 0, bytes = 0;
    int pins = 0;
    std::list<std::string>::iterator lru;
  };
  bool alloc_locked(uint64_t bytes, uint64_t* off);
  void free_locked(uint64_t off, uint64_t bytes);

  mutable std::mutex mu_;
  uint8_t* slab_ = nullptr;
  bool pinned_ = true;
  uint64_t cap_ = 0, used_ = 0;
  std::unordered_map<std::string, Entry> map_;
  std::list<std::string> lru_;             // front = most recent
  std::map<uint64_t, uint64_t>* free_ = nullptr;  // offset -> length (first fit, coalesced)
  uint64_t hits_ = 0, misses_ = 0, evictions_ = 0;
};

}  // namespace lakeb::weights
