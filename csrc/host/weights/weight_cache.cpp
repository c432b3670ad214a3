#include "weights/weight_cache.h"

#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <stdexcept>

namespace lakeb::weights {

namespace {
constexpr uint64_t kAlign = 256;
uint64_t round_up(uint64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }
}  // namespace

WeightCache::WeightCache(uint64_t capacity_bytes, bool pinned) : pinned_(pinned), cap_(round_up(capacity_bytes)) {
  if (cap_ == 0) throw std::invalid_argument("WeightCache: capacity must be > 0");
  void* p = nullptr;
  if (pinned_ && cudaHostAlloc(&p, cap_, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    pinned_ = false;  // no GPU here: pageable memory keeps the host-side contract working
    p = nullptr;
  }
  if (!p) p = std::aligned_alloc(kAlign, cap_);
  if (!p) throw std::runtime_error("WeightCache: out of host memory");
  slab_ = static_cast<uint8_t*>(p);
  free_ = new std::map<uint64_t, uint64_t>{{0, cap_}};
}

WeightCache::~WeightCache() {
  if (pinned_)
    cudaFreeHost(slab_);
  else
    std::free(slab_);
  delete free_;
}

std::string WeightCache::key(const std::string& model, const std::string& revision, const std::string& name) {
  return model + '\0' + revision + '\0' + name;
}

bool WeightCache::alloc_locked(uint64_t bytes, uint64_t* off) {
  for (;;) {
    for (auto it = free_->begin(); it != free_->end(); ++it) {
      if (it->second >= bytes) {
        *off = it->first;
        const uint64_t rest = it->second - bytes;
        const uint64_t at = it->first + bytes;
        free_->erase(it);
        if (rest) (*free_)[at] = rest;
        used_ += bytes;
        return true;
      }
    }
    // evict the least recently used unpinned entry and retry
    auto victim = lru_.end();
    for (auto it = lru_.rbegin(); it != lru_.rend(); ++it) {
      if (map_[*it].pins == 0) {
        victim = std::next(it).base();
        break;
      }
    }
    if (victim == lru_.end()) return false;
    Entry e = map_[*victim];
    map_.erase(*victim);
    lru_.erase(victim);
    free_locked(e.off, e.bytes);
    evictions_++;
  }
}

void WeightCache::free_locked(uint64_t off, uint64_t bytes) {
  used_ -= bytes;
  auto it = free_->emplace(off, bytes).first;
  auto next = std::next(it);
  if (next != free_->end() && it->first + it->second == next->first) {
    it->second += next->second;
    free_->erase(next);
  }
  if (it != free_->begin()) {
    auto prev = std::prev(it);
    if (prev->first + prev->second == it->first) {
      prev->second += it->second;
      free_->erase(it);
    }
  }
}

bool WeightCache::put(const std::string& k, uintptr_t src, uint64_t bytes, bool device) {
  const uint64_t need = round_up(bytes);
  std::lock_guard<std::mutex> g(mu_);
  auto it = map_.find(k);
  if (it != map_.end()) {
    if (it->second.bytes == bytes) return true;  // already staged
    if (it->second.pins) return false;
    free_locked(it->second.off, round_up(it->second.bytes));
    lru_.erase(it->second.lru);
    map_.erase(it);
  }
  uint64_t off = 0;
  if (need > cap_ || !alloc_locked(need, &off)) return false;
  void* dst = slab_ + off;
  if (device) {
    if (cudaMemcpy(dst, reinterpret_cast<const void*>(src), bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
      cudaGetLastError();
      free_locked(off, need);
      return false;
    }
  } else {
    std::memcpy(dst, reinterpret_cast<const void*>(src), bytes);
  }
  lru_.push_front(k);
  map_[k] = Entry{off, bytes, 0, lru_.begin()};
  return true;
}

bool WeightCache::contains(const std::string& k) const {
  std::lock_guard<std::mutex> g(mu_);
  return map_.count(k) != 0;
}

uint64_t WeightCache::size_of(const std::string& k) const {
  std::lock_guard<std::mutex> g(mu_);
  auto it = map_.find(k);
  return it == map_.end() ? 0 : it->second.bytes;
}

bool WeightCache::load_to(const std::string& k, uintptr_t dst, uint64_t stream) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = map_.find(k);
  if (it == map_.end()) {
    misses_++;
    return false;
  }
  hits_++;
  lru_.splice(lru_.begin(), lru_, it->second.lru);
  cudaError_t e = cudaMemcpyAsync(reinterpret_cast<void*>(dst), slab_ + it->second.off, it->second.bytes,
                                  cudaMemcpyHostToDevice, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string("WeightCache::load_to: ") + cudaGetErrorString(e));
  }
  return true;
}

bool WeightCache::read(const std::string& k, uintptr_t dst, uint64_t bytes) const {
  std::lock_guard<std::mutex> g(mu_);
  auto it = map_.find(k);
  if (it == map_.end() || bytes > it->second.bytes) return false;
  std::memcpy(reinterpret_cast<void*>(dst), slab_ + it->second.off, bytes);
  return true;
}

void WeightCache::pin(const std::string& k) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = map_.find(k);
  if (it != map_.end()) it->second.pins++;
}

void WeightCache::unpin(const std::string& k) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = map_.find(k);
  if (it != map_.end() && it->second.pins > 0) it->second.pins--;
}

bool WeightCache::erase(const std::string& k) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = map_.find(k);
  if (it == map_.end() || it->second.pins) return false;
  free_locked(it->second.off, round_up(it->second.bytes));
  lru_.erase(it->second.lru);
  map_.erase(it);
  return true;
}

uint64_t WeightCache::used() const {
  std::lock_guard<std::mutex> g(mu_);
  return used_;
}

size_t WeightCache::entries() const {
  std::lock_guard<std::mutex> g(mu_);
  return map_.size();
}

}  // namespace lakeb::weights
