#include "tier/tier.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <stdexcept>

#include "common/hash.h"

namespace lakeb::tier {
namespace {
[[noreturn]] void fail(const std::string& m) { throw std::invalid_argument(m); }

void mkdirs(const std::string& path) {
  std::string cur;
  for (size_t i = 0; i < path.size(); ++i) {
    cur.push_back(path[i]);
    if (path[i] == '/' || i + 1 == path.size()) ::mkdir(cur.c_str(), 0755);
  }
}

bool pwrite_all(int fd, const uint8_t* p, uint64_t n, uint64_t off) {
  while (n) {
    ssize_t w = ::pwrite(fd, p, n, static_cast<off_t>(off));
    if (w < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    p += w;
    n -= uint64_t(w);
    off += uint64_t(w);
  }
  return true;
}
bool pread_all(int fd, uint8_t* p, uint64_t n, uint64_t off) {
  while (n) {
    ssize_t r = ::pread(fd, p, n, static_cast<off_t>(off));
    if (r < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    if (r == 0) return false;
    p += r;
    n -= uint64_t(r);
    off += uint64_t(r);
  }
  return true;
}
struct RecordHeader {
  char magic[4];
  uint16_t version;
  uint16_t header_bytes;
  uint32_t flags;
  uint32_t reserved;
  uint64_t payload_bytes;
  uint8_t block_hash[32];
  uint64_t checksum;
};
static_assert(sizeof(RecordHeader) == kBlockHeaderBytes, "block record header is 64 bytes");

inline uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
// SplitMix64's finalizer (S. Vigna): full avalanche of a 64-bit state.
inline uint64_t mix_final(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
}  // namespace

// Word-wise multiply-rotate hash over the payload with a SplitMix64 finish: not cryptographic,
// it detects torn, stale and bit-flipped records (a flipped bit changes every output bit).
uint64_t payload_checksum(const uint8_t* p, uint64_t n) {
  uint64_t h = 0x9e3779b97f4a7c15ull ^ n;
  uint64_t i = 0;
  for (; i + 8 <= n; i += 8) {
    uint64_t w;
    std::memcpy(&w, p + i, 8);
    h = rotl64(h ^ (w * 0x9e3779b97f4a7c15ull), 29) * 0xc2b2ae3d27d4eb4full;
  }
  uint64_t tail = 0;
  for (uint64_t k = 0; i + k < n; ++k) tail |= uint64_t(p[i + k]) << (8 * k);
  return mix_final(h ^ tail);
}

// ------------------------------------------------------------------ segment arena
SegmentArena::SegmentArena(uint64_t slot_bytes, size_t per_seg)
    : slot_bytes_(slot_bytes ? slot_bytes : 4096), per_seg_(per_seg ? per_seg : 64) {}

std::optional<Placement> SegmentArena::placement(const std::string& h) const {
  auto it = where_.find(h);
  if (it == where_.end()) return std::nullopt;
  return it->second;
}

Placement SegmentArena::alloc(const std::string& h) {
  if (auto p = placement(h)) return *p;
  for (auto& [seg, slots] : segs_)
    for (size_t i = 0; i < slots.size(); ++i)
      if (slots[i].empty()) {
        slots[i] = h;
        Placement pl{seg, uint64_t(i) * slot_bytes_};
        where_[h] = pl;
        return pl;
      }
  uint64_t seg = segs_.empty() ? 1 : segs_.rbegin()->first + 1;
  auto& slots = segs_[seg];
  slots.assign(per_seg_, std::string());
  slots[0] = h;
  Placement pl{seg, 0};
  where_[h] = pl;
  return pl;
}

Placement SegmentArena::place_at(const std::string& h, uint64_t seg, uint64_t offset) {
  if (offset % slot_bytes_) fail("place_at: offset not slot aligned");
  size_t idx = offset / slot_bytes_;
  if (idx >= per_seg_) fail("place_at: offset beyond segment capacity");
  auto& slots = segs_[seg];
  if (slots.empty()) slots.assign(per_seg_, std::string());
  if (!slots[idx].empty() && slots[idx] != h) fail("place_at: slot occupied");
  free(h);
  slots[idx] = h;
  Placement pl{seg, offset};
  where_[h] = pl;
  return pl;
}

Placement SegmentArena::alloc_spare(const std::string& h) { return alloc(spare_key(h)); }

void SegmentArena::commit_spare(const std::string& h) {
  auto sp = where_.find(spare_key(h));
  if (sp == where_.end()) fail("commit_spare: no spare slot");
  const Placement pl = sp->second;
  where_.erase(sp);
  free(h);
  segs_[pl.segment_id][pl.offset / slot_bytes_] = h;
  where_[h] = pl;
}

void SegmentArena::drop_spare(const std::string& h) { free(spare_key(h)); }

bool SegmentArena::free(const std::string& h) {
  auto it = where_.find(h);
  if (it == where_.end()) return false;
  auto& slots = segs_[it->second.segment_id];
  slots[it->second.offset / slot_bytes_].clear();
  where_.erase(it);
  return true;
}

std::vector<Relocate> SegmentArena::compact(uint64_t seg) {
  std::vector<Relocate> out;
  auto it = segs_.find(seg);
  if (it == segs_.end()) return out;
  auto& slots = it->second;
  size_t lo = 0, hi = slots.size();
  while (true) {
    while (lo < slots.size() && !slots[lo].empty()) ++lo;
    while (hi > 0 && slots[hi - 1].empty()) --hi;
    if (lo >= hi) break;
    const std::string h = slots[hi - 1];
    Relocate r{h, Placement{seg, uint64_t(hi - 1) * slot_bytes_}, Placement{seg, uint64_t(lo) * slot_bytes_}};
    slots[lo] = h;
    slots[hi - 1].clear();
    where_[h] = r.to;
    out.push_back(r);
  }
  return out;
}

Relocate SegmentArena::relocate(const std::string& h, uint64_t seg, uint64_t offset) {
  auto from = placement(h);
  if (!from) fail("relocate: unknown block");
  Relocate r{h, *from, Placement{seg, offset}};
  place_at(h, seg, offset);
  return r;
}

double SegmentArena::utilization(uint64_t seg) const {
  auto it = segs_.find(seg);
  if (it == segs_.end() || it->second.empty()) return 0.0;
  size_t used = 0;
  for (auto& s : it->second) used += !s.empty();
  return double(used) / double(it->second.size());
}

size_t SegmentArena::dense_prefix_slots(uint64_t seg) const {
  auto it = segs_.find(seg);
  if (it == segs_.end()) return 0;
  size_t n = 0;
  while (n < it->second.size() && !it->second[n].empty()) ++n;
  return n;
}

bool SegmentArena::has_holes(uint64_t seg) const {
  auto it = segs_.find(seg);
  if (it == segs_.end()) return false;
  bool seen_empty = false;
  for (auto& s : it->second) {
    if (s.empty()) seen_empty = true;
    else if (seen_empty) return true;
  }
  return false;
}

std::vector<uint64_t> SegmentArena::segment_ids() const {
  std::vector<uint64_t> out;
  for (auto& [k, v] : segs_) out.push_back(k);
  return out;
}

std::vector<std::string> SegmentArena::hashes_in_segment(uint64_t seg) const {
  std::vector<std::string> out;
  auto it = segs_.find(seg);
  if (it == segs_.end()) return out;
  for (auto& s : it->second)
    if (!s.empty()) out.push_back(s);
  return out;
}

// ------------------------------------------------------------------ bandwidth pool
BandwidthPool::BandwidthPool(uint64_t budget, uint64_t window) : budget_(budget), window_(window ? window : 1000) {}
void BandwidthPool::roll(uint64_t now) {
  if (now >= window_start_ + window_ || now < window_start_) {
    window_start_ = now - (now % window_);
    used_ = 0;
  }
}
bool BandwidthPool::try_consume(uint64_t bytes, uint64_t now) {
  if (paused_) return false;
  roll(now);
  if (used_ + bytes > budget_ && used_ > 0) return false;  // an oversize single item may use a fresh window
  used_ += bytes;
  return true;
}
uint64_t BandwidthPool::remaining(uint64_t now) {
  roll(now);
  return used_ >= budget_ ? 0 : budget_ - used_;
}

// ------------------------------------------------------------------ engine
TierEngine::TierEngine(TierCaps caps, uint64_t block_bytes, uint8_t* l1_base, const std::string& l2_dir,
                       const std::string& l3_dir, const std::string& model_key)
    : caps_(caps),
      block_bytes_(block_bytes),
      l1_base_(l1_base),
      l2_dir_(l2_dir),
      l3_dir_(l3_dir),
      model_key_(model_key),
      arena_(block_bytes + kBlockHeaderBytes, 64) {
  if (!block_bytes_) fail("TierEngine: block_bytes must be > 0");
  if (l2_dir_.empty()) fail("TierEngine: an L2 directory is required (L2 is the durable recovery point)");
  mkdirs(l2_dir_);
  if (!l3_dir_.empty()) mkdirs(l3_dir_ + "/" + model_key_);
  for (int64_t s = int64_t(caps_.l1) - 1; s >= 0; --s) free_slots_.push_back(s);
}
TierEngine::~TierEngine() {
  for (auto& [seg, fd] : seg_fds_) ::close(fd);
}

void TierEngine::touch(std::list<std::string>& order,
                       std::unordered_map<std::string, std::list<std::string>::iterator>& pos, const std::string& h) {
  auto it = pos.find(h);
  if (it != pos.end()) order.erase(it->second);
  order.push_back(h);
  pos[h] = std::prev(order.end());
}

std::string TierEngine::seg_path(uint64_t seg) const { return l2_dir_ + "/seg_" + std::to_string(seg) + ".bin"; }
std::string TierEngine::l3_path(const std::string& h) const { return l3_dir_ + "/" + model_key_ + "/" + to_hex(h); }

int TierEngine::segment_fd(uint64_t seg) const {
  std::lock_guard<std::mutex> g(fd_mu_);
  auto it = seg_fds_.find(seg);
  if (it != seg_fds_.end()) return it->second;
  int fd = ::open(seg_path(seg).c_str(), O_RDWR | O_CREAT, 0644);
  if (fd >= 0) seg_fds_[seg] = fd;
  return fd;
}

bool TierEngine::write_record(int fd, const std::string& h, const uint8_t* bytes, uint64_t off) const {
  RecordHeader hd{};
  std::memcpy(hd.magic, kBlockMagic, 4);
  hd.version = kBlockFormatVersion;
  hd.header_bytes = kBlockHeaderBytes;
  hd.payload_bytes = block_bytes_;
  std::memcpy(hd.block_hash, h.data(), std::min<size_t>(h.size(), 32));
  hd.checksum = payload_checksum(bytes, block_bytes_);
  return pwrite_all(fd, bytes, block_bytes_, off + kBlockHeaderBytes) &&
         pwrite_all(fd, reinterpret_cast<const uint8_t*>(&hd), kBlockHeaderBytes, off);
}

bool TierEngine::read_record(int fd, const std::string& h, uint8_t* dst, uint64_t off) const {
  RecordHeader hd;
  uint8_t want[32] = {0};
  std::memcpy(want, h.data(), std::min<size_t>(h.size(), 32));
  const bool ok = pread_all(fd, reinterpret_cast<uint8_t*>(&hd), kBlockHeaderBytes, off) &&
                  std::memcmp(hd.magic, kBlockMagic, 4) == 0 && hd.version == kBlockFormatVersion &&
                  hd.header_bytes == kBlockHeaderBytes && hd.payload_bytes == block_bytes_ &&
                  std::memcmp(hd.block_hash, want, 32) == 0 &&
                  pread_all(fd, dst, block_bytes_, off + kBlockHeaderBytes) &&
                  payload_checksum(dst, block_bytes_) == hd.checksum;
  if (!ok) {
    std::lock_guard<std::mutex> g(fd_mu_);
    ++corrupt_reads_;
  }
  return ok;
}

// The record is on the device (fdatasync) before the write reports success: PutEnd registers
// the block as durable right after this returns.
bool TierEngine::write_l2(const std::string& h, const uint8_t* bytes) {
  Placement pl = arena_.alloc(h);
  const int fd = segment_fd(pl.segment_id);
  return fd >= 0 && write_record(fd, h, bytes, pl.offset) && ::fdatasync(fd) == 0;
}
// Copy-on-write overwrite of a resident block: the new record goes to a spare slot and
// replaces the old one only once it is on the device, so a failed write leaves the previous
// record readable where the control plane last saw it.
bool TierEngine::overwrite_l2(const std::string& h, const uint8_t* bytes) {
  const Placement pl = arena_.alloc_spare(h);
  const int fd = segment_fd(pl.segment_id);
  if (fd < 0 || !write_record(fd, h, bytes, pl.offset) || ::fdatasync(fd) != 0) {
    arena_.drop_spare(h);
    return false;
  }
  arena_.commit_spare(h);
  return true;
}
bool TierEngine::read_l2(const std::string& h, uint8_t* dst) const {
  auto pl = arena_.placement(h);
  if (!pl) return false;
  const int fd = segment_fd(pl->segment_id);
  return fd >= 0 && read_record(fd, h, dst, pl->offset);
}
// L3 objects are written to a temporary name, synced and renamed, then the directory entry
// is synced, so a crash leaves either the old state or the whole record.
bool TierEngine::write_l3(const std::string& h, const uint8_t* bytes) {
  if (l3_dir_.empty()) return false;
  std::string tmp = l3_path(h) + ".tmp";
  int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
  if (fd < 0) return false;
  bool ok = write_record(fd, h, bytes, 0) && ::fdatasync(fd) == 0;
  ::close(fd);
  ok = ok && ::rename(tmp.c_str(), l3_path(h).c_str()) == 0;
  if (ok) {
    int dfd = ::open((l3_dir_ + "/" + model_key_).c_str(), O_RDONLY | O_DIRECTORY);
    if (dfd >= 0) {
      ::fsync(dfd);
      ::close(dfd);
    }
  }
  return ok;
}
bool TierEngine::read_l3(const std::string& h, uint8_t* dst) const {
  if (l3_dir_.empty()) return false;
  int fd = ::open(l3_path(h).c_str(), O_RDONLY);
  if (fd < 0) return false;
  bool ok = read_record(fd, h, dst, 0);
  ::close(fd);
  return ok;
}
bool TierEngine::l3_present(const std::string& h) const {
  if (l3_dir_.empty()) return false;
  struct stat st;
  return ::stat(l3_path(h).c_str(), &st) == 0;
}
size_t TierEngine::l3_len() const {
  // counted lazily by the caller through directory listings; keep a cheap estimate here
  return 0;
}

int64_t TierEngine::l0_page(const std::string& h) const {
  auto it = l0_.find(h);
  return it == l0_.end() ? -1 : it->second;
}
int64_t TierEngine::l1_slot(const std::string& h) const {
  auto it = l1_.find(h);
  return it == l1_.end() ? -1 : it->second;
}
TierId TierEngine::local_tier(const std::string& h) const {
  if (l0_.count(h)) return TierId::L0;
  if (l1_.count(h)) return TierId::L1;
  if (l2_.count(h)) return TierId::L2;
  if (l3_present(h)) return TierId::L3;
  return TierId::None;
}
uint32_t TierEngine::hit_count(const std::string& h) const {
  auto it = hits_.find(h);
  return it == hits_.end() ? 0 : it->second;
}
uint32_t TierEngine::pin_count(const std::string& h) const {
  auto it = pins_.find(h);
  return it == pins_.end() ? 0 : it->second;
}
void TierEngine::unpin(const std::string& h) {
  auto it = pins_.find(h);
  if (it == pins_.end() || it->second == 0) fail("unpin: block not pinned");
  if (--it->second == 0) pins_.erase(it);
}

void TierEngine::note_l0(const std::string& h, int64_t page) {
  l0_[h] = page;
  touch(l0_order_, l0_pos_, h);
}
void TierEngine::drop_l0(const std::string& h) {
  l0_.erase(h);
  auto it = l0_pos_.find(h);
  if (it != l0_pos_.end()) {
    l0_order_.erase(it->second);
    l0_pos_.erase(it);
  }
}

void TierEngine::l2_forget(const std::string& h) {
  l2_.erase(h);
  arena_.free(h);
  auto it = l2_pos_.find(h);
  if (it != l2_pos_.end()) {
    l2_order_.erase(it->second);
    l2_pos_.erase(it);
  }
}

// Two-phase: the victims (least recently written, unpinned; a pinned block keeps its LRU
// position) are chosen and their L3 objects written before any leaves L2, so a cap that cannot
// be met (every candidate pinned) or an L3 write that fails changes nothing (an L3 object this
// call created is removed again).
SideEffects TierEngine::ensure_l2_cap() {
  SideEffects fx;
  if (!caps_.l2) return fx;
  size_t evictable = l2_.size();
  std::vector<std::string> victims;
  for (auto& h : l2_order_) {
    if (evictable <= caps_.l2) break;
    if (pin_count(h)) continue;
    victims.push_back(h);
    --evictable;
  }
  if (evictable > caps_.l2) fail("l2 over cap: all victims pinned (unpin before put)");
  std::vector<uint8_t> buf(block_bytes_);
  std::vector<std::string> created;
  for (auto& v : victims) {
    if (l3_present(v)) continue;
    if (read_l2(v, buf.data()) && write_l3(v, buf.data())) {
      created.push_back(v);
      continue;
    }
    for (auto& c : created) ::unlink(l3_path(c).c_str());
    fail("l2 over cap: moving a block to L3 failed");
  }
  for (auto& v : victims) {
    l2_forget(v);
    fx.l2_demoted_to_l3.push_back(v);
  }
  return fx;
}

std::pair<TierId, SideEffects> TierEngine::put_durable(const std::string& h, const uint8_t* bytes) {
  if (l2_.count(h)) {
    // Blocks are named by the chain hash of their content, so an overwrite carries the same
    // bytes (it refreshes a torn record); the resident count is unchanged, so no cap demotion.
    if (!overwrite_l2(h, bytes)) fail("put_durable: L2 write failed (the previous record is kept)");
    touch(l2_order_, l2_pos_, h);
    return {TierId::L2, SideEffects{}};
  }
  if (!write_l2(h, bytes)) {
    arena_.free(h);
    fail("put_durable: L2 write failed");
  }
  l2_.insert(h);
  touch(l2_order_, l2_pos_, h);
  SideEffects fx;
  try {
    fx = ensure_l2_cap();
  } catch (...) {
    l2_forget(h);  // two-phase: undo the insert, leave no state change behind
    throw;
  }
  if (l2_.count(h)) return {TierId::L2, fx};
  if (l3_present(h)) return {TierId::L3, fx};
  fail("put_durable: block lost after L2 cap demote");
}

bool TierEngine::read_host(const std::string& h, uint8_t* dst) const {
  auto it = l1_.find(h);
  if (it != l1_.end()) {
    std::memcpy(dst, l1_ptr(it->second), block_bytes_);
    return true;
  }
  if (l2_.count(h) && read_l2(h, dst)) return true;
  return read_l3(h, dst);
}

AccessKind TierEngine::probe(const std::string& h) {
  AccessKind k = AccessKind::Miss;
  if (l0_.count(h)) k = AccessKind::L0Hit;
  else if (l1_.count(h)) k = AccessKind::L1Hit;
  else if (l2_.count(h)) k = AccessKind::L2Hit;
  else if (l3_present(h)) k = AccessKind::L3Hit;
  if (k != AccessKind::Miss) {
    uint32_t c = ++hits_[h];
    if (k == AccessKind::L0Hit && one_shot_.count(h) && c >= admit_after_) one_shot_.erase(h);
  }
  stats.record(k);
  return k;
}

uint64_t TierEngine::estimate_promote_cost(const std::string& h) const {
  switch (local_tier(h)) {
    case TierId::L0: return 0;
    case TierId::L1: return block_bytes_;
    case TierId::L2: return 2 * block_bytes_;
    case TierId::L3: return 3 * block_bytes_;
    default: return UINT64_MAX;
  }
}

int64_t TierEngine::alloc_l1_slot(SideEffects* fx) {
  if (!free_slots_.empty()) {
    int64_t s = free_slots_.back();
    free_slots_.pop_back();
    return s;
  }
  // evict the LRU unpinned L1 copy that has durable backing
  for (auto& h : l1_order_) {
    if (pin_count(h) || !has_durable_backing(h)) continue;
    int64_t s = l1_[h];
    l1_.erase(h);
    auto it = l1_pos_.find(h);
    l1_order_.erase(it->second);
    l1_pos_.erase(it);
    (void)fx;
    return s;
  }
  return -1;
}

BeginPromote TierEngine::begin_promote(const std::string& h) {
  if (l0_.count(h)) return BeginPromote::AlreadyL0;
  if (inflight_.count(h)) return BeginPromote::AlreadyInFlight;
  if (local_tier(h) == TierId::None) return BeginPromote::Missing;
  inflight_.insert(h);
  return BeginPromote::Started;
}

std::optional<std::string> TierEngine::evict_l0_pressure_victim() const {
  // one-shot blocks first, then LRU; pinned and non-durable blocks stay
  for (int pass = 0; pass < 2; ++pass)
    for (auto& h : l0_order_) {
      if (pin_count(h) || !has_durable_backing(h)) continue;
      if (pass == 0 && !one_shot_.count(h)) continue;
      return h;
    }
  return std::nullopt;
}

std::optional<DeviceCopy> TierEngine::demote_l0(const std::string& h) {
  auto it = l0_.find(h);
  if (it == l0_.end()) return std::nullopt;
  if (!has_durable_backing(h)) fail("demote_l0: no durable backing (write L2 first)");
  if (pin_count(h)) fail("demote_l0: block pinned");
  DeviceCopy c;
  c.hash = h;
  c.page = it->second;
  c.to_device = false;
  SideEffects fx;
  auto l1 = l1_.find(h);
  if (l1 != l1_.end()) {
    c.slot = l1->second;
  } else {
    c.slot = alloc_l1_slot(&fx);
    if (c.slot >= 0) {
      l1_[h] = c.slot;
      touch(l1_order_, l1_pos_, h);
    }
  }
  drop_l0(h);
  one_shot_.erase(h);
  return c;
}

std::optional<DeviceCopy> TierEngine::promote_to_l0(const std::string& h, std::vector<DeviceCopy>* evict,
                                                    SideEffects* fx, const std::function<int64_t()>& alloc_page) {
  if (l0_.count(h)) {
    touch(l0_order_, l0_pos_, h);
    return std::nullopt;
  }
  // stage into L1
  int64_t slot = l1_slot(h);
  if (slot < 0) {
    slot = alloc_l1_slot(fx);
    if (slot < 0) fail("promote_to_l0: no free L1 slot");
    uint8_t* dst = l1_ptr(slot);
    bool ok = false;
    if (l2_.count(h)) ok = read_l2(h, dst);
    if (!ok) ok = read_l3(h, dst);
    if (!ok) {
      free_slots_.push_back(slot);
      fail("promote_to_l0: block not found in L2/L3");
    }
    l1_[h] = slot;
    touch(l1_order_, l1_pos_, h);
  }
  if (!l2_.count(h) && l3_present(h)) rehydrate_l2(h, l1_ptr(slot), fx);
  // reserve an L0 page, demoting under pressure
  int64_t page = -1;
  if (l0_.size() < caps_.l0) page = alloc_page ? alloc_page() : -1;
  while (page < 0) {
    auto v = evict_l0_pressure_victim();
    if (!v) fail("promote_to_l0: L0 full and every resident block is pinned or not durable");
    auto c = demote_l0(*v);
    if (c && evict) evict->push_back(*c);
    if (fx) fx->l0_demoted.push_back(*v);
    page = c ? c->page : -1;
  }
  note_l0(h, page);
  if (hit_count(h) < admit_after_) one_shot_.insert(h);
  DeviceCopy cp{h, page, slot, true};
  return cp;
}

bool TierEngine::demote_l2_to_l3(const std::string& h) {
  if (!l2_.count(h)) return false;
  if (pin_count(h)) fail("demote_l2_to_l3: block pinned");
  if (!l3_present(h)) {
    std::vector<uint8_t> buf(block_bytes_);
    if (!read_l2(h, buf.data())) fail("demote_l2_to_l3: L2 read failed");
    if (!write_l3(h, buf.data())) fail("demote_l2_to_l3: L3 write failed");
  }
  l2_forget(h);
  return true;
}

// A block read back from L3 gets an L2 record again (the node's local recovery point for its
// working set), under the L2 cap; with every L2 resident pinned it stays L3-only.
void TierEngine::rehydrate_l2(const std::string& h, const uint8_t* bytes, SideEffects* fx) {
  bool room = !caps_.l2 || l2_.size() < caps_.l2;
  for (auto it = l2_order_.begin(); !room && it != l2_order_.end(); ++it) room = pin_count(*it) == 0;
  if (!room) return;  // the cap could only be met by demoting this block again
  if (!write_l2(h, bytes)) {
    arena_.free(h);
    return;
  }
  l2_.insert(h);
  touch(l2_order_, l2_pos_, h);
  try {
    SideEffects d = ensure_l2_cap();
    if (fx) fx->l2_demoted_to_l3.insert(fx->l2_demoted_to_l3.end(), d.l2_demoted_to_l3.begin(), d.l2_demoted_to_l3.end());
  } catch (const std::invalid_argument&) {  // an L3 write of the victim failed: stay L3-only
    l2_forget(h);
  }
}

void TierEngine::discard(const std::string& h) {
  drop_l0(h);
  auto l1 = l1_.find(h);
  if (l1 != l1_.end()) {
    free_slots_.push_back(l1->second);
    l1_.erase(l1);
    auto it = l1_pos_.find(h);
    if (it != l1_pos_.end()) {
      l1_order_.erase(it->second);
      l1_pos_.erase(it);
    }
  }
  if (l2_.count(h)) l2_forget(h);
  pins_.erase(h);
  hits_.erase(h);
  one_shot_.erase(h);
  inflight_.erase(h);
}

std::vector<Relocate> TierEngine::compact_l2_segment(uint64_t seg) {
  // read every block first, then rewrite at the compacted slots
  std::vector<std::pair<std::string, std::vector<uint8_t>>> data;
  for (auto& h : arena_.hashes_in_segment(seg)) {
    std::vector<uint8_t> b(block_bytes_);
    if (!read_l2(h, b.data())) fail("compact: L2 read failed");
    data.emplace_back(h, std::move(b));
  }
  auto moves = arena_.compact(seg);
  for (auto& mv : moves)
    for (auto& [h, b] : data)
      if (h == mv.hash) write_l2(h, b.data());
  return moves;
}

Relocate TierEngine::colocate_l2_move(const std::string& h, uint64_t seg, uint64_t offset) {
  std::vector<uint8_t> buf(block_bytes_);
  if (!read_l2(h, buf.data())) fail("colocate: L2 read failed");
  Relocate r = arena_.relocate(h, seg, offset);
  write_l2(h, buf.data());
  return r;
}

// ------------------------------------------------------------------ pipeline
TierPipeline::TierPipeline(TierEngine* e, BandwidthPool* bw, std::string node) : eng_(e), bw_(bw), node_(std::move(node)) {}

std::pair<size_t, std::vector<LocationEvent>> TierPipeline::tick(size_t max_steps, uint64_t now_ms,
                                                                 const std::function<int64_t()>& alloc_page,
                                                                 std::vector<DeviceCopy>* copies) {
  std::vector<LocationEvent> ev;
  size_t done = 0, failed = 0;
  std::deque<Action> retry;
  while (done < max_steps && !q_.empty()) {
    Action a = q_.front();
    q_.pop_front();
    uint64_t cost = a.kind == ActionKind::Promote || a.kind == ActionKind::FillMiss ? eng_->estimate_promote_cost(a.hash)
                                                                                    : eng_->block_bytes();
    if (cost == UINT64_MAX) cost = eng_->block_bytes();
    if (!bw_->try_consume(cost, now_ms)) {
      q_.push_front(a);  // budget exhausted for this window
      break;
    }
    try {
      switch (a.kind) {
        case ActionKind::Promote:
        case ActionKind::FillMiss: {
          SideEffects fx;
          std::vector<DeviceCopy> ev_copies;
          const bool was_l2 = eng_->is_l2_durable(a.hash);
          auto c = eng_->promote_to_l0(a.hash, &ev_copies, &fx, alloc_page);
          for (auto& v : fx.l2_demoted_to_l3) {  // the cap demotions of an L3 block's rehydration
            if (v == a.hash) continue;
            ev.push_back({LocKind::Absent, v, 3, node_, 0, 0});
            ev.push_back({LocKind::L3Present, v, 4, node_, 0, 0});
          }
          if (!was_l2 && eng_->is_l2_durable(a.hash)) {
            auto pl = eng_->l2_placement(a.hash);
            ev.push_back({LocKind::Present, a.hash, 3, node_, pl ? pl->segment_id : 0, pl ? pl->offset : 0});
          }
          for (auto& x : ev_copies) {
            copies->push_back(x);
            ev.push_back({LocKind::Absent, x.hash, 1, node_, 0, 0});
            ev.push_back({LocKind::Present, x.hash, 2, node_, 0, uint64_t(x.slot)});
          }
          if (c) {
            copies->push_back(*c);
            ev.push_back({LocKind::Present, a.hash, 1, node_, 0, uint64_t(c->page)});
          }
          eng_->finish_promote(a.hash);
          break;
        }
        case ActionKind::DemoteL0: {
          auto c = eng_->demote_l0(a.hash);
          if (c) {
            copies->push_back(*c);
            ev.push_back({LocKind::Absent, a.hash, 1, node_, 0, 0});
            if (c->slot >= 0) ev.push_back({LocKind::Present, a.hash, 2, node_, 0, uint64_t(c->slot)});
          }
          break;
        }
        case ActionKind::DemoteL2:
          if (eng_->demote_l2_to_l3(a.hash)) {
            ev.push_back({LocKind::Absent, a.hash, 3, node_, 0, 0});
            ev.push_back({LocKind::L3Present, a.hash, 4, node_, 0, 0});
          }
          break;
        case ActionKind::CompactSegment:
          for (auto& mv : eng_->compact_l2_segment(a.segment_id))
            ev.push_back({LocKind::Moved, mv.hash, 3, node_, mv.to.segment_id, mv.to.offset});
          break;
        case ActionKind::CoLocateMove: {
          auto mv = eng_->colocate_l2_move(a.hash, a.segment_id, a.offset);
          ev.push_back({LocKind::Moved, mv.hash, 3, node_, mv.to.segment_id, mv.to.offset});
          break;
        }
      }
      ++done;
    } catch (const std::exception&) {
      if (++a.failures < kMaxFailures) retry.push_back(a);
      if (++failed >= max_steps) break;  // a tick spends at most max_steps attempts on failures
    }
  }
  for (auto& a : retry) q_.push_back(a);
  return {done, ev};
}

// ------------------------------------------------------------------ writeback batcher
std::vector<std::string> WritebackBatcher::push(const std::string& h) {
  buf_.push_back(h);
  if (buf_.size() >= batch_) return drain();
  return {};
}
std::vector<std::string> WritebackBatcher::drain() {
  std::vector<std::string> out;
  out.swap(buf_);
  if (!out.empty()) ++flushes_;
  return out;
}

}  // namespace lakeb::tier
