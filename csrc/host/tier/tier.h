// Local tiered KV store of one node: L0 = HBM pages of the device arena,
// L1 = slots of a pinned host buffer, L2 = NVMe segment files (durable
// recovery point), L3 = object directory (source of truth).
//
// Block bytes move L1 <-> L2 <-> L3 inside this library (file I/O on the
// pinned slots); L0 <-> L1 moves are device copies issued by the caller on a
// side CUDA stream (the engine hands out page/slot pairs). Capacity is per
// tier in blocks with LRU order, local pins, one-shot admission (a block
// promoted to L0 counts as one-shot until it has been hit promote_admit_after
// times; one-shot blocks are evicted first), promote de-duplication and side
// effects (L0 demotions, L2->L3 demotions) reported to the control plane.
//
// Behaviour follows rust/tiered-store/src/{engine,pipeline,segment,bandwidth,
// writeback,stats}.rs of the reference, which keeps bytes in hash maps; here
// the tiers hold real memory and files.
#pragma once
#include <cstdint>
#include <deque>
#include <functional>
#include <list>
#include <mutex>
#include <map>
#include <optional>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace lakeb::tier {

enum class TierId : int { L0 = 0, L1 = 1, L2 = 2, L3 = 3, None = 4 };
enum class AccessKind : int { L0Hit = 0, L1Hit = 1, L2Hit = 2, L3Hit = 3, Miss = 4 };

struct TierCaps {
  size_t l0 = 64, l1 = 256, l2 = 1024;
};

// ---------------------------------------------------------------- segment arena
struct Placement {
  uint64_t segment_id = 0;
  uint64_t offset = 0;
};
struct Relocate {
  std::string hash;
  Placement from, to;
};

// L2 slot layout: fixed-size slots, `slots_per_segment` slots per segment file.
class SegmentArena {
 public:
  SegmentArena(uint64_t slot_bytes = 4096, size_t slots_per_segment = 64);
  uint64_t slot_bytes() const { return slot_bytes_; }
  size_t slots_per_segment() const { return per_seg_; }
  std::optional<Placement> placement(const std::string& h) const;
  Placement alloc(const std::string& h);
  // A second slot for a new record of `h` while its current slot stays valid; commit_spare
  // makes it h's placement (freeing the old slot), drop_spare gives it back.
  Placement alloc_spare(const std::string& h);
  void commit_spare(const std::string& h);
  void drop_spare(const std::string& h);
  Placement place_at(const std::string& h, uint64_t segment_id, uint64_t offset);
  bool free(const std::string& h);
  std::vector<Relocate> compact(uint64_t segment_id);
  Relocate relocate(const std::string& h, uint64_t segment_id, uint64_t offset);
  double utilization(uint64_t segment_id) const;
  size_t dense_prefix_slots(uint64_t segment_id) const;
  bool has_holes(uint64_t segment_id) const;
  std::vector<uint64_t> segment_ids() const;
  std::vector<std::string> hashes_in_segment(uint64_t segment_id) const;

 private:
  static std::string spare_key(const std::string& h) { return std::string("\0spare:", 7) + h; }
  uint64_t slot_bytes_;
  size_t per_seg_;
  std::map<uint64_t, std::vector<std::string>> segs_;  // segment -> slot owners ("" = free)
  std::unordered_map<std::string, Placement> where_;
};

// ---------------------------------------------------------------- bandwidth pool
// Token bucket for background traffic: `budget_bytes` per `window_ms`.
class BandwidthPool {
 public:
  BandwidthPool(uint64_t budget_bytes = 100ull << 20, uint64_t window_ms = 1000);
  bool try_consume(uint64_t bytes, uint64_t now_ms);
  void set_paused(bool p) { paused_ = p; }
  bool paused() const { return paused_; }
  uint64_t remaining(uint64_t now_ms);

 private:
  void roll(uint64_t now_ms);
  uint64_t budget_, window_, used_ = 0, window_start_ = 0;
  bool paused_ = false;
};

// ---------------------------------------------------------------- hit stats
struct HitStats {
  uint64_t counts[5] = {0, 0, 0, 0, 0};
  // modelled cost per access (microseconds) for L0..L3 hits and a miss (recompute)
  double cost_us[5] = {1.0, 20.0, 200.0, 5000.0, 0.0};
  void record(AccessKind k) { counts[int(k)]++; }
  uint64_t total() const { return counts[0] + counts[1] + counts[2] + counts[3] + counts[4]; }
  double hit_rate() const { return total() ? double(total() - counts[4]) / double(total()) : 0.0; }
  double l0_hit_rate() const { return total() ? double(counts[0]) / double(total()) : 0.0; }
  double modelled_cost_us() const {
    double c = 0;
    for (int i = 0; i < 5; ++i) c += cost_us[i] * double(counts[i]);
    return c;
  }
};

struct SideEffects {
  std::vector<std::string> l0_demoted;
  std::vector<std::string> l2_demoted_to_l3;
};

// Device copy the caller must perform (L0 page <-> L1 slot).
struct DeviceCopy {
  std::string hash;
  int64_t page = -1;  // device arena page
  int64_t slot = -1;  // pinned host slot
  bool to_device = true;
};

enum class BeginPromote : int { Started = 0, AlreadyInFlight = 1, AlreadyL0 = 2, Missing = 3 };

// On-disk record of one block at L2 (a segment slot) and L3 (an object file): a 64-byte
// header, then the payload. The header names the block (its 32-byte chain hash), the payload
// length and a 64-bit checksum of the payload, so a torn, stale or foreign slot is detected
// on read (the read fails and the block counts as missing) instead of returning wrong KV.
constexpr uint64_t kBlockHeaderBytes = 64;
constexpr char kBlockMagic[4] = {'L', 'K', 'B', 'K'};
constexpr uint16_t kBlockFormatVersion = 1;
uint64_t payload_checksum(const uint8_t* p, uint64_t n);

class TierEngine {
 public:
  // l1_base: pinned host buffer of l1 caps * block_bytes bytes (owned by the caller).
  TierEngine(TierCaps caps, uint64_t block_bytes, uint8_t* l1_base, const std::string& l2_dir,
             const std::string& l3_dir, const std::string& model_key = "model");
  ~TierEngine();

  TierCaps caps() const { return caps_; }
  uint64_t block_bytes() const { return block_bytes_; }
  void set_promote_admit_after(uint32_t n) { admit_after_ = n; }

  // residency
  TierId local_tier(const std::string& h) const;
  bool in_l0(const std::string& h) const { return l0_.count(h) != 0; }
  int64_t l0_page(const std::string& h) const;
  int64_t l1_slot(const std::string& h) const;
  uint8_t* l1_ptr(int64_t slot) const { return l1_base_ + uint64_t(slot) * block_bytes_; }
  bool is_l2_durable(const std::string& h) const { return l2_.count(h) != 0; }
  bool l3_present(const std::string& h) const;
  bool has_durable_backing(const std::string& h) const { return is_l2_durable(h) || l3_present(h); }
  std::optional<Placement> l2_placement(const std::string& h) const { return arena_.placement(h); }
  size_t l0_len() const { return l0_.size(); }
  size_t l1_len() const { return l1_.size(); }
  size_t l2_len() const { return l2_.size(); }
  // L2 residents from least to most recently written (the cap-demotion order)
  std::vector<std::string> l2_order() const { return {l2_order_.begin(), l2_order_.end()}; }
  size_t l3_len() const;
  uint32_t hit_count(const std::string& h) const;
  bool is_one_shot(const std::string& h) const { return one_shot_.count(h) != 0; }

  // pins
  void pin(const std::string& h) { pins_[h]++; }
  void unpin(const std::string& h);
  uint32_t pin_count(const std::string& h) const;

  // L0 bookkeeping (device pages are owned by the engine's block pool)
  void note_l0(const std::string& h, int64_t page);
  void drop_l0(const std::string& h);

  // durable write: bytes (host) -> L2 segment slot; demotes L2 -> L3 over the cap. On an
  // error nothing changed: a new block is absent from L2 and L3, an overwritten one keeps its
  // previous record, and the L2 LRU order is the one before the call.
  std::pair<TierId, SideEffects> put_durable(const std::string& h, const uint8_t* bytes);
  // copy a block's bytes into `dst` from the fastest host tier (L1 > L2 > L3)
  bool read_host(const std::string& h, uint8_t* dst) const;

  AccessKind probe(const std::string& h);
  uint64_t estimate_promote_cost(const std::string& h) const;

  // Bring a block into an L1 slot (from L2/L3) and reserve an L0 page for it.
  // Returns the device copy to perform (L1 slot -> L0 page); an L0 victim that
  // must first be copied out is reported in `evict` (page -> its L1 slot). A block
  // read from L3 also gets an L2 record again under the L2 cap (its demotions are
  // reported in fx->l2_demoted_to_l3); with every L2 resident pinned it stays L3-only.
  std::optional<DeviceCopy> promote_to_l0(const std::string& h, std::vector<DeviceCopy>* evict, SideEffects* fx,
                                          const std::function<int64_t()>& alloc_page);
  BeginPromote begin_promote(const std::string& h);
  void finish_promote(const std::string& h) { inflight_.erase(h); }
  size_t promote_inflight_len() const { return inflight_.size(); }
  // L0 -> L1 (needs durable backing); returns the device copy page -> slot
  std::optional<DeviceCopy> demote_l0(const std::string& h);
  std::optional<std::string> evict_l0_pressure_victim() const;
  bool demote_l2_to_l3(const std::string& h);
  void discard(const std::string& h);

  // defrag on the L2 arena (moves file bytes too)
  std::vector<Relocate> compact_l2_segment(uint64_t segment_id);
  Relocate colocate_l2_move(const std::string& h, uint64_t segment_id, uint64_t offset);
  SegmentArena& arena() { return arena_; }
  HitStats stats;
  uint64_t corrupt_reads() const { return corrupt_reads_; }  // records that failed validation
  uint64_t record_bytes() const { return block_bytes_ + kBlockHeaderBytes; }

 private:
  static void touch(std::list<std::string>& order, std::unordered_map<std::string, std::list<std::string>::iterator>& pos,
                    const std::string& h);
  std::string seg_path(uint64_t seg) const;
  std::string l3_path(const std::string& h) const;
  bool write_l2(const std::string& h, const uint8_t* bytes);
  bool overwrite_l2(const std::string& h, const uint8_t* bytes);
  void l2_forget(const std::string& h);
  void rehydrate_l2(const std::string& h, const uint8_t* bytes, SideEffects* fx);
  bool read_l2(const std::string& h, uint8_t* dst) const;
  bool write_l3(const std::string& h, const uint8_t* bytes);
  bool read_l3(const std::string& h, uint8_t* dst) const;
  bool write_record(int fd, const std::string& h, const uint8_t* bytes, uint64_t off) const;
  bool read_record(int fd, const std::string& h, uint8_t* dst, uint64_t off) const;
  int segment_fd(uint64_t seg) const;
  SideEffects ensure_l2_cap();
  int64_t alloc_l1_slot(SideEffects* fx);

  TierCaps caps_;
  uint64_t block_bytes_;
  uint8_t* l1_base_;
  std::string l2_dir_, l3_dir_, model_key_;
  std::unordered_map<std::string, int64_t> l0_;  // hash -> device page
  std::unordered_map<std::string, int64_t> l1_;  // hash -> host slot
  std::unordered_set<std::string> l2_;
  std::vector<int64_t> free_slots_;
  std::list<std::string> l0_order_, l1_order_, l2_order_;
  std::unordered_map<std::string, std::list<std::string>::iterator> l0_pos_, l1_pos_, l2_pos_;
  std::unordered_map<std::string, uint32_t> pins_, hits_;
  std::unordered_set<std::string> one_shot_, inflight_;
  uint32_t admit_after_ = 2;
  SegmentArena arena_;
  mutable std::mutex fd_mu_;
  mutable std::unordered_map<uint64_t, int> seg_fds_;  // open segment files, closed with the engine
  mutable uint64_t corrupt_reads_ = 0;
};

// ---------------------------------------------------------------- pipeline
enum class ActionKind : int { Promote = 0, FillMiss = 1, DemoteL0 = 2, DemoteL2 = 3, CompactSegment = 4, CoLocateMove = 5 };
struct Action {
  ActionKind kind = ActionKind::Promote;
  std::string hash;
  uint64_t segment_id = 0;
  uint64_t offset = 0;
  int failures = 0;
};
enum class LocKind : int { Present = 0, Absent = 1, Moved = 2, L3Present = 3 };
struct LocationEvent {
  LocKind kind = LocKind::Present;
  std::string hash;
  int tier = 0;  // proto Tier numbering: L0=1, L1=2, L2=3, L3=4
  std::string node_id;
  uint64_t segment_id = 0, offset = 0;
};

class TierPipeline {
 public:
  static constexpr int kMaxFailures = 3;
  TierPipeline(TierEngine* engine, BandwidthPool* bw, std::string node_id);
  void enqueue(const Action& a) { q_.push_back(a); }
  size_t pending() const { return q_.size(); }
  const std::string& node_id() const { return node_; }
  // Run up to max_steps actions and return how many succeeded. An action that fails goes
  // back to the queue until it has failed kMaxFailures times, then it is dropped; one the
  // bandwidth window cannot pay for ends the tick and stays at the front. `alloc_page`
  // provides L0 pages; device copies produced by promotions/demotions are appended to `copies`.
  std::pair<size_t, std::vector<LocationEvent>> tick(size_t max_steps, uint64_t now_ms,
                                                     const std::function<int64_t()>& alloc_page,
                                                     std::vector<DeviceCopy>* copies);

 private:
  TierEngine* eng_;
  BandwidthPool* bw_;
  std::string node_;
  std::deque<Action> q_;
};

// ---------------------------------------------------------------- writeback batcher
// Collects full blocks produced by decode and flushes them every `batch` blocks;
// drain() flushes the remainder at the request barrier.
class WritebackBatcher {
 public:
  explicit WritebackBatcher(size_t batch = 4) : batch_(batch ? batch : 1) {}
  // returns a batch to flush when the threshold is reached
  std::vector<std::string> push(const std::string& h);
  std::vector<std::string> drain();
  size_t pending() const { return buf_.size(); }
  uint64_t flushes() const { return flushes_; }

 private:
  size_t batch_;
  std::vector<std::string> buf_;
  uint64_t flushes_ = 0;
};

}  // namespace lakeb::tier
