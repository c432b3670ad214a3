// Location-view authority of the KV storage pool.
//
// One namespace per (model_id, revision); inside it one pool view per
// pool_kind (TARGET / DRAFT). A pool view holds every registered block keyed
// by its flat chain hash, the lineage of each block (a 64-bit positional hash
// of the whole prefix, so a flat hash reached through a different prefix is
// a miss), per-kind reference counts, an inactive (evictable) index with
// leaf-only, frequency-bucketed eviction, per-(block, node) hit counts and
// placement marks. Every state change emits view events that are committed to
// a bounded replay log (seq 0 is reserved for snapshots).
//
// Behaviour follows the reference control plane
// (rust/controlplane/src/authority.rs:358-1593, quota.rs, view.rs,
//  placement.rs, shard.rs, reconcile.rs, defrag.rs); the data structures are
// this file's own (no Dynamo registry).
#pragma once
#include <cstdint>
#include <deque>
#include <functional>
#include <list>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "authority/types.h"

namespace lakeb::cp {

constexpr size_t kInactiveCap = 4096;
constexpr uint8_t kFreqThresholds[3] = {3, 8, 15};
constexpr size_t kViewLogCap = 1024;
constexpr uint64_t kDefaultOrphanTtlMs = 30000;
constexpr uint32_t kDefaultVnodes = 64;
constexpr uint32_t kFollowHitThreshold = 2;
constexpr size_t kFollowEvalLimit = 16;
constexpr size_t kAnchorDepthCap = 8;
constexpr uint64_t kDefaultSlotBytes = 4096;

// Count-min sketch with 4-bit saturating counters and periodic halving
// (TinyLFU admission/frequency estimate).
class FrequencySketch {
 public:
  explicit FrequencySketch(size_t width = 4096);
  void touch(uint64_t key);
  uint8_t estimate(uint64_t key) const;

 private:
  size_t width_;
  std::vector<uint8_t> rows_[4];
  uint64_t adds_ = 0;
  uint64_t reset_at_;
};

// Zero-ref (evictable) blocks of one pool view, keyed by lineage.
//
// Entries are split by shape: a leaf (no registered child) can go now, an inner
// block waits until its last registered child is gone (the authority reports that
// through set_leaf). A batch eviction ranks the current leaves once by (frequency
// bucket, release order), takes the coldest, and ranks again only if the removals
// turned parents into leaves and the batch is still short: one pass per lineage
// level instead of one scan per victim.
//
// The index holds at most `cap` entries. A release past the cap is not dropped:
// it waits in an overflow FIFO and enters the index as room frees up, so every
// zero-ref block eventually becomes evictable and quota planning can count it.
class InactiveIndex {
 public:
  explicit InactiveIndex(size_t cap) : cap_(cap) {}
  bool has(uint64_t lin) const;                 // indexed (not waiting in overflow)
  size_t size() const { return indexed_; }      // indexed entries (<= cap)
  size_t waiting() const { return spill_.size(); }
  size_t evictable() const { return indexed_ + spill_.size(); }
  size_t cap() const { return cap_; }
  void release(uint64_t lin, bool leaf);        // ref total reached zero
  bool retain(uint64_t lin);                    // ref total left zero (or the block is gone)
  void set_leaf(uint64_t lin, bool leaf);       // child count crossed zero
  // Takes up to n coldest leaves. `drop` removes each victim's block (which may turn
  // its parent into a leaf through set_leaf) before the next one is taken.
  size_t evict(size_t n, const std::function<uint8_t(uint64_t)>& freq, const std::function<void(uint64_t)>& drop);

 private:
  struct Slot {
    uint64_t tick = 0;
    bool leaf = true;
    bool spilled = false;
  };
  void admit(uint64_t lin, Slot& s);  // overflow or indexed
  void refill();

  size_t cap_;
  uint64_t tick_ = 0;
  size_t indexed_ = 0;
  std::unordered_map<uint64_t, Slot> slots_;
  std::map<uint64_t, uint64_t> leaves_;  // release tick -> lineage (indexed leaves)
  std::list<uint64_t> spill_;            // overflow, oldest first
  std::unordered_map<uint64_t, std::list<uint64_t>::iterator> spill_at_;
};

struct RefAccounts {
  int64_t request = 0;
  int64_t writeback = 0;
  int64_t total() const { return request + writeback; }
  int64_t& bucket(int kind) { return kind == WRITEBACK ? writeback : request; }
  int64_t get(int kind) const { return kind == WRITEBACK ? writeback : request; }
};

struct Entry {
  uint64_t lineage = 0;
  uint64_t parent = 0;  // parent lineage (0 = root)
  BlockMeta meta;
  uint64_t block_id = 0;
  std::vector<std::string> prefix_chain;
  int64_t registered_children = 0;
};

struct PoolView {
  explicit PoolView(size_t cap) : inactive(cap) {}
  std::unordered_map<std::string, Entry> by_flat;
  std::unordered_map<uint64_t, std::string> lin_to_flat;
  std::unordered_map<uint64_t, RefAccounts> refs;
  InactiveIndex inactive;
  FrequencySketch freq;
  std::unordered_map<std::string, std::map<std::string, uint32_t>> hit_counts;
  std::set<std::pair<std::string, std::string>> placement_marks;
  uint64_t next_block_id = 1;
};

struct Namespace {
  ModelDescriptor desc;
  std::map<int, std::unique_ptr<PoolView>> pools;
  int64_t used_bytes = 0;
  int64_t bytes_per_block() const { return desc.bytes_per_block > 0 ? int64_t(desc.bytes_per_block) : 1; }
};

struct OrphanEntry {
  std::string node_id;
  uint64_t marked_at_ms = 0;
};

class Authority {
 public:
  explicit Authority(size_t inactive_cap = kInactiveCap, int64_t pool_capacity_bytes = 0);

  // ----- models / quota
  void register_model(const ModelDescriptor& d);
  void deregister_model(const std::string& model_id, const std::string& revision);
  bool has_namespace(const std::string& model_id, const std::string& revision) const;
  void set_quota(const std::string& model_id, const std::string& revision, const Quota& q);
  Quota get_quota(const std::string& model_id, const std::string& revision) const;
  int64_t used_bytes(const std::string& model_id, const std::string& revision) const;
  std::vector<ModelDescriptor> models() const;

  // ----- blocks
  RegisterResult preflight_register(const std::string& model_id, const std::string& revision, int pool_kind,
                                    const std::vector<std::string>& block_hashes) const;
  RegisterResult register_blocks(const std::string& node_id, const std::vector<std::string>& prefix_hashes,
                                 std::vector<BlockMeta> metas);
  LookupResult lookup_prefix(const std::string& model_id, const std::string& revision, int pool_kind,
                             const std::vector<std::string>& prefix_hashes, const std::string& requester);
  std::vector<BlockMeta> locate(const std::vector<KVBlockID>& ids) const;
  void report_refs(const std::vector<RefDelta>& deltas);  // all-or-nothing
  std::pair<int64_t, int64_t> refs_by_kind(const KVBlockID& id) const;
  void complete_barrier(const std::string& request_id, const std::string& node_id);
  bool barrier_completed(const std::string& request_id) const;
  void publish_location(const KVBlockID& id, int tier, const std::string& node_id, uint64_t segment_id,
                        uint64_t offset, bool present);
  void set_l3_present(const KVBlockID& id, bool present);
  size_t evict_n(const std::string& model_id, const std::string& revision, int pool_kind, size_t n);
  size_t inactive_len(const std::string& model_id, const std::string& revision, int pool_kind) const;
  size_t block_count(const std::string& model_id, const std::string& revision) const;

  // ----- view log
  ViewUpdate commit_pending();  // seq = next; empty events allowed (anchor)
  std::vector<ViewUpdate> replay_after(uint64_t from_seq, bool* ok) const;
  ViewUpdate snapshot() const;  // seq 0, REGISTERED for every block
  uint64_t last_seq() const { return next_seq_ - 1; }
  // Committed updates kept for resuming subscribers (older resume points get a snapshot).
  void set_view_log_cap(size_t n);
  size_t view_log_cap() const { return log_cap_; }
  size_t pending_events() const { return pending_.size(); }

  // ----- reconcile / GC
  void report_orphans(const std::vector<OrphanReport>& reports);
  std::vector<KVBlockID> discard_blocks(const std::vector<KVBlockID>& ids);
  std::vector<KVBlockID> sweep_orphans(uint64_t ttl_ms);
  std::pair<std::vector<KVBlockID>, std::vector<KVBlockID>> gc_cold(const std::string& model_id,
                                                                   const std::string& revision, int pool_kind,
                                                                   size_t n);
  std::pair<uint32_t, std::vector<KVBlockID>> reconcile_dead_node(const std::string& node_id);
  size_t orphan_count() const { return orphans_.size(); }
  void set_clock(std::function<uint64_t()> now_ms) { now_ms_ = std::move(now_ms); }

  // ----- checkpoint
  CheckpointSnapshot export_snapshot();
  void import_snapshot(const CheckpointSnapshot& snap);

  // ----- shard ring / hits / placement
  ShardMap shard_map() const;
  std::vector<ShardMigration> join_shard_node(const std::string& node_id, uint32_t vnodes,
                                              std::vector<KVBlockID>* warmup);
  std::pair<std::vector<ShardMigration>, std::vector<KVBlockID>> drain_shard_node(const std::string& node_id);
  void remove_shard_node(const std::string& node_id);
  std::string shard_owner(const std::string& block_hash) const;
  std::vector<std::string> ready_nodes() const;
  void report_hits(const std::string& node_id, const std::vector<KVBlockID>& ids,
                   std::vector<PlacementPlan>* follow_plans);
  uint32_t hit_count(const KVBlockID& id) const;
  uint32_t hit_count_on(const KVBlockID& id, const std::string& node) const;
  std::vector<KVBlockID> warmup_plan(const std::string& node_id, size_t k) const;
  bool preplace_on_register(const std::string& model_id, const std::string& revision, int pool_kind,
                            const std::vector<std::string>& prefix_hashes, PlacementPlan* out);

  // ----- defrag
  double l2_fragmentation_ratio(const std::string& model_id, const std::string& revision, int pool_kind,
                                uint64_t slot_bytes) const;
  std::vector<DefragMove> plan_defrag(const std::string& model_id, const std::string& revision, int pool_kind,
                                      int mode, uint64_t slot_bytes) const;
  size_t relocate_in_view(const std::vector<DefragMove>& moves);
  void set_background_paused(bool p) { bg_paused_ = p; }
  bool background_paused() const { return bg_paused_; }

  static int resolve_pool_kind(int raw);
  static std::vector<uint64_t> lineage_from_prefix(const std::vector<std::string>& prefix_hashes);

 private:
  struct BlockKey {
    std::string model_id, revision;
    int pool_kind;
    std::string flat;
    bool operator<(const BlockKey& o) const {
      return std::tie(model_id, revision, pool_kind, flat) < std::tie(o.model_id, o.revision, o.pool_kind, o.flat);
    }
  };
  static BlockKey key_of(const KVBlockID& id);
  Namespace* ns(const std::string& m, const std::string& r);
  const Namespace* ns(const std::string& m, const std::string& r) const;
  PoolView* pool(Namespace* n, int pk, bool create);
  const PoolView* pool(const Namespace* n, int pk) const;
  Entry* find(const KVBlockID& id, PoolView** pv = nullptr, Namespace** nsp = nullptr);
  const Entry* find(const KVBlockID& id) const;
  // admission (own eviction, hard limit, borrowing against pool capacity)
  struct AdmitPlan {
    bool accept = true;
    size_t evict_own = 0;      // own zero-ref blocks to evict first
    int64_t from_lenders = 0;  // bytes to take back from namespaces above their soft quota
    BackpressureSignal bp;
  };
  AdmitPlan plan_admit(const Namespace& n, size_t fresh_blocks) const;
  int64_t pool_used_bytes() const;
  int64_t lendable_bytes(const Namespace& n) const;
  int64_t take_from_lenders(const Namespace* borrower, int64_t bytes);
  // eviction
  size_t evict_in(Namespace* n, PoolView* p, size_t count);
  size_t evict_ns(Namespace* n, size_t count);
  void remove_entry(PoolView* p, const std::string& flat);
  void link_child(PoolView* p, uint64_t parent, int step);
  // view events
  void emit_upsert(int kind, const BlockMeta& m);
  void emit_invalidated(const KVBlockID& id);
  // refs: settle a block's zero crossing after its ledger changed from `was` (held_between:
  // it was referenced at some point in between, so ending at zero is a release)
  void settle_refs(PoolView* p, const Entry& e, const RefAccounts& was, bool held_between);
  // registration
  struct RegisterBatch {
    Namespace* n = nullptr;
    int pool_kind = TARGET;
    std::vector<size_t> pos;  // prefix index of each meta
    size_t fresh = 0;         // distinct hashes not yet registered
  };
  RegisterBatch check_register(const std::vector<std::string>& prefix_hashes, const std::vector<BlockMeta>& metas,
                               bool need_durable);
  void rebuild_ring();
  std::vector<std::pair<std::string, KVBlockID>> all_block_keys() const;
  std::string owner_on(const std::map<uint64_t, std::string>& ring, const std::string& key) const;

  std::map<std::pair<std::string, std::string>, std::unique_ptr<Namespace>> namespaces_;
  size_t inactive_cap_;
  int64_t pool_capacity_bytes_;
  std::unordered_map<std::string, std::string> barriers_;
  std::map<BlockKey, OrphanEntry> orphans_;
  std::map<std::string, std::map<BlockKey, RefAccounts>> node_refs_;
  std::function<uint64_t()> now_ms_;
  uint64_t checkpoint_seq_ = 0;
  // view log
  std::deque<ViewUpdate> log_;
  size_t log_cap_ = kViewLogCap;
  uint64_t next_seq_ = 1;
  std::vector<ViewEvent> pending_;
  // shard ring
  struct NodeState {
    uint32_t vnodes = kDefaultVnodes;
    bool draining = false;
    std::vector<uint64_t> hashes;
  };
  std::map<std::string, NodeState> nodes_;
  std::map<uint64_t, std::string> ring_;
  uint64_t generation_ = 0;
  bool bg_paused_ = false;
};

}  // namespace lakeb::cp
