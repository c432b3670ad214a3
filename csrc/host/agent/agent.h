// Storage agent core of a node: the durable-first block commit protocol
// (PutEnd), the control-plane port it talks through, application of tier
// location events to the authority, and the backpressure memory the agent
// returns on load reports.
//
// PutEnd order (each step has its own rollback):
//   admit preflight -> flush to L2 only -> pin -> publish collateral L2->L3
//   demotions -> RegisterBlocks (discard on failure) -> REQUEST hold +1 ->
//   WRITEBACK +1 -> RequestBarrier -> WRITEBACK -1 -> hold -1 -> unpin.
// The writeback / hold flags make commit_through retry-safe.
//
// Behaviour follows rust/storage-agent/src/{putend,cp_port,lib}.rs of the
// reference; the port is a C++ interface that Python can implement (fault
// injection in tests).
#pragma once
#include <chrono>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "authority/authority.h"
#include "tier/tier.h"

namespace lakeb::agent {

class ControlPlanePort {
 public:
  virtual ~ControlPlanePort() = default;
  virtual void admit_register_blocks(const std::string& node_id, const std::vector<std::string>& prefix,
                                     const std::vector<cp::BlockMeta>& metas) = 0;
  virtual void register_blocks(const std::string& node_id, const std::vector<std::string>& prefix,
                               const std::vector<cp::BlockMeta>& metas) = 0;
  virtual void report_refs(const std::vector<cp::RefDelta>& deltas) = 0;
  virtual void request_barrier(const std::string& request_id, const std::string& node_id) = 0;
  virtual void publish_location(const cp::KVBlockID& id, int tier, const std::string& node_id, uint64_t segment_id,
                                uint64_t offset, bool present) = 0;
  virtual void set_l3_present(const cp::KVBlockID& id, bool present) = 0;
};

// Port bound to an in-process authority (commits view events after each call).
class AuthorityPort : public ControlPlanePort {
 public:
  explicit AuthorityPort(cp::Authority* a) : a_(a) {}
  void admit_register_blocks(const std::string& node_id, const std::vector<std::string>& prefix,
                             const std::vector<cp::BlockMeta>& metas) override;
  void register_blocks(const std::string& node_id, const std::vector<std::string>& prefix,
                       const std::vector<cp::BlockMeta>& metas) override;
  void report_refs(const std::vector<cp::RefDelta>& deltas) override;
  void request_barrier(const std::string& request_id, const std::string& node_id) override;
  void publish_location(const cp::KVBlockID& id, int tier, const std::string& node_id, uint64_t segment_id,
                        uint64_t offset, bool present) override;
  void set_l3_present(const cp::KVBlockID& id, bool present) override;

 private:
  cp::Authority* a_;
};

class PutEndSession {
 public:
  // node_id: the node that commits (its refs, register hold and barrier). storage_node: the node
  // whose L2 holds the blocks (their L2 locations); empty = node_id. They differ when several
  // engines share one pool node's tiers.
  PutEndSession(std::string request_id, std::string node_id, std::string model_id, std::string revision = "",
                std::string storage_node = "");
  void put_start(const std::string& block_hash, const uint8_t* bytes, size_t n);
  // Extend the prefix chain with a block that is already durable (no bytes, not re-registered).
  void add_prefix(const std::string& block_hash) {
    if (!blocks_.empty()) throw std::invalid_argument("add_prefix: chain blocks must precede new blocks");
    prefix_.push_back(block_hash);
  }
  std::vector<cp::BlockMeta> metas(const tier::TierEngine& store) const;
  std::vector<std::string> flush_durable(tier::TierEngine& store);
  void commit_through(ControlPlanePort& cp, tier::TierEngine& store);
  bool all_durable() const;
  bool writeback_open() const { return writeback_open_; }
  bool register_hold_open() const { return hold_open_; }
  const std::vector<std::string>& prefix_hashes() const { return prefix_; }
  const std::string& request_id() const { return request_id_; }

 private:
  struct Pending {
    cp::KVBlockID id;
    std::vector<uint8_t> bytes;
    bool durable = false;
  };
  std::vector<cp::RefDelta> deltas(int kind, int32_t d) const;
  bool release_hold(ControlPlanePort& cp);
  std::string request_id_, node_id_, model_id_, revision_, storage_node_;
  std::vector<std::string> prefix_;
  std::vector<Pending> blocks_;
  bool writeback_open_ = false;
  bool hold_open_ = false;
};

// Apply tier location events to the authority: best effort and idempotent
// (unknown blocks are skipped). Returns the number applied.
size_t apply_location_events(ControlPlanePort& cp, const std::string& model_id, const std::string& revision,
                             int pool_kind, const std::vector<tier::LocationEvent>& events);

// Backpressure memory: the last hard-quota signal stays "fresh" for ttl_s and is
// attached to load-report acks.
// Defrag moves the control plane planned (Authority::plan_defrag) queued on this node's tier
// pipeline: segment compactions and co-locate moves. A move addressed to another node is
// skipped (moving a block across nodes needs a transfer). Returns the number queued.
size_t enqueue_defrag_moves(tier::TierPipeline& pipe, const std::vector<cp::DefragMove>& moves);
// The control plane's PauseBackground switch applied to the node's background bandwidth: a
// paused pool admits no pipeline action (promotions, demotions and defrag wait).
inline void sync_background_pause(tier::BandwidthPool& bw, bool paused) { bw.set_paused(paused); }

class BackpressureMemory {
 public:
  explicit BackpressureMemory(double ttl_s = 30.0) : ttl_(ttl_s) {}
  void record(const cp::BackpressureSignal& s);
  bool fresh(cp::BackpressureSignal* out) const;
  void clear() { has_ = false; }

 private:
  double ttl_;
  bool has_ = false;
  cp::BackpressureSignal last_;
  std::chrono::steady_clock::time_point at_;
};

}  // namespace lakeb::agent
