// Request-control-plane core of the Router: execution-mode selection,
// prefix-affinity / rendezvous node choice, the priority queue with
// preemption and per-model backpressure, the read-only replica of the pool's
// location view, the queue-depth autoscaler, the node registry and the batched
// hot-hit set.
//
// Decisions are synchronous and thread-safe; the asyncio front end
// (lake_b200/router/http.py) drives them. Behaviour follows go/router/
// {modeselect,affinity,pq,mirror,autoscale}.go of the reference; the HRW score
// keeps its byte layout fnv1a64(u64-LE len(key) || key || node) so pool-side
// pre-placement and router cold-path choices agree.
#pragma once
#include <chrono>
#include <cstdint>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

#include "authority/types.h"

namespace lakeb::router {

enum class ExecMode : int { Colocated = 0, PDDisagg = 1, DDirect = 2 };
enum class Role : int { Hybrid = 0, Prefill = 1, Decode = 2 };

constexpr double kTransferBWThresholdGBps = 1.0;
constexpr int64_t kDefaultAffinityGuard = 8;
constexpr size_t kAnchorDepth = 8;

struct PrefixHint {
  int computed_tokens = 0;
  int reused_blocks = 0;
  int local_hit_blocks = 0;
  bool local_hit = false;
};

ExecMode select_exec_mode(const PrefixHint& hint, int prompt_len, Role role, double bw_gbps);
std::string prefix_anchor(const std::vector<std::string>& hashes);

// ---------------------------------------------------------------- view mirror
struct MirrorBlock {
  std::string hash;
  bool local_hit = false;
};

class ViewMirror {
 public:
  // Returns 0 on success, or the expected seq when the update leaves a gap
  // (the caller then resumes from last_seq()).
  uint64_t apply(const cp::ViewUpdate& u);
  uint64_t last_seq() const;
  // Contiguous prefix match; local_hit = an L0 copy on `requester`.
  std::vector<MirrorBlock> prefix_lookup(const std::string& model, const std::string& revision, int pool_kind,
                                         const std::vector<std::string>& hashes, const std::string& requester) const;
  size_t size() const;

 private:
  struct Entry {
    std::vector<cp::Location> locations;
    bool l3_present = false;
    int block_kind = 0;
  };
  using NsKey = std::tuple<std::string, std::string, int>;
  void upsert(const cp::ViewEvent& e);
  mutable std::mutex mu_;
  uint64_t last_seq_ = 0;
  std::map<NsKey, std::unordered_map<std::string, Entry>> blocks_;
};

// ---------------------------------------------------------------- node registry
class NodeRegistry {
 public:
  explicit NodeRegistry(const std::vector<std::string>& initial = {});
  std::vector<std::string> ready_ids() const;
  void inc_inflight(const std::string& id);
  void dec_inflight(const std::string& id);
  int64_t inflight(const std::string& id) const;
  void add(const std::string& id);
  bool mark_draining(const std::string& id);
  void unmark_draining(const std::string& id);
  void remove(const std::string& id);
  std::vector<std::string> draining() const;
  std::string last_ready() const;
  std::string next_id() const;
  size_t count() const;

 private:
  mutable std::mutex mu_;
  std::vector<std::string> order_;
  std::set<std::string> draining_;
  std::unordered_map<std::string, int64_t> inflight_;
};

// Prefix-affinity node choice: hot path = best contiguous local-L0 prefix under
// the in-flight guard; cold path = rendezvous hash of the routing key.
std::string pick_node(const NodeRegistry& nodes, const ViewMirror* mirror, const std::string& model,
                      const std::vector<std::string>& hashes, const std::string& routing_key, int64_t guard);

// ---------------------------------------------------------------- priority queue
struct LoadReport {
  std::string node_id;
  uint32_t queue_len = 0, in_flight = 0, remaining_cap = 0;
};

class PQScheduler {
 public:
  PQScheduler(int max_inflight, double bp_ttl_s);
  // Enqueue; returns the ticket. If the new request outranks the lowest-priority
  // running one while all slots are busy, that ticket is returned in `preempt`.
  uint64_t submit(int priority, const std::string& model, uint64_t* preempt);
  // Tickets to start now (priority desc, FIFO within a priority; backpressured
  // models are skipped, not dropped).
  std::vector<uint64_t> start_eligible();
  // A running ticket ended; preempted tickets are requeued with a fresh wait clock.
  void finish(uint64_t ticket, bool preempted);
  bool cancel(uint64_t ticket);  // waiting -> removed; running -> marked abandoned
  void set_backpressure(const std::string& model);
  bool backpressured(const std::string& model) const;
  double next_backpressure_expiry_s() const;  // seconds until the earliest expiry of a queued model, <0 none
  void set_max_inflight(int n);
  LoadReport load_snapshot(const std::string& node_id) const;
  std::vector<double> wait_samples() const;
  size_t queue_len() const;
  size_t in_flight() const;

 private:
  using Clock = std::chrono::steady_clock;
  struct Req {
    uint64_t ticket;
    int priority;
    std::string model;
    uint64_t seq;
    Clock::time_point enq;
    double wait = 0;
    bool abandoned = false;
  };
  void insert_locked(Req r);
  mutable std::mutex mu_;
  int max_inflight_;
  double bp_ttl_;
  uint64_t next_ticket_ = 1, seq_ = 0;
  std::vector<Req> queue_;
  std::map<uint64_t, Req> running_;
  std::map<std::string, Clock::time_point> bp_;
  std::vector<double> waits_;
};

// ---------------------------------------------------------------- autoscaler
enum class ScaleDecision : int { None = 0, ScaleOut = 1, ScaleIn = 2 };
struct AutoscaleConfig {
  int min_nodes = 1, max_nodes = 8, scale_out_queue_len = 4, scale_in_queue_len = 0, sustain_periods = 3;
  double cooldown_s = 10.0;
};
class Autoscaler {
 public:
  explicit Autoscaler(AutoscaleConfig c);
  ScaleDecision evaluate(double now_s, int queue_len, int in_flight, int node_count);

 private:
  AutoscaleConfig c_;
  int over_ = 0, under_ = 0;
  double last_ = -1e18;
};

// Batched (node, block) hit reports for the control plane.
class HotSet {
 public:
  explicit HotSet(size_t cap = 4096) : cap_(cap) {}
  void add(const std::string& node, const std::vector<cp::KVBlockID>& ids);
  std::map<std::string, std::vector<cp::KVBlockID>> drain();
  size_t size() const;

 private:
  mutable std::mutex mu_;
  size_t cap_;
  std::set<std::string> seen_;
  std::map<std::string, std::vector<cp::KVBlockID>> by_node_;
};

}  // namespace lakeb::router
