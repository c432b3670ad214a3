#include "router/router.h"

#include <algorithm>

#include "common/hash.h"

namespace lakeb::router {

ExecMode select_exec_mode(const PrefixHint& hint, int prompt_len, Role role, double bw_gbps) {
  if (prompt_len > 0 && hint.local_hit && hint.computed_tokens > 0) return ExecMode::DDirect;
  if (hint.reused_blocks > 0 && bw_gbps > 0 && bw_gbps < kTransferBWThresholdGBps) return ExecMode::Colocated;
  if (role == Role::Prefill || role == Role::Decode) return ExecMode::PDDisagg;
  return ExecMode::Colocated;
}

std::string prefix_anchor(const std::vector<std::string>& hashes) {
  if (hashes.empty()) return std::string();
  return hashes[std::min(hashes.size(), kAnchorDepth) - 1];
}

// ------------------------------------------------------------------ mirror
uint64_t ViewMirror::apply(const cp::ViewUpdate& u) {
  std::lock_guard<std::mutex> g(mu_);
  if (u.seq == 0) {  // snapshot reset
    blocks_.clear();
    last_seq_ = 0;
    for (auto& e : u.events) upsert(e);
    return 0;
  }
  if (u.events.empty()) {  // anchor: advances the sequence only
    if (u.seq > last_seq_) last_seq_ = u.seq;
    return 0;
  }
  if (u.seq <= last_seq_) return 0;               // duplicate
  if (u.seq != last_seq_ + 1) return last_seq_ + 1;  // gap
  last_seq_ = u.seq;
  for (auto& e : u.events) {
    if (e.kind == cp::INVALIDATED) {
      auto it = blocks_.find({e.id.model_id, e.id.revision, e.id.pool_kind ? e.id.pool_kind : int(cp::TARGET)});
      if (it != blocks_.end()) it->second.erase(e.id.block_hash);
    } else {
      upsert(e);
    }
  }
  return 0;
}

void ViewMirror::upsert(const cp::ViewEvent& e) {
  auto& ns = blocks_[{e.id.model_id, e.id.revision, e.id.pool_kind ? e.id.pool_kind : int(cp::TARGET)}];
  auto& ent = ns[e.id.block_hash];
  ent.locations = e.locations;
  ent.l3_present = e.l3_present;
  if (e.kind == cp::REGISTERED) ent.block_kind = e.block_kind;
}

uint64_t ViewMirror::last_seq() const {
  std::lock_guard<std::mutex> g(mu_);
  return last_seq_;
}

size_t ViewMirror::size() const {
  std::lock_guard<std::mutex> g(mu_);
  size_t n = 0;
  for (auto& [k, v] : blocks_) n += v.size();
  return n;
}

std::vector<MirrorBlock> ViewMirror::prefix_lookup(const std::string& model, const std::string& revision,
                                                   int pool_kind, const std::vector<std::string>& hashes,
                                                   const std::string& requester) const {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<MirrorBlock> out;
  auto it = blocks_.find({model, revision, pool_kind ? pool_kind : int(cp::TARGET)});
  if (it == blocks_.end()) return out;
  for (auto& h : hashes) {
    auto b = it->second.find(h);
    if (b == it->second.end()) break;
    bool local = false;
    for (auto& l : b->second.locations) local |= (l.tier == cp::L0 && l.node_id == requester);
    out.push_back(MirrorBlock{h, local});
  }
  return out;
}

// ------------------------------------------------------------------ registry
NodeRegistry::NodeRegistry(const std::vector<std::string>& initial) {
  for (auto& id : initial) add(id);
}
std::vector<std::string> NodeRegistry::ready_ids() const {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<std::string> out;
  for (auto& id : order_)
    if (!draining_.count(id)) out.push_back(id);
  return out;
}
void NodeRegistry::inc_inflight(const std::string& id) {
  std::lock_guard<std::mutex> g(mu_);
  inflight_[id]++;
}
void NodeRegistry::dec_inflight(const std::string& id) {
  std::lock_guard<std::mutex> g(mu_);
  inflight_[id]--;
}
int64_t NodeRegistry::inflight(const std::string& id) const {
  std::lock_guard<std::mutex> g(mu_);
  auto it = inflight_.find(id);
  return it == inflight_.end() ? 0 : it->second;
}
void NodeRegistry::add(const std::string& id) {
  std::lock_guard<std::mutex> g(mu_);
  if (std::find(order_.begin(), order_.end(), id) == order_.end()) order_.push_back(id);
  draining_.erase(id);
}
bool NodeRegistry::mark_draining(const std::string& id) {
  std::lock_guard<std::mutex> g(mu_);
  if (std::find(order_.begin(), order_.end(), id) == order_.end()) return false;
  return draining_.insert(id).second;
}
void NodeRegistry::unmark_draining(const std::string& id) {
  std::lock_guard<std::mutex> g(mu_);
  draining_.erase(id);
}
void NodeRegistry::remove(const std::string& id) {
  std::lock_guard<std::mutex> g(mu_);
  order_.erase(std::remove(order_.begin(), order_.end(), id), order_.end());
  draining_.erase(id);
  inflight_.erase(id);
}
std::vector<std::string> NodeRegistry::draining() const {
  std::lock_guard<std::mutex> g(mu_);
  return std::vector<std::string>(draining_.begin(), draining_.end());
}
std::string NodeRegistry::last_ready() const {
  std::lock_guard<std::mutex> g(mu_);
  for (auto it = order_.rbegin(); it != order_.rend(); ++it)
    if (!draining_.count(*it)) return *it;
  return std::string();
}
std::string NodeRegistry::next_id() const {
  std::lock_guard<std::mutex> g(mu_);
  for (size_t i = 0;; ++i) {
    std::string id = "worker-" + std::to_string(i);
    if (std::find(order_.begin(), order_.end(), id) == order_.end()) return id;
  }
}
size_t NodeRegistry::count() const {
  std::lock_guard<std::mutex> g(mu_);
  return order_.size() - draining_.size();
}

std::string pick_node(const NodeRegistry& nodes, const ViewMirror* mirror, const std::string& model,
                      const std::vector<std::string>& hashes, const std::string& routing_key, int64_t guard) {
  auto ids = nodes.ready_ids();
  if (ids.empty()) return "worker-0";
  if (ids.size() == 1) return ids[0];
  if (guard <= 0) guard = kDefaultAffinityGuard;
  if (mirror) {
    std::vector<std::pair<int, std::string>> cands;
    for (auto& id : ids) {
      int score = 0;
      for (auto& b : mirror->prefix_lookup(model, "", cp::TARGET, hashes, id)) {
        if (!b.local_hit) break;
        ++score;
      }
      if (score > 0) cands.emplace_back(score, id);
    }
    std::stable_sort(cands.begin(), cands.end(), [](auto& a, auto& b) {
      return a.first != b.first ? a.first > b.first : a.second < b.second;
    });
    for (auto& [s, id] : cands)
      if (nodes.inflight(id) < guard) return id;
  }
  std::vector<std::string> eligible;
  for (auto& id : ids)
    if (nodes.inflight(id) < guard) eligible.push_back(id);
  if (eligible.empty()) eligible = ids;
  std::string best = eligible[0];
  uint64_t best_score = hrw_score(routing_key, best);
  for (size_t i = 1; i < eligible.size(); ++i) {
    uint64_t s = hrw_score(routing_key, eligible[i]);
    if (s > best_score || (s == best_score && eligible[i] < best)) {
      best = eligible[i];
      best_score = s;
    }
  }
  return best;
}

// ------------------------------------------------------------------ PQ
PQScheduler::PQScheduler(int max_inflight, double bp_ttl_s)
    : max_inflight_(max_inflight > 0 ? max_inflight : 1), bp_ttl_(bp_ttl_s) {}

void PQScheduler::insert_locked(Req r) {
  auto pos = std::find_if(queue_.begin(), queue_.end(), [&](const Req& q) {
    return q.priority < r.priority || (q.priority == r.priority && q.seq > r.seq);
  });
  queue_.insert(pos, std::move(r));
}

uint64_t PQScheduler::submit(int priority, const std::string& model, uint64_t* preempt) {
  std::lock_guard<std::mutex> g(mu_);
  Req r{next_ticket_++, priority, model, ++seq_, Clock::now()};
  uint64_t t = r.ticket;
  insert_locked(r);
  if (preempt) *preempt = 0;
  if (int(running_.size()) >= max_inflight_) {
    auto bp = bp_.find(model);
    bool blocked = bp != bp_.end() && Clock::now() < bp->second;
    if (!blocked) {
      const Req* victim = nullptr;
      for (auto& [tk, q] : running_) {
        if (q.abandoned) continue;
        if (!victim || q.priority < victim->priority || (q.priority == victim->priority && q.seq > victim->seq))
          victim = &q;
      }
      if (victim && priority > victim->priority && preempt) *preempt = victim->ticket;
    }
  }
  return t;
}

std::vector<uint64_t> PQScheduler::start_eligible() {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<uint64_t> out;
  auto now = Clock::now();
  while (int(running_.size()) < max_inflight_) {
    auto it = std::find_if(queue_.begin(), queue_.end(), [&](const Req& q) {
      auto bp = bp_.find(q.model);
      return !(bp != bp_.end() && now < bp->second);
    });
    if (it == queue_.end()) break;
    Req r = *it;
    queue_.erase(it);
    r.wait = std::chrono::duration<double>(now - r.enq).count();
    running_[r.ticket] = r;
    out.push_back(r.ticket);
  }
  return out;
}

void PQScheduler::finish(uint64_t ticket, bool preempted) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = running_.find(ticket);
  if (it == running_.end()) return;
  Req r = it->second;
  running_.erase(it);
  if (r.abandoned) return;
  if (preempted) {
    r.enq = Clock::now();
    insert_locked(r);
    return;
  }
  if (waits_.size() >= 4096) waits_.erase(waits_.begin());
  waits_.push_back(r.wait);
}

bool PQScheduler::cancel(uint64_t ticket) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = std::find_if(queue_.begin(), queue_.end(), [&](const Req& q) { return q.ticket == ticket; });
  if (it != queue_.end()) {
    queue_.erase(it);
    return true;
  }
  auto r = running_.find(ticket);
  if (r != running_.end()) r->second.abandoned = true;
  return false;
}

void PQScheduler::set_backpressure(const std::string& model) {
  std::lock_guard<std::mutex> g(mu_);
  bp_[model] = Clock::now() + std::chrono::duration_cast<Clock::duration>(std::chrono::duration<double>(bp_ttl_));
}
bool PQScheduler::backpressured(const std::string& model) const {
  std::lock_guard<std::mutex> g(mu_);
  auto it = bp_.find(model);
  return it != bp_.end() && Clock::now() < it->second;
}
double PQScheduler::next_backpressure_expiry_s() const {
  std::lock_guard<std::mutex> g(mu_);
  auto now = Clock::now();
  double best = -1;
  for (auto& q : queue_) {
    auto it = bp_.find(q.model);
    if (it == bp_.end() || now >= it->second) continue;
    double d = std::chrono::duration<double>(it->second - now).count();
    if (best < 0 || d < best) best = d;
  }
  return best;
}
void PQScheduler::set_max_inflight(int n) {
  std::lock_guard<std::mutex> g(mu_);
  max_inflight_ = n > 0 ? n : 1;
}
LoadReport PQScheduler::load_snapshot(const std::string& node_id) const {
  std::lock_guard<std::mutex> g(mu_);
  int rem = max_inflight_ - int(running_.size());
  return LoadReport{node_id, uint32_t(queue_.size()), uint32_t(running_.size()), uint32_t(rem < 0 ? 0 : rem)};
}
std::vector<double> PQScheduler::wait_samples() const {
  std::lock_guard<std::mutex> g(mu_);
  return waits_;
}
size_t PQScheduler::queue_len() const {
  std::lock_guard<std::mutex> g(mu_);
  return queue_.size();
}
size_t PQScheduler::in_flight() const {
  std::lock_guard<std::mutex> g(mu_);
  return running_.size();
}

// ------------------------------------------------------------------ autoscaler
Autoscaler::Autoscaler(AutoscaleConfig c) : c_(c) {
  if (c_.min_nodes <= 0) c_.min_nodes = 1;
  if (c_.max_nodes <= 0) c_.max_nodes = 8;
  if (c_.scale_out_queue_len <= 0) c_.scale_out_queue_len = 4;
  if (c_.sustain_periods <= 0) c_.sustain_periods = 3;
  if (c_.cooldown_s <= 0) c_.cooldown_s = 10.0;
}

ScaleDecision Autoscaler::evaluate(double now, int queue_len, int in_flight, int node_count) {
  bool over = queue_len >= c_.scale_out_queue_len;
  bool under = queue_len <= c_.scale_in_queue_len && in_flight <= 1;
  if (over) {
    over_++;
    under_ = 0;
  } else if (under) {
    under_++;
    over_ = 0;
  } else {
    over_ = under_ = 0;
  }
  if (now - last_ < c_.cooldown_s) return ScaleDecision::None;
  if (over_ >= c_.sustain_periods && node_count < c_.max_nodes) {
    over_ = 0;
    last_ = now;
    return ScaleDecision::ScaleOut;
  }
  if (under_ >= c_.sustain_periods && node_count > c_.min_nodes) {
    under_ = 0;
    last_ = now;
    return ScaleDecision::ScaleIn;
  }
  return ScaleDecision::None;
}

// ------------------------------------------------------------------ hot set
void HotSet::add(const std::string& node, const std::vector<cp::KVBlockID>& ids) {
  std::lock_guard<std::mutex> g(mu_);
  for (auto& id : ids) {
    if (seen_.size() >= cap_) return;
    std::string k = node + "\x1f" + id.model_id + "\x1f" + id.revision + "\x1f" + std::to_string(id.pool_kind) + "\x1f" +
                    id.block_hash;
    if (!seen_.insert(k).second) continue;
    by_node_[node].push_back(id);
  }
}
std::map<std::string, std::vector<cp::KVBlockID>> HotSet::drain() {
  std::lock_guard<std::mutex> g(mu_);
  std::map<std::string, std::vector<cp::KVBlockID>> out;
  out.swap(by_node_);
  seen_.clear();
  return out;
}
size_t HotSet::size() const {
  std::lock_guard<std::mutex> g(mu_);
  return seen_.size();
}

}  // namespace lakeb::router
