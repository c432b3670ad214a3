#include "agent/agent.h"

#include <stdexcept>

namespace lakeb::agent {

using cp::BlockMeta;
using cp::KVBlockID;
using cp::Location;
using cp::RefDelta;

// ------------------------------------------------------------------ authority port
void AuthorityPort::admit_register_blocks(const std::string&, const std::vector<std::string>& prefix,
                                          const std::vector<BlockMeta>& metas) {
  if (metas.empty()) return;
  std::vector<std::string> hs;
  for (auto& m : metas) hs.push_back(m.id.block_hash);
  auto r = a_->preflight_register(metas[0].id.model_id, metas[0].id.revision, metas[0].id.pool_kind, hs);
  (void)prefix;
  if (!r.accepted)
    throw std::runtime_error("admit: rejected (" + r.backpressure.reason + ", deficit " +
                             std::to_string(r.backpressure.deficit_bytes) + " bytes)");
}
void AuthorityPort::register_blocks(const std::string& node_id, const std::vector<std::string>& prefix,
                                    const std::vector<BlockMeta>& metas) {
  auto r = a_->register_blocks(node_id, prefix, metas);
  a_->commit_pending();
  if (!r.accepted) throw std::runtime_error("register: rejected (" + r.backpressure.reason + ")");
}
void AuthorityPort::report_refs(const std::vector<RefDelta>& d) { a_->report_refs(d); }
void AuthorityPort::request_barrier(const std::string& rid, const std::string& node) { a_->complete_barrier(rid, node); }
void AuthorityPort::publish_location(const KVBlockID& id, int tier, const std::string& node, uint64_t seg, uint64_t off,
                                     bool present) {
  a_->publish_location(id, tier, node, seg, off, present);
  a_->commit_pending();
}
void AuthorityPort::set_l3_present(const KVBlockID& id, bool present) {
  a_->set_l3_present(id, present);
  a_->commit_pending();
}

// ------------------------------------------------------------------ PutEnd
PutEndSession::PutEndSession(std::string rid, std::string node, std::string model, std::string rev,
                             std::string storage_node)
    : request_id_(std::move(rid)),
      node_id_(std::move(node)),
      model_id_(std::move(model)),
      revision_(std::move(rev)),
      storage_node_(storage_node.empty() ? node_id_ : std::move(storage_node)) {}

void PutEndSession::put_start(const std::string& h, const uint8_t* bytes, size_t n) {
  prefix_.push_back(h);
  Pending p;
  p.id = KVBlockID{model_id_, h, cp::TARGET, "public", revision_};
  p.bytes.assign(bytes, bytes + n);
  blocks_.push_back(std::move(p));
}

std::vector<BlockMeta> PutEndSession::metas(const tier::TierEngine& store) const {
  std::vector<BlockMeta> out;
  for (auto& b : blocks_) {
    BlockMeta m;
    m.id = b.id;
    m.block_kind = cp::T_TYPE;
    if (store.is_l2_durable(b.id.block_hash)) {
      auto pl = store.l2_placement(b.id.block_hash);
      m.locations.push_back(Location{cp::L2, storage_node_, pl ? pl->segment_id : 1, pl ? pl->offset : 0});
    }
    m.l3_present = store.l3_present(b.id.block_hash);
    out.push_back(std::move(m));
  }
  return out;
}

std::vector<std::string> PutEndSession::flush_durable(tier::TierEngine& store) {
  std::vector<std::string> demoted;
  for (auto& b : blocks_) {
    if (b.bytes.size() != store.block_bytes())
      throw std::invalid_argument("flush: block size mismatch (" + std::to_string(b.bytes.size()) + " vs " +
                                  std::to_string(store.block_bytes()) + ")");
    // A block is named by the chain hash of its content: one that is already durable (an
    // earlier attempt of this commit, or another request's) is not written again, so a retry
    // neither moves its L2 record away from the slot the control plane was told about nor
    // brings a block the cap moved to L3 back into L2.
    if (!store.has_durable_backing(b.id.block_hash)) {
      auto [t, fx] = store.put_durable(b.id.block_hash, b.bytes.data());
      (void)t;
      demoted.insert(demoted.end(), fx.l2_demoted_to_l3.begin(), fx.l2_demoted_to_l3.end());
    }
    b.durable = store.has_durable_backing(b.id.block_hash);
    if (!b.durable) throw std::runtime_error("flush: block not settled on L2|L3");
  }
  return demoted;
}

bool PutEndSession::all_durable() const {
  for (auto& b : blocks_)
    if (!b.durable) return false;
  return true;
}

std::vector<RefDelta> PutEndSession::deltas(int kind, int32_t d) const {
  std::vector<RefDelta> out;
  for (auto& b : blocks_) out.push_back(RefDelta{b.id, kind, d, node_id_});
  return out;
}

bool PutEndSession::release_hold(ControlPlanePort& cp) {
  if (!hold_open_) return true;
  try {
    cp.report_refs(deltas(cp::REQUEST, -1));
    hold_open_ = false;
  } catch (...) {
  }
  return !hold_open_;
}

void PutEndSession::commit_through(ControlPlanePort& cp, tier::TierEngine& store) {
  if (blocks_.empty()) return;
  cp.admit_register_blocks(node_id_, prefix_, metas(store));
  auto demoted = flush_durable(store);
  if (!all_durable()) throw std::runtime_error("commit: not settled on L2|L3");
  for (auto& b : blocks_) store.pin(b.id.block_hash);
  auto unpin_all = [&] {
    for (auto& b : blocks_) {
      try {
        store.unpin(b.id.block_hash);
      } catch (...) {
      }
    }
  };
  try {
    for (auto& h : demoted) {
      bool ours = false;
      for (auto& b : blocks_) ours |= b.id.block_hash == h;
      if (ours) continue;
      KVBlockID id{model_id_, h, cp::TARGET, "public", revision_};
      cp.publish_location(id, cp::L2, storage_node_, 0, 0, false);
      cp.set_l3_present(id, true);
    }
  } catch (...) {
    unpin_all();
    throw;
  }
  try {
    cp.register_blocks(node_id_, prefix_, metas(store));
  } catch (...) {
    for (auto& b : blocks_) {
      try {
        store.unpin(b.id.block_hash);
      } catch (...) {
      }
      b.durable = false;
    }
    throw;
  }
  try {
    for (auto& b : blocks_) {
      if (store.l3_present(b.id.block_hash)) cp.set_l3_present(b.id, true);
      if (!store.is_l2_durable(b.id.block_hash)) cp.publish_location(b.id, cp::L2, storage_node_, 0, 0, false);
    }
    if (!hold_open_) {
      cp.report_refs(deltas(cp::REQUEST, +1));
      hold_open_ = true;
    }
  } catch (...) {
    unpin_all();
    throw;
  }
  if (!writeback_open_) {
    try {
      cp.report_refs(deltas(cp::WRITEBACK, +1));
      writeback_open_ = true;
    } catch (...) {
      release_hold(cp);
      unpin_all();
      throw;
    }
  }
  try {
    cp.request_barrier(request_id_, node_id_);
  } catch (const std::exception& e) {
    bool rolled = false;
    try {
      cp.report_refs(deltas(cp::WRITEBACK, -1));
      writeback_open_ = false;
      rolled = true;
    } catch (const std::exception& re) {
      unpin_all();
      throw std::runtime_error(std::string(e.what()) + "; writeback rollback failed after barrier error: " + re.what());
    }
    unpin_all();
    (void)rolled;
    throw std::runtime_error(std::string(e.what()) +
                             "; barrier failed - REQUEST register-hold retained, block frozen pending retry/discard");
  }
  if (writeback_open_) {
    try {
      cp.report_refs(deltas(cp::WRITEBACK, -1));
      writeback_open_ = false;
    } catch (const std::exception& e) {
      bool retained = !release_hold(cp);
      unpin_all();
      throw std::runtime_error(std::string(e.what()) +
                               "; barrier succeeded but WRITEBACK -1 failed: refs retain +1 pending node reconcile" +
                               (retained ? "; REQUEST register-hold release also failed" : ""));
    }
  }
  if (hold_open_) {
    try {
      cp.report_refs(deltas(cp::REQUEST, -1));
      hold_open_ = false;
    } catch (const std::exception& e) {
      unpin_all();
      throw std::runtime_error(std::string(e.what()) + "; register-hold release failed after barrier");
    }
  }
  for (auto& b : blocks_) store.unpin(b.id.block_hash);
}

// ------------------------------------------------------------------ location events
size_t apply_location_events(ControlPlanePort& cp, const std::string& model_id, const std::string& revision,
                             int pool_kind, const std::vector<tier::LocationEvent>& events) {
  size_t n = 0;
  for (auto& e : events) {
    KVBlockID id{model_id, e.hash, pool_kind, "public", revision};
    try {
      switch (e.kind) {
        case tier::LocKind::Present:
          cp.publish_location(id, e.tier, e.node_id, e.segment_id, e.offset, true);
          break;
        case tier::LocKind::Absent:
          cp.publish_location(id, e.tier, e.node_id, 0, 0, false);
          break;
        case tier::LocKind::Moved:
          cp.publish_location(id, e.tier, e.node_id, e.segment_id, e.offset, true);
          break;
        case tier::LocKind::L3Present:
          cp.set_l3_present(id, true);
          break;
      }
      ++n;
    } catch (...) {
      // best effort: an unknown block (never registered) is skipped
    }
  }
  return n;
}

size_t enqueue_defrag_moves(tier::TierPipeline& pipe, const std::vector<cp::DefragMove>& moves) {
  size_t n = 0;
  for (auto& m : moves) {
    if (!m.node_id.empty() && m.node_id != pipe.node_id()) continue;
    tier::Action a;
    if (m.compact_segment) {
      a.kind = tier::ActionKind::CompactSegment;
      a.segment_id = m.segment_id;
    } else if (!m.id.block_hash.empty()) {
      a.kind = tier::ActionKind::CoLocateMove;
      a.hash = m.id.block_hash;
      a.segment_id = m.to_segment;
      a.offset = m.to_offset;
    } else {
      continue;
    }
    pipe.enqueue(a);
    ++n;
  }
  return n;
}

// ------------------------------------------------------------------ backpressure
void BackpressureMemory::record(const cp::BackpressureSignal& s) {
  last_ = s;
  has_ = true;
  at_ = std::chrono::steady_clock::now();
}
bool BackpressureMemory::fresh(cp::BackpressureSignal* out) const {
  if (!has_) return false;
  double age = std::chrono::duration<double>(std::chrono::steady_clock::now() - at_).count();
  if (age > ttl_) return false;
  if (out) *out = last_;
  return true;
}

}  // namespace lakeb::agent
