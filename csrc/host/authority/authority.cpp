#include "authority/authority.h"

#include <algorithm>
#include <chrono>
#include <stdexcept>
#include <tuple>

#include "common/hash.h"

namespace lakeb::cp {

namespace {
uint64_t wall_ms() {
  return static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::system_clock::now().time_since_epoch())
          .count());
}
[[noreturn]] void fail(const std::string& msg) { throw std::invalid_argument(msg); }
bool has_tier(const BlockMeta& m, int tier) {
  for (auto& l : m.locations)
    if (l.tier == tier) return true;
  return false;
}
bool has_tier_on(const BlockMeta& m, int tier, const std::string& node) {
  for (auto& l : m.locations)
    if (l.tier == tier && l.node_id == node) return true;
  return false;
}
const char* ref_kind_name(int k) { return k == WRITEBACK ? "WRITEBACK" : "REQUEST"; }
int resolve_ref_kind(int raw) {
  if (raw == REQUEST || raw == WRITEBACK) return raw;
  fail("RefDelta: unsupported ref_kind " + std::to_string(raw) + " (want REQUEST/WRITEBACK)");
}
uint8_t bucket_of(uint8_t f) {
  if (f < kFreqThresholds[0]) return 0;
  if (f < kFreqThresholds[1]) return 1;
  if (f < kFreqThresholds[2]) return 2;
  return 3;
}
}  // namespace

// ------------------------------------------------------------------ sketch
FrequencySketch::FrequencySketch(size_t width) : width_(width), reset_at_(uint64_t(width) * 10) {
  for (auto& r : rows_) r.assign(width_, 0);
}
void FrequencySketch::touch(uint64_t key) {
  for (int i = 0; i < 4; ++i) {
    auto& c = rows_[i][mix64(key + 0x9e3779b97f4a7c15ull * (i + 1)) % width_];
    if (c < 15) ++c;
  }
  if (++adds_ >= reset_at_) {  // aging: halve all counters
    for (auto& r : rows_)
      for (auto& c : r) c >>= 1;
    adds_ /= 2;
  }
}
uint8_t FrequencySketch::estimate(uint64_t key) const {
  uint8_t m = 15;
  for (int i = 0; i < 4; ++i) m = std::min(m, rows_[i][mix64(key + 0x9e3779b97f4a7c15ull * (i + 1)) % width_]);
  return m;
}

// ------------------------------------------------------------------ inactive index
bool InactiveIndex::insert(uint64_t lin) {
  if (order_.count(lin) || order_.size() >= cap_) return false;
  order_[lin] = tick_++;
  return true;
}
bool InactiveIndex::take(uint64_t lin) { return order_.erase(lin) != 0; }
std::vector<uint64_t> InactiveIndex::allocate(size_t n, const std::function<bool(uint64_t)>& is_leaf,
                                              const std::function<uint8_t(uint64_t)>& freq) {
  std::vector<uint64_t> out;
  while (out.size() < n && !order_.empty()) {
    // candidates: leaves; order by (frequency bucket, insertion tick)
    uint64_t best = 0;
    std::pair<uint8_t, uint64_t> best_key{255, ~0ull};
    bool found = false;
    for (auto& [lin, tick] : order_) {
      if (!is_leaf(lin)) continue;
      std::pair<uint8_t, uint64_t> k{bucket_of(freq(lin)), tick};
      if (!found || k < best_key) {
        best_key = k;
        best = lin;
        found = true;
      }
    }
    if (!found) break;
    order_.erase(best);
    out.push_back(best);
  }
  return out;
}

// ------------------------------------------------------------------ authority basics
Authority::Authority(size_t inactive_cap, int64_t pool_capacity_bytes)
    : inactive_cap_(std::max<size_t>(1, inactive_cap)), pool_capacity_bytes_(pool_capacity_bytes), now_ms_(wall_ms) {}

int Authority::resolve_pool_kind(int raw) {
  if (raw == POOL_UNSPECIFIED) return TARGET;
  if (raw == TARGET || raw == DRAFT) return raw;
  fail("unsupported pool_kind " + std::to_string(raw));
}

std::vector<uint64_t> Authority::lineage_from_prefix(const std::vector<std::string>& prefix_hashes) {
  std::vector<uint64_t> out;
  out.reserve(prefix_hashes.size());
  uint64_t parent = 0;
  for (size_t i = 0; i < prefix_hashes.size(); ++i) {
    uint64_t h = hash64(prefix_hashes[i], parent ^ mix64(i + 1));
    if (h == 0) h = 1;
    out.push_back(h);
    parent = h;
  }
  return out;
}

Authority::BlockKey Authority::key_of(const KVBlockID& id) {
  return BlockKey{id.model_id, id.revision, resolve_pool_kind(id.pool_kind), id.block_hash};
}

Namespace* Authority::ns(const std::string& m, const std::string& r) {
  auto it = namespaces_.find({m, r});
  return it == namespaces_.end() ? nullptr : it->second.get();
}
const Namespace* Authority::ns(const std::string& m, const std::string& r) const {
  auto it = namespaces_.find({m, r});
  return it == namespaces_.end() ? nullptr : it->second.get();
}
PoolView* Authority::pool(Namespace* n, int pk, bool create) {
  auto it = n->pools.find(pk);
  if (it != n->pools.end()) return it->second.get();
  if (!create) return nullptr;
  auto& p = n->pools[pk];
  p = std::make_unique<PoolView>(inactive_cap_);
  return p.get();
}
const PoolView* Authority::pool(const Namespace* n, int pk) const {
  auto it = n->pools.find(pk);
  return it == n->pools.end() ? nullptr : it->second.get();
}
Entry* Authority::find(const KVBlockID& id, PoolView** pv, Namespace** nsp) {
  Namespace* n = ns(id.model_id, id.revision);
  if (!n) return nullptr;
  PoolView* p = pool(n, resolve_pool_kind(id.pool_kind), false);
  if (!p) return nullptr;
  auto it = p->by_flat.find(id.block_hash);
  if (it == p->by_flat.end()) return nullptr;
  if (pv) *pv = p;
  if (nsp) *nsp = n;
  return &it->second;
}
const Entry* Authority::find(const KVBlockID& id) const {
  const Namespace* n = ns(id.model_id, id.revision);
  if (!n) return nullptr;
  const PoolView* p = pool(n, resolve_pool_kind(id.pool_kind));
  if (!p) return nullptr;
  auto it = p->by_flat.find(id.block_hash);
  return it == p->by_flat.end() ? nullptr : &it->second;
}

// ------------------------------------------------------------------ models
void Authority::register_model(const ModelDescriptor& d) {
  if (d.model_id.empty()) fail("RegisterModel: model_id required");
  if (d.quota.soft_bytes < 0 || d.quota.hard_bytes < 0) fail("quota: soft/hard_bytes must be non-negative");
  if (d.quota.hard_bytes > 0 && d.quota.soft_bytes > d.quota.hard_bytes)
    fail("quota: soft_bytes must be <= hard_bytes when hard>0");
  auto* n = ns(d.model_id, d.revision);
  if (n) {
    const auto& a = n->desc;
    if (a.num_layers != d.num_layers || a.hash_algo != d.hash_algo || a.block_tokens != d.block_tokens ||
        a.bytes_per_block != d.bytes_per_block)
      fail("RegisterModel: descriptor conflicts with the registered identity of (" + d.model_id + ", " + d.revision +
           ")");
    n->desc.quota = d.quota;  // idempotent re-register may update the quota
    return;
  }
  auto ns_ptr = std::make_unique<Namespace>();
  ns_ptr->desc = d;
  namespaces_[{d.model_id, d.revision}] = std::move(ns_ptr);
}

void Authority::deregister_model(const std::string& model_id, const std::string& revision) {
  auto it = namespaces_.find({model_id, revision});
  if (it == namespaces_.end()) fail("DeregisterModel: unknown namespace (" + model_id + ")");
  for (auto& [pk, p] : it->second->pools)
    for (auto& [flat, e] : p->by_flat) emit_invalidated(e.meta.id);
  namespaces_.erase(it);
}

bool Authority::has_namespace(const std::string& m, const std::string& r) const { return ns(m, r) != nullptr; }

void Authority::set_quota(const std::string& m, const std::string& r, const Quota& q) {
  auto* n = ns(m, r);
  if (!n) fail("SetModelQuota: unknown namespace (" + m + ")");
  if (q.soft_bytes < 0 || q.hard_bytes < 0) fail("quota: soft/hard_bytes must be non-negative");
  if (q.hard_bytes > 0 && q.soft_bytes > q.hard_bytes) fail("quota: soft_bytes must be <= hard_bytes when hard>0");
  n->desc.quota = q;
}
Quota Authority::get_quota(const std::string& m, const std::string& r) const {
  auto* n = ns(m, r);
  if (!n) fail("GetModelQuota: unknown namespace (" + m + ")");
  return n->desc.quota;
}
int64_t Authority::used_bytes(const std::string& m, const std::string& r) const {
  auto* n = ns(m, r);
  return n ? n->used_bytes : 0;
}
std::vector<ModelDescriptor> Authority::models() const {
  std::vector<ModelDescriptor> out;
  for (auto& [k, n] : namespaces_) out.push_back(n->desc);
  return out;
}

// ------------------------------------------------------------------ quota admission
int64_t Authority::free_bytes() const {
  if (pool_capacity_bytes_ <= 0) return INT64_MAX / 4;
  int64_t used = 0;
  for (auto& [k, n] : namespaces_) used += n->used_bytes;
  return std::max<int64_t>(0, pool_capacity_bytes_ - used);
}

int64_t Authority::reclaimable_borrowed(const std::string& m, const std::string& r) const {
  int64_t total = 0;
  for (auto& [k, n] : namespaces_) {
    if (k.first == m && k.second == r) continue;
    int64_t soft = n->desc.quota.soft_bytes;
    int64_t over = soft > 0 ? std::max<int64_t>(0, n->used_bytes - soft) : 0;
    if (over <= 0) continue;
    int64_t inactive = 0;
    for (auto& [pk, p] : n->pools) inactive += int64_t(p->inactive.size());
    total += std::min(over, inactive * n->bytes_per_block());
  }
  return total;
}

void Authority::reclaim_borrowed(const std::string& m, const std::string& r, int64_t want) {
  int64_t freed = 0;
  for (auto& [k, n] : namespaces_) {
    if (freed >= want) break;
    if (k.first == m && k.second == r) continue;
    int64_t soft = n->desc.quota.soft_bytes;
    int64_t over = soft > 0 ? std::max<int64_t>(0, n->used_bytes - soft) : 0;
    if (over <= 0) continue;
    int64_t bpb = n->bytes_per_block();
    int64_t target = std::min(want - freed, over);
    size_t blocks = size_t(std::max<int64_t>(1, (target + bpb - 1) / bpb));
    auto removed = evict_ns(n.get(), blocks, k.first, k.second);
    freed += int64_t(removed.size()) * bpb;
  }
}

Authority::AdmitPlan Authority::plan_admit(const std::string& m, const std::string& r, size_t new_blocks) const {
  AdmitPlan plan;
  if (new_blocks == 0) return plan;
  const Namespace* n = ns(m, r);
  if (!n) fail("admit: unknown namespace (" + m + ")");
  const Quota& q = n->desc.quota;
  int64_t bpb = n->bytes_per_block();
  int64_t used = n->used_bytes;
  int64_t delta = int64_t(new_blocks) * bpb;
  size_t inactive_n = 0;
  for (auto& [pk, p] : n->pools) inactive_n += p->inactive.size();
  int64_t inactive_bytes = int64_t(inactive_n) * bpb;
  auto reject = [&](int64_t used_b, int64_t deficit, const char* reason) {
    plan.accept = false;
    plan.bp = BackpressureSignal{m, r, used_b, q.soft_bytes, q.hard_bytes, deficit, reason};
    return plan;
  };
  if (q.hard_bytes > 0 && used + delta > q.hard_bytes) {
    int64_t need = used + delta - q.hard_bytes;
    if (inactive_bytes < need) return reject(used, need - inactive_bytes, "HARD_QUOTA");
  }
  size_t own = 0;
  if (q.hard_bytes > 0 && used + delta > q.hard_bytes)
    own = std::max(own, size_t((used + delta - q.hard_bytes + bpb - 1) / bpb));
  if (q.soft_bytes > 0 && used + delta > q.soft_bytes)
    own = std::max(own, size_t((used + delta - q.soft_bytes + bpb - 1) / bpb));
  own = std::min(own, inactive_n);
  int64_t sim_used = used - int64_t(own) * bpb;
  int64_t reclaim = 0;
  if (q.borrow_enabled && q.soft_bytes > 0) {
    int64_t projected = sim_used + delta;
    if (projected > q.soft_bytes) {
      int64_t need_borrow = projected - q.soft_bytes;
      int64_t fr = free_bytes();
      if (pool_capacity_bytes_ > 0) fr = std::max<int64_t>(0, fr + int64_t(own) * bpb);
      if (fr < need_borrow) {
        int64_t want = need_borrow - fr;
        int64_t avail = reclaimable_borrowed(m, r);
        if (avail < want && pool_capacity_bytes_ > 0 && (q.hard_bytes == 0 || projected <= q.hard_bytes))
          return reject(projected, want - avail, "POOL_CAPACITY");
        reclaim = std::min(want, avail);
      }
    }
  }
  if (q.hard_bytes > 0 && sim_used + delta > q.hard_bytes)
    return reject(sim_used, sim_used + delta - q.hard_bytes, "HARD_QUOTA");
  plan.own_evict = own;
  plan.reclaim = reclaim;
  return plan;
}

RegisterResult Authority::preflight_register(const std::string& model_id, const std::string& revision, int pool_kind,
                                             const std::vector<std::string>& block_hashes) const {
  int pk = resolve_pool_kind(pool_kind);
  const Namespace* n = ns(model_id, revision);
  if (!n) fail("AdmitRegisterBlocks: model not registered (" + model_id + "); call RegisterModel first");
  const PoolView* p = pool(n, pk);
  std::unordered_set<std::string> seen;
  size_t fresh = 0;
  for (auto& h : block_hashes) {
    if (!seen.insert(h).second) continue;
    if (!p || !p->by_flat.count(h)) ++fresh;
  }
  AdmitPlan plan = plan_admit(model_id, revision, fresh);
  RegisterResult res;
  res.accepted = plan.accept;
  res.backpressure = plan.bp;
  return res;
}

// ------------------------------------------------------------------ register
RegisterResult Authority::register_blocks(const std::string& node_id, const std::vector<std::string>& prefix_hashes,
                                          std::vector<BlockMeta> metas) {
  RegisterResult res;
  if (metas.empty()) return res;
  const std::string model_id = metas.front().id.model_id;
  const std::string revision = metas.front().id.revision;
  const int pk = resolve_pool_kind(metas.front().id.pool_kind);
  if (prefix_hashes.empty()) fail("RegisterBlocks: prefix_hashes required (lineage)");
  std::unordered_map<std::string, size_t> index_of;
  for (size_t i = 0; i < prefix_hashes.size(); ++i) index_of.emplace(prefix_hashes[i], i);
  std::vector<size_t> positions;
  for (auto& m : metas) {
    if (m.id.model_id != model_id) fail("RegisterBlocks: mixed model_id " + model_id + " vs " + m.id.model_id);
    if (m.id.revision != revision) fail("RegisterBlocks: mixed revision");
    if (resolve_pool_kind(m.id.pool_kind) != pk) fail("RegisterBlocks: mixed pool_kind");
    auto it = index_of.find(m.id.block_hash);
    if (it == index_of.end()) fail("RegisterBlocks: block hash not in prefix_hashes");
    positions.push_back(it->second);
  }
  std::sort(positions.begin(), positions.end());
  positions.erase(std::unique(positions.begin(), positions.end()), positions.end());
  for (size_t i = 1; i < positions.size(); ++i)
    if (positions[i] != positions[i - 1] + 1)
      fail("RegisterBlocks: blocks must be a contiguous segment of prefix_hashes");
  Namespace* n = ns(model_id, revision);
  if (!n) fail("RegisterBlocks: model not registered (" + model_id + "); call RegisterModel first");
  // count new flats
  PoolView* p = pool(n, pk, true);
  std::unordered_set<std::string> seen;
  size_t fresh = 0;
  for (auto& m : metas)
    if (seen.insert(m.id.block_hash).second && !p->by_flat.count(m.id.block_hash)) ++fresh;
  AdmitPlan plan = plan_admit(model_id, revision, fresh);
  if (!plan.accept) {
    res.accepted = false;
    res.backpressure = plan.bp;
    return res;
  }
  // validate durability before any mutation
  for (auto& m : metas)
    if (m.locations.empty() && !m.l3_present) fail("RegisterBlocks: need L2 location or l3_present (durable first)");
  if (plan.own_evict) evict_ns(n, plan.own_evict, model_id, revision);
  if (plan.reclaim) reclaim_borrowed(model_id, revision, plan.reclaim);
  p = pool(n, pk, true);

  auto lineage = lineage_from_prefix(prefix_hashes);
  int64_t bpb = n->bytes_per_block();
  for (auto& m : metas) {
    m.id.pool_kind = pk;
    for (auto& l : m.locations)
      if (l.node_id.empty()) l.node_id = node_id;
    size_t pos = index_of[m.id.block_hash];
    uint64_t lin = lineage[pos];
    auto it = p->by_flat.find(m.id.block_hash);
    bool is_new = it == p->by_flat.end();
    Entry e;
    if (!is_new) {
      e = it->second;
    } else {
      e.block_id = p->next_block_id++;
      n->used_bytes += bpb;
      e.parent = pos ? lineage[pos - 1] : 0;
      if (e.parent) {
        auto pit = p->lin_to_flat.find(e.parent);
        if (pit != p->lin_to_flat.end()) p->by_flat[pit->second].registered_children++;
      }
    }
    e.lineage = lin;
    e.meta = m;
    e.prefix_chain.assign(prefix_hashes.begin(), prefix_hashes.begin() + pos + 1);
    p->lin_to_flat[lin] = m.id.block_hash;
    p->by_flat[m.id.block_hash] = e;
    p->freq.touch(lin);
    emit_upsert(is_new ? REGISTERED : MOVED, m);
    orphans_.erase(key_of(m.id));
  }
  return res;
}

// ------------------------------------------------------------------ lookup / locate
LookupResult Authority::lookup_prefix(const std::string& model_id, const std::string& revision, int pool_kind,
                                      const std::vector<std::string>& prefix_hashes, const std::string& requester) {
  LookupResult r;
  if (prefix_hashes.empty()) return r;
  int pk;
  try {
    pk = resolve_pool_kind(pool_kind);
  } catch (...) {
    return r;
  }
  Namespace* n = ns(model_id, revision);
  if (!n) return r;
  PoolView* p = pool(n, pk, false);
  if (!p) return r;
  auto lineage = lineage_from_prefix(prefix_hashes);
  bool all_local = true;
  for (size_t i = 0; i < prefix_hashes.size(); ++i) {
    auto it = p->by_flat.find(prefix_hashes[i]);
    if (it == p->by_flat.end() || it->second.lineage != lineage[i]) {
      all_local = false;
      break;
    }
    p->freq.touch(lineage[i]);
    ReusableBlock rb;
    rb.id = it->second.meta.id;
    rb.meta = it->second.meta;
    auto rit = p->refs.find(lineage[i]);
    rb.meta.ref_count = rit == p->refs.end() ? 0 : uint32_t(std::max<int64_t>(0, rit->second.total()));
    rb.local_hit = has_tier_on(rb.meta, L0, requester);
    if (!rb.local_hit) all_local = false;
    r.blocks.push_back(std::move(rb));
    r.hit_length++;
  }
  r.all_local_hit = all_local && r.hit_length > 0;
  return r;
}

std::vector<BlockMeta> Authority::locate(const std::vector<KVBlockID>& ids) const {
  std::vector<BlockMeta> out;
  for (auto& id : ids) {
    try {
      if (const Entry* e = find(id)) out.push_back(e->meta);
    } catch (...) {
    }
  }
  return out;
}

// ------------------------------------------------------------------ refs
void Authority::apply_ref(const RefDelta& d, bool track_node) {
  PoolView* p = nullptr;
  Entry* e = find(d.id, &p);
  if (!e) fail("RefDelta: unknown block_hash");
  int kind = resolve_ref_kind(d.kind);
  auto& acc = p->refs[e->lineage];
  int64_t before = acc.total();
  int64_t after_b = acc.bucket(kind) + d.delta;
  if (after_b < 0) fail(std::string("RefDelta: ref_count underflow (kind=") + ref_kind_name(kind) + ")");
  acc.bucket(kind) = after_b;
  int64_t after = acc.total();
  if (before > 0 && after == 0) {
    p->inactive.insert(e->lineage);
  } else if (before == 0 && after > 0) {
    p->inactive.take(e->lineage);
  }
  if (track_node && !d.node_id.empty() && d.delta != 0) {
    auto& held = node_refs_[d.node_id];
    auto bk = key_of(d.id);
    auto& a = held[bk];
    a.bucket(kind) += d.delta;
    if (a.total() <= 0) held.erase(bk);
  }
}

void Authority::report_refs(const std::vector<RefDelta>& deltas) {
  // project the whole batch first: any failure leaves state untouched
  std::map<std::pair<const PoolView*, uint64_t>, RefAccounts> proj;
  std::map<std::pair<std::string, BlockKey>, RefAccounts> proj_node;
  for (size_t i = 0; i < deltas.size(); ++i) {
    const auto& d = deltas[i];
    const std::string at = "ReportRef batch[" + std::to_string(i) + "]: ";
    PoolView* p = nullptr;
    Entry* e = nullptr;
    try {
      e = find(d.id, &p);
    } catch (const std::exception& ex) {
      fail(at + ex.what());
    }
    if (!e) fail(at + "unknown block_hash");
    int kind;
    try {
      kind = resolve_ref_kind(d.kind);
    } catch (const std::exception& ex) {
      fail(at + ex.what());
    }
    std::pair<const PoolView*, uint64_t> key{p, e->lineage};
    auto it = proj.find(key);
    if (it == proj.end()) {
      auto rit = p->refs.find(e->lineage);
      it = proj.emplace(key, rit == p->refs.end() ? RefAccounts{} : rit->second).first;
    }
    int64_t next = it->second.bucket(kind) + d.delta;
    if (next < 0) fail(at + "ref_count underflow (kind=" + ref_kind_name(kind) + ")");
    it->second.bucket(kind) = next;
    if (!d.node_id.empty() && d.delta != 0) {
      auto nk = std::make_pair(d.node_id, key_of(d.id));
      auto nit = proj_node.find(nk);
      if (nit == proj_node.end()) {
        RefAccounts cur;
        auto hit = node_refs_.find(d.node_id);
        if (hit != node_refs_.end()) {
          auto b = hit->second.find(nk.second);
          if (b != hit->second.end()) cur = b->second;
        }
        nit = proj_node.emplace(nk, cur).first;
      }
      int64_t nn = nit->second.bucket(kind) + d.delta;
      if (nn < 0) fail(at + "node_ref underflow (kind=" + ref_kind_name(kind) + ")");
      nit->second.bucket(kind) = nn;
    }
  }
  for (auto& d : deltas) apply_ref(d, true);
}

std::pair<int64_t, int64_t> Authority::refs_by_kind(const KVBlockID& id) const {
  const Namespace* n = ns(id.model_id, id.revision);
  if (!n) return {0, 0};
  const PoolView* p = pool(n, resolve_pool_kind(id.pool_kind));
  if (!p) return {0, 0};
  auto it = p->by_flat.find(id.block_hash);
  if (it == p->by_flat.end()) return {0, 0};
  auto r = p->refs.find(it->second.lineage);
  if (r == p->refs.end()) return {0, 0};
  return {r->second.request, r->second.writeback};
}

void Authority::complete_barrier(const std::string& request_id, const std::string& node_id) {
  if (request_id.empty()) fail("RequestBarrier: request_id required");
  if (node_id.empty()) fail("RequestBarrier: node_id required");
  barriers_[request_id] = node_id;
}
bool Authority::barrier_completed(const std::string& request_id) const { return barriers_.count(request_id) != 0; }

void Authority::publish_location(const KVBlockID& id, int tier, const std::string& node_id, uint64_t segment_id,
                                 uint64_t offset, bool present) {
  if (tier == L3) fail("publish_location: L3 is expressed by l3_present, never as a Location");
  Entry* e = find(id);
  if (!e) fail("publish_location: unknown block");
  auto& locs = e->meta.locations;
  auto same = [&](const Location& l) { return l.tier == tier && l.node_id == node_id; };
  locs.erase(std::remove_if(locs.begin(), locs.end(), same), locs.end());
  if (present) locs.push_back(Location{tier, node_id, segment_id, offset});
  emit_upsert(MOVED, e->meta);
}

void Authority::set_l3_present(const KVBlockID& id, bool present) {
  Entry* e = find(id);
  if (!e) fail("set_l3_present: unknown block");
  e->meta.l3_present = present;
  emit_upsert(MOVED, e->meta);
}

size_t Authority::inactive_len(const std::string& m, const std::string& r, int pool_kind) const {
  const Namespace* n = ns(m, r);
  if (!n) return 0;
  const PoolView* p = pool(n, resolve_pool_kind(pool_kind));
  return p ? p->inactive.size() : 0;
}

size_t Authority::block_count(const std::string& m, const std::string& r) const {
  const Namespace* n = ns(m, r);
  if (!n) return 0;
  size_t c = 0;
  for (auto& [pk, p] : n->pools) c += p->by_flat.size();
  return c;
}

// ------------------------------------------------------------------ eviction
void Authority::remove_entry(PoolView* p, const std::string& flat) {
  auto it = p->by_flat.find(flat);
  if (it == p->by_flat.end()) return;
  const Entry& e = it->second;
  if (e.parent) {
    auto pit = p->lin_to_flat.find(e.parent);
    if (pit != p->lin_to_flat.end()) {
      auto fit = p->by_flat.find(pit->second);
      if (fit != p->by_flat.end()) fit->second.registered_children--;
    }
  }
  p->inactive.take(e.lineage);
  p->refs.erase(e.lineage);
  p->lin_to_flat.erase(e.lineage);
  p->hit_counts.erase(flat);
  for (auto m = p->placement_marks.begin(); m != p->placement_marks.end();)
    m = m->first == flat ? p->placement_marks.erase(m) : std::next(m);
  p->by_flat.erase(it);
}

std::vector<std::string> Authority::drop_victims(PoolView* p, size_t n) {
  auto is_leaf = [p](uint64_t lin) {
    auto f = p->lin_to_flat.find(lin);
    if (f == p->lin_to_flat.end()) return true;
    return p->by_flat[f->second].registered_children <= 0;
  };
  auto freq = [p](uint64_t lin) { return p->freq.estimate(lin); };
  std::vector<std::string> removed;
  for (uint64_t lin : p->inactive.allocate(n, is_leaf, freq)) {
    auto r = p->refs.find(lin);
    if (r != p->refs.end() && r->second.total() > 0) continue;
    auto f = p->lin_to_flat.find(lin);
    if (f == p->lin_to_flat.end()) continue;
    std::string flat = f->second;
    emit_invalidated(p->by_flat[flat].meta.id);
    remove_entry(p, flat);
    removed.push_back(flat);
  }
  return removed;
}

std::vector<std::pair<int, std::string>> Authority::evict_ns(Namespace* n, size_t count, const std::string&,
                                                              const std::string&) {
  std::vector<std::pair<int, std::string>> out;
  size_t left = count;
  for (auto& [pk, p] : n->pools) {  // std::map: TARGET before DRAFT
    if (!left) break;
    for (auto& f : drop_victims(p.get(), left)) {
      out.emplace_back(pk, f);
      --left;
    }
  }
  n->used_bytes = std::max<int64_t>(0, n->used_bytes - int64_t(out.size()) * n->bytes_per_block());
  return out;
}

size_t Authority::evict_n(const std::string& m, const std::string& r, int pool_kind, size_t n) {
  Namespace* ns_ = ns(m, r);
  if (!ns_) return 0;
  PoolView* p = pool(ns_, resolve_pool_kind(pool_kind), false);
  if (!p) return 0;
  auto removed = drop_victims(p, n);
  ns_->used_bytes = std::max<int64_t>(0, ns_->used_bytes - int64_t(removed.size()) * ns_->bytes_per_block());
  return removed.size();
}

// ------------------------------------------------------------------ view log
void Authority::emit_upsert(int kind, const BlockMeta& m) {
  ViewEvent e;
  e.kind = kind;
  e.id = m.id;
  e.locations = m.locations;
  e.l3_present = m.l3_present;
  e.block_kind = kind == REGISTERED ? m.block_kind : 0;
  pending_.push_back(std::move(e));
}
void Authority::emit_invalidated(const KVBlockID& id) {
  ViewEvent e;
  e.kind = INVALIDATED;
  e.id = id;
  pending_.push_back(std::move(e));
}

ViewUpdate Authority::commit_pending() {
  ViewUpdate u;
  u.seq = next_seq_++;
  u.events = std::move(pending_);
  pending_.clear();
  log_.push_back(u);
  while (log_.size() > kViewLogCap) log_.pop_front();
  return u;
}

std::vector<ViewUpdate> Authority::replay_after(uint64_t from_seq, bool* ok) const {
  std::vector<ViewUpdate> out;
  *ok = false;
  if (from_seq == 0 || from_seq >= next_seq_) return out;
  uint64_t floor = log_.empty() ? next_seq_ : log_.front().seq;
  if (from_seq + 1 < floor) return out;
  for (auto& u : log_)
    if (u.seq > from_seq) out.push_back(u);
  *ok = true;
  return out;
}

ViewUpdate Authority::snapshot() const {
  ViewUpdate u;
  u.seq = 0;
  for (auto& [k, n] : namespaces_)
    for (auto& [pk, p] : n->pools)
      for (auto& [flat, e] : p->by_flat) {
        ViewEvent ev;
        ev.kind = REGISTERED;
        ev.id = e.meta.id;
        ev.locations = e.meta.locations;
        ev.l3_present = e.meta.l3_present;
        ev.block_kind = e.meta.block_kind;
        u.events.push_back(std::move(ev));
      }
  return u;
}

// ------------------------------------------------------------------ reconcile / GC
void Authority::report_orphans(const std::vector<OrphanReport>& reports) {
  uint64_t now = now_ms_();
  for (auto& r : reports)
    for (auto& id : r.ids) {
      auto k = key_of(id);
      if (const Entry* e = find(id)) {
        (void)e;
        continue;  // registered: not an orphan
      }
      orphans_.emplace(k, OrphanEntry{r.node_id, r.marked_at_ms ? r.marked_at_ms : now});
    }
}

std::vector<KVBlockID> Authority::discard_blocks(const std::vector<KVBlockID>& ids) {
  std::vector<KVBlockID> out;
  for (auto& id : ids) {
    orphans_.erase(key_of(id));
    Namespace* n = nullptr;
    PoolView* p = nullptr;
    Entry* e = find(id, &p, &n);
    if (!e) continue;
    auto r = p->refs.find(e->lineage);
    if (r != p->refs.end() && r->second.total() > 0)
      fail("DiscardBlocks: block still referenced (refs=" + std::to_string(r->second.total()) + ")");
    emit_invalidated(e->meta.id);
    remove_entry(p, id.block_hash);
    n->used_bytes = std::max<int64_t>(0, n->used_bytes - n->bytes_per_block());
    out.push_back(id);
  }
  return out;
}

std::vector<KVBlockID> Authority::sweep_orphans(uint64_t ttl_ms) {
  if (!ttl_ms) ttl_ms = kDefaultOrphanTtlMs;
  uint64_t now = now_ms_();
  std::vector<KVBlockID> out;
  for (auto it = orphans_.begin(); it != orphans_.end();) {
    if (now >= it->second.marked_at_ms && now - it->second.marked_at_ms >= ttl_ms) {
      KVBlockID id{it->first.model_id, it->first.flat, it->first.pool_kind, "public", it->first.revision};
      out.push_back(id);
      it = orphans_.erase(it);
    } else {
      ++it;
    }
  }
  return out;
}

std::pair<std::vector<KVBlockID>, std::vector<KVBlockID>> Authority::gc_cold(const std::string& m,
                                                                             const std::string& r, int pool_kind,
                                                                             size_t count) {
  std::vector<KVBlockID> discarded, stripped;
  if (!count) return {discarded, stripped};
  Namespace* n = ns(m, r);
  if (!n) fail("gc_cold: unknown namespace (" + m + ")");
  PoolView* p = pool(n, resolve_pool_kind(pool_kind), false);
  if (!p) return {discarded, stripped};
  auto is_leaf = [p](uint64_t lin) {
    auto f = p->lin_to_flat.find(lin);
    return f == p->lin_to_flat.end() || p->by_flat[f->second].registered_children <= 0;
  };
  auto freq = [p](uint64_t lin) { return p->freq.estimate(lin); };
  std::vector<uint64_t> reinsert;
  for (uint64_t lin : p->inactive.allocate(count, is_leaf, freq)) {
    auto rf = p->refs.find(lin);
    if (rf != p->refs.end() && rf->second.total() > 0) continue;
    auto f = p->lin_to_flat.find(lin);
    if (f == p->lin_to_flat.end()) continue;
    Entry& e = p->by_flat[f->second];
    bool durable = has_tier(e.meta, L2) || e.meta.l3_present;
    auto& locs = e.meta.locations;
    locs.erase(std::remove_if(locs.begin(), locs.end(), [](const Location& l) { return l.tier == L0 || l.tier == L1; }),
               locs.end());
    if (durable) {
      emit_upsert(MOVED, e.meta);
      stripped.push_back(e.meta.id);
      reinsert.push_back(lin);
    } else {
      KVBlockID id = e.meta.id;
      emit_invalidated(id);
      remove_entry(p, f->second);
      n->used_bytes = std::max<int64_t>(0, n->used_bytes - n->bytes_per_block());
      discarded.push_back(id);
    }
  }
  for (uint64_t lin : reinsert) p->inactive.insert(lin);
  return {discarded, stripped};
}

std::pair<uint32_t, std::vector<KVBlockID>> Authority::reconcile_dead_node(const std::string& node_id) {
  if (node_id.empty()) fail("reconcile_dead_node: node_id required");
  uint32_t cleared = 0;
  std::vector<KVBlockID> stripped;
  auto held = node_refs_.find(node_id);
  if (held != node_refs_.end()) {
    auto copy = held->second;
    for (auto& [bk, acc] : copy) {
      KVBlockID id{bk.model_id, bk.flat, bk.pool_kind, "public", bk.revision};
      for (int kind : {REQUEST, WRITEBACK}) {
        int64_t v = acc.get(kind);
        if (v <= 0) continue;
        try {
          apply_ref(RefDelta{id, kind, int32_t(-v), node_id}, false);
          cleared++;
        } catch (...) {
        }
      }
    }
    node_refs_.erase(node_id);
  }
  for (auto& [k, n] : namespaces_)
    for (auto& [pk, p] : n->pools)
      for (auto& [flat, e] : p->by_flat) {
        auto& locs = e.meta.locations;
        size_t before = locs.size();
        locs.erase(std::remove_if(locs.begin(), locs.end(),
                                  [&](const Location& l) { return l.tier == L0 && l.node_id == node_id; }),
                   locs.end());
        if (locs.size() != before) {
          emit_upsert(MOVED, e.meta);
          stripped.push_back(e.meta.id);
        }
      }
  return {cleared, stripped};
}

// ------------------------------------------------------------------ checkpoint
CheckpointSnapshot Authority::export_snapshot() {
  CheckpointSnapshot s;
  s.seq = ++checkpoint_seq_;
  for (auto& [k, n] : namespaces_) {
    s.models.push_back(n->desc);
    for (auto& [pk, p] : n->pools)
      for (auto& [flat, e] : p->by_flat) s.blocks.push_back(CheckpointBlock{e.meta, e.prefix_chain});
  }
  // parents before children so import can rebuild the lineage tree in order
  std::stable_sort(s.blocks.begin(), s.blocks.end(),
                   [](const CheckpointBlock& a, const CheckpointBlock& b) { return a.prefix_chain.size() < b.prefix_chain.size(); });
  return s;
}

void Authority::import_snapshot(const CheckpointSnapshot& snap) {
  namespaces_.clear();
  orphans_.clear();
  node_refs_.clear();
  for (auto& d : snap.models) register_model(d);
  std::vector<CheckpointBlock> blocks = snap.blocks;
  std::stable_sort(blocks.begin(), blocks.end(),
                   [](const CheckpointBlock& a, const CheckpointBlock& b) { return a.prefix_chain.size() < b.prefix_chain.size(); });
  for (auto& b : blocks) {
    Namespace* n = ns(b.meta.id.model_id, b.meta.id.revision);
    if (!n) fail("RestoreCheckpoint: block of an unregistered model");
    if (b.prefix_chain.empty() || b.prefix_chain.back() != b.meta.id.block_hash)
      fail("RestoreCheckpoint: prefix_chain must end with the block hash");
    PoolView* p = pool(n, resolve_pool_kind(b.meta.id.pool_kind), true);
    auto lin = lineage_from_prefix(b.prefix_chain);
    Entry e;
    e.lineage = lin.back();
    e.parent = lin.size() > 1 ? lin[lin.size() - 2] : 0;
    e.meta = b.meta;
    e.meta.ref_count = 0;
    e.block_id = p->next_block_id++;
    e.prefix_chain = b.prefix_chain;
    if (e.parent) {
      auto pit = p->lin_to_flat.find(e.parent);
      if (pit != p->lin_to_flat.end()) p->by_flat[pit->second].registered_children++;
    }
    p->lin_to_flat[e.lineage] = b.meta.id.block_hash;
    p->by_flat[b.meta.id.block_hash] = e;
    n->used_bytes += n->bytes_per_block();
  }
  checkpoint_seq_ = std::max(checkpoint_seq_, snap.seq);
  // restore publishes a fresh snapshot: the replay log restarts
  log_.clear();
  pending_.clear();
}

// ------------------------------------------------------------------ shard ring
void Authority::rebuild_ring() {
  ring_.clear();
  for (auto& [id, st] : nodes_)
    if (!st.draining)
      for (uint64_t h : st.hashes) ring_[h] = id;
}

std::string Authority::owner_on(const std::map<uint64_t, std::string>& ring, const std::string& key) const {
  if (ring.empty()) return std::string();
  uint64_t h = hash64(key, 0x5eed);
  auto it = ring.lower_bound(h);
  if (it == ring.end()) it = ring.begin();
  return it->second;
}

std::string Authority::shard_owner(const std::string& block_hash) const { return owner_on(ring_, block_hash); }

std::vector<std::string> Authority::ready_nodes() const {
  std::vector<std::string> out;
  for (auto& [id, st] : nodes_)
    if (!st.draining) out.push_back(id);
  return out;
}

ShardMap Authority::shard_map() const {
  ShardMap m;
  m.generation = generation_;
  m.default_vnode_count = kDefaultVnodes;
  for (auto& [id, st] : nodes_) m.nodes.push_back(ShardEntry{id, st.vnodes, st.draining, st.hashes});
  return m;
}

std::vector<std::pair<std::string, KVBlockID>> Authority::all_block_keys() const {
  std::vector<std::pair<std::string, KVBlockID>> out;
  for (auto& [k, n] : namespaces_)
    for (auto& [pk, p] : n->pools)
      for (auto& [flat, e] : p->by_flat) out.emplace_back(flat, e.meta.id);
  return out;
}

std::vector<ShardMigration> Authority::join_shard_node(const std::string& node_id, uint32_t vnodes,
                                                       std::vector<KVBlockID>* warmup) {
  if (node_id.empty()) fail("JoinShardNode: node_id required");
  if (!vnodes) vnodes = kDefaultVnodes;
  auto before = ring_;
  NodeState st;
  st.vnodes = vnodes;
  std::set<uint64_t> hs;
  for (uint32_t i = 0; i < vnodes; ++i) {
    std::string buf = node_id;
    for (int b = 0; b < 4; ++b) buf.push_back(char((i >> (8 * b)) & 0xff));
    hs.insert(hash64(buf, 0x5eed));
  }
  uint64_t salt = 0;
  while (hs.size() < vnodes) hs.insert(hash64(node_id + "#" + std::to_string(salt++), 0x5eed));
  st.hashes.assign(hs.begin(), hs.end());
  auto prev = nodes_.find(node_id);
  if (prev != nodes_.end() && !prev->second.draining) fail("JoinShardNode: node already joined: " + node_id);
  nodes_[node_id] = st;
  rebuild_ring();
  generation_++;
  std::vector<ShardMigration> migs;
  for (auto& [flat, id] : all_block_keys()) {
    std::string a = owner_on(before, flat), b = owner_on(ring_, flat);
    if (b == node_id && a != b) migs.push_back(ShardMigration{id, a, b, false});
  }
  if (warmup) *warmup = warmup_plan(node_id, 64);
  return migs;
}

std::pair<std::vector<ShardMigration>, std::vector<KVBlockID>> Authority::drain_shard_node(const std::string& node_id) {
  auto it = nodes_.find(node_id);
  if (it == nodes_.end()) fail("DrainShardNode: unknown node " + node_id);
  auto before = ring_;
  it->second.draining = true;
  rebuild_ring();
  generation_++;
  std::vector<ShardMigration> migs;
  std::vector<KVBlockID> push_l2;
  for (auto& [k, n] : namespaces_)
    for (auto& [pk, p] : n->pools)
      for (auto& [flat, e] : p->by_flat) {
        std::string a = owner_on(before, flat);
        bool on_node = false;
        for (auto& l : e.meta.locations) on_node |= l.node_id == node_id;
        bool durable_elsewhere = e.meta.l3_present;
        for (auto& l : e.meta.locations) durable_elsewhere |= (l.tier == L2 && l.node_id != node_id);
        if (a == node_id || on_node) {
          std::string b = owner_on(ring_, flat);
          migs.push_back(ShardMigration{e.meta.id, node_id, b, on_node && !durable_elsewhere});
        }
        if (on_node && !durable_elsewhere) push_l2.push_back(e.meta.id);
      }
  return {migs, push_l2};
}

void Authority::remove_shard_node(const std::string& node_id) {
  auto it = nodes_.find(node_id);
  if (it == nodes_.end()) fail("RemoveShardNode: unknown node " + node_id);
  if (!it->second.draining) fail("RemoveShardNode: drain the node first: " + node_id);
  for (auto& [k, n] : namespaces_)
    for (auto& [pk, p] : n->pools)
      for (auto& [flat, e] : p->by_flat)
        for (auto& l : e.meta.locations)
          if (l.node_id == node_id && l.tier != L0)
            fail("RemoveShardNode: placements remain on " + node_id + " (move L1/L2 copies first)");
  nodes_.erase(it);
  rebuild_ring();
  generation_++;
}

// ------------------------------------------------------------------ hits / placement
void Authority::report_hits(const std::string& node_id, const std::vector<KVBlockID>& ids,
                            std::vector<PlacementPlan>* follow) {
  std::map<std::string, std::vector<KVBlockID>> cand;
  size_t evaluated = 0;
  for (auto& id : ids) {
    PoolView* p = nullptr;
    Entry* e = nullptr;
    try {
      e = find(id, &p);
    } catch (...) {
      continue;
    }
    if (!e) continue;
    uint32_t& c = p->hit_counts[id.block_hash][node_id];
    c++;
    p->freq.touch(e->lineage);
    if (!follow || node_id.empty()) continue;
    if (c < kFollowHitThreshold || evaluated >= kFollowEvalLimit) continue;
    if (has_tier_on(e->meta, L0, node_id)) continue;
    if (p->placement_marks.count({id.block_hash, node_id})) continue;
    evaluated++;
    // co-locate the ancestors that are not yet on the node (root first)
    for (auto& anc : e->prefix_chain) {
      auto ai = p->by_flat.find(anc);
      if (ai == p->by_flat.end()) continue;
      if (has_tier_on(ai->second.meta, L0, node_id) || p->placement_marks.count({anc, node_id})) continue;
      p->placement_marks.insert({anc, node_id});
      cand[node_id].push_back(ai->second.meta.id);
    }
  }
  if (follow)
    for (auto& [node, v] : cand) follow->push_back(PlacementPlan{node, v});
}

uint32_t Authority::hit_count(const KVBlockID& id) const {
  const Namespace* n = ns(id.model_id, id.revision);
  if (!n) return 0;
  const PoolView* p = pool(n, resolve_pool_kind(id.pool_kind));
  if (!p) return 0;
  auto it = p->hit_counts.find(id.block_hash);
  if (it == p->hit_counts.end()) return 0;
  uint32_t s = 0;
  for (auto& [node, c] : it->second) s += c;
  return s;
}

uint32_t Authority::hit_count_on(const KVBlockID& id, const std::string& node) const {
  const Namespace* n = ns(id.model_id, id.revision);
  if (!n) return 0;
  const PoolView* p = pool(n, resolve_pool_kind(id.pool_kind));
  if (!p) return 0;
  auto it = p->hit_counts.find(id.block_hash);
  if (it == p->hit_counts.end()) return 0;
  auto c = it->second.find(node);
  return c == it->second.end() ? 0 : c->second;
}

std::vector<KVBlockID> Authority::warmup_plan(const std::string& node_id, size_t k) const {
  std::vector<std::pair<uint32_t, KVBlockID>> owned;
  for (auto& [key, n] : namespaces_)
    for (auto& [pk, p] : n->pools)
      for (auto& [flat, e] : p->by_flat) {
        if (owner_on(ring_, flat) != node_id) continue;
        uint32_t hits = 0;
        auto it = p->hit_counts.find(flat);
        if (it != p->hit_counts.end())
          for (auto& [nd, c] : it->second) hits += c;
        if (hits) owned.emplace_back(hits, e.meta.id);
      }
  std::stable_sort(owned.begin(), owned.end(), [](auto& a, auto& b) { return a.first > b.first; });
  std::vector<KVBlockID> out;
  for (size_t i = 0; i < owned.size() && i < k; ++i) out.push_back(owned[i].second);
  return out;
}

bool Authority::preplace_on_register(const std::string& model_id, const std::string& revision, int pool_kind,
                                     const std::vector<std::string>& prefix_hashes, PlacementPlan* out) {
  if (prefix_hashes.empty()) return false;
  const std::string& anchor = prefix_hashes[std::min(prefix_hashes.size(), kAnchorDepthCap) - 1];
  auto nodes = ready_nodes();
  if (nodes.empty()) return false;
  std::string home;
  uint64_t best = 0;
  for (auto& nd : nodes) {  // max score; ties go to the smaller node id
    uint64_t s = hrw_score(anchor, nd);
    if (home.empty() || s > best || (s == best && nd < home)) {
      best = s;
      home = nd;
    }
  }
  Namespace* n = ns(model_id, revision);
  if (!n) return false;
  PoolView* p = pool(n, resolve_pool_kind(pool_kind), false);
  if (!p) return false;
  PlacementPlan plan;
  plan.node_id = home;
  for (auto& flat : prefix_hashes) {
    auto it = p->by_flat.find(flat);
    if (it == p->by_flat.end()) continue;
    if (has_tier_on(it->second.meta, L0, home)) continue;
    if (p->placement_marks.count({flat, home})) continue;
    plan.ids.push_back(it->second.meta.id);
  }
  if (plan.ids.empty()) return false;
  for (auto& id : plan.ids) p->placement_marks.insert({id.block_hash, home});
  *out = plan;
  return true;
}

// ------------------------------------------------------------------ defrag
double Authority::l2_fragmentation_ratio(const std::string& m, const std::string& r, int pool_kind,
                                         uint64_t slot_bytes) const {
  if (!slot_bytes) slot_bytes = kDefaultSlotBytes;
  const Namespace* n = ns(m, r);
  if (!n) return 0.0;
  const PoolView* p = pool(n, resolve_pool_kind(pool_kind));
  if (!p) return 0.0;
  // per (node, segment): occupied slots vs highest slot index + 1
  std::map<std::pair<std::string, uint64_t>, std::pair<uint64_t, uint64_t>> seg;  // used, span
  for (auto& [flat, e] : p->by_flat)
    for (auto& l : e.meta.locations)
      if (l.tier == L2) {
        auto& s = seg[{l.node_id, l.segment_id}];
        s.first++;
        s.second = std::max<uint64_t>(s.second, l.offset / slot_bytes + 1);
      }
  uint64_t used = 0, span = 0;
  for (auto& [k, v] : seg) {
    used += v.first;
    span += v.second;
  }
  return span ? 1.0 - double(used) / double(span) : 0.0;
}

std::vector<DefragMove> Authority::plan_defrag(const std::string& m, const std::string& r, int pool_kind, int mode,
                                               uint64_t slot_bytes) const {
  if (!slot_bytes) slot_bytes = kDefaultSlotBytes;
  if (mode == DEFRAG_MODE_UNSPECIFIED) mode = BOTH;
  std::vector<DefragMove> moves;
  const Namespace* n = ns(m, r);
  if (!n) fail("TriggerDefrag: unknown namespace (" + m + ")");
  const PoolView* p = pool(n, resolve_pool_kind(pool_kind));
  if (!p) return moves;
  // occupancy per (node, segment)
  std::map<std::pair<std::string, uint64_t>, std::set<uint64_t>> occ;
  for (auto& [flat, e] : p->by_flat)
    for (auto& l : e.meta.locations)
      if (l.tier == L2) occ[{l.node_id, l.segment_id}].insert(l.offset / slot_bytes);
  if (mode == COMPACT || mode == BOTH) {
    // move the highest slots of each segment into its lowest holes
    for (auto& [key, slots] : occ) {
      std::set<uint64_t> cur = slots;
      uint64_t hole = 0;
      while (true) {
        while (cur.count(hole)) hole++;
        if (cur.empty() || *cur.rbegin() <= hole) break;
        uint64_t top = *cur.rbegin();
        for (auto& [flat, e] : p->by_flat)
          for (auto& l : e.meta.locations)
            if (l.tier == L2 && l.node_id == key.first && l.segment_id == key.second && l.offset / slot_bytes == top) {
              DefragMove mv{e.meta.id, key.first, key.second, l.offset, key.second, hole * slot_bytes, true, key.second};
              moves.push_back(mv);
            }
        cur.erase(top);
        cur.insert(hole);
      }
    }
  }
  if (mode == COLOCATE || mode == BOTH) {
    // children whose L2 copy sits on a different segment than their parent move next to it
    for (auto& [flat, e] : p->by_flat) {
      if (!e.parent) continue;
      auto pf = p->lin_to_flat.find(e.parent);
      if (pf == p->lin_to_flat.end()) continue;
      const Entry& par = p->by_flat.at(pf->second);
      const Location* pl = nullptr;
      for (auto& l : par.meta.locations)
        if (l.tier == L2) pl = &l;
      if (!pl) continue;
      for (auto& l : e.meta.locations) {
        if (l.tier != L2 || l.node_id != pl->node_id || l.segment_id == pl->segment_id) continue;
        auto& slots = occ[{pl->node_id, pl->segment_id}];
        uint64_t s = pl->offset / slot_bytes + 1;
        while (slots.count(s) && s < 64) s++;
        if (s >= 64) continue;
        slots.insert(s);
        moves.push_back(DefragMove{e.meta.id, l.node_id, l.segment_id, l.offset, pl->segment_id, s * slot_bytes, false,
                                   pl->segment_id});
      }
    }
  }
  return moves;
}

size_t Authority::relocate_in_view(const std::vector<DefragMove>& moves) {
  size_t n = 0;
  for (auto& mv : moves) {
    Entry* e = find(mv.id);
    if (!e) continue;
    for (auto& l : e->meta.locations)
      if (l.tier == L2 && l.node_id == mv.node_id && l.segment_id == mv.from_segment && l.offset == mv.from_offset) {
        l.segment_id = mv.to_segment;
        l.offset = mv.to_offset;
        emit_upsert(MOVED, e->meta);
        n++;
        break;
      }
  }
  return n;
}

}  // namespace lakeb::cp
