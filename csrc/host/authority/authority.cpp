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
bool InactiveIndex::has(uint64_t lin) const {
  auto it = slots_.find(lin);
  return it != slots_.end() && !it->second.spilled;
}

void InactiveIndex::admit(uint64_t lin, Slot& s) {
  if (indexed_ >= cap_) {
    s.spilled = true;
    spill_at_[lin] = spill_.insert(spill_.end(), lin);
    return;
  }
  s.spilled = false;
  s.tick = tick_++;
  ++indexed_;
  if (s.leaf) leaves_.emplace(s.tick, lin);
}

void InactiveIndex::release(uint64_t lin, bool leaf) {
  if (slots_.count(lin)) return;  // already zero-ref
  Slot& s = slots_[lin];
  s.leaf = leaf;
  admit(lin, s);
}

bool InactiveIndex::retain(uint64_t lin) {
  auto it = slots_.find(lin);
  if (it == slots_.end()) return false;
  Slot s = it->second;
  slots_.erase(it);
  if (s.spilled) {
    auto at = spill_at_.find(lin);
    spill_.erase(at->second);
    spill_at_.erase(at);
    return true;
  }
  if (s.leaf) leaves_.erase(s.tick);
  --indexed_;
  refill();
  return true;
}

void InactiveIndex::set_leaf(uint64_t lin, bool leaf) {
  auto it = slots_.find(lin);
  if (it == slots_.end() || it->second.leaf == leaf) return;
  Slot& s = it->second;
  s.leaf = leaf;
  if (s.spilled) return;
  if (leaf)
    leaves_.emplace(s.tick, lin);
  else
    leaves_.erase(s.tick);
}

void InactiveIndex::refill() {
  while (indexed_ < cap_ && !spill_.empty()) {
    uint64_t lin = spill_.front();
    spill_.pop_front();
    spill_at_.erase(lin);
    admit(lin, slots_[lin]);
  }
}

size_t InactiveIndex::evict(size_t n, const std::function<uint8_t(uint64_t)>& freq,
                            const std::function<void(uint64_t)>& drop) {
  size_t taken = 0;
  while (taken < n && !leaves_.empty()) {
    // rank this pass's leaves: coldest bucket first, oldest release first inside a bucket
    std::vector<uint64_t> ranked[4];
    for (auto& [tick, lin] : leaves_) ranked[bucket_of(freq(lin))].push_back(lin);
    for (auto& tier : ranked)
      for (uint64_t lin : tier) {
        if (taken == n) break;
        auto it = slots_.find(lin);
        if (it == slots_.end() || it->second.spilled || !it->second.leaf) continue;  // changed by a drop
        leaves_.erase(it->second.tick);
        slots_.erase(it);
        --indexed_;
        drop(lin);
        ++taken;
      }
    refill();
  }
  return taken;
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

// ------------------------------------------------------------------ admission
// A namespace's usage has three levels: up to its soft quota the bytes are its own
// reservation; between soft and hard they are borrowed (only with borrow_enabled, and
// only while the pool has room); the hard quota is never crossed. Admitting `fresh`
// blocks first makes room from the namespace's own zero-ref blocks, down to whichever
// of its two limits is tighter. What still lies above the hard quota is refused as
// HARD_QUOTA. A borrower that would push the pool past its capacity takes the excess
// back from namespaces that are themselves above their soft quota (their zero-ref
// blocks), largest excess first; if they cannot cover it, the admission is refused
// as POOL_CAPACITY. A refused admission changes nothing.
int64_t Authority::pool_used_bytes() const {
  int64_t used = 0;
  for (auto& kv : namespaces_) used += kv.second->used_bytes;
  return used;
}

int64_t Authority::lendable_bytes(const Namespace& n) const {
  const int64_t soft = n.desc.quota.soft_bytes;
  if (soft <= 0 || n.used_bytes <= soft) return 0;
  size_t zero_ref = 0;
  for (auto& kv : n.pools) zero_ref += kv.second->inactive.evictable();
  return std::min<int64_t>(n.used_bytes - soft, int64_t(zero_ref) * n.bytes_per_block());
}

int64_t Authority::take_from_lenders(const Namespace* borrower, int64_t bytes) {
  std::vector<std::pair<int64_t, Namespace*>> lenders;  // (lendable bytes, namespace)
  for (auto& kv : namespaces_)
    if (kv.second.get() != borrower)
      if (int64_t l = lendable_bytes(*kv.second)) lenders.emplace_back(l, kv.second.get());
  std::stable_sort(lenders.begin(), lenders.end(), [](auto& x, auto& y) { return x.first > y.first; });
  int64_t got = 0;
  for (auto& [lendable, n] : lenders) {
    if (got >= bytes) break;
    const int64_t unit = n->bytes_per_block();
    const int64_t ask = std::min(lendable, bytes - got);
    got += int64_t(evict_ns(n, size_t((ask + unit - 1) / unit))) * unit;
  }
  return got;
}

Authority::AdmitPlan Authority::plan_admit(const Namespace& n, size_t fresh_blocks) const {
  AdmitPlan plan;
  if (!fresh_blocks) return plan;
  constexpr int64_t kUnbounded = INT64_MAX / 4;
  const Quota& q = n.desc.quota;
  const int64_t unit = n.bytes_per_block();
  const int64_t incoming = int64_t(fresh_blocks) * unit;
  const int64_t hard = q.hard_bytes > 0 ? q.hard_bytes : kUnbounded;
  const int64_t soft = q.soft_bytes > 0 ? q.soft_bytes : kUnbounded;
  auto refuse = [&](int64_t used, int64_t short_by, const char* why) {
    plan.accept = false;
    plan.bp = BackpressureSignal{n.desc.model_id, n.desc.revision, used, q.soft_bytes, q.hard_bytes, short_by, why};
    return plan;
  };

  size_t own_zero_ref = 0;
  for (auto& kv : n.pools) own_zero_ref += kv.second->inactive.evictable();
  const int64_t over_limit = n.used_bytes + incoming - std::min(hard, soft);
  if (over_limit > 0) plan.evict_own = std::min<size_t>(own_zero_ref, size_t((over_limit + unit - 1) / unit));
  const int64_t freed = int64_t(plan.evict_own) * unit;
  const int64_t after = n.used_bytes - freed + incoming;
  if (after > hard) return refuse(n.used_bytes, after - hard, "HARD_QUOTA");

  if (q.borrow_enabled && after > soft && pool_capacity_bytes_ > 0) {
    const int64_t pool_after = pool_used_bytes() - freed + incoming;
    const int64_t excess = pool_after - pool_capacity_bytes_;
    if (excess > 0) {
      int64_t lendable = 0;
      for (auto& kv : namespaces_)
        if (kv.second.get() != &n) lendable += lendable_bytes(*kv.second);
      if (lendable < excess) return refuse(after, excess - lendable, "POOL_CAPACITY");
      plan.from_lenders = excess;
    }
  }
  return plan;
}

Authority::RegisterBatch Authority::check_register(const std::vector<std::string>& prefix_hashes,
                                                   const std::vector<BlockMeta>& metas, bool need_durable) {
  RegisterBatch b;
  const KVBlockID& first = metas.front().id;
  b.pool_kind = resolve_pool_kind(first.pool_kind);
  if (prefix_hashes.empty()) fail("RegisterBlocks: prefix_hashes required (lineage)");
  std::unordered_map<std::string, size_t> at;
  for (size_t i = 0; i < prefix_hashes.size(); ++i) at.emplace(prefix_hashes[i], i);
  std::set<size_t> covered;
  for (auto& m : metas) {
    if (m.id.model_id != first.model_id) fail("RegisterBlocks: mixed model_id " + first.model_id + " vs " + m.id.model_id);
    if (m.id.revision != first.revision) fail("RegisterBlocks: mixed revision");
    if (resolve_pool_kind(m.id.pool_kind) != b.pool_kind) fail("RegisterBlocks: mixed pool_kind");
    auto it = at.find(m.id.block_hash);
    if (it == at.end()) fail("RegisterBlocks: block hash not in prefix_hashes");
    b.pos.push_back(it->second);
    covered.insert(it->second);
    if (need_durable && m.locations.empty() && !m.l3_present)
      fail("RegisterBlocks: need L2 location or l3_present (durable first)");
  }
  if (*covered.rbegin() - *covered.begin() + 1 != covered.size())
    fail("RegisterBlocks: blocks must be a contiguous segment of prefix_hashes");
  b.n = ns(first.model_id, first.revision);
  if (!b.n) fail("RegisterBlocks: model not registered (" + first.model_id + "); call RegisterModel first");
  const PoolView* p = pool(b.n, b.pool_kind);
  for (size_t i : covered)
    if (!p || !p->by_flat.count(prefix_hashes[i])) ++b.fresh;
  return b;
}

RegisterResult Authority::preflight_register(const std::string& model_id, const std::string& revision, int pool_kind,
                                             const std::vector<std::string>& block_hashes) const {
  const int pk = resolve_pool_kind(pool_kind);
  const Namespace* n = ns(model_id, revision);
  if (!n) fail("AdmitRegisterBlocks: model not registered (" + model_id + "); call RegisterModel first");
  const PoolView* p = pool(n, pk);
  std::set<std::string> fresh;
  for (auto& h : block_hashes)
    if (!p || !p->by_flat.count(h)) fresh.insert(h);
  AdmitPlan plan = plan_admit(*n, fresh.size());
  RegisterResult res;
  res.accepted = plan.accept;
  res.backpressure = plan.bp;
  return res;
}

RegisterResult Authority::register_blocks(const std::string& node_id, const std::vector<std::string>& prefix_hashes,
                                          std::vector<BlockMeta> metas) {
  RegisterResult res;
  if (metas.empty()) return res;
  RegisterBatch b = check_register(prefix_hashes, metas, true);
  AdmitPlan plan = plan_admit(*b.n, b.fresh);
  if (!plan.accept) {
    res.accepted = false;
    res.backpressure = plan.bp;
    return res;
  }
  if (plan.evict_own) evict_ns(b.n, plan.evict_own);
  if (plan.from_lenders) take_from_lenders(b.n, plan.from_lenders);

  PoolView* p = pool(b.n, b.pool_kind, true);
  const auto lineage = lineage_from_prefix(prefix_hashes);
  for (size_t i = 0; i < metas.size(); ++i) {
    BlockMeta& m = metas[i];
    const size_t pos = b.pos[i];
    m.id.pool_kind = b.pool_kind;
    for (auto& l : m.locations)
      if (l.node_id.empty()) l.node_id = node_id;
    auto [it, inserted] = p->by_flat.try_emplace(m.id.block_hash);
    Entry& e = it->second;
    if (inserted) {
      e.block_id = p->next_block_id++;
      e.parent = pos ? lineage[pos - 1] : 0;
      b.n->used_bytes += b.n->bytes_per_block();
      link_child(p, e.parent, +1);
    }
    e.lineage = lineage[pos];
    e.meta = m;
    e.prefix_chain.assign(prefix_hashes.begin(), prefix_hashes.begin() + pos + 1);
    p->lin_to_flat[e.lineage] = m.id.block_hash;
    p->freq.touch(e.lineage);
    emit_upsert(inserted ? REGISTERED : MOVED, m);
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
void Authority::settle_refs(PoolView* p, const Entry& e, const RefAccounts& was, bool held_between) {
  const auto it = p->refs.find(e.lineage);
  const int64_t now = it == p->refs.end() ? 0 : it->second.total();
  if ((was.total() > 0 || held_between) && now == 0)
    p->inactive.release(e.lineage, e.registered_children <= 0);
  else if (was.total() == 0 && now > 0)
    p->inactive.retain(e.lineage);
}

// A batch applies delta by delta to the block ledgers and to the per-node ledgers that
// let a dead node's references be released later. The first write to each ledger cell
// saves the cell's old value; a failing delta puts every saved value back, so a batch is
// all-or-nothing. Zero crossings (block becomes evictable or stops being so) are settled
// once per block after the whole batch went through.
void Authority::report_refs(const std::vector<RefDelta>& deltas) {
  struct BlockCell {
    PoolView* p;
    const Entry* e;
    RefAccounts was;
    bool held = false;  // referenced at some point inside the batch
  };
  std::vector<BlockCell> blocks;
  std::map<std::pair<const PoolView*, uint64_t>, size_t> block_at;
  std::map<std::pair<std::string, BlockKey>, std::pair<bool, RefAccounts>> node_was;  // existed, value
  auto rollback = [&]() {
    for (auto& c : blocks) {
      if (c.was.request == 0 && c.was.writeback == 0)
        c.p->refs.erase(c.e->lineage);
      else
        c.p->refs[c.e->lineage] = c.was;
    }
    for (auto& [k, v] : node_was) {
      if (v.first)
        node_refs_[k.first][k.second] = v.second;
      else if (auto h = node_refs_.find(k.first); h != node_refs_.end()) {
        h->second.erase(k.second);
        if (h->second.empty()) node_refs_.erase(h);
      }
    }
  };
  for (size_t i = 0; i < deltas.size(); ++i) {
    const RefDelta& d = deltas[i];
    std::string err;
    try {
      PoolView* p = nullptr;
      const Entry* e = find(d.id, &p);
      if (!e) throw std::invalid_argument("unknown block_hash");
      const int kind = resolve_ref_kind(d.kind);
      auto key = std::make_pair(static_cast<const PoolView*>(p), e->lineage);
      if (!block_at.count(key)) {
        auto cur = p->refs.find(e->lineage);
        block_at[key] = blocks.size();
        blocks.push_back(BlockCell{p, e, cur == p->refs.end() ? RefAccounts{} : cur->second});
      }
      RefAccounts& acc = p->refs[e->lineage];
      if (acc.get(kind) + d.delta < 0)
        throw std::invalid_argument(std::string("ref_count underflow (kind=") + ref_kind_name(kind) + ")");
      if (!d.node_id.empty() && d.delta != 0) {
        const BlockKey bk = key_of(d.id);
        auto nk = std::make_pair(d.node_id, bk);
        auto& held = node_refs_[d.node_id];
        auto hit = held.find(bk);
        if (!node_was.count(nk)) node_was[nk] = {hit != held.end(), hit != held.end() ? hit->second : RefAccounts{}};
        RefAccounts& mine = held[bk];
        if (mine.get(kind) + d.delta < 0)
          throw std::invalid_argument(std::string("node_ref underflow (kind=") + ref_kind_name(kind) + ")");
        mine.bucket(kind) += d.delta;
        if (mine.total() == 0) held.erase(bk);
        if (held.empty()) node_refs_.erase(d.node_id);
      }
      acc.bucket(kind) += d.delta;
      if (acc.total() > 0) blocks[block_at[key]].held = true;
    } catch (const std::exception& ex) {
      err = "ReportRef batch[" + std::to_string(i) + "]: " + ex.what();
    }
    if (!err.empty()) {
      rollback();
      fail(err);
    }
  }
  for (auto& c : blocks) {
    auto it = c.p->refs.find(c.e->lineage);
    if (it != c.p->refs.end() && it->second.total() == 0) c.p->refs.erase(it);
    settle_refs(c.p, *c.e, c.was, c.held);
  }
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
  if (tier == L0 && !present) {
    // the copy a placement plan put there is gone: the node may be planned again
    PoolView* p = nullptr;
    find(id, &p);
    p->placement_marks.erase({id.block_hash, node_id});
  }
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
void Authority::link_child(PoolView* p, uint64_t parent, int step) {
  if (!parent) return;
  auto f = p->lin_to_flat.find(parent);
  if (f == p->lin_to_flat.end()) return;
  auto pe = p->by_flat.find(f->second);
  if (pe == p->by_flat.end()) return;
  Entry& par = pe->second;
  const bool was_leaf = par.registered_children <= 0;
  par.registered_children = std::max<int64_t>(0, par.registered_children + step);
  const bool leaf = par.registered_children <= 0;
  if (leaf != was_leaf) p->inactive.set_leaf(parent, leaf);
}

void Authority::remove_entry(PoolView* p, const std::string& flat) {
  auto it = p->by_flat.find(flat);
  if (it == p->by_flat.end()) return;
  const uint64_t lin = it->second.lineage, parent = it->second.parent;
  p->inactive.retain(lin);
  p->refs.erase(lin);
  p->lin_to_flat.erase(lin);
  p->hit_counts.erase(flat);
  p->placement_marks.erase(p->placement_marks.lower_bound({flat, std::string()}),
                           p->placement_marks.lower_bound({flat + '\0', std::string()}));
  p->by_flat.erase(it);
  link_child(p, parent, -1);
}

size_t Authority::evict_in(Namespace* n, PoolView* p, size_t count) {
  auto freq = [p](uint64_t lin) { return p->freq.estimate(lin); };
  auto drop = [&](uint64_t lin) {
    auto f = p->lin_to_flat.find(lin);
    if (f == p->lin_to_flat.end()) return;
    const std::string flat = f->second;
    emit_invalidated(p->by_flat[flat].meta.id);
    remove_entry(p, flat);
  };
  const size_t gone = p->inactive.evict(count, freq, drop);
  n->used_bytes = std::max<int64_t>(0, n->used_bytes - int64_t(gone) * n->bytes_per_block());
  return gone;
}

size_t Authority::evict_ns(Namespace* n, size_t count) {
  size_t gone = 0;
  for (auto& kv : n->pools) {  // TARGET before DRAFT
    if (gone >= count) break;
    gone += evict_in(n, kv.second.get(), count - gone);
  }
  return gone;
}

size_t Authority::evict_n(const std::string& m, const std::string& r, int pool_kind, size_t n) {
  Namespace* space = ns(m, r);
  if (!space) return 0;
  PoolView* p = pool(space, resolve_pool_kind(pool_kind), false);
  return p ? evict_in(space, p, n) : 0;
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
  while (log_.size() > log_cap_) log_.pop_front();
  return u;
}

void Authority::set_view_log_cap(size_t n) {
  log_cap_ = n ? n : 1;
  while (log_.size() > log_cap_) log_.pop_front();
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
      fail("DiscardBlocks: block still referenced (global_refs=" + std::to_string(r->second.total()) + ")");
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

// Cold GC: the coldest zero-ref leaves lose their L0/L1 copies. A block with a durable
// copy (L2 or L3) stays registered and evictable; any other block leaves the view.
std::pair<std::vector<KVBlockID>, std::vector<KVBlockID>> Authority::gc_cold(const std::string& m,
                                                                             const std::string& r, int pool_kind,
                                                                             size_t count) {
  std::vector<KVBlockID> discarded, stripped;
  if (!count) return {discarded, stripped};
  Namespace* n = ns(m, r);
  if (!n) fail("gc_cold: unknown namespace (" + m + ")");
  PoolView* p = pool(n, resolve_pool_kind(pool_kind), false);
  if (!p) return {discarded, stripped};
  std::vector<uint64_t> keep;
  auto freq = [p](uint64_t lin) { return p->freq.estimate(lin); };
  auto visit = [&](uint64_t lin) {
    auto f = p->lin_to_flat.find(lin);
    if (f == p->lin_to_flat.end()) return;
    Entry& e = p->by_flat[f->second];
    auto& locs = e.meta.locations;
    locs.erase(std::remove_if(locs.begin(), locs.end(), [](const Location& l) { return l.tier == L0 || l.tier == L1; }),
               locs.end());
    if (has_tier(e.meta, L2) || e.meta.l3_present) {
      emit_upsert(MOVED, e.meta);
      stripped.push_back(e.meta.id);
      keep.push_back(lin);
      return;
    }
    discarded.push_back(e.meta.id);
    emit_invalidated(e.meta.id);
    remove_entry(p, f->second);
    n->used_bytes = std::max<int64_t>(0, n->used_bytes - n->bytes_per_block());
  };
  p->inactive.evict(count, freq, visit);
  for (uint64_t lin : keep) {  // durable: back among the zero-ref blocks (newest release)
    auto f = p->lin_to_flat.find(lin);
    p->inactive.release(lin, f == p->lin_to_flat.end() || p->by_flat[f->second].registered_children <= 0);
  }
  return {discarded, stripped};
}

// A node that died holds references it will never release, and L0 copies that are gone.
// Its per-node ledger is released block by block (each kind it held), and every L0
// location on it is stripped from the view. Returns the number of blocks whose
// references were released and the blocks that lost an L0 location.
std::pair<uint32_t, std::vector<KVBlockID>> Authority::reconcile_dead_node(const std::string& node_id) {
  if (node_id.empty()) fail("reconcile_dead_node: node_id required");
  uint32_t released = 0;
  auto held = node_refs_.find(node_id);
  if (held != node_refs_.end()) {
    for (auto& [bk, mine] : held->second) {
      PoolView* p = nullptr;
      KVBlockID id{bk.model_id, bk.flat, bk.pool_kind, "public", bk.revision};
      const Entry* e = find(id, &p);
      if (!e) continue;
      RefAccounts& acc = p->refs[e->lineage];
      const RefAccounts was = acc;
      acc.request = std::max<int64_t>(0, acc.request - mine.request);
      acc.writeback = std::max<int64_t>(0, acc.writeback - mine.writeback);
      if (acc.total() == 0) p->refs.erase(e->lineage);
      settle_refs(p, *e, was, false);
      ++released;
    }
    node_refs_.erase(held);
  }
  std::vector<KVBlockID> stripped;
  auto on_node_l0 = [&](const Location& l) { return l.tier == L0 && l.node_id == node_id; };
  for (auto& [k, n] : namespaces_)
    for (auto& [pk, p] : n->pools)
      for (auto& [flat, e] : p->by_flat) {
        auto& locs = e.meta.locations;
        auto tail = std::remove_if(locs.begin(), locs.end(), on_node_l0);
        if (tail == locs.end()) continue;
        locs.erase(tail, locs.end());
        emit_upsert(MOVED, e.meta);
        stripped.push_back(e.meta.id);
      }
  return {released, stripped};
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
  // every block must fit its model's hard quota before anything is replaced: a restore
  // that silently dropped blocks would report success for a partial view
  std::map<std::pair<std::string, std::string>, int64_t> need;
  for (auto& b : snap.blocks) need[{b.meta.id.model_id, b.meta.id.revision}] += 1;
  for (auto& d : snap.models) {
    const int64_t unit = d.bytes_per_block > 0 ? int64_t(d.bytes_per_block) : 1;
    const int64_t bytes = need[{d.model_id, d.revision}] * unit;
    if (d.quota.hard_bytes > 0 && bytes > d.quota.hard_bytes)
      fail("import_snapshot register rejected: (" + d.model_id + ", " + d.revision + ") holds " +
           std::to_string(bytes) + " bytes over its hard quota " + std::to_string(d.quota.hard_bytes));
  }
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
    p->lin_to_flat[e.lineage] = b.meta.id.block_hash;
    p->by_flat[b.meta.id.block_hash] = e;
    link_child(p, e.parent, +1);
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

// The hottest blocks (summed hits over every node) that the node does not already hold
// in L0, hottest first.
std::vector<KVBlockID> Authority::warmup_plan(const std::string& node_id, size_t k) const {
  std::vector<std::pair<uint32_t, KVBlockID>> hot;
  for (auto& kv : namespaces_)
    for (auto& pv : kv.second->pools) {
      const PoolView& p = *pv.second;
      for (auto& [flat, per_node] : p.hit_counts) {
        uint32_t hits = 0;
        for (auto& nc : per_node) hits += nc.second;
        auto e = p.by_flat.find(flat);
        if (!hits || e == p.by_flat.end() || has_tier_on(e->second.meta, L0, node_id)) continue;
        hot.emplace_back(hits, e->second.meta.id);
      }
    }
  std::stable_sort(hot.begin(), hot.end(), [](auto& x, auto& y) {
    return x.first != y.first ? x.first > y.first : x.second.block_hash < y.second.block_hash;
  });
  std::vector<KVBlockID> out;
  for (size_t i = 0; i < hot.size() && i < k; ++i) out.push_back(hot[i].second);
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
// L2 segments of one pool view, per (node, segment): occupied slot indices and whether a
// referenced block (which defrag must not move) sits in the segment.
namespace {
struct SegmentUse {
  std::set<uint64_t> slots;
  bool frozen = false;
};
std::map<std::pair<std::string, uint64_t>, SegmentUse> l2_segments(const PoolView& p, uint64_t slot_bytes) {
  std::map<std::pair<std::string, uint64_t>, SegmentUse> segs;
  for (auto& [flat, e] : p.by_flat) {
    auto r = p.refs.find(e.lineage);
    const bool held = r != p.refs.end() && r->second.total() > 0;
    for (auto& l : e.meta.locations)
      if (l.tier == L2) {
        auto& u = segs[{l.node_id, l.segment_id}];
        u.slots.insert(l.offset / slot_bytes);
        u.frozen |= held;
      }
  }
  return segs;
}
bool has_holes(const std::set<uint64_t>& slots) { return !slots.empty() && *slots.rbegin() + 1 != slots.size(); }
}  // namespace

// Share of the movable (unfrozen) L2 segments that have holes below their highest slot.
double Authority::l2_fragmentation_ratio(const std::string& m, const std::string& r, int pool_kind,
                                         uint64_t slot_bytes) const {
  if (!slot_bytes) slot_bytes = kDefaultSlotBytes;
  const Namespace* n = ns(m, r);
  if (!n) return 0.0;
  const PoolView* p = pool(n, resolve_pool_kind(pool_kind));
  if (!p) return 0.0;
  size_t movable = 0, holey = 0;
  for (auto& [key, u] : l2_segments(*p, slot_bytes)) {
    if (u.frozen) continue;
    ++movable;
    holey += has_holes(u.slots);
  }
  return movable ? double(holey) / double(movable) : 0.0;
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
  // occupancy per (node, segment), and the blocks in each occupied slot
  std::map<std::pair<std::string, uint64_t>, std::set<uint64_t>> occ;
  std::map<std::tuple<std::string, uint64_t, uint64_t>, std::vector<std::pair<KVBlockID, uint64_t>>> in_slot;
  for (auto& [flat, e] : p->by_flat)
    for (auto& l : e.meta.locations)
      if (l.tier == L2) {
        const uint64_t slot = l.offset / slot_bytes;
        occ[{l.node_id, l.segment_id}].insert(slot);
        in_slot[{l.node_id, l.segment_id, slot}].emplace_back(e.meta.id, l.offset);
      }
  if (mode == COMPACT || mode == BOTH) {
    // fill each segment's lowest holes with its highest occupied slots
    const auto segs = l2_segments(*p, slot_bytes);
    for (auto& [key, slots] : occ) {
      if (segs.at(key).frozen) continue;  // a referenced block must not move
      std::set<uint64_t> cur = slots;
      uint64_t hole = 0;
      for (;;) {
        while (cur.count(hole)) ++hole;
        if (cur.empty() || *cur.rbegin() <= hole) break;
        const uint64_t top = *cur.rbegin();
        for (auto& [id, offset] : in_slot[{key.first, key.second, top}])
          moves.push_back(DefragMove{id, key.first, key.second, offset, key.second, hole * slot_bytes, true, key.second});
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
