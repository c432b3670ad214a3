// pybind11 module lake_b200._host: the host-side C++ components (control-plane
// authority, hashing, and the tier/router/agent cores registered by their own
// translation units through register_* functions).
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "authority/authority.h"
#include "common/hash.h"

namespace py = pybind11;
using namespace lakeb;
using namespace lakeb::cp;

void register_tier(py::module_& m);
void register_router(py::module_& m);
void register_agent(py::module_& m);
void register_transfer(py::module_& m);
void register_weights(py::module_& m);

namespace {

py::bytes B(const std::string& s) { return py::bytes(s); }

template <class T>
void bytes_field(py::class_<T>& c, const char* name, std::string T::*field) {
  c.def_property(
      name, [field](const T& self) { return py::bytes(self.*field); },
      [field](T& self, const py::bytes& v) { self.*field = std::string(v); });
}

std::vector<std::string> to_strs(const std::vector<py::bytes>& v) {
  std::vector<std::string> out;
  out.reserve(v.size());
  for (auto& b : v) out.emplace_back(b);
  return out;
}

}  // namespace

PYBIND11_MODULE(_host, m) {
  m.doc() = "lake_b200 host components (C++)";
  py::register_exception<std::invalid_argument>(m, "HostError", PyExc_ValueError);

  // ---------------------------------------------------------------- hashing
  m.def("chain_block_hashes",
        [](const std::vector<uint32_t>& toks, size_t bs, bool full_only, const py::bytes& parent) {
          std::vector<py::bytes> out;
          for (auto& h : chain_block_hashes(toks, bs, full_only, std::string(parent))) out.push_back(B(h));
          return out;
        },
        py::arg("tokens"), py::arg("block_size"), py::arg("full_only") = false, py::arg("parent") = py::bytes(""));
  m.def("sha256", [](const py::bytes& b) {
    std::string s(b);
    auto d = sha256(reinterpret_cast<const uint8_t*>(s.data()), s.size());
    return B(std::string(reinterpret_cast<const char*>(d.data()), d.size()));
  });
  m.def("hrw_score", [](const py::bytes& key, const std::string& node) { return hrw_score(std::string(key), node); });
  m.def("fnv1a64", [](const py::bytes& b) {
    std::string s(b);
    return fnv1a64_update(kFnvOffset, s.data(), s.size());
  });

  // ---------------------------------------------------------------- value types
  py::class_<KVBlockID> kid(m, "KVBlockID");
  kid.def(py::init<>())
      .def(py::init([](const std::string& model_id, const py::bytes& h, int pool_kind, const std::string& revision,
                       const std::string& scope) {
             return KVBlockID{model_id, std::string(h), pool_kind, scope, revision};
           }),
           py::arg("model_id"), py::arg("block_hash"), py::arg("pool_kind") = int(TARGET), py::arg("revision") = "",
           py::arg("scope") = "public")
      .def_readwrite("model_id", &KVBlockID::model_id)
      .def_readwrite("pool_kind", &KVBlockID::pool_kind)
      .def_readwrite("scope", &KVBlockID::scope)
      .def_readwrite("revision", &KVBlockID::revision);
  bytes_field(kid, "block_hash", &KVBlockID::block_hash);

  py::class_<Location>(m, "Location")
      .def(py::init<>())
      .def(py::init([](int tier, const std::string& node, uint64_t seg, uint64_t off) {
             return Location{tier, node, seg, off};
           }),
           py::arg("tier"), py::arg("node_id") = "", py::arg("segment_id") = 0, py::arg("offset") = 0)
      .def_readwrite("tier", &Location::tier)
      .def_readwrite("node_id", &Location::node_id)
      .def_readwrite("segment_id", &Location::segment_id)
      .def_readwrite("offset", &Location::offset);

  py::class_<BlockMeta>(m, "BlockMeta")
      .def(py::init<>())
      .def(py::init([](const KVBlockID& id, const std::vector<Location>& locs, bool l3, int kind) {
             BlockMeta b;
             b.id = id;
             b.locations = locs;
             b.l3_present = l3;
             b.block_kind = kind;
             return b;
           }),
           py::arg("id"), py::arg("locations") = std::vector<Location>{}, py::arg("l3_present") = false,
           py::arg("block_kind") = int(T_TYPE))
      .def_readwrite("id", &BlockMeta::id)
      .def_readwrite("block_kind", &BlockMeta::block_kind)
      .def_readwrite("locations", &BlockMeta::locations)
      .def_readwrite("l3_present", &BlockMeta::l3_present)
      .def_readwrite("ref_count", &BlockMeta::ref_count);

  py::class_<Quota>(m, "Quota")
      .def(py::init([](int64_t s, int64_t h, bool b) { return Quota{s, h, b}; }), py::arg("soft_bytes") = 0,
           py::arg("hard_bytes") = 0, py::arg("borrow_enabled") = false)
      .def_readwrite("soft_bytes", &Quota::soft_bytes)
      .def_readwrite("hard_bytes", &Quota::hard_bytes)
      .def_readwrite("borrow_enabled", &Quota::borrow_enabled);

  py::class_<BackpressureSignal>(m, "BackpressureSignal")
      .def(py::init<>())
      .def_readwrite("model_id", &BackpressureSignal::model_id)
      .def_readwrite("revision", &BackpressureSignal::revision)
      .def_readwrite("used_bytes", &BackpressureSignal::used_bytes)
      .def_readwrite("soft_bytes", &BackpressureSignal::soft_bytes)
      .def_readwrite("hard_bytes", &BackpressureSignal::hard_bytes)
      .def_readwrite("deficit_bytes", &BackpressureSignal::deficit_bytes)
      .def_readwrite("reason", &BackpressureSignal::reason);

  py::class_<ModelDescriptor>(m, "ModelDescriptor")
      .def(py::init([](const std::string& model_id, const std::string& revision, uint32_t num_layers,
                       uint32_t block_tokens, uint64_t bytes_per_block, int hash_algo, const Quota& q) {
             return ModelDescriptor{model_id, revision, num_layers, block_tokens, bytes_per_block, hash_algo, q};
           }),
           py::arg("model_id"), py::arg("revision") = "", py::arg("num_layers") = 0, py::arg("block_tokens") = 16,
           py::arg("bytes_per_block") = 0, py::arg("hash_algo") = 1, py::arg("quota") = Quota{})
      .def_readwrite("model_id", &ModelDescriptor::model_id)
      .def_readwrite("revision", &ModelDescriptor::revision)
      .def_readwrite("num_layers", &ModelDescriptor::num_layers)
      .def_readwrite("block_tokens", &ModelDescriptor::block_tokens)
      .def_readwrite("bytes_per_block", &ModelDescriptor::bytes_per_block)
      .def_readwrite("hash_algo", &ModelDescriptor::hash_algo)
      .def_readwrite("quota", &ModelDescriptor::quota);

  py::class_<ViewEvent>(m, "ViewEvent")
      .def(py::init<>())
      .def_readwrite("kind", &ViewEvent::kind)
      .def_readwrite("id", &ViewEvent::id)
      .def_readwrite("locations", &ViewEvent::locations)
      .def_readwrite("l3_present", &ViewEvent::l3_present)
      .def_readwrite("block_kind", &ViewEvent::block_kind);
  py::class_<ViewUpdate>(m, "ViewUpdate")
      .def(py::init<>())
      .def_readwrite("seq", &ViewUpdate::seq)
      .def_readwrite("events", &ViewUpdate::events);

  py::class_<ReusableBlock>(m, "ReusableBlock")
      .def_readonly("id", &ReusableBlock::id)
      .def_readonly("meta", &ReusableBlock::meta)
      .def_readonly("local_hit", &ReusableBlock::local_hit);
  py::class_<LookupResult>(m, "LookupResult")
      .def_readonly("blocks", &LookupResult::blocks)
      .def_readonly("hit_length", &LookupResult::hit_length)
      .def_readonly("all_local_hit", &LookupResult::all_local_hit);

  py::class_<RefDelta>(m, "RefDelta")
      .def(py::init([](const KVBlockID& id, int kind, int32_t delta, const std::string& node) {
             return RefDelta{id, kind, delta, node};
           }),
           py::arg("id"), py::arg("kind"), py::arg("delta"), py::arg("node_id") = "")
      .def_readwrite("id", &RefDelta::id)
      .def_readwrite("kind", &RefDelta::kind)
      .def_readwrite("delta", &RefDelta::delta)
      .def_readwrite("node_id", &RefDelta::node_id);

  py::class_<RegisterResult>(m, "RegisterResult")
      .def_readonly("accepted", &RegisterResult::accepted)
      .def_readonly("backpressure", &RegisterResult::backpressure);

  py::class_<OrphanReport>(m, "OrphanReport")
      .def(py::init([](const std::string& node, const std::vector<KVBlockID>& ids, uint64_t at) {
             return OrphanReport{node, ids, at};
           }),
           py::arg("node_id"), py::arg("ids"), py::arg("marked_at_ms") = 0);

  py::class_<CheckpointBlock> cb(m, "CheckpointBlock");
  cb.def(py::init<>())
      .def_readwrite("meta", &CheckpointBlock::meta)
      .def_property(
          "prefix_chain",
          [](const CheckpointBlock& c) {
            std::vector<py::bytes> o;
            for (auto& s : c.prefix_chain) o.push_back(B(s));
            return o;
          },
          [](CheckpointBlock& c, const std::vector<py::bytes>& v) { c.prefix_chain = to_strs(v); });
  py::class_<CheckpointSnapshot>(m, "CheckpointSnapshot")
      .def(py::init<>())
      .def_readwrite("seq", &CheckpointSnapshot::seq)
      .def_readwrite("models", &CheckpointSnapshot::models)
      .def_readwrite("blocks", &CheckpointSnapshot::blocks);

  py::class_<DefragMove>(m, "DefragMove")
      .def(py::init<>())
      .def_readwrite("id", &DefragMove::id)
      .def_readwrite("node_id", &DefragMove::node_id)
      .def_readwrite("from_segment", &DefragMove::from_segment)
      .def_readwrite("from_offset", &DefragMove::from_offset)
      .def_readwrite("to_segment", &DefragMove::to_segment)
      .def_readwrite("to_offset", &DefragMove::to_offset)
      .def_readwrite("compact_segment", &DefragMove::compact_segment)
      .def_readwrite("segment_id", &DefragMove::segment_id);

  py::class_<ShardEntry>(m, "ShardEntry")
      .def_readonly("node_id", &ShardEntry::node_id)
      .def_readonly("vnode_count", &ShardEntry::vnode_count)
      .def_readonly("draining", &ShardEntry::draining)
      .def_readonly("vnode_hashes", &ShardEntry::vnode_hashes);
  py::class_<ShardMap>(m, "ShardMap")
      .def_readonly("generation", &ShardMap::generation)
      .def_readonly("default_vnode_count", &ShardMap::default_vnode_count)
      .def_readonly("nodes", &ShardMap::nodes);
  py::class_<ShardMigration>(m, "ShardMigration")
      .def_readonly("id", &ShardMigration::id)
      .def_readonly("from_node", &ShardMigration::from_node)
      .def_readonly("to_node", &ShardMigration::to_node)
      .def_readonly("push_l2_first", &ShardMigration::push_l2_first);
  py::class_<PlacementPlan>(m, "PlacementPlan")
      .def_readonly("node_id", &PlacementPlan::node_id)
      .def_readonly("ids", &PlacementPlan::ids);

  // ---------------------------------------------------------------- authority
  py::class_<Authority>(m, "Authority")
      .def(py::init<size_t, int64_t>(), py::arg("inactive_cap") = kInactiveCap, py::arg("pool_capacity_bytes") = 0)
      .def("register_model", &Authority::register_model)
      .def("deregister_model", &Authority::deregister_model)
      .def("has_namespace", &Authority::has_namespace)
      .def("set_quota", &Authority::set_quota)
      .def("get_quota", &Authority::get_quota)
      .def("used_bytes", &Authority::used_bytes)
      .def("models", &Authority::models)
      .def("preflight_register",
           [](const Authority& a, const std::string& m, const std::string& r, int pk, const std::vector<py::bytes>& h) {
             return a.preflight_register(m, r, pk, to_strs(h));
           })
      .def("register_blocks",
           [](Authority& a, const std::string& node, const std::vector<py::bytes>& prefix,
              const std::vector<BlockMeta>& metas) { return a.register_blocks(node, to_strs(prefix), metas); })
      .def("lookup_prefix",
           [](Authority& a, const std::string& m, const std::string& r, int pk, const std::vector<py::bytes>& prefix,
              const std::string& requester) { return a.lookup_prefix(m, r, pk, to_strs(prefix), requester); },
           py::arg("model_id"), py::arg("revision"), py::arg("pool_kind"), py::arg("prefix_hashes"),
           py::arg("requester") = "")
      .def("locate", &Authority::locate)
      .def("report_refs", &Authority::report_refs)
      .def("refs_by_kind", &Authority::refs_by_kind)
      .def("complete_barrier", &Authority::complete_barrier)
      .def("barrier_completed", &Authority::barrier_completed)
      .def("publish_location", &Authority::publish_location, py::arg("id"), py::arg("tier"), py::arg("node_id"),
           py::arg("segment_id") = 1, py::arg("offset") = 0, py::arg("present") = true)
      .def("set_l3_present", &Authority::set_l3_present)
      .def("evict_n", &Authority::evict_n)
      .def("inactive_len", &Authority::inactive_len)
      .def("block_count", &Authority::block_count)
      .def("commit_pending", &Authority::commit_pending)
      .def("replay_after",
           [](const Authority& a, uint64_t seq) -> py::object {
             bool ok = false;
             auto v = a.replay_after(seq, &ok);
             if (!ok) return py::none();
             return py::cast(v);
           })
      .def("snapshot", &Authority::snapshot)
      .def("last_seq", &Authority::last_seq)
      .def("set_view_log_cap", &Authority::set_view_log_cap)
      .def("view_log_cap", &Authority::view_log_cap)
      .def("pending_events", &Authority::pending_events)
      .def("report_orphans", &Authority::report_orphans)
      .def("discard_blocks", &Authority::discard_blocks)
      .def("sweep_orphans", &Authority::sweep_orphans)
      .def("gc_cold", &Authority::gc_cold)
      .def("reconcile_dead_node", &Authority::reconcile_dead_node)
      .def("orphan_count", &Authority::orphan_count)
      .def("set_clock", &Authority::set_clock)
      .def("export_snapshot", &Authority::export_snapshot)
      .def("import_snapshot", &Authority::import_snapshot)
      .def("shard_map", &Authority::shard_map)
      .def("join_shard_node",
           [](Authority& a, const std::string& node, uint32_t vnodes) {
             std::vector<KVBlockID> warm;
             auto migs = a.join_shard_node(node, vnodes, &warm);
             return py::make_tuple(migs, warm);
           },
           py::arg("node_id"), py::arg("vnode_count") = 0)
      .def("drain_shard_node", &Authority::drain_shard_node)
      .def("remove_shard_node", &Authority::remove_shard_node)
      .def("shard_owner", [](const Authority& a, const py::bytes& h) { return a.shard_owner(std::string(h)); })
      .def("ready_nodes", &Authority::ready_nodes)
      .def("report_hits",
           [](Authority& a, const std::string& node, const std::vector<KVBlockID>& ids) {
             std::vector<PlacementPlan> plans;
             a.report_hits(node, ids, &plans);
             return plans;
           })
      .def("hit_count", &Authority::hit_count)
      .def("hit_count_on", &Authority::hit_count_on)
      .def("warmup_plan", &Authority::warmup_plan)
      .def("preplace_on_register",
           [](Authority& a, const std::string& m, const std::string& r, int pk,
              const std::vector<py::bytes>& prefix) -> py::object {
             PlacementPlan p;
             if (!a.preplace_on_register(m, r, pk, to_strs(prefix), &p)) return py::none();
             return py::cast(p);
           })
      .def("l2_fragmentation_ratio", &Authority::l2_fragmentation_ratio)
      .def("plan_defrag", &Authority::plan_defrag)
      .def("relocate_in_view", &Authority::relocate_in_view)
      .def("set_background_paused", &Authority::set_background_paused)
      .def("background_paused", &Authority::background_paused);

  register_tier(m);
  register_router(m);
  register_agent(m);
  register_transfer(m);
  register_weights(m);
}
