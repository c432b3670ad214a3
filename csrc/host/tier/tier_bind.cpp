#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "tier/tier.h"

namespace py = pybind11;
using namespace lakeb::tier;

void register_tier(py::module_& m) {
  py::enum_<TierId>(m, "TierId")
      .value("L0", TierId::L0)
      .value("L1", TierId::L1)
      .value("L2", TierId::L2)
      .value("L3", TierId::L3)
      .value("NONE", TierId::None);
  py::enum_<AccessKind>(m, "AccessKind")
      .value("L0_HIT", AccessKind::L0Hit)
      .value("L1_HIT", AccessKind::L1Hit)
      .value("L2_HIT", AccessKind::L2Hit)
      .value("L3_HIT", AccessKind::L3Hit)
      .value("MISS", AccessKind::Miss);
  py::enum_<BeginPromote>(m, "BeginPromote")
      .value("STARTED", BeginPromote::Started)
      .value("ALREADY_IN_FLIGHT", BeginPromote::AlreadyInFlight)
      .value("ALREADY_L0", BeginPromote::AlreadyL0)
      .value("MISSING", BeginPromote::Missing);

  py::class_<TierCaps>(m, "TierCaps")
      .def(py::init([](size_t l0, size_t l1, size_t l2) { return TierCaps{l0, l1, l2}; }), py::arg("l0") = 64,
           py::arg("l1") = 256, py::arg("l2") = 1024)
      .def_readwrite("l0", &TierCaps::l0)
      .def_readwrite("l1", &TierCaps::l1)
      .def_readwrite("l2", &TierCaps::l2);

  py::class_<Placement>(m, "Placement")
      .def_readonly("segment_id", &Placement::segment_id)
      .def_readonly("offset", &Placement::offset);
  py::class_<Relocate>(m, "Relocate")
      .def_property_readonly("hash", [](const Relocate& r) { return py::bytes(r.hash); })
      .def_readonly("src", &Relocate::from)
      .def_readonly("dst", &Relocate::to);

  py::class_<SegmentArena>(m, "SegmentArena")
      .def(py::init<uint64_t, size_t>(), py::arg("slot_bytes") = 4096, py::arg("slots_per_segment") = 64)
      .def("alloc", [](SegmentArena& a, const py::bytes& h) { return a.alloc(std::string(h)); })
      .def("place_at",
           [](SegmentArena& a, const py::bytes& h, uint64_t s, uint64_t o) { return a.place_at(std::string(h), s, o); })
      .def("free", [](SegmentArena& a, const py::bytes& h) { return a.free(std::string(h)); })
      .def("placement", [](const SegmentArena& a, const py::bytes& h) { return a.placement(std::string(h)); })
      .def("compact", &SegmentArena::compact)
      .def("relocate",
           [](SegmentArena& a, const py::bytes& h, uint64_t s, uint64_t o) { return a.relocate(std::string(h), s, o); })
      .def("utilization", &SegmentArena::utilization)
      .def("dense_prefix_slots", &SegmentArena::dense_prefix_slots)
      .def("has_holes", &SegmentArena::has_holes)
      .def("segment_ids", &SegmentArena::segment_ids);

  py::class_<BandwidthPool>(m, "BandwidthPool")
      .def(py::init<uint64_t, uint64_t>(), py::arg("budget_bytes") = 100ull << 20, py::arg("window_ms") = 1000)
      .def("try_consume", &BandwidthPool::try_consume)
      .def("remaining", &BandwidthPool::remaining)
      .def("set_paused", &BandwidthPool::set_paused)
      .def("paused", &BandwidthPool::paused);

  py::class_<HitStats>(m, "HitStats")
      .def_property_readonly("counts", [](const HitStats& s) {
        return std::vector<uint64_t>(s.counts, s.counts + 5);
      })
      .def("hit_rate", &HitStats::hit_rate)
      .def("l0_hit_rate", &HitStats::l0_hit_rate)
      .def("modelled_cost_us", &HitStats::modelled_cost_us)
      .def("total", &HitStats::total);

  py::class_<SideEffects>(m, "SideEffects")
      .def(py::init<>())
      .def_property_readonly("l0_demoted",
                             [](const SideEffects& f) {
                               std::vector<py::bytes> o;
                               for (auto& h : f.l0_demoted) o.push_back(py::bytes(h));
                               return o;
                             })
      .def_property_readonly("l2_demoted_to_l3", [](const SideEffects& f) {
        std::vector<py::bytes> o;
        for (auto& h : f.l2_demoted_to_l3) o.push_back(py::bytes(h));
        return o;
      });

  py::class_<DeviceCopy>(m, "DeviceCopy")
      .def_property_readonly("hash", [](const DeviceCopy& c) { return py::bytes(c.hash); })
      .def_readonly("page", &DeviceCopy::page)
      .def_readonly("slot", &DeviceCopy::slot)
      .def_readonly("to_device", &DeviceCopy::to_device);

  py::class_<TierEngine>(m, "TierEngine", py::dynamic_attr())
      .def(py::init([](TierCaps caps, uint64_t block_bytes, uintptr_t l1_base, const std::string& l2_dir,
                       const std::string& l3_dir, const std::string& key) {
             return new TierEngine(caps, block_bytes, reinterpret_cast<uint8_t*>(l1_base), l2_dir, l3_dir, key);
           }),
           py::arg("caps"), py::arg("block_bytes"), py::arg("l1_base"), py::arg("l2_dir"), py::arg("l3_dir"),
           py::arg("model_key") = "model")
      .def("caps", &TierEngine::caps)
      .def("block_bytes", &TierEngine::block_bytes)
      .def("set_promote_admit_after", &TierEngine::set_promote_admit_after)
      .def("local_tier", [](const TierEngine& e, const py::bytes& h) { return e.local_tier(std::string(h)); })
      .def("l0_page", [](const TierEngine& e, const py::bytes& h) { return e.l0_page(std::string(h)); })
      .def("l1_slot", [](const TierEngine& e, const py::bytes& h) { return e.l1_slot(std::string(h)); })
      .def("is_l2_durable", [](const TierEngine& e, const py::bytes& h) { return e.is_l2_durable(std::string(h)); })
      .def("l3_present", [](const TierEngine& e, const py::bytes& h) { return e.l3_present(std::string(h)); })
      .def("has_durable_backing",
           [](const TierEngine& e, const py::bytes& h) { return e.has_durable_backing(std::string(h)); })
      .def("l2_placement", [](const TierEngine& e, const py::bytes& h) { return e.l2_placement(std::string(h)); })
      .def("l0_len", &TierEngine::l0_len)
      .def("l1_len", &TierEngine::l1_len)
      .def("l2_len", &TierEngine::l2_len)
      .def("l2_order",
           [](const TierEngine& e) {
             py::list o;
             for (auto& h : e.l2_order()) o.append(py::bytes(h));
             return o;
           })
      .def("corrupt_reads", &TierEngine::corrupt_reads)
      .def("record_bytes", &TierEngine::record_bytes)
      .def("hit_count", [](const TierEngine& e, const py::bytes& h) { return e.hit_count(std::string(h)); })
      .def("is_one_shot", [](const TierEngine& e, const py::bytes& h) { return e.is_one_shot(std::string(h)); })
      .def("pin", [](TierEngine& e, const py::bytes& h) { e.pin(std::string(h)); })
      .def("unpin", [](TierEngine& e, const py::bytes& h) { e.unpin(std::string(h)); })
      .def("pin_count", [](const TierEngine& e, const py::bytes& h) { return e.pin_count(std::string(h)); })
      .def("note_l0", [](TierEngine& e, const py::bytes& h, int64_t page) { e.note_l0(std::string(h), page); })
      .def("drop_l0", [](TierEngine& e, const py::bytes& h) { e.drop_l0(std::string(h)); })
      .def("put_durable",
           [](TierEngine& e, const py::bytes& h, uintptr_t src) {
             return e.put_durable(std::string(h), reinterpret_cast<const uint8_t*>(src));
           })
      .def("put_durable_bytes",
           [](TierEngine& e, const py::bytes& h, const py::bytes& data) {
             std::string d(data);
             if (d.size() != e.block_bytes()) throw std::invalid_argument("put_durable_bytes: size mismatch");
             return e.put_durable(std::string(h), reinterpret_cast<const uint8_t*>(d.data()));
           })
      .def("read_host",
           [](const TierEngine& e, const py::bytes& h, uintptr_t dst) {
             return e.read_host(std::string(h), reinterpret_cast<uint8_t*>(dst));
           })
      .def("read_bytes",
           [](const TierEngine& e, const py::bytes& h) -> py::object {
             std::string buf(e.block_bytes(), '\0');
             if (!e.read_host(std::string(h), reinterpret_cast<uint8_t*>(&buf[0]))) return py::none();
             return py::bytes(buf);
           })
      .def("probe", [](TierEngine& e, const py::bytes& h) { return e.probe(std::string(h)); })
      .def("estimate_promote_cost",
           [](const TierEngine& e, const py::bytes& h) { return e.estimate_promote_cost(std::string(h)); })
      .def("promote_to_l0",
           [](TierEngine& e, const py::bytes& h, const std::function<int64_t()>& alloc) {
             std::vector<DeviceCopy> ev;
             SideEffects fx;
             auto c = e.promote_to_l0(std::string(h), &ev, &fx, alloc);
             return py::make_tuple(c, ev, fx);
           })
      .def("begin_promote", [](TierEngine& e, const py::bytes& h) { return e.begin_promote(std::string(h)); })
      .def("finish_promote", [](TierEngine& e, const py::bytes& h) { e.finish_promote(std::string(h)); })
      .def("promote_inflight_len", &TierEngine::promote_inflight_len)
      .def("demote_l0", [](TierEngine& e, const py::bytes& h) { return e.demote_l0(std::string(h)); })
      .def("evict_l0_pressure_victim",
           [](const TierEngine& e) -> py::object {
             auto v = e.evict_l0_pressure_victim();
             if (!v) return py::none();
             return py::bytes(*v);
           })
      .def("demote_l2_to_l3", [](TierEngine& e, const py::bytes& h) { return e.demote_l2_to_l3(std::string(h)); })
      .def("discard", [](TierEngine& e, const py::bytes& h) { e.discard(std::string(h)); })
      .def("compact_l2_segment", &TierEngine::compact_l2_segment)
      .def("colocate_l2_move",
           [](TierEngine& e, const py::bytes& h, uint64_t s, uint64_t o) {
             return e.colocate_l2_move(std::string(h), s, o);
           })
      .def_readonly("stats", &TierEngine::stats);

  py::enum_<ActionKind>(m, "ActionKind")
      .value("PROMOTE", ActionKind::Promote)
      .value("FILL_MISS", ActionKind::FillMiss)
      .value("DEMOTE_L0", ActionKind::DemoteL0)
      .value("DEMOTE_L2", ActionKind::DemoteL2)
      .value("COMPACT_SEGMENT", ActionKind::CompactSegment)
      .value("COLOCATE_MOVE", ActionKind::CoLocateMove);
  py::enum_<LocKind>(m, "LocKind")
      .value("PRESENT", LocKind::Present)
      .value("ABSENT", LocKind::Absent)
      .value("MOVED", LocKind::Moved)
      .value("L3_PRESENT", LocKind::L3Present);
  py::class_<Action>(m, "Action")
      .def(py::init([](ActionKind k, const py::bytes& h, uint64_t seg, uint64_t off) {
             Action a;
             a.kind = k;
             a.hash = std::string(h);
             a.segment_id = seg;
             a.offset = off;
             return a;
           }),
           py::arg("kind"), py::arg("hash") = py::bytes(""), py::arg("segment_id") = 0, py::arg("offset") = 0);
  py::class_<LocationEvent>(m, "LocationEvent")
      .def(py::init([](LocKind k, const py::bytes& h, int tier, const std::string& node, uint64_t seg, uint64_t off) {
             return LocationEvent{k, std::string(h), tier, node, seg, off};
           }),
           py::arg("kind"), py::arg("hash"), py::arg("tier"), py::arg("node_id"), py::arg("segment_id") = 0,
           py::arg("offset") = 0)
      .def_readonly("kind", &LocationEvent::kind)
      .def_property_readonly("hash", [](const LocationEvent& e) { return py::bytes(e.hash); })
      .def_readonly("tier", &LocationEvent::tier)
      .def_readonly("node_id", &LocationEvent::node_id)
      .def_readonly("segment_id", &LocationEvent::segment_id)
      .def_readonly("offset", &LocationEvent::offset);
  py::class_<TierPipeline>(m, "TierPipeline")
      .def(py::init<TierEngine*, BandwidthPool*, std::string>(), py::keep_alive<1, 2>(), py::keep_alive<1, 3>())
      .def("enqueue", &TierPipeline::enqueue)
      .def("pending", &TierPipeline::pending)
      .def("node_id", &TierPipeline::node_id)
      .def("tick", [](TierPipeline& p, size_t steps, uint64_t now_ms, const std::function<int64_t()>& alloc) {
        std::vector<DeviceCopy> copies;
        auto r = p.tick(steps, now_ms, alloc, &copies);
        return py::make_tuple(r.first, r.second, copies);
      });

  py::class_<WritebackBatcher>(m, "WritebackBatcher")
      .def(py::init<size_t>(), py::arg("batch") = 4)
      .def("push",
           [](WritebackBatcher& w, const py::bytes& h) {
             std::vector<py::bytes> o;
             for (auto& x : w.push(std::string(h))) o.push_back(py::bytes(x));
             return o;
           })
      .def("drain",
           [](WritebackBatcher& w) {
             std::vector<py::bytes> o;
             for (auto& x : w.drain()) o.push_back(py::bytes(x));
             return o;
           })
      .def("pending", &WritebackBatcher::pending)
      .def("flushes", &WritebackBatcher::flushes);
}
