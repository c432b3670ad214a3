#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "router/router.h"

namespace py = pybind11;
using namespace lakeb::router;

namespace {
std::vector<std::string> strs(const std::vector<py::bytes>& v) {
  std::vector<std::string> o;
  for (auto& b : v) o.emplace_back(b);
  return o;
}
}  // namespace

void register_router(py::module_& m) {
  py::enum_<ExecMode>(m, "ExecMode")
      .value("COLOCATED", ExecMode::Colocated)
      .value("PD_DISAGG", ExecMode::PDDisagg)
      .value("D_DIRECT", ExecMode::DDirect);
  py::enum_<Role>(m, "Role").value("HYBRID", Role::Hybrid).value("PREFILL", Role::Prefill).value("DECODE", Role::Decode);
  py::class_<PrefixHint>(m, "PrefixHint")
      .def(py::init([](int c, int r, int l, bool lh) { return PrefixHint{c, r, l, lh}; }), py::arg("computed_tokens") = 0,
           py::arg("reused_blocks") = 0, py::arg("local_hit_blocks") = 0, py::arg("local_hit") = false)
      .def_readwrite("computed_tokens", &PrefixHint::computed_tokens)
      .def_readwrite("reused_blocks", &PrefixHint::reused_blocks)
      .def_readwrite("local_hit_blocks", &PrefixHint::local_hit_blocks)
      .def_readwrite("local_hit", &PrefixHint::local_hit);
  m.def("select_exec_mode", &select_exec_mode);
  m.def("prefix_anchor", [](const std::vector<py::bytes>& h) { return py::bytes(prefix_anchor(strs(h))); });
  m.attr("TRANSFER_BW_THRESHOLD_GBPS") = kTransferBWThresholdGBps;

  py::class_<MirrorBlock>(m, "MirrorBlock")
      .def_property_readonly("hash", [](const MirrorBlock& b) { return py::bytes(b.hash); })
      .def_readonly("local_hit", &MirrorBlock::local_hit);
  py::class_<ViewMirror>(m, "ViewMirror")
      .def(py::init<>())
      .def("apply", &ViewMirror::apply)
      .def("last_seq", &ViewMirror::last_seq)
      .def("size", &ViewMirror::size)
      .def("prefix_lookup", [](const ViewMirror& v, const std::string& model, const std::string& rev, int pk,
                               const std::vector<py::bytes>& h, const std::string& req) {
        return v.prefix_lookup(model, rev, pk, strs(h), req);
      });

  py::class_<NodeRegistry>(m, "NodeRegistry")
      .def(py::init<const std::vector<std::string>&>(), py::arg("initial") = std::vector<std::string>{})
      .def("ready_ids", &NodeRegistry::ready_ids)
      .def("inc_inflight", &NodeRegistry::inc_inflight)
      .def("dec_inflight", &NodeRegistry::dec_inflight)
      .def("inflight", &NodeRegistry::inflight)
      .def("add", &NodeRegistry::add)
      .def("mark_draining", &NodeRegistry::mark_draining)
      .def("unmark_draining", &NodeRegistry::unmark_draining)
      .def("remove", &NodeRegistry::remove)
      .def("draining", &NodeRegistry::draining)
      .def("last_ready", &NodeRegistry::last_ready)
      .def("next_id", &NodeRegistry::next_id)
      .def("count", &NodeRegistry::count);
  m.def("pick_node",
        [](const NodeRegistry& n, const ViewMirror* mirror, const std::string& model, const std::vector<py::bytes>& h,
           const py::bytes& key, int64_t guard) { return pick_node(n, mirror, model, strs(h), std::string(key), guard); },
        py::arg("nodes"), py::arg("mirror"), py::arg("model"), py::arg("hashes"), py::arg("routing_key"),
        py::arg("guard") = kDefaultAffinityGuard);

  py::class_<LoadReport>(m, "LoadReport")
      .def_readonly("node_id", &LoadReport::node_id)
      .def_readonly("queue_len", &LoadReport::queue_len)
      .def_readonly("in_flight", &LoadReport::in_flight)
      .def_readonly("remaining_cap", &LoadReport::remaining_cap);
  py::class_<PQScheduler>(m, "PQScheduler")
      .def(py::init<int, double>(), py::arg("max_inflight"), py::arg("bp_ttl_s") = 5.0)
      .def("submit",
           [](PQScheduler& s, int prio, const std::string& model) {
             uint64_t pre = 0;
             uint64_t t = s.submit(prio, model, &pre);
             return py::make_tuple(t, pre ? py::object(py::int_(pre)) : py::object(py::none()));
           })
      .def("start_eligible", &PQScheduler::start_eligible)
      .def("finish", &PQScheduler::finish, py::arg("ticket"), py::arg("preempted") = false)
      .def("cancel", &PQScheduler::cancel)
      .def("set_backpressure", &PQScheduler::set_backpressure)
      .def("backpressured", &PQScheduler::backpressured)
      .def("next_backpressure_expiry_s", &PQScheduler::next_backpressure_expiry_s)
      .def("set_max_inflight", &PQScheduler::set_max_inflight)
      .def("load_snapshot", &PQScheduler::load_snapshot)
      .def("wait_samples", &PQScheduler::wait_samples)
      .def("queue_len", &PQScheduler::queue_len)
      .def("in_flight", &PQScheduler::in_flight);

  py::enum_<ScaleDecision>(m, "ScaleDecision")
      .value("NONE", ScaleDecision::None)
      .value("SCALE_OUT", ScaleDecision::ScaleOut)
      .value("SCALE_IN", ScaleDecision::ScaleIn);
  py::class_<AutoscaleConfig>(m, "AutoscaleConfig")
      .def(py::init([](int mn, int mx, int out, int in, int sus, double cool) {
             return AutoscaleConfig{mn, mx, out, in, sus, cool};
           }),
           py::arg("min_nodes") = 1, py::arg("max_nodes") = 8, py::arg("scale_out_queue_len") = 4,
           py::arg("scale_in_queue_len") = 0, py::arg("sustain_periods") = 3, py::arg("cooldown_s") = 10.0);
  py::class_<Autoscaler>(m, "Autoscaler")
      .def(py::init<AutoscaleConfig>())
      .def("evaluate", &Autoscaler::evaluate);
  py::class_<HotSet>(m, "HotSet")
      .def(py::init<size_t>(), py::arg("cap") = 4096)
      .def("add", &HotSet::add)
      .def("drain", &HotSet::drain)
      .def("size", &HotSet::size);
}
