#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "agent/agent.h"

namespace py = pybind11;
using namespace lakeb;
using namespace lakeb::agent;

namespace {
std::vector<std::string> strs(const std::vector<py::bytes>& v) {
  std::vector<std::string> o;
  for (auto& b : v) o.emplace_back(b);
  return o;
}
std::vector<py::bytes> pybytes(const std::vector<std::string>& v) {
  std::vector<py::bytes> o;
  for (auto& s : v) o.push_back(py::bytes(s));
  return o;
}

// Lets Python implement a control-plane port (fault-injection doubles in tests,
// or a gRPC client in the agent process).
class PyPort : public ControlPlanePort {
 public:
  using ControlPlanePort::ControlPlanePort;
  void admit_register_blocks(const std::string& node, const std::vector<std::string>& prefix,
                             const std::vector<cp::BlockMeta>& metas) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(this, "admit_register_blocks");
    if (f) f(node, pybytes(prefix), metas);
  }
  void register_blocks(const std::string& node, const std::vector<std::string>& prefix,
                       const std::vector<cp::BlockMeta>& metas) override {
    PYBIND11_OVERRIDE_PURE_NAME(void, ControlPlanePort, "register_blocks", register_blocks, node, pybytes(prefix), metas);
  }
  void report_refs(const std::vector<cp::RefDelta>& d) override {
    PYBIND11_OVERRIDE_PURE(void, ControlPlanePort, report_refs, d);
  }
  void request_barrier(const std::string& rid, const std::string& node) override {
    PYBIND11_OVERRIDE_PURE(void, ControlPlanePort, request_barrier, rid, node);
  }
  void publish_location(const cp::KVBlockID& id, int tier, const std::string& node, uint64_t seg, uint64_t off,
                        bool present) override {
    PYBIND11_OVERRIDE_PURE(void, ControlPlanePort, publish_location, id, tier, node, seg, off, present);
  }
  void set_l3_present(const cp::KVBlockID& id, bool present) override {
    PYBIND11_OVERRIDE_PURE(void, ControlPlanePort, set_l3_present, id, present);
  }
};
}  // namespace

void register_agent(py::module_& m) {
  py::class_<ControlPlanePort, PyPort>(m, "ControlPlanePort")
      .def(py::init<>())
      .def("admit_register_blocks",
           [](ControlPlanePort& p, const std::string& node, const std::vector<py::bytes>& prefix,
              const std::vector<cp::BlockMeta>& metas) { p.admit_register_blocks(node, strs(prefix), metas); })
      .def("register_blocks",
           [](ControlPlanePort& p, const std::string& node, const std::vector<py::bytes>& prefix,
              const std::vector<cp::BlockMeta>& metas) { p.register_blocks(node, strs(prefix), metas); })
      .def("report_refs", &ControlPlanePort::report_refs)
      .def("request_barrier", &ControlPlanePort::request_barrier)
      .def("publish_location", &ControlPlanePort::publish_location)
      .def("set_l3_present", &ControlPlanePort::set_l3_present);
  py::class_<AuthorityPort, ControlPlanePort>(m, "AuthorityPort")
      .def(py::init<cp::Authority*>(), py::keep_alive<1, 2>());

  py::class_<PutEndSession>(m, "PutEndSession")
      .def(py::init<std::string, std::string, std::string, std::string, std::string>(), py::arg("request_id"),
           py::arg("node_id"), py::arg("model_id"), py::arg("revision") = "", py::arg("storage_node") = "")
      .def("put_start",
           [](PutEndSession& s, const py::bytes& h, const py::bytes& data) {
             std::string d(data);
             s.put_start(std::string(h), reinterpret_cast<const uint8_t*>(d.data()), d.size());
           })
      .def("put_start_ptr",
           [](PutEndSession& s, const py::bytes& h, uintptr_t ptr, size_t n) {
             s.put_start(std::string(h), reinterpret_cast<const uint8_t*>(ptr), n);
           })
      .def("add_prefix", [](PutEndSession& s, const py::bytes& h) { s.add_prefix(std::string(h)); })
      .def("metas", &PutEndSession::metas)
      .def("flush_durable", [](PutEndSession& s, tier::TierEngine& st) { return pybytes(s.flush_durable(st)); })
      .def("commit_through", &PutEndSession::commit_through, py::call_guard<py::gil_scoped_release>())
      .def("all_durable", &PutEndSession::all_durable)
      .def("writeback_open", &PutEndSession::writeback_open)
      .def("register_hold_open", &PutEndSession::register_hold_open)
      .def("prefix_hashes", [](const PutEndSession& s) { return pybytes(s.prefix_hashes()); });

  m.def("apply_location_events", &apply_location_events, py::arg("port"), py::arg("model_id"), py::arg("revision"),
        py::arg("pool_kind"), py::arg("events"));

  m.def("enqueue_defrag_moves", &enqueue_defrag_moves, py::arg("pipeline"), py::arg("moves"));
  m.def("sync_background_pause", &sync_background_pause, py::arg("bandwidth"), py::arg("paused"));
  py::class_<BackpressureMemory>(m, "BackpressureMemory")
      .def(py::init<double>(), py::arg("ttl_s") = 30.0)
      .def("record", &BackpressureMemory::record)
      .def("fresh",
           [](const BackpressureMemory& b) -> py::object {
             cp::BackpressureSignal s;
             if (!b.fresh(&s)) return py::none();
             return py::cast(s);
           })
      .def("clear", &BackpressureMemory::clear);
}
