#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "transfer/transfer.h"

namespace py = pybind11;
using namespace lakeb;

void register_transfer(py::module_& m) {
  m.attr("SEG_HOST") = int(SEG_HOST);
  m.attr("SEG_PINNED") = int(SEG_PINNED);
  m.attr("SEG_DEVICE") = int(SEG_DEVICE);
  m.attr("SEG_EXTERNAL") = int(SEG_EXTERNAL);

  py::class_<TransferOp>(m, "TransferOp")
      .def(py::init([](int tier, const std::string& node, uint64_t ss, uint64_t so, uint64_t ds, uint64_t dof,
                       uint64_t len) { return TransferOp{tier, node, ss, so, ds, dof, len}; }),
           py::arg("src_tier"), py::arg("src_node"), py::arg("src_segment"), py::arg("src_offset"),
           py::arg("dst_segment"), py::arg("dst_offset"), py::arg("length"));
  py::class_<TaskStatus>(m, "TaskStatus")
      .def_readonly("state", &TaskStatus::state)
      .def_readonly("bytes_done", &TaskStatus::bytes_done);

  py::class_<TransferEngine>(m, "TransferEngine")
      .def(py::init<std::string>(), py::arg("node_id") = "node-0")
      .def_property_readonly("node_id", &TransferEngine::node_id)
      .def("open_segment", &TransferEngine::open_segment, py::arg("name"), py::arg("capacity"),
           py::arg("kind") = int(SEG_HOST), py::arg("device") = -1)
      .def("register_segment", &TransferEngine::register_segment, py::arg("name"), py::arg("ptr"),
           py::arg("capacity"), py::arg("device") = -1)
      .def("free_segment", &TransferEngine::free_segment)
      .def("write_segment",
           [](TransferEngine& e, uint64_t id, uint64_t off, const py::bytes& b) {
             e.write_segment(id, off, std::string(b));
           })
      .def("read_segment",
           [](TransferEngine& e, uint64_t id, uint64_t off, uint64_t len) {
             std::string s;
             {
               py::gil_scoped_release r;
               s = e.read_segment(id, off, len);
             }
             return py::bytes(s);
           })
      .def("segment_ptr", &TransferEngine::segment_ptr)
      .def("allocate_batch_id", &TransferEngine::allocate_batch_id)
      .def("submit_transfer", &TransferEngine::submit_transfer, py::call_guard<py::gil_scoped_release>())
      .def("get_transfer_status", &TransferEngine::get_transfer_status)
      .def("wait_batch", &TransferEngine::wait_batch, py::call_guard<py::gil_scoped_release>())
      .def("free_batch_id", &TransferEngine::free_batch_id, py::call_guard<py::gil_scoped_release>())
      .def("segment_count", &TransferEngine::segment_count)
      .def("batch_count", &TransferEngine::batch_count)
      .def_property_readonly("bytes_moved", &TransferEngine::bytes_moved);

  py::class_<ByteStore>(m, "ByteStore")
      .def(py::init<uint64_t>(), py::arg("capacity_bytes") = 0)
      .def_static("key",
                  [](const std::string& m, const std::string& r, int pk, const py::bytes& h) {
                    return py::bytes(ByteStore::key(m, r, pk, std::string(h)));
                  })
      .def("put", [](ByteStore& s, const py::bytes& k, const py::bytes& d) { s.put(std::string(k), std::string(d)); })
      .def("get",
           [](ByteStore& s, const py::bytes& k) -> py::object {
             std::string out;
             if (!s.get(std::string(k), &out)) return py::none();
             return py::bytes(out);
           })
      .def("contains", [](const ByteStore& s, const py::bytes& k) { return s.contains(std::string(k)); })
      .def("erase", [](ByteStore& s, const py::bytes& k) { return s.erase(std::string(k)); })
      .def("__len__", &ByteStore::size)
      .def_property_readonly("bytes", &ByteStore::bytes)
      .def_property_readonly("evictions", &ByteStore::evictions);
}
