#include <pybind11/pybind11.h>

#include "weights/weight_cache.h"

namespace py = pybind11;
using lakeb::weights::WeightCache;

void register_weights(py::module_& m) {
  py::class_<WeightCache>(m, "WeightCache")
      .def(py::init<uint64_t, bool>(), py::arg("capacity_bytes"), py::arg("pinned") = true)
      .def_static("key", &WeightCache::key)
      .def("put", &WeightCache::put, py::arg("key"), py::arg("src"), py::arg("nbytes"), py::arg("device") = false,
           py::call_guard<py::gil_scoped_release>())
      .def("contains", &WeightCache::contains)
      .def("size_of", &WeightCache::size_of)
      .def("load_to", &WeightCache::load_to, py::arg("key"), py::arg("dst"), py::arg("stream"))
      .def("read", &WeightCache::read)
      .def("pin", &WeightCache::pin)
      .def("unpin", &WeightCache::unpin)
      .def("erase", &WeightCache::erase)
      .def_property_readonly("capacity", &WeightCache::capacity)
      .def_property_readonly("used", &WeightCache::used)
      .def_property_readonly("entries", &WeightCache::entries)
      .def_property_readonly("hits", &WeightCache::hits)
      .def_property_readonly("misses", &WeightCache::misses)
      .def_property_readonly("evictions", &WeightCache::evictions);
}
