// pybind11 bindings of the host-side runtime (module ``meshy_b200._native``).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>

#include "column_store.h"

namespace py = pybind11;
using meshy::ColumnStore;
using meshy::PageAllocator;

static std::vector<std::vector<std::string>> to_cols(const std::vector<std::vector<py::bytes>>& v) {
  std::vector<std::vector<std::string>> out(v.size());
  for (size_t f = 0; f < v.size(); ++f) {
    out[f].reserve(v[f].size());
    for (auto& b : v[f]) out[f].emplace_back(std::string(b));
  }
  return out;
}

PYBIND11_MODULE(_native, m) {
  m.doc() = "meshy_b200 host runtime: column store (data plane), KV page allocator";
  py::class_<ColumnStore>(m, "ColumnStore")
      .def(py::init<>())
      .def("put_rows",
           [](ColumnStore& s, const std::string& part, const std::vector<std::string>& fields,
              const std::vector<std::vector<py::bytes>>& values) {
             auto cols = to_cols(values);
             py::gil_scoped_release nogil;
             return s.put_rows(part, fields, cols);
           })
      .def("put_columns",
           [](ColumnStore& s, const std::string& part, const std::vector<int64_t>& idx,
              const std::vector<std::string>& fields, const std::vector<std::vector<py::bytes>>& values) {
             auto cols = to_cols(values);
             py::gil_scoped_release nogil;
             return s.put_columns(part, idx, fields, cols);
           })
      .def("get_meta",
           [](ColumnStore& s, const std::string& part, const std::vector<std::string>& fields, int64_t batch_size,
              int mode, const std::string& task, int64_t wait_ms) {
             py::gil_scoped_release nogil;
             return s.get_meta(part, fields, batch_size, mode, task, wait_ms);
           },
           py::arg("part"), py::arg("fields"), py::arg("batch_size"), py::arg("mode"), py::arg("task"),
           py::arg("wait_ms") = 0)
      .def("get_data",
           [](ColumnStore& s, const std::string& part, const std::vector<int64_t>& idx,
              const std::vector<std::string>& fields) {
             std::vector<std::vector<std::string>> data;
             {
               py::gil_scoped_release nogil;
               data = s.get_data(part, idx, fields);
             }
             py::list out;
             for (auto& col : data) {
               py::list c;
               for (auto& b : col) c.append(py::bytes(b));
               out.append(c);
             }
             return out;
           })
      .def("clear", &ColumnStore::clear)
      .def("clear_partition", &ColumnStore::clear_partition)
      .def("reset_consumption", &ColumnStore::reset_consumption)
      .def("partitions", &ColumnStore::partitions)
      .def("num_rows", &ColumnStore::num_rows)
      .def("status", &ColumnStore::status);

  py::class_<PageAllocator>(m, "PageAllocator")
      .def(py::init<int64_t, int64_t>(), py::arg("n_pages"), py::arg("reserved") = 1)
      .def("allocate", &PageAllocator::allocate)
      .def("free", &PageAllocator::free)
      .def("retain", &PageAllocator::retain)
      .def_property_readonly("num_free", &PageAllocator::num_free)
      .def_property_readonly("num_pages", &PageAllocator::num_pages);
}
