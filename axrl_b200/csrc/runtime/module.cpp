// Host runtime module axrl_b200._runtime: KV block manager, shared-memory segments,
// VMM tagged allocator.
#include <pybind11/pybind11.h>

namespace py = pybind11;

namespace ax_rt {
void bind_block_manager(py::module_& m);
void bind_shm(py::module_& m);
void bind_vmm(py::module_& m);
}  // namespace ax_rt

PYBIND11_MODULE(_runtime, m) {
  m.doc() = "axrl_b200 native host runtime";
  ax_rt::bind_block_manager(m);
  ax_rt::bind_shm(m);
  ax_rt::bind_vmm(m);
}
