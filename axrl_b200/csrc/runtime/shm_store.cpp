// Shared-memory segments for the host data plane (handle-based tensor store).
//
// Reference counterpart: TensorHandle over Ray plasma (axrl/utils/tensor_store.py:27-91).
// A producer writes a payload into a named POSIX shared-memory segment and passes a small
// handle (segment name, offset, shape, dtype) through the control plane; consumers map the
// segment read-only and build zero-copy views.  Segments can optionally be page-locked with
// cudaHostRegister so host->device copies from them are asynchronous DMA.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <pybind11/pybind11.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <stdexcept>
#include <string>

namespace py = pybind11;

namespace ax_rt {

class ShmSegment {
 public:
  ShmSegment(const std::string& name, int64_t size, bool create) : name_(name), size_(size), owner_(create) {
    int flags = create ? (O_CREAT | O_EXCL | O_RDWR) : O_RDWR;
    fd_ = shm_open(name.c_str(), flags, 0600);
    if (fd_ < 0) throw std::runtime_error("shm_open(" + name + "): " + std::strerror(errno));
    if (create) {
      if (ftruncate(fd_, size) != 0) {
        int e = errno;
        ::close(fd_);
        shm_unlink(name.c_str());
        throw std::runtime_error(std::string("ftruncate: ") + std::strerror(e));
      }
    } else {
      struct stat st;
      fstat(fd_, &st);
      size_ = st.st_size;
    }
    ptr_ = size_ > 0 ? mmap(nullptr, size_, PROT_READ | PROT_WRITE, MAP_SHARED, fd_, 0) : nullptr;
    if (size_ > 0 && ptr_ == MAP_FAILED) {
      int e = errno;
      ::close(fd_);
      throw std::runtime_error(std::string("mmap: ") + std::strerror(e));
    }
  }
  ~ShmSegment() { close(); }

  void close() {
    if (registered_) {
      cudaHostUnregister(ptr_);
      registered_ = false;
    }
    if (ptr_ && ptr_ != MAP_FAILED) munmap(ptr_, size_);
    ptr_ = nullptr;
    if (fd_ >= 0) ::close(fd_);
    fd_ = -1;
  }

  // Page-lock for async H2D; returns false (no error) when no CUDA device is present.
  bool pin() {
    if (registered_ || !ptr_) return registered_;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
      cudaGetLastError();
      return false;
    }
    registered_ = cudaHostRegister(ptr_, size_, cudaHostRegisterPortable) == cudaSuccess;
    if (!registered_) cudaGetLastError();
    return registered_;
  }

  void unlink() { shm_unlink(name_.c_str()); }
  int64_t address() const { return (int64_t)(uintptr_t)ptr_; }
  int64_t size() const { return size_; }
  const std::string& name() const { return name_; }
  bool pinned() const { return registered_; }
  py::memoryview view() { return py::memoryview::from_memory(ptr_, size_, false); }

 private:
  std::string name_;
  int64_t size_;
  bool owner_;
  int fd_ = -1;
  void* ptr_ = nullptr;
  bool registered_ = false;
};

void bind_shm(py::module_& m) {
  py::class_<ShmSegment>(m, "ShmSegment")
      .def(py::init<const std::string&, int64_t, bool>(), py::arg("name"), py::arg("size"), py::arg("create"))
      .def("close", &ShmSegment::close)
      .def("pin", &ShmSegment::pin)
      .def("unlink", &ShmSegment::unlink)
      .def("view", &ShmSegment::view)
      .def_property_readonly("address", &ShmSegment::address)
      .def_property_readonly("size", &ShmSegment::size)
      .def_property_readonly("name", &ShmSegment::name)
      .def_property_readonly("pinned", &ShmSegment::pinned);
}

}  // namespace ax_rt
