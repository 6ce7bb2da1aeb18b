// Tagged virtual-memory allocator: release and re-map GPU memory at the same addresses.
//
// Reference counterpart: torch_memory_saver (an LD_PRELOAD cudaMalloc hook used through
// axrl/ray/ray_utils.py:33-41 and axrl/worker/megatron_worker.py:1463-1480) that lets the
// trainer and the rollout engine time-slice one GPU.
//
// Every allocation reserves its own virtual range (cuMemAddressReserve) backed by one
// physical allocation (cuMemCreate + cuMemMap).  `pause(tag)` optionally copies the
// contents to pinned host memory, then unmaps and releases the physical memory while
// keeping the virtual range; `resume(tag)` creates new physical memory, maps it at the same
// address and restores the contents.  Tensors that point into a paused range keep their
// addresses and become valid again after resume.
//
// torch integration: ax_vmm_malloc / ax_vmm_free have the signature expected by
// torch.cuda.memory.CUDAPluggableAllocator; allocations made while a tag is active
// (set_tag) belong to that tag.  Use it through a torch.cuda.MemPool so only the tensors
// created inside `use_mem_pool` are routed here.
#include <cuda.h>
#include <cuda_runtime.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

namespace ax_rt {

// Driver entry points are resolved at run time through the CUDA runtime, so this module
// loads (and its host-only parts work) on machines without a GPU driver.
struct Drv {
  CUresult (*Init)(unsigned int) = nullptr;
  CUresult (*GetErrorString)(CUresult, const char**) = nullptr;
  CUresult (*MemGetAllocationGranularity)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags) = nullptr;
  CUresult (*MemAddressReserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long) = nullptr;
  CUresult (*MemAddressFree)(CUdeviceptr, size_t) = nullptr;
  CUresult (*MemCreate)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long) = nullptr;
  CUresult (*MemRelease)(CUmemGenericAllocationHandle) = nullptr;
  CUresult (*MemMap)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long) = nullptr;
  CUresult (*MemUnmap)(CUdeviceptr, size_t) = nullptr;
  CUresult (*MemSetAccess)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t) = nullptr;

  template <class F>
  static void get(const char* name, F& fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
      throw std::runtime_error(std::string("CUDA driver entry point unavailable: ") + name);
    fn = reinterpret_cast<F>(p);
  }
  static Drv& d() {
    static Drv x = [] {
      Drv r;
      get("cuInit", r.Init);
      get("cuGetErrorString", r.GetErrorString);
      get("cuMemGetAllocationGranularity", r.MemGetAllocationGranularity);
      get("cuMemAddressReserve", r.MemAddressReserve);
      get("cuMemAddressFree", r.MemAddressFree);
      get("cuMemCreate", r.MemCreate);
      get("cuMemRelease", r.MemRelease);
      get("cuMemMap", r.MemMap);
      get("cuMemUnmap", r.MemUnmap);
      get("cuMemSetAccess", r.MemSetAccess);
      return r;
    }();
    return x;
  }
};

#define VMM_CHECK(x)                                                                \
  do {                                                                              \
    CUresult _r = (x);                                                              \
    if (_r != CUDA_SUCCESS) {                                                       \
      const char* _s = nullptr;                                                     \
      Drv::d().GetErrorString(_r, &_s);                                             \
      throw std::runtime_error(std::string(#x " failed: ") + (_s ? _s : "unknown")); \
    }                                                                               \
  } while (0)

struct Region {
  CUdeviceptr ptr = 0;
  size_t size = 0;  // rounded to granularity
  size_t user_size = 0;
  int device = 0;
  std::string tag;
  CUmemGenericAllocationHandle handle = 0;
  bool mapped = false;
  void* backup = nullptr;  // pinned host copy while paused (optional)
};

class VmmAllocator {
 public:
  static VmmAllocator& get() {
    static VmmAllocator a;
    return a;
  }

  void set_tag(const std::string& t) {
    std::lock_guard<std::mutex> g(mu_);
    tag_ = t;
  }
  std::string tag() {
    std::lock_guard<std::mutex> g(mu_);
    return tag_;
  }

  void* malloc(size_t size, int device) {
    std::lock_guard<std::mutex> g(mu_);
    Drv::d().Init(0);
    CUmemAllocationProp prop = props(device);
    size_t gran = 0;
    VMM_CHECK(Drv::d().MemGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM));
    size_t sz = ((size + gran - 1) / gran) * gran;
    if (sz == 0) sz = gran;
    Region r;
    r.size = sz;
    r.user_size = size;
    r.device = device;
    r.tag = tag_;
    VMM_CHECK(Drv::d().MemAddressReserve(&r.ptr, sz, 0, 0, 0));
    map_new(r);
    regions_[r.ptr] = r;
    return (void*)r.ptr;
  }

  void free(void* p) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = regions_.find((CUdeviceptr)p);
    if (it == regions_.end()) return;
    Region& r = it->second;
    if (r.mapped) {
      Drv::d().MemUnmap(r.ptr, r.size);
      Drv::d().MemRelease(r.handle);
    }
    if (r.backup) cudaFreeHost(r.backup);
    Drv::d().MemAddressFree(r.ptr, r.size);
    regions_.erase(it);
  }

  // Release physical memory of every region with `tag`.  Returns bytes released.
  int64_t pause(const std::string& tag, bool backup) {
    std::lock_guard<std::mutex> g(mu_);
    int64_t total = 0;
    cudaDeviceSynchronize();
    for (auto& kv : regions_) {
      Region& r = kv.second;
      if (r.tag != tag || !r.mapped) continue;
      if (backup) {
        if (!r.backup && cudaHostAlloc(&r.backup, r.user_size, cudaHostAllocDefault) != cudaSuccess)
          throw std::runtime_error("pinned backup allocation failed");
        if (cudaMemcpy(r.backup, (void*)r.ptr, r.user_size, cudaMemcpyDeviceToHost) != cudaSuccess)
          throw std::runtime_error("backup copy failed");
      }
      VMM_CHECK(Drv::d().MemUnmap(r.ptr, r.size));
      VMM_CHECK(Drv::d().MemRelease(r.handle));
      r.mapped = false;
      total += (int64_t)r.size;
    }
    return total;
  }

  int64_t resume(const std::string& tag) {
    std::lock_guard<std::mutex> g(mu_);
    int64_t total = 0;
    for (auto& kv : regions_) {
      Region& r = kv.second;
      if (r.tag != tag || r.mapped) continue;
      map_new(r);
      if (r.backup) {
        if (cudaMemcpy((void*)r.ptr, r.backup, r.user_size, cudaMemcpyHostToDevice) != cudaSuccess)
          throw std::runtime_error("restore copy failed");
        cudaFreeHost(r.backup);
        r.backup = nullptr;
      }
      total += (int64_t)r.size;
    }
    return total;
  }

  py::dict stats() {
    std::lock_guard<std::mutex> g(mu_);
    py::dict d;
    for (auto& kv : regions_) {
      const Region& r = kv.second;
      std::string key = r.tag + (r.mapped ? ":mapped" : ":paused");
      int64_t prev = d.contains(key.c_str()) ? d[key.c_str()].cast<int64_t>() : 0;
      d[key.c_str()] = prev + (int64_t)r.size;
    }
    return d;
  }

 private:
  CUmemAllocationProp props(int device) {
    CUmemAllocationProp prop = {};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = device;
    return prop;
  }
  void map_new(Region& r) {
    CUmemAllocationProp prop = props(r.device);
    VMM_CHECK(Drv::d().MemCreate(&r.handle, r.size, &prop, 0));
    VMM_CHECK(Drv::d().MemMap(r.ptr, r.size, 0, r.handle, 0));
    CUmemAccessDesc acc = {};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = r.device;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    VMM_CHECK(Drv::d().MemSetAccess(r.ptr, r.size, &acc, 1));
    r.mapped = true;
  }

  std::mutex mu_;
  std::string tag_ = "default";
  std::map<CUdeviceptr, Region> regions_;
};

void bind_vmm(py::module_& m) {
  m.def("vmm_set_tag", [](const std::string& t) { VmmAllocator::get().set_tag(t); });
  m.def("vmm_tag", []() { return VmmAllocator::get().tag(); });
  m.def("vmm_pause", [](const std::string& t, bool backup) { return VmmAllocator::get().pause(t, backup); }, py::arg("tag"),
        py::arg("backup") = false);
  m.def("vmm_resume", [](const std::string& t) { return VmmAllocator::get().resume(t); });
  m.def("vmm_stats", []() { return VmmAllocator::get().stats(); });
  m.def("vmm_malloc", [](int64_t size, int device) { return (int64_t)(uintptr_t)VmmAllocator::get().malloc(size, device); });
  m.def("vmm_free", [](int64_t ptr) { VmmAllocator::get().free((void*)(uintptr_t)ptr); });
}

}  // namespace ax_rt

// C ABI for torch.cuda.memory.CUDAPluggableAllocator.
extern "C" {
void* ax_vmm_malloc(ssize_t size, int device, cudaStream_t) {
  try {
    return ax_rt::VmmAllocator::get().malloc((size_t)size, device);
  } catch (...) {
    return nullptr;
  }
}
void ax_vmm_free(void* ptr, ssize_t, int, cudaStream_t) {
  try {
    ax_rt::VmmAllocator::get().free(ptr);
  } catch (...) {
  }
}
}
