// Device helpers and launch utilities shared by the sm_100a kernels.  Pure CUDA: no torch
// headers, so translation units that only hold kernels and raw-pointer launchers compile in
// seconds.  Torch-facing wrappers include common.cuh, which adds the tensor types on top.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <mutex>
#include <set>
#include <sstream>
#include <stdexcept>
#include <string>
#include <tuple>
#include <utility>

namespace ax {
namespace detail {
inline void cat_args(std::ostringstream&) {}
template <typename T, typename... R>
inline void cat_args(std::ostringstream& os, const T& v, const R&... r) {
  os << v;
  cat_args(os, r...);
}
}  // namespace detail

// Throws std::runtime_error (a Python RuntimeError through the bindings) with the message parts.
template <typename... A>
[[noreturn]] inline void fail(const char* file, int line, const A&... parts) {
  std::ostringstream os;
  detail::cat_args(os, parts...);
  os << " (" << file << ":" << line << ")";
  throw std::runtime_error(os.str());
}
}  // namespace ax

#define AX_REQUIRE(cond, ...)                                   \
  do {                                                          \
    if (!(cond)) ::ax::fail(__FILE__, __LINE__, __VA_ARGS__);   \
  } while (0)
#define AX_CUDA_OK(expr)                                                                       \
  do {                                                                                         \
    cudaError_t _e = (expr);                                                                   \
    if (_e != cudaSuccess) ::ax::fail(__FILE__, __LINE__, "CUDA error ", cudaGetErrorString(_e)); \
  } while (0)
#define AX_LAUNCH_OK() AX_CUDA_OK(cudaGetLastError())

namespace ax {

// Device scratch memory for launchers that need a temporary buffer (CUTLASS workspaces, grouped
// GEMM argument arrays).  The torch glue implements these with the caching allocator on the
// given stream, so a buffer freed right after the launch is reused only by later work on that
// stream.
void* scratch_alloc(size_t bytes, cudaStream_t st);
void scratch_free(void* p);

struct Scratch {
  void* ptr = nullptr;
  Scratch(size_t bytes, cudaStream_t st) : ptr(bytes ? scratch_alloc(bytes, st) : nullptr) {}
  ~Scratch() {
    if (ptr) scratch_free(ptr);
  }
  Scratch(const Scratch&) = delete;
  Scratch& operator=(const Scratch&) = delete;
};

using bf16 = __nv_bfloat16;
using bf162 = __nv_bfloat162;

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Raise a kernel's dynamic shared memory limit on the current device.  The attribute is per
// device, so the (kernel, device, bytes) triples already set are remembered, not one flag per process.
inline void smem_attr(const void* kern, int bytes) {
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, int>> done;
  int dev = 0;
  AX_CUDA_OK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> g(mu);
  const auto key = std::make_tuple(kern, dev, bytes);
  if (done.count(key)) return;
  AX_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert(key);
}

// 16-byte vector of 8 bf16.
struct alignas(16) V8 {
  bf162 h[4];
};

__device__ __forceinline__ void load8(const bf16* p, float (&f)[8]) {
  V8 v = *reinterpret_cast<const V8*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(bf16* p, const float (&f)[8]) {
  V8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<V8*>(p) = v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `sh` must hold >= 32 floats.  All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* sh) {
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  v = lane < nw ? sh[lane] : 0.f;
  return warp_sum(v);
}

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with launch_pdl() may be scheduled while its stream predecessor is still
// running: as soon as every CTA of the predecessor has executed pdl_trigger() (or exited).  Every
// thread of such a kernel executes pdl_wait() before it reads memory that earlier work writes and
// before it writes memory that earlier work may still read; pdl_wait() returns once the
// predecessor grid has completed and its writes are visible.  Only reads of data that no recent
// kernel writes (weights during a rollout, see weights_static()) may be issued before it.  Every
// kernel launched this way waits unconditionally, so a grid completes only after its predecessor,
// and ordering stays transitive along the stream.  Kernels on the decode path trigger before they
// wait: a successor then becomes resident as soon as SM room frees up and streams its weights during
// the tail of this grid and its predecessor (its own pdl_wait() still orders every dependent access).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool& pdl_enabled() {
  static bool on = [] {
    const char* e = std::getenv("AXRL_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Set while the rollout engine decodes: the weight matrices are then read-only, so weight-streaming
// GEMMs may start loading them before their predecessor finishes.
inline bool& weights_static() {
  static bool on = false;
  return on;
}

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  AX_CUDA_OK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

}  // namespace ax
