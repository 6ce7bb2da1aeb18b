// NVLink collective kernels over symmetric memory (peer pointers and NVLS multicast).
//
// * p2p_reduce_shard     – reduce-scatter step of the distributed optimizer: pull every peer's
//                          fp32 gradient slice of this rank's shard (P2P loads), sum, write the
//                          local shard, accumulate its squared norm.
// * p2p_broadcast_shard  – all-gather step: cast the updated fp32 master shard to bf16 and store it
//                          into every peer's parameter buffer (P2P stores).
// * mc_reduce_shard / mc_broadcast_shard – the same two steps through an NVLS multicast address:
//                          one multimem.ld_reduce sums all ranks inside the switch, one multimem.st
//                          writes all ranks.
// * flag_signal / flag_wait_bounded – cross-GPU flags with a bounded wait: the waiting kernel gives
//                          up after `timeout_ns` (globaltimer) and writes an error status instead of
//                          spinning forever, so a missing peer becomes a host-visible error.
//
// Reference counterpart: Megatron's NCCL reduce-scatter / all-gather of the distributed
// optimizer (axrl/worker/megatron_worker.py:905-930); NCCL is kept as the baseline.
#include "common.cuh"

namespace ax {

// ---------------------------------------------------------------------------- P2P
__global__ void p2p_reduce_shard_k(const int64_t* __restrict__ ptrs, float* __restrict__ local, long s0, long n, int world,
                                   float* __restrict__ sq) {
  __shared__ float sh[32];
  float acc = 0.f;
  long n4 = n / 4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(ptrs[r]) + s0) + i;
      float4 v = *src;
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    reinterpret_cast<float4*>(local + s0)[i] = s;
    acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
  }
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) atomicAdd(sq, acc);
}

__global__ void p2p_broadcast_shard_k(const int64_t* __restrict__ ptrs, const float* __restrict__ master, long s0, long n, int world) {
  long n8 = n / 8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    float f[8];
    float4 a = reinterpret_cast<const float4*>(master)[2 * i], b = reinterpret_cast<const float4*>(master)[2 * i + 1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    V8 v;
#pragma unroll
    for (int j = 0; j < 4; ++j) v.h[j] = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
    for (int r = 0; r < world; ++r) reinterpret_cast<V8*>(reinterpret_cast<bf16*>(ptrs[r]) + s0)[i] = v;
  }
}

// ---------------------------------------------------------------------------- NVLS multicast
__global__ void mc_reduce_shard_k(uint64_t mc_base, float* __restrict__ local, long s0, long n, float* __restrict__ sq) {
  __shared__ float sh[32];
  float acc = 0.f;
  long n4 = n / 4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    uint64_t addr = mc_base + (uint64_t)(s0 + 4 * i) * 4;
    float x, y, z, w;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(x), "=f"(y), "=f"(z), "=f"(w) : "l"(addr) : "memory");
    reinterpret_cast<float4*>(local + s0)[i] = make_float4(x, y, z, w);
    acc += x * x + y * y + z * z + w * w;
  }
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) atomicAdd(sq, acc);
}

__global__ void mc_broadcast_shard_k(uint64_t mc_base, const float* __restrict__ master, long s0, long n) {
  long n8 = n / 8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    float4 a = reinterpret_cast<const float4*>(master)[2 * i], b = reinterpret_cast<const float4*>(master)[2 * i + 1];
    bf162 h0 = __floats2bfloat162_rn(a.x, a.y), h1 = __floats2bfloat162_rn(a.z, a.w);
    bf162 h2 = __floats2bfloat162_rn(b.x, b.y), h3 = __floats2bfloat162_rn(b.z, b.w);
    uint64_t addr = mc_base + (uint64_t)(s0 + 8 * i) * 2;
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(addr), "r"(*reinterpret_cast<uint32_t*>(&h0)),
                 "r"(*reinterpret_cast<uint32_t*>(&h1)), "r"(*reinterpret_cast<uint32_t*>(&h2)), "r"(*reinterpret_cast<uint32_t*>(&h3))
                 : "memory");
  }
}

// ---------------------------------------------------------------------------- bounded flags
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Set peer's flag slot to `value` (release semantics at system scope).
__global__ void flag_signal_k(int64_t peer_flag_addr, int slot, int value) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    int* f = reinterpret_cast<int*>(peer_flag_addr) + slot;
    __threadfence_system();
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f), "r"(value) : "memory");
  }
}

// Wait until local flag slot == value or timeout_ns elapses.  status[0] = 0 ok, 1 timed out.
// On success the flag is reset to 0 so the slot can be reused.
__global__ void flag_wait_bounded_k(int* flag, int slot, int value, uint64_t timeout_ns, int* status) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  uint64_t t0 = gtimer();
  int v = 0;
  while (true) {
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(flag + slot) : "memory");
    if (v == value) {
      flag[slot] = 0;
      status[0] = 0;
      return;
    }
    if (gtimer() - t0 > timeout_ns) {
      status[0] = 1;
      return;
    }
    __nanosleep(200);
  }
}

static int comm_ctas(long n) { return (int)std::max<long>(1, std::min<long>((n + 255) / 256, num_sms() * 4)); }

void p2p_reduce_shard(at::Tensor ptrs, at::Tensor local, int64_t s0, int64_t n, int64_t world, at::Tensor sq) {
  AX_CHECK(n % 4 == 0 && s0 % 4 == 0, "shard must be 16-byte aligned");
  if (n == 0) return;
  p2p_reduce_shard_k<<<comm_ctas(n / 4), 256, 0, stream()>>>(ptrs.data_ptr<int64_t>(), local.data_ptr<float>(), s0, n, (int)world,
                                                            sq.data_ptr<float>());
  AX_LAUNCH_OK();
}

void p2p_broadcast_shard(at::Tensor ptrs, at::Tensor master, int64_t s0, int64_t n, int64_t world) {
  AX_CHECK(n % 8 == 0 && s0 % 8 == 0, "shard must be 16-byte aligned");
  if (n == 0) return;
  p2p_broadcast_shard_k<<<comm_ctas(n / 8), 256, 0, stream()>>>(ptrs.data_ptr<int64_t>(), master.data_ptr<float>(), s0, n, (int)world);
  AX_LAUNCH_OK();
}

void mc_reduce_shard(int64_t mc_ptr, at::Tensor local, int64_t s0, int64_t n, at::Tensor sq) {
  AX_CHECK(mc_ptr != 0 && n % 4 == 0 && s0 % 4 == 0, "NVLS group address and 16-byte aligned shard required");
  if (n == 0) return;
  mc_reduce_shard_k<<<comm_ctas(n / 4), 256, 0, stream()>>>((uint64_t)mc_ptr, local.data_ptr<float>(), s0, n, sq.data_ptr<float>());
  AX_LAUNCH_OK();
}

void mc_broadcast_shard(int64_t mc_ptr, at::Tensor master, int64_t s0, int64_t n) {
  AX_CHECK(mc_ptr != 0 && n % 8 == 0 && s0 % 8 == 0, "NVLS group address and 16-byte aligned shard required");
  if (n == 0) return;
  mc_broadcast_shard_k<<<comm_ctas(n / 8), 256, 0, stream()>>>((uint64_t)mc_ptr, master.data_ptr<float>(), s0, n);
  AX_LAUNCH_OK();
}

void flag_signal(int64_t peer_flag_addr, int64_t slot, int64_t value) {
  flag_signal_k<<<1, 32, 0, stream()>>>(peer_flag_addr, (int)slot, (int)value);
  AX_LAUNCH_OK();
}

void flag_wait_bounded(at::Tensor flags, int64_t slot, int64_t value, int64_t timeout_ns, at::Tensor status) {
  flag_wait_bounded_k<<<1, 32, 0, stream()>>>(flags.data_ptr<int>(), (int)slot, (int)value, (uint64_t)timeout_ns, status.data_ptr<int>());
  AX_LAUNCH_OK();
}

}  // namespace ax
