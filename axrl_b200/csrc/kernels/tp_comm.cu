// Tensor-parallel (sequence-parallel) row collectives over NVLink peer memory.
//
// The trainer's TP group keeps symmetric buffers (same size on every rank, every rank maps every
// peer's copy) for the all-gather input of column-parallel GEMMs and for the reduce-scatter slots
// of row-parallel GEMMs.  Data moves with P2P stores issued by tp_push_k; readiness travels in
// per-channel epoch flags:
//
//   flags[ch][src] (int, in each rank's symmetric flag array) = last epoch at which rank `src`
//   signalled channel `ch` to this rank.  Epochs only grow, so a waiter tests `>= epoch` and no
//   flag is ever reset.
//
// A push of epoch e on data channel c to the ranks in dst_mask:
//   1. block 0 tells every peer "my buffer of channel c may be overwritten for epoch e" (free
//      channel c + kFreeBase; idempotent, so every push of the epoch may repeat it);
//   2. every block waits until each destination peer has said the same (its previous readers of
//      the buffer have finished: that peer's push is stream-ordered after them);
//   3. the blocks copy the payload into each destination rank's buffer (P2P stores; the own rank
//      is a local copy);
//   4. the last block to finish (ticket counter) fences and sets flags[c][self] = e on every
//      destination peer.
// Consumers wait for the data flag of the source they need (tp_wait_k) and then read their own
// local buffer, so the GEMMs that consume gathered rows never read another GPU's memory.
//
// Every wait is bounded by `timeout_ns` (globaltimer): on expiry the kernel records a status code
// (1 = free-barrier timeout, 2 = data timeout) in `status`, skips the dependent work and returns,
// so a missing peer becomes an error the host reads instead of a hung GPU.
//
// Reference counterpart: Megatron's sequence-parallel all-gather / reduce-scatter around
// Column/RowParallelLinear (NCCL), selected by provider.sequence_parallel
// (axrl/worker/megatron_worker.py:825).
#include "common.cuh"

namespace ax {
namespace tpc {

constexpr int kMaxTP = 8;
constexpr int kFreeBase = 16;  // free channel of data channel c is c + kFreeBase
constexpr int kChannels = 32;

struct Peers {
  int64_t p[kMaxTP];
};

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until flags[ch][s] >= epoch for every s in `mask`; false on timeout.
__device__ bool wait_mask(const int* flags, int ch, unsigned mask, int epoch, uint64_t timeout_ns) {
  uint64_t t0 = gtimer();
  for (int s = 0; s < kMaxTP; ++s) {
    if (!(mask >> s & 1u)) continue;
    const int* f = flags + ch * kMaxTP + s;
    while (ld_acquire(f) < epoch) {
      if (gtimer() - t0 > timeout_ns) return false;
      __nanosleep(128);
    }
  }
  return true;
}

// dst rank d receives src[d * src_stride16 ...][0, n16) at its buffer + dst_off16 (16-byte units).
__global__ void tp_push_k(const uint4* __restrict__ src, long n16, long src_stride16, Peers dst, long dst_off16, Peers flags,
                          const int* __restrict__ my_flags, int ch, int epoch, int world, int self, unsigned dst_mask,
                          unsigned* ticket, uint64_t timeout_ns, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      for (int p = 0; p < world; ++p)
        if (p != self) st_release(reinterpret_cast<int*>(flags.p[p]) + (ch + kFreeBase) * kMaxTP + self, epoch);
    }
    ok = wait_mask(my_flags, ch + kFreeBase, dst_mask & ~(1u << self), epoch, timeout_ns);
    if (!ok) atomicCAS(status, 0, 1);
  }
  __syncthreads();
  if (ok) {
    const long stride = (long)gridDim.x * blockDim.x;
    for (int k = 0; k < world; ++k) {
      int d = (self + 1 + k) % world;  // peers first, own copy last; ranks start on different peers
      if (!(dst_mask >> d & 1u)) continue;
      const uint4* s = src + (long)d * src_stride16;
      uint4* o = reinterpret_cast<uint4*>(dst.p[d]) + dst_off16;
      for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) o[i] = s[i];
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned t = atomicAdd(ticket, 1u);
    if (t == gridDim.x - 1) {
      *ticket = 0u;  // every block of this launch has arrived; the next launch is stream-ordered
      __threadfence_system();
      for (int p = 0; p < world; ++p)
        if (p != self && (dst_mask >> p & 1u)) st_release(reinterpret_cast<int*>(flags.p[p]) + ch * kMaxTP + self, epoch);
    }
  }
}

__global__ void tp_wait_k(const int* __restrict__ my_flags, int ch, unsigned mask, int epoch, uint64_t timeout_ns, int* status) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    if (!wait_mask(my_flags, ch, mask, epoch, timeout_ns)) atomicCAS(status, 0, 2);
  }
}

// out[i] = sum_s slots[s][i] (+ residual[i]), fp32 accumulation, 8 bf16 per thread step.
__global__ void tp_reduce_slots_k(const bf16* __restrict__ slots, long n, int world, const bf16* __restrict__ residual,
                                  bf16* __restrict__ out) {
  const long n8 = n / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    float acc[8], f[8];
    if (residual) load8(residual + i * 8, acc);
    else
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int s = 0; s < world; ++s) {
      load8(slots + (long)s * n + i * 8, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
    store8(out + i * 8, acc);
  }
}

static Peers to_peers(const at::Tensor& t) {
  AX_CHECK(t.device().is_cpu() && t.scalar_type() == at::kLong && t.numel() <= kMaxTP, "peer table: int64 CPU tensor");
  Peers p{};
  for (int i = 0; i < t.numel(); ++i) p.p[i] = t.data_ptr<int64_t>()[i];
  return p;
}

}  // namespace tpc

// Push `src` (chunk d at d * src_stride_bytes, or the same chunk for every rank when the stride is
// 0) into the symmetric buffer of every rank in `dst_mask` at `dst_off_bytes`, then signal data
// channel `ch` to those ranks.
void tp_push(at::Tensor src, int64_t chunk_bytes, int64_t src_stride_bytes, at::Tensor dst_ptrs, int64_t dst_off_bytes,
             at::Tensor flag_ptrs, at::Tensor my_flags, int64_t ch, int64_t epoch, int64_t self, int64_t dst_mask, at::Tensor ticket,
             int64_t timeout_ns, at::Tensor status, int64_t ctas) {
  int world = dst_ptrs.numel();
  AX_CHECK(world >= 1 && world <= tpc::kMaxTP && self < world, "world size");
  AX_CHECK(ch >= 0 && ch < tpc::kFreeBase, "channel");
  AX_CHECK(chunk_bytes % 16 == 0 && src_stride_bytes % 16 == 0 && dst_off_bytes % 16 == 0, "16-byte granularity");
  AX_CHECK(reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0, "src alignment");
  AX_CHECK(my_flags.scalar_type() == at::kInt && my_flags.numel() >= tpc::kChannels * tpc::kMaxTP, "flags");
  tpc::tp_push_k<<<(int)ctas, 512, 0, stream()>>>(reinterpret_cast<const uint4*>(src.data_ptr()), chunk_bytes / 16, src_stride_bytes / 16,
                                                 tpc::to_peers(dst_ptrs), dst_off_bytes / 16, tpc::to_peers(flag_ptrs),
                                                 my_flags.data_ptr<int>(), (int)ch, (int)epoch, world, (int)self,
                                                 (unsigned)dst_mask, reinterpret_cast<unsigned*>(ticket.data_ptr<int>()) + ch, (uint64_t)timeout_ns,
                                                 status.data_ptr<int>());
  AX_LAUNCH_OK();
}

void tp_wait(at::Tensor my_flags, int64_t ch, int64_t mask, int64_t epoch, int64_t timeout_ns, at::Tensor status) {
  tpc::tp_wait_k<<<1, 32, 0, stream()>>>(my_flags.data_ptr<int>(), (int)ch, (unsigned)mask, (int)epoch, (uint64_t)timeout_ns,
                                        status.data_ptr<int>());
  AX_LAUNCH_OK();
}

void tp_reduce_slots(at::Tensor slots, int64_t world, int64_t n, c10::optional<at::Tensor> residual, at::Tensor out) {
  AX_CHECK(n % 8 == 0, "row payload must be a multiple of 8 elements");
  AX_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == n, "out");
  if (n == 0) return;
  int ctas = (int)std::min<long>((n / 8 + 255) / 256, (long)num_sms() * 8);
  tpc::tp_reduce_slots_k<<<ctas, 256, 0, stream()>>>(reinterpret_cast<const bf16*>(slots.data_ptr()), n, (int)world,
                                                    residual ? reinterpret_cast<const bf16*>(residual->data_ptr()) : nullptr,
                                                    reinterpret_cast<bf16*>(out.data_ptr()));
  AX_LAUNCH_OK();
}

}  // namespace ax
