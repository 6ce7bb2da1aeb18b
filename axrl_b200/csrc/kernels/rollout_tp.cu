// Tensor-parallel rollout collectives over NVLink peer memory, safe inside CUDA graphs.
//
// tp_ar_rms_k: one-shot all-reduce of the row-parallel projection partials fused with the
//   residual add and the next RMSNorm:
//     h = residual + sum_peers partial_p ;  x = h * rsqrt(mean(h^2) + eps) * w
//   Every rank's GEMM has written its partial into its own symmetric buffer; each block of the
//   kernel meets its counterpart blocks on the other ranks at a flag barrier, then reads its rows
//   of every peer's partial with P2P loads.
// tp_gather_cols_k: all-gather of vocabulary-sharded logits rows (B, V/tp) into (B, V).
//
// Graph safety: the barrier epoch is not a kernel argument (arguments are frozen in a captured
// graph) but a per-block counter in device memory that the kernel increments itself; all ranks run
// the same sequence of launches, so their counters agree.  Flag slots are per (block, source rank);
// a waiter tests `>= epoch`.  The host alternates two buffers between consecutive calls so a GEMM
// never overwrites a partial that a slower peer may still be reading.
// Every wait is bounded (globaltimer) and records status 2 on expiry instead of hanging.
//
// Reference counterpart: SGLang / FlashInfer custom all-reduce (+ fused RMSNorm) used by the
// rollout engines (guarded in axrl/worker/sglang_worker.py:125-152).
#include "common.cuh"

namespace ax {
namespace rtp {

constexpr int kMaxTP = 8;
constexpr int kBlocks = 32;  // fixed grid: every launch uses the same per-block counters

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

// flags layout: [kBlocks][kMaxTP] ints per rank; counters: [kBlocks] ints per rank (local).
__device__ bool block_barrier(Peers flags, int* my_flags, int* ctr, int world, int self, uint64_t timeout_ns, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const int epoch = ctr[blockIdx.x] + 1;
    __threadfence_system();  // this rank's partial (written by the preceding GEMM) is visible
    for (int p = 0; p < world; ++p)
      if (p != self) st_release(reinterpret_cast<int*>(flags.p[p]) + blockIdx.x * kMaxTP + self, epoch);
    bool good = true;
    uint64_t t0 = gtimer();
    for (int p = 0; p < world && good; ++p) {
      if (p == self) continue;
      while (ld_acquire(my_flags + blockIdx.x * kMaxTP + p) < epoch) {
        if (gtimer() - t0 > timeout_ns) {
          good = false;
          atomicCAS(status, 0, 2);
          break;
        }
        __nanosleep(64);
      }
    }
    ctr[blockIdx.x] = epoch;
    ok = good;
  }
  __syncthreads();
  return ok;
}

// rows x H bf16; partials at bufs.p[r] + off (elements).  H % 8 == 0, H <= 8 * 4 * blockDim.
__global__ void __launch_bounds__(512) tp_ar_rms_k(Peers bufs, long off, int rows, int H, const bf16* __restrict__ residual,
                                                   const bf16* __restrict__ w, float eps, bf16* __restrict__ out_h,
                                                   bf16* __restrict__ out_x, Peers flags, int* my_flags, int* ctr, int world, int self,
                                                   uint64_t timeout_ns, int* status) {
  if (!block_barrier(flags, my_flags, ctr, world, self, timeout_ns, status)) return;
  __shared__ float red[32];
  const int n8 = H / 8;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    float acc[4][8];
    float ss = 0.f;
    int cnt = 0;
    for (int i = threadIdx.x, j = 0; i < n8; i += blockDim.x, ++j) {
      float v[8];
      if (residual) load8(residual + (long)r * H + i * 8, v);
      else
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = 0.f;
      for (int p = 0; p < world; ++p) {
        float f[8];
        load8(reinterpret_cast<const bf16*>(bufs.p[p]) + off + (long)r * H + i * 8, f);
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] += f[t];
      }
      // round to bf16 first: the residual stream is stored in bf16
      bf16 hb[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        hb[t] = __float2bfloat16(v[t]);
        acc[j][t] = __bfloat162float(hb[t]);
        ss += acc[j][t] * acc[j][t];
      }
      if (out_h) *reinterpret_cast<V8*>(out_h + (long)r * H + i * 8) = *reinterpret_cast<V8*>(hb);
      cnt = j + 1;
    }
    ss = block_sum(ss, red);
    const float rstd = rsqrtf(ss / H + eps);
    for (int i = threadIdx.x, j = 0; j < cnt; i += blockDim.x, ++j) {
      float wf[8], x[8];
      load8(w + i * 8, wf);
#pragma unroll
      for (int t = 0; t < 8; ++t) x[t] = acc[j][t] * rstd * wf[t];
      store8(out_x + (long)r * H + i * 8, x);
    }
  }
}

// out[b, p*Vs + c] = shard_p[b, c] (bf16), shards at bufs.p[p] + off.
__global__ void tp_gather_cols_k(Peers bufs, long off, int rows, int Vs, bf16* __restrict__ out, Peers flags, int* my_flags, int* ctr,
                                 int world, int self, uint64_t timeout_ns, int* status) {
  if (!block_barrier(flags, my_flags, ctr, world, self, timeout_ns, status)) return;
  const int n8 = Vs / 8;
  const long total = (long)rows * n8 * world;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int p = (int)(i / ((long)rows * n8));
    const long rem = i % ((long)rows * n8);
    const int b = (int)(rem / n8), c = (int)(rem % n8);
    const V8 v = *reinterpret_cast<const V8*>(reinterpret_cast<const bf16*>(bufs.p[p]) + off + (long)b * Vs + c * 8);
    *reinterpret_cast<V8*>(out + (long)b * Vs * world + (long)p * Vs + c * 8) = v;
  }
}

static Peers to_peers(const at::Tensor& t) {
  AX_CHECK(t.device().is_cpu() && t.scalar_type() == at::kLong && t.numel() <= kMaxTP, "peer table: int64 CPU tensor");
  Peers p{};
  for (int i = 0; i < t.numel(); ++i) p.p[i] = t.data_ptr<int64_t>()[i];
  return p;
}

}  // namespace rtp

void tp_ar_rms(at::Tensor buf_ptrs, int64_t off, int64_t rows, int64_t H, c10::optional<at::Tensor> residual, at::Tensor w, double eps,
               c10::optional<at::Tensor> out_h, at::Tensor out_x, at::Tensor flag_ptrs, at::Tensor my_flags, at::Tensor ctr, int64_t self,
               int64_t timeout_ns, at::Tensor status) {
  AX_CHECK(H % 8 == 0 && H <= 8 * 4 * 512, "hidden size");
  AX_CHECK(ctr.numel() >= rtp::kBlocks && my_flags.numel() >= rtp::kBlocks * rtp::kMaxTP, "counters / flags");
  rtp::tp_ar_rms_k<<<rtp::kBlocks, 512, 0, stream()>>>(
      rtp::to_peers(buf_ptrs), (long)off, (int)rows, (int)H, residual ? (const bf16*)residual->data_ptr() : nullptr,
      (const bf16*)w.data_ptr(), (float)eps, out_h ? (bf16*)out_h->data_ptr() : nullptr, (bf16*)out_x.data_ptr(), rtp::to_peers(flag_ptrs),
      my_flags.data_ptr<int>(), ctr.data_ptr<int>(), (int)buf_ptrs.numel(), (int)self, (uint64_t)timeout_ns, status.data_ptr<int>());
  AX_LAUNCH_OK();
}

void tp_gather_cols(at::Tensor buf_ptrs, int64_t off, int64_t rows, int64_t Vs, at::Tensor out, at::Tensor flag_ptrs, at::Tensor my_flags,
                    at::Tensor ctr, int64_t self, int64_t timeout_ns, at::Tensor status) {
  AX_CHECK(Vs % 8 == 0 && out.scalar_type() == at::kBFloat16 && out.is_contiguous(), "logits layout");
  rtp::tp_gather_cols_k<<<rtp::kBlocks, 512, 0, stream()>>>(rtp::to_peers(buf_ptrs), (long)off, (int)rows, (int)Vs, (bf16*)out.data_ptr(),
                                                           rtp::to_peers(flag_ptrs), my_flags.data_ptr<int>(), ctr.data_ptr<int>(),
                                                           (int)buf_ptrs.numel(), (int)self, (uint64_t)timeout_ns, status.data_ptr<int>());
  AX_LAUNCH_OK();
}

}  // namespace ax
