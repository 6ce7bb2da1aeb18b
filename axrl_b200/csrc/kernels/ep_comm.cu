// Expert-parallel dispatch / combine over NVLink peer memory, with no host synchronisation.
//
// Every EP rank holds E_l = E / P experts.  A source rank sorts its (token, k) assignments by
// global expert and pushes its per-expert counts into every rank's symmetric count table
// (tp_push of csrc/kernels/tp_comm.cu), so every rank knows the full count matrix C[s][e].
// From C each rank derives, on the device (ep_plan_k):
//   * the owner layout of its receive buffer: rows grouped by local expert, then by source rank,
//     so the received rows are already in grouped-GEMM order (offsets[el] = first row of local
//     expert el; the grouped expert GEMM consumes them directly);
//   * dst_start[e]: where this source's rows for global expert e start in the owner's buffer;
//   * for each (local expert el, source s) block of its own buffer: the first row position and the
//     first row index in the source's sorted order.
// ep_transfer_k then moves rows with P2P stores, one warp per row:
//   mode 0 (source -> owner, "dispatch"): sorted row j of this rank goes to its owner's buffer;
//   mode 1 (owner -> source, "combine"):  owner row p goes back to row j of its source's buffer.
// The backward of dispatch is a combine of the row gradients and vice versa.
//
// Flow control follows tp_comm.cu: before the first store into a peer's buffer every block waits
// for that peer's "free" flag of this epoch (the peer's previous readers of the buffer have
// finished); after the stores the last block sets the data flag on every peer.  All waits are
// bounded (globaltimer) and report through `status` (1 free timeout, 3 capacity overflow).
// Rows that would land beyond a buffer's capacity are dropped and flagged (status 3).
//
// Reference counterpart: Megatron's alltoall token dispatcher (NCCL all-to-all + permute / unpermute)
// selected by moe_token_dispatcher_type="alltoall" (axrl/worker/megatron_worker.py:833).
#include "common.cuh"

namespace ax {
namespace epc {

constexpr int kMaxEP = 8;
constexpr int kMaxTP = 8;
constexpr int kMaxE = 1024;  // experts per layer
constexpr int kFreeBase = 16;

struct Peers {
  int64_t p[kMaxEP];
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

// One block.  C: (P, E) int32 counts (row s = rank s's rows per global expert).
// Outputs (int32): offsets[E_l+1] (this rank's receive layout), dst_start[E] (where this rank's rows
// for expert e start at their owner), blk_pos[E_l*P], blk_src[E_l*P] (block (el, s) of this rank's
// buffer: first position, first row in source s's sorted order), totals[2] = {rows received, rows sent}.
__global__ void ep_plan_k(const int* __restrict__ C, int P, int E, int self, int* offsets, int* dst_start, int* blk_pos, int* blk_src,
                          int* totals) {
  const int El = E / P;
  if (threadIdx.x != 0) return;  // tiny (P*E <= 8*1024): one thread keeps it simple and exact
  // receive layout of this rank
  int pos = 0;
  for (int el = 0; el < El; ++el) {
    offsets[el] = pos;
    int e = self * El + el;
    for (int s = 0; s < P; ++s) {
      int src_start = 0;
      for (int e2 = 0; e2 < e; ++e2) src_start += C[s * E + e2];
      blk_pos[el * P + s] = pos;
      blk_src[el * P + s] = src_start;
      pos += C[s * E + e];
    }
  }
  offsets[El] = pos;
  totals[0] = pos;
  // where this rank's rows go at each owner
  int sent = 0;
  for (int d = 0; d < P; ++d) {
    int base = 0;
    for (int el = 0; el < El; ++el) {
      int e = d * El + el;
      int before = 0;
      for (int s = 0; s < self; ++s) before += C[s * E + e];
      dst_start[e] = base + before;
      for (int s = 0; s < P; ++s) base += C[s * E + e];
      sent += C[self * E + e];
    }
  }
  totals[1] = sent;
}

// mode 0: rows of this rank's sorted order (n = totals[1]) -> owners' buffers; with `src_idx`, sorted
//         row r is row src_idx[r] of `rows` (the token rows, gathered on the fly).
// mode 1: rows of this rank's receive buffer (n = totals[0]) -> sources' buffers.
__global__ void ep_transfer_k(int mode, const uint4* __restrict__ rows, const int64_t* __restrict__ src_idx, int row16,
                              const int* __restrict__ C, int P, int E, int self,
                              const int* __restrict__ dst_start, const int* __restrict__ offsets, const int* __restrict__ blk_pos,
                              const int* __restrict__ blk_src, const int* __restrict__ totals, Peers dst, long dst_cap_rows, Peers flags,
                              const int* __restrict__ my_flags, int ch, int epoch, unsigned* ticket, uint64_t timeout_ns,
                              int* status) {
  __shared__ int ok;
  const int El = E / P;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0)
      for (int p = 0; p < P; ++p)
        if (p != self) st_release(reinterpret_cast<int*>(flags.p[p]) + (ch + kFreeBase) * kMaxTP + self, epoch);
    bool good = true;
    uint64_t t0 = gtimer();
    for (int p = 0; p < P && good; ++p) {
      if (p == self) continue;
      const int* f = my_flags + (ch + kFreeBase) * kMaxTP + p;
      while (ld_acquire(f) < epoch) {
        if (gtimer() - t0 > timeout_ns) {
          good = false;
          break;
        }
        __nanosleep(128);
      }
    }
    ok = good;
    if (!good) atomicCAS(status, 0, 1);
  }
  // row -> (expert / local expert) lookups by binary search over prefix sums staged in shared memory
  __shared__ int pre[kMaxE + 1];
  if (threadIdx.x == 0) {
    if (mode == 0) {  // this rank's sorted rows: exclusive prefix of its per-expert counts
      int a = 0;
      for (int e = 0; e < E; ++e) {
        pre[e] = a;
        a += C[self * E + e];
      }
      pre[E] = a;
    } else {
      for (int el = 0; el <= El; ++el) pre[el] = offsets[el];
    }
  }
  __syncthreads();
  if (ok) {
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x / 32;
    const long n = mode == 0 ? totals[1] : totals[0];
    const int nb = mode == 0 ? E : El;
    for (long r = (long)blockIdx.x * warps + threadIdx.x / 32; r < n; r += (long)gridDim.x * warps) {
      int lo = 0, hi = nb;  // first index with pre[index] > r, minus one: pre[x] <= r < pre[x + 1]
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (pre[mid] <= r) lo = mid + 1;
        else hi = mid;
      }
      const int x = lo - 1;
      int peer;
      long at;
      if (mode == 0) {
        peer = x / El;
        at = dst_start[x] + (r - pre[x]);
      } else {
        int s = 0;
        while (s + 1 < P && blk_pos[x * P + s + 1] <= r) ++s;
        peer = s;
        at = blk_src[x * P + s] + (r - blk_pos[x * P + s]);
      }
      if (at >= dst_cap_rows) {
        if (lane == 0) atomicCAS(status, 0, 3);
        continue;
      }
      const uint4* __restrict__ src = rows + (src_idx != nullptr ? src_idx[r] : r) * row16;
      uint4* __restrict__ out = reinterpret_cast<uint4*>(dst.p[peer]) + at * row16;
      for (int i0 = 0; i0 < row16; i0 += 8 * 32) {  // eight 16-byte loads in flight per lane, then the stores
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i0 + j * 32 + lane < row16) v[j] = src[i0 + j * 32 + lane];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i0 + j * 32 + lane < row16) out[i0 + j * 32 + lane] = v[j];
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned t = atomicAdd(ticket, 1u);
    if (t == gridDim.x - 1) {
      *ticket = 0u;
      __threadfence_system();
      for (int p = 0; p < P; ++p)
        if (p != self) st_release(reinterpret_cast<int*>(flags.p[p]) + ch * kMaxTP + self, epoch);
    }
  }
}

static Peers to_peers(const at::Tensor& t) {
  AX_CHECK(t.device().is_cpu() && t.scalar_type() == at::kLong && t.numel() <= kMaxEP, "peer table: int64 CPU tensor");
  Peers p{};
  for (int i = 0; i < t.numel(); ++i) p.p[i] = t.data_ptr<int64_t>()[i];
  return p;
}

}  // namespace epc

// plan: (C (P,E) int32 device, self) -> fills offsets, dst_start, blk_pos, blk_src, totals (device int32)
void ep_plan(at::Tensor C, int64_t self, at::Tensor offsets, at::Tensor dst_start, at::Tensor blk_pos, at::Tensor blk_src,
             at::Tensor totals) {
  AX_CHECK(C.scalar_type() == at::kInt && C.dim() == 2 && C.is_contiguous(), "C: (P, E) int32");
  int P = C.size(0), E = C.size(1);
  AX_CHECK(P <= epc::kMaxEP && E % P == 0 && E <= epc::kMaxE, "EP shape");
  epc::ep_plan_k<<<1, 32, 0, stream()>>>(C.data_ptr<int>(), P, E, (int)self, offsets.data_ptr<int>(), dst_start.data_ptr<int>(),
                                        blk_pos.data_ptr<int>(), blk_src.data_ptr<int>(), totals.data_ptr<int>());
  AX_LAUNCH_OK();
}

void ep_transfer(int64_t mode, at::Tensor rows, at::Tensor C, int64_t self, at::Tensor dst_start, at::Tensor offsets, at::Tensor blk_pos,
                 at::Tensor blk_src, at::Tensor totals, at::Tensor dst_ptrs, int64_t dst_cap_rows, at::Tensor flag_ptrs,
                 at::Tensor my_flags, int64_t ch, int64_t epoch, at::Tensor ticket, int64_t timeout_ns, at::Tensor status, int64_t ctas,
                 c10::optional<at::Tensor> src_idx) {
  AX_CHECK(rows.is_cuda() && rows.is_contiguous() && rows.dim() == 2, "rows");
  AX_CHECK(C.dim() == 2 && C.size(1) <= epc::kMaxE && C.size(0) <= epc::kMaxEP, "C: (P <= 8, E <= 1024)");
  const int64_t* idx = nullptr;
  if (src_idx.has_value()) {
    AX_CHECK(mode == 0 && src_idx->is_cuda() && src_idx->scalar_type() == at::kLong && src_idx->is_contiguous(), "src_idx: int64 (mode 0)");
    idx = src_idx->data_ptr<int64_t>();
  }
  long row_bytes = rows.size(1) * rows.element_size();
  AX_CHECK(row_bytes % 16 == 0, "row bytes must be a multiple of 16");
  int P = C.size(0), E = C.size(1);
  epc::ep_transfer_k<<<(int)ctas, 256, 0, stream()>>>(
      (int)mode, reinterpret_cast<const uint4*>(rows.data_ptr()), idx, (int)(row_bytes / 16), C.data_ptr<int>(), P, E, (int)self,
      dst_start.data_ptr<int>(), offsets.data_ptr<int>(), blk_pos.data_ptr<int>(), blk_src.data_ptr<int>(), totals.data_ptr<int>(),
      epc::to_peers(dst_ptrs), (long)dst_cap_rows, epc::to_peers(flag_ptrs), my_flags.data_ptr<int>(), (int)ch, (int)epoch,
      reinterpret_cast<unsigned*>(ticket.data_ptr<int>()) + ch, (uint64_t)timeout_ns, status.data_ptr<int>());
  AX_LAUNCH_OK();
}

}  // namespace ax
