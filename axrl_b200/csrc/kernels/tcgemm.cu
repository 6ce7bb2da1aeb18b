// Hand-written persistent bf16 GEMM on the 5th-generation tensor cores, with epilogues that can
// write tiles straight into another GPU's memory (the fused GEMM -> reduce-scatter of tensor
// parallelism).  Reference counterpart: the TP row-parallel linear + sequence-parallel
// reduce-scatter of Megatron / TransformerEngine (axrl/worker/megatron_worker.py:833-870), which
// runs a cuBLAS GEMM and then an NCCL reduce-scatter.
//
//   D[M, N] = A[M, K] @ B[N, K]^T (+ C[M, N])      bf16 in, fp32 accumulate
//
// Either operand may be K-major (reduction dimension contiguous: the forward x @ W^T) or MN-major
// (loaded as 64 x 64 boxes, the descriptor's leading offset stepping from one 64-wide block to
// the next): the data-gradient GEMM dY @ W reads W MN-major, the weight-gradient GEMM dY^T @ X
// reads both operands MN-major and accumulates into an fp32 gradient (mode F32ACC).
//
// One CTA per SM walks output tiles of 128 x 256 (grouped raster: GROUP_M row tiles share the
// column tiles they visit, so weight tiles stay in L2):
//
//   warp 0      TMA producer: A (128 x 64) and B (256 x 64) K-slices into a 4-stage ring
//               (cp.async.bulk.tensor, 128-byte swizzle, no multicast).
//   warp 1      MMA issuer (one thread) and TMEM owner: four tcgen05.mma (M 128, N 256, K 16) per
//               K-slice into one of two 256-column fp32 accumulators, so the epilogue of tile t
//               overlaps the main loop of tile t + 1.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time (warp w reads TMEM lanes 32 (w % 4)),
//               optional residual, bf16 conversion, and the store:
//                 mode LOCAL   D row-major in this GPU's memory;
//                 mode F32ACC  fp32 D row-major, added to (or replacing) what it holds;
//                 mode SLOTS   row r of the output belongs to TP rank r / rows_per_rank; the tile
//                              is stored into that rank's receive slot for this rank
//                              (peer[owner] + (rank * rows_per_rank + r % rows_per_rank) * N),
//                              with plain stores over NVLink, so the transfer of every tile
//                              overlaps the MMAs of the next one.  Synchronisation follows the
//                              TP channel protocol of tp_comm.cu: CTA 0 declares this rank's
//                              receive buffer free for the epoch, every epilogue waits (bounded)
//                              until each peer has declared the same before its first store, and
//                              the last CTA to finish fences and raises the epoch's data flag on
//                              every peer.
//
//   mode AGATHER (all-gather -> GEMM of tensor parallelism): A is the gathered activation (world x
//                rows_per_rank rows) in this rank's gather buffer, where the caller has placed this
//                rank's own rows.  Four extra warps per CTA pull the other ranks' rows from their
//                gather buffers over NVLink (16-byte loads, each row crossing the link once) into
//                this rank's buffer, every CTA a share of every chunk; a chunk is complete when its
//                copy counter reaches the call's target, and the TMA producer waits (bounded) for
//                that before loading A tiles of the chunk.  Row tiles are visited this rank's chunk
//                first, so the local MMAs cover the transfers.  Handshakes on the TP channel: CTA 0
//                raises this rank's data flag on every peer (its rows are in place), copy warps
//                wait for each peer's data flag before reading it, and the CTA that completes a
//                peer's chunk tells that peer its buffer is free again.
//
// Every mbarrier wait is bounded: on expiry the CTA records an error code, drains what it issued,
// frees its TMEM and exits.  TMA reads only this GPU's memory.
#include <cuda.h>

#include <vector>

#include "../cuda_common.cuh"

namespace ax {
namespace tg {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, GROUP_M = 8;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr long WAIT_LIMIT = 1L << 26;
enum { B_FULL = 0, B_EMPTY = STAGES, B_ACC_FULL = 2 * STAGES, B_ACC_EMPTY = 2 * STAGES + 2, B_DRAIN = 2 * STAGES + 4, NBAR = 2 * STAGES + 5 };
enum Mode { LOCAL = 0, SLOTS = 1, F32ACC = 2, AGATHER = 3 };
constexpr int threads_of(int mode) { return mode == AGATHER ? 320 : THREADS; }  // AGATHER: warps 6-9 copy

struct Params {
  int M, N, K;
  int tiles_m, tiles_n;
  bf16* d;               // LOCAL: D (M x N)
  float* d32;            // F32ACC: D (M x N) fp32
  int accumulate;        // F32ACC: D += A @ B (else D = A @ B)
  const bf16* c;         // optional residual (M x N), LOCAL mode
  const int64_t* peers;  // SLOTS: receive buffer of every TP rank (device pointers as int64)
  int rank, rows_per_rank;
  int* err;
  // SLOTS: channel flags (tp_comm.cu layout: flags[ch][src]) of every rank and of this rank
  const int64_t* flag_peers;
  const int* my_flags;
  int ch, epoch, world;
  unsigned* ticket;
  unsigned long long timeout_ns;
  int* status;
  // AGATHER: every rank's gather buffer (world x rows_per_rank rows of K), this rank's copy counters
  // (one per source chunk, monotonic) and the counter value of a complete chunk for this call
  const int64_t* src_peers;
  int* ag_cnt;
  int ag_target;
};

constexpr int kMaxTP = 8, kFreeBase = 16;
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ int ld_acquire(const int* f) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* f, int v) { asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f), "r"(v) : "memory"); }
// Every peer has declared this channel's buffer free for `epoch` (bounded).
__device__ bool peers_free(const Params& p) {
  const uint64_t t0 = gtimer();
  for (int s = 0; s < p.world; ++s) {
    if (s == p.rank) continue;
    const int* f = p.my_flags + (p.ch + kFreeBase) * kMaxTP + s;
    while (ld_acquire(f) < p.epoch) {
      if (gtimer() - t0 > p.timeout_ns) return false;
      __nanosleep(64);
    }
  }
  return true;
}

__device__ __forceinline__ uint32_t s32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* b, int n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void arrive(uint64_t* b) { asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s32(b)) : "memory"); }
__device__ __forceinline__ bool try_wait(uint64_t* b, uint32_t ph) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(ok) : "r"(s32(b)), "r"(ph) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait(uint64_t* b, uint32_t ph, volatile int* abort, int* err, int code) {
  for (long it = 0; !try_wait(b, ph); ++it) {
    if (*abort) return false;
    if (it > WAIT_LIMIT) {
      *abort = 1;
      atomicCAS(err, 0, code);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* m, int x, int y, uint64_t* b) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(s32(dst)),
               "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(s32(b))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(s32(b)) : "memory");
}
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d), "l"(a),
               "l"(b), "r"(idesc), "r"(acc)
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%"
      "25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]),
        "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// K-major, 128-byte swizzle shared-memory descriptor (rows of 128 bytes, 8-row groups 1024 bytes apart)
__device__ __forceinline__ uint64_t desc_k128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// MN-major, 128-byte swizzle descriptor: 64-element blocks of 8 KB (64 K rows x 128 bytes) one after
// the other (leading offset), 8-row groups 1024 bytes apart
__device__ __forceinline__ uint64_t desc_mn128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)(8192 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// kind::f16 instruction descriptor: bf16 x bf16 -> fp32, M = 128, N = BN; bits 15 / 16 mark an
// MN-major A / B
template <bool A_MN, bool B_MN>
constexpr uint32_t idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}
constexpr uint32_t IDESC = idesc<false, false>();

// Tile t of the grouped raster -> (row tile, column tile); `rot` rotates the row tiles (AGATHER:
// this rank's chunk first).
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn, int rot = 0) {
  const int per_group = GROUP_M * tiles_n;
  const int g = t / per_group, first = g * GROUP_M;
  const int rows = min(GROUP_M, tiles_m - first);
  const int in = t - g * per_group;
  tm = (first + in % rows + rot) % tiles_m;
  tn = in / rows;
}
__device__ __forceinline__ int ld_acquire_gpu(const int* f) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}

template <int MODE, bool A_MN = false, bool B_MN = false>
__global__ void __launch_bounds__(threads_of(MODE), 1) gemm_k(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                                                              Params p) {
  extern __shared__ char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + STAGES * STAGE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBAR);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = p.tiles_m * p.tiles_n, kslices = (p.K + BK - 1) / BK;  // a ragged last slice reads zeros
  const int rot = MODE == AGATHER ? p.rank * (p.rows_per_rank / BM) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar[B_FULL + s], 1);
      mbar_init(&bar[B_EMPTY + s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bar[B_ACC_FULL + a], 1);
      mbar_init(&bar[B_ACC_EMPTY + a], 4);
    }
    mbar_init(&bar[B_DRAIN], 1);
    *abort = 0;
    tmem_slot[2] = 0u;  // epilogue warps finished (SLOTS completion count)
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&ta)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tb)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      int it = 0;  // global K-slice counter (ring position)
      unsigned ready = MODE == AGATHER ? (1u << p.rank) : 0u;  // AGATHER: source chunks complete in this buffer
      for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, p.tiles_m, p.tiles_n, tm, tn, rot);
        if constexpr (MODE == AGATHER) {
          const int c = tm * BM / p.rows_per_rank;
          if (!(ready & (1u << c))) {
            const uint64_t t0 = gtimer();
            while (ld_acquire_gpu(p.ag_cnt + c) < p.ag_target) {
              if (*abort) break;
              if (gtimer() - t0 > p.timeout_ns) {
                atomicCAS(p.status, 0, 2);
                *abort = 1;
                break;
              }
              __nanosleep(64);
            }
            if (*abort) break;
            asm volatile("fence.proxy.async.global;" ::: "memory");  // the copies are visible to the TMA reads
            ready |= 1u << c;
          }
        }
        for (int kb = 0; kb < kslices; ++kb, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !wait(&bar[B_EMPTY + s], ((it / STAGES) - 1) & 1, abort, p.err, 1)) break;
          expect_tx(&bar[B_FULL + s], STAGE_BYTES);
          char* st = sm + s * STAGE_BYTES;
          if constexpr (A_MN) {
#pragma unroll
            for (int i = 0; i < BM / 64; ++i) tma2d(st + i * 8192, &ta, tm * BM + i * 64, kb * BK, &bar[B_FULL + s]);
          } else {
            tma2d(st, &ta, kb * BK, tm * BM, &bar[B_FULL + s]);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int i = 0; i < BN / 64; ++i) tma2d(st + A_BYTES + i * 8192, &tb, tn * BN + i * 64, kb * BK, &bar[B_FULL + s]);
          } else {
            tma2d(st + A_BYTES, &tb, kb * BK, tn * BN, &bar[B_FULL + s]);
          }
        }
      }
      if (*abort) {  // every copy this CTA started lands before shared memory is released
        int zero = 0;
        for (int i = max(0, it - STAGES); i < it; ++i) wait(&bar[B_FULL + i % STAGES], (i / STAGES) & 1, (volatile int*)&zero, p.err, 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0, ti = 0;
      for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, ++ti) {
        const int a = ti & 1;
        if (ti >= 2 && !wait(&bar[B_ACC_EMPTY + a], ((ti >> 1) - 1) & 1, abort, p.err, 2)) break;
        fence_after();
        bool ok = true;
        for (int kb = 0; kb < kslices; ++kb, ++it) {
          const int s = it % STAGES;
          if (!wait(&bar[B_FULL + s], (it / STAGES) & 1, abort, p.err, 3)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t sa = s32(sm + s * STAGE_BYTES), sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t da = A_MN ? desc_mn128(sa + kk * 2048) : desc_k128(sa + kk * 32);
            const uint64_t db = B_MN ? desc_mn128(sb + kk * 2048) : desc_k128(sb + kk * 32);
            mma(tmem + a * BN, da, db, idesc<A_MN, B_MN>(), (kb | kk) ? 1u : 0u);
          }
          commit(&bar[B_EMPTY + s]);
        }
        if (!ok) break;
        commit(&bar[B_ACC_FULL + a]);
      }
      commit(&bar[B_DRAIN]);  // nothing issued here may still run when TMEM is freed
      int zero = 0;
      wait(&bar[B_DRAIN], 0, (volatile int*)&zero, p.err, 4);
    }
  } else if (MODE == AGATHER && warp >= 6) {
    // ---------------------------------------------------------------- copy warps (AGATHER): pull peer chunks
    const int cw = warp - 6;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the preceding kernels (this rank's rows) are complete
    if (blockIdx.x == 0 && cw == 0 && lane == 0)  // this rank's rows are in place in its gather buffer
      for (int s = 0; s < p.world; ++s)
        if (s != p.rank) st_release(reinterpret_cast<int*>(p.flag_peers[s]) + p.ch * kMaxTP + p.rank, p.epoch);
    const long row16 = (long)p.K * 2 / 16;
    const int per_cta = (p.rows_per_rank + gridDim.x - 1) / gridDim.x;
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(p.src_peers[p.rank]));
    volatile uint32_t* s_ok = tmem_slot + 3;  // the copy warps' shared decision for the current chunk
    for (int k = 1; k < p.world; ++k) {
      const int s = (p.rank + k) % p.world;
      if (cw == 0 && lane == 0) {  // the peer's rows are in place (one poller, bounded)
        uint32_t ok = 1;
        const uint64_t t0 = gtimer();
        const int* f = p.my_flags + p.ch * kMaxTP + s;
        while (ld_acquire(f) < p.epoch) {
          if (*abort || gtimer() - t0 > p.timeout_ns) {
            ok = 0;
            break;
          }
          __nanosleep(128);
        }
        if (!ok && !*abort) {
          atomicCAS(p.status, 0, 2);
          *abort = 1;
        }
        *s_ok = ok;
      }
      asm volatile("bar.sync 2, 128;" ::: "memory");
      const bool go = *s_ok != 0;
      asm volatile("bar.sync 2, 128;" ::: "memory");  // every copy warp read the decision before the next chunk's
      if (!go) break;
      const long r0 = (long)s * p.rows_per_rank + (long)blockIdx.x * per_cta;
      const long r1 = min((long)(s + 1) * p.rows_per_rank, r0 + per_cta);
      const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(p.src_peers[s]));
      if (r0 < r1) {
        const long v1 = r1 * row16;
        for (long v = r0 * row16 + (cw * 32 + lane); v < v1; v += 4 * 4 * 32) {  // four 16-byte loads in flight per lane
          uint4 a[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (v + u * 128 < v1) a[u] = src[v + u * 128];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (v + u * 128 < v1) dst[v + u * 128] = a[u];
        }
      }
      asm volatile("bar.sync 2, 128;" ::: "memory");  // the four copy warps finished this CTA's share
      if (cw == 0 && lane == 0) {
        __threadfence();
        asm volatile("fence.proxy.async.global;" ::: "memory");
        if (atomicAdd(p.ag_cnt + s, 1) + 1 == p.ag_target)  // the chunk is complete here: the peer may reuse its rows
          st_release(reinterpret_cast<int*>(p.flag_peers[s]) + (p.ch + kFreeBase) * kMaxTP + p.rank, p.epoch);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    if (MODE == SLOTS) {
      if (blockIdx.x == 0 && warp == 2 && lane == 0)  // this rank's receive buffer may be overwritten
        for (int s = 0; s < p.world; ++s)
          if (s != p.rank) st_release(reinterpret_cast<int*>(p.flag_peers[s]) + (p.ch + kFreeBase) * kMaxTP + p.rank, p.epoch);
      int ok = 1;
      if (lane == 0 && !peers_free(p)) {
        ok = 0;
        atomicCAS(p.status, 0, 1);
        *abort = 1;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) goto epilogue_done;
    }
    {
    int ti = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++ti) {
      const int a = ti & 1;
      if (!__all_sync(0xffffffffu, wait(&bar[B_ACC_FULL + a], (ti >> 1) & 1, abort, p.err, 5))) break;
      fence_after();
      int tm, tn;
      tile_coords(t, p.tiles_m, p.tiles_n, tm, tn, rot);
      const int row = tm * BM + q * 32 + lane;
      if constexpr (MODE == F32ACC) {
        float* d = row < p.M ? p.d32 + (long)row * p.N : nullptr;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(lane_base + a * BN + c * 32, r);
          const int col = tn * BN + c * 32;
          if (d != nullptr && col < p.N) {
            float4* d4 = reinterpret_cast<float4*>(d + col);
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              float4 o = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]), __uint_as_float(r[4 * v + 2]),
                                     __uint_as_float(r[4 * v + 3]));
              if (p.accumulate) {
                const float4 old = d4[v];
                o.x += old.x, o.y += old.y, o.z += old.z, o.w += old.w;
              }
              d4[v] = o;
            }
          }
        }
        fence_before();
        __syncwarp();
        if (lane == 0) arrive(&bar[B_ACC_EMPTY + a]);
        continue;
      }
      bf16* dst = nullptr;
      const bf16* res = nullptr;
      if (row < p.M) {
        if (MODE == LOCAL || MODE == AGATHER) {
          dst = p.d + (long)row * p.N;
          if (p.c) res = p.c + (long)row * p.N;
        } else {
          const int owner = row / p.rows_per_rank;
          bf16* base = reinterpret_cast<bf16*>(p.peers[owner]);
          dst = base + ((long)p.rank * p.rows_per_rank + row % p.rows_per_rank) * p.N;
        }
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(lane_base + a * BN + c * 32, r);
        const int col = tn * BN + c * 32;
        if (dst != nullptr && col < p.N) {
          uint4 out[4];
          uint32_t* w = reinterpret_cast<uint32_t*>(out);
          if (res != nullptr) {
            const uint4* rs = reinterpret_cast<const uint4*>(res + col);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 x = rs[v];
              const bf162* h = reinterpret_cast<const bf162*>(&x);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float2 f = __bfloat1622float2(h[e]);
                bf162 o = __floats2bfloat162_rn(__uint_as_float(r[v * 8 + 2 * e]) + f.x, __uint_as_float(r[v * 8 + 2 * e + 1]) + f.y);
                w[v * 4 + e] = *reinterpret_cast<uint32_t*>(&o);
              }
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              bf162 o = __floats2bfloat162_rn(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
              w[e] = *reinterpret_cast<uint32_t*>(&o);
            }
          }
          uint4* d4 = reinterpret_cast<uint4*>(dst + col);
#pragma unroll
          for (int v = 0; v < 4; ++v) d4[v] = out[v];
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) arrive(&bar[B_ACC_EMPTY + a]);
    }
    }
    if (MODE == SLOTS) {
      // the last epilogue warp of the last CTA publishes the epoch's data flag on every peer
      __threadfence_system();
      __syncwarp();
      if (lane == 0) {
        unsigned* done_warps = reinterpret_cast<unsigned*>(tmem_slot + 2);
        if (atomicAdd(done_warps, 1u) == 3u && !*abort) {
          const unsigned t = atomicAdd(p.ticket, 1u);
          if (t == gridDim.x - 1) {
            *p.ticket = 0u;  // every CTA of this launch arrived; the next launch is stream-ordered
            __threadfence_system();
            for (int s = 0; s < p.world; ++s)
              if (s != p.rank) st_release(reinterpret_cast<int*>(p.flag_peers[s]) + p.ch * kMaxTP + p.rank, p.epoch);
          }
        }
      }
    }
  epilogue_done:;
  }
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------------------------- weight streaming (decode)
// Y[M, N] = X[M, K] @ W[N, K]^T (+ R) for M <= 64 token rows, computed transposed on the tensor
// cores: Y^T tile (128 weight rows x NTOK tokens) = W tile (128 x K, the MMA's M) @ X^T.  At decode
// sizes the GEMM is a read of W, so the grid is one CTA per SM and every CTA streams the same
// number of (128-row W tile, 64-wide K slab) units, a contiguous range in tile-major order:
//
//   warp 0      TMA producer: W slab (16 KB) + X slab (NTOK x 64) into an 8-stage ring; with
//               `prefetch_w` (weights read-only during the rollout) the first W slabs are issued
//               before waiting for the preceding kernel (programmatic dependent launch).
//   warp 1      MMA issuer: four tcgen05.mma (M 128, N NTOK, K 16) per slab into one of two TMEM
//               accumulators; a run of slabs of one W tile is a segment.
//   warps 2-5   epilogue per segment, warp w owning weight rows 32 (w % 4) .. +31 of the tile (its
//               TMEM lanes): a segment that covers the whole K range stores bf16 (+ R) directly;
//               otherwise the fp32 partial is added to a workspace (red.global.add) and the
//               stripe's arrival counter is advanced by the slabs covered; the warp that completes
//               the stripe adds R, stores bf16 and zeroes the workspace stripe and counter, so the
//               workspace is clean for the next call without a memset.  Calls sharing a workspace
//               must be stream-ordered.
namespace sk {
constexpr int BW = 128, BK = 64, STAGES = 8, THREADS = 192;
constexpr uint32_t TMEM_COLS = 128;  // two accumulators of up to 64 columns
enum { B_FULL = 0, B_EMPTY = STAGES, B_ACC_FULL = 2 * STAGES, B_ACC_EMPTY = 2 * STAGES + 2, B_DRAIN = 2 * STAGES + 4, NBAR = 2 * STAGES + 5 };

struct Params {
  int M, N, K;
  int kslabs, units, per;
  const bf16* r;
  bf16* y;
  float* ws;  // M x N fp32, zero between calls
  int* cnt;   // 4 counters per W tile, zero between calls
  int* err;
  int prefetch_w;
};

__device__ __forceinline__ void red_add(float* p, float v) { asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory"); }

template <int NTOK>
__device__ __forceinline__ void flush_stripe(const Params& p, int tile, int slabs, const uint32_t (&v)[NTOK], int lane, int q) {
  const int n = tile * BW + q * 32 + lane;
  const bool full = slabs == p.kslabs;
  if (full) {
    if (n < p.N)
#pragma unroll 4
      for (int t = 0; t < NTOK; ++t) {
        if (t >= p.M) break;
        float f = __uint_as_float(v[t]);
        if (p.r) f += __bfloat162float(p.r[(long)t * p.N + n]);
        p.y[(long)t * p.N + n] = __float2bfloat16_rn(f);
      }
    return;
  }
  if (n < p.N)
#pragma unroll 4
    for (int t = 0; t < NTOK; ++t) {
      if (t >= p.M) break;
      red_add(p.ws + (long)t * p.N + n, __uint_as_float(v[t]));
    }
  __threadfence();
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    int* c = p.cnt + tile * 4 + q;
    last = atomicAdd(c, slabs) + slabs == p.kslabs;
    if (last) *c = 0;  // every contributor has arrived: reset for the next call
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();
  if (n < p.N)
    for (int t0 = 0; t0 < p.M; t0 += 8) {  // eight independent loads in flight per thread, then the stores
      float f[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) f[u] = t0 + u < p.M ? __ldcg(p.ws + (long)(t0 + u) * p.N + n) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (t0 + u >= p.M) break;
        const long at = (long)(t0 + u) * p.N + n;
        p.ws[at] = 0.f;
        float v = f[u];
        if (p.r) v += __bfloat162float(p.r[at]);
        p.y[at] = __float2bfloat16_rn(v);
      }
    }
}

template <int NTOK>
__global__ void __launch_bounds__(THREADS, 1) stream_k(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, Params p) {
  constexpr int W_BYTES = BW * BK * 2, X_BYTES = NTOK * BK * 2, STAGE = W_BYTES + X_BYTES;
  constexpr uint32_t IDS = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NTOK >> 3) << 17) | ((uint32_t)(BW >> 4) << 24);
  extern __shared__ char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + STAGES * STAGE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBAR);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = blockIdx.x * p.per, u1 = min(p.units, u0 + p.per);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tg::mbar_init(&bar[B_FULL + s], 1);
      tg::mbar_init(&bar[B_EMPTY + s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tg::mbar_init(&bar[B_ACC_FULL + a], 1);
      tg::mbar_init(&bar[B_ACC_EMPTY + a], 4);
    }
    tg::mbar_init(&bar[B_DRAIN], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tg::s32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tg::fence_before();
  __syncthreads();
  tg::fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const int n_units = max(0, u1 - u0);
      int pre = 0;
      if (p.prefetch_w) {  // weight slabs do not depend on the preceding kernel
        pre = min(n_units, STAGES);
        for (int i = 0; i < pre; ++i) {
          const int u = u0 + i;
          tg::expect_tx(&bar[B_FULL + i], STAGE);
          tg::tma2d(sm + i * STAGE, &tw, (u % p.kslabs) * BK, (u / p.kslabs) * BW, &bar[B_FULL + i]);
        }
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int i = 0; i < pre; ++i) {
        const int u = u0 + i;
        tg::tma2d(sm + i * STAGE + W_BYTES, &tx, (u % p.kslabs) * BK, 0, &bar[B_FULL + i]);
      }
      int i = pre;
      for (; i < n_units; ++i) {
        const int s = i % STAGES, u = u0 + i;
        if (i >= STAGES && !tg::wait(&bar[B_EMPTY + s], ((i / STAGES) - 1) & 1, abort, p.err, 21)) break;
        tg::expect_tx(&bar[B_FULL + s], STAGE);
        tg::tma2d(sm + s * STAGE, &tw, (u % p.kslabs) * BK, (u / p.kslabs) * BW, &bar[B_FULL + s]);
        tg::tma2d(sm + s * STAGE + W_BYTES, &tx, (u % p.kslabs) * BK, 0, &bar[B_FULL + s]);
      }
      if (*abort) {
        int zero = 0;
        for (int k = max(0, i - STAGES); k < i; ++k) tg::wait(&bar[B_FULL + k % STAGES], (k / STAGES) & 1, (volatile int*)&zero, p.err, 21);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int i = 0, seg = 0;
      bool ok = true;
      while (ok && u0 + i < u1) {
        const int tile = (u0 + i) / p.kslabs, a = seg & 1;
        if (seg >= 2 && !tg::wait(&bar[B_ACC_EMPTY + a], ((seg >> 1) - 1) & 1, abort, p.err, 22)) break;
        tg::fence_after();
        int j = 0;
        for (; u0 + i < u1 && (u0 + i) / p.kslabs == tile; ++i, ++j) {
          const int s = i % STAGES;
          if (!tg::wait(&bar[B_FULL + s], (i / STAGES) & 1, abort, p.err, 23)) {
            ok = false;
            break;
          }
          tg::fence_after();
          const uint32_t sw = tg::s32(sm + s * STAGE), sx = sw + W_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) tg::mma(tmem + a * 64, tg::desc_k128(sw + kk * 32), tg::desc_k128(sx + kk * 32), IDS, (j | kk) ? 1u : 0u);
          tg::commit(&bar[B_EMPTY + s]);
        }
        if (!ok) break;
        tg::commit(&bar[B_ACC_FULL + a]);
        ++seg;
      }
      tg::commit(&bar[B_DRAIN]);
      int zero = 0;
      tg::wait(&bar[B_DRAIN], 0, (volatile int*)&zero, p.err, 24);
    }
  } else {
    const int q = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    int i = 0, seg = 0;
    while (u0 + i < u1) {
      const int tile = (u0 + i) / p.kslabs, a = seg & 1;
      int slabs = 0;
      while (u0 + i < u1 && (u0 + i) / p.kslabs == tile) ++i, ++slabs;
      if (!__all_sync(0xffffffffu, tg::wait(&bar[B_ACC_FULL + a], (seg >> 1) & 1, abort, p.err, 25))) break;
      tg::fence_after();
      uint32_t v[NTOK];
      {
        uint32_t t32[32];
        tg::tmem_ld32(lane_base + a * 64, t32);
#pragma unroll
        for (int e = 0; e < 32 && e < NTOK; ++e) v[e] = t32[e];
        if constexpr (NTOK == 64) {
          tg::tmem_ld32(lane_base + a * 64 + 32, t32);
#pragma unroll
          for (int e = 0; e < 32; ++e) v[32 + e] = t32[e];
        }
      }
      tg::fence_before();
      __syncwarp();
      if (lane == 0) tg::arrive(&bar[B_ACC_EMPTY + a]);  // the accumulator may be reused while this stripe is stored
      flush_stripe<NTOK>(p, tile, slabs, v, lane, q);
      ++seg;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tg::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}
}  // namespace sk

// ---------------------------------------------------------------------------------- weight streaming, cluster split-K
// Same product as stream_k (Y^T tile of 128 weight rows x NTOK tokens = W tile @ X^T on the tensor
// cores, M <= 128 token rows), on a fixed grid instead of persistent units: CTA (t, s) streams the
// K slabs [s * per, (s + 1) * per) of weight tile t, and the `splits` CTAs of a tile form one
// thread-block cluster.  The split-K partials are reduced over distributed shared memory, in a
// fixed order, so the result is deterministic and there is no workspace, counter or global atomic
// (a scattered fp32 reduction of M x N x splits values is what limits the persistent kernel at 32-64
// rows).  Two CTAs fit on an SM, and `splits` is the largest count (<= 8) whose grid is resident in
// one wave.
//
//   warp 0      TMA producer: W slab (128 x 64) + X slab (NTOK x 64) per stage; with `prefetch_w`
//               the first W slabs are requested before the preceding kernel has finished.
//   warp 1      TMEM owner and MMA issuer: four tcgen05.mma (M 128, N NTOK, K 16) per slab.
//   warps 2-5   epilogue: TMEM -> this CTA's fp32 partial in shared memory (token-major rows of
//               128 floats, over the drained stage ring); after a cluster barrier, cluster rank r
//               sums its 1/splits share of the tile's M x 128 outputs over every rank's partial
//               (ld.shared::cluster, ranks in order), adds R and stores bf16.
//   all         a second cluster barrier keeps every partial alive until its readers are done.
// Every mbarrier wait is bounded; every thread reaches both cluster barriers whatever happened.
namespace cs {
constexpr int BW = 128, BK = 64, THREADS = 192, MAX_SPLITS = 16;  // > 8: non-portable cluster sizes
// Input transform applied to each X slab in shared memory before its MMAs (warps 2-5):
//   X_PLAIN   none;
//   X_RMS     X = RMSNorm(H) with weight g: the slab becomes bf16(H * g) and the per-token sums of
//             squares are accumulated; the token's 1/rms scales its outputs after the cluster
//             reduction (the MMA is linear in each token row), so the normalised activation is never
//             written to memory;
//   X_SWIGLU  X = silu(G) * U from the fused gate/up activation [M, 2K] (gate columns [0, K), up
//             columns [K, 2K)); both slabs are loaded and the product replaces the gate slab.
enum XMode { X_PLAIN = 0, X_RMS = 1, X_SWIGLU = 2 };
template <int NTOK, int XM>
constexpr int stage_bytes() {
  return BW * BK * 2 + NTOK * BK * 2 * (XM == X_SWIGLU ? 2 : 1);
}
template <int NTOK, int XM>
constexpr int stages() {
  return (100 * 1024) / stage_bytes<NTOK, XM>() < 5 ? (100 * 1024) / stage_bytes<NTOK, XM>() : 5;
}
template <int NTOK, int XM>
constexpr int smem_bytes() {
  return stages<NTOK, XM>() * stage_bytes<NTOK, XM>() + (3 * stages<NTOK, XM>() + 1) * 8 + 16 + 5 * NTOK * 4 + 1024;
}

struct Params {
  int M, N, K, kslabs, per;
  const bf16* r;
  bf16* y;
  int* err;
  int prefetch_w;
  const bf16* g;  // X_RMS: norm weight [K]
  float eps;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_rank(uint32_t local_addr, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(local_addr), "r"(rank));
  return ra;
}
__device__ __forceinline__ float4 ld_cluster4(uint32_t local_addr, uint32_t rank) {
  const uint32_t ra = map_rank(local_addr, rank);
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(ra) : "memory");
  return v;
}
__device__ __forceinline__ float ld_cluster1(uint32_t local_addr, uint32_t rank) {
  const uint32_t ra = map_rank(local_addr, rank);
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}
__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }

template <int NTOK, int XM>
__global__ void __launch_bounds__(THREADS, 1) stream_cluster_k(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx,
                                                               Params p) {
  constexpr int S = stages<NTOK, XM>(), W_BYTES = BW * BK * 2, X_BYTES = NTOK * BK * 2, STAGE = stage_bytes<NTOK, XM>();
  constexpr uint32_t TCOLS = NTOK < 32 ? 32 : NTOK;
  constexpr uint32_t IDS = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NTOK >> 3) << 17) | ((uint32_t)(BW >> 4) << 24);
  static_assert(NTOK * BW * 4 <= S * STAGE, "the partial must fit over the stage ring");
  static_assert(S >= 2, "at least two stages");
  extern __shared__ char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + S * STAGE);
  uint64_t* empty = full + S;
  uint64_t* xready = full + 2 * S;
  uint64_t* acc_bar = full + 3 * S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 3 * S + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* ssq = reinterpret_cast<float*>(tmem_slot + 4);  // X_RMS: this CTA's per-token partial sums of squares
  float* ssq_w = ssq + NTOK;                             // X_RMS: the same per transform warp
  float* part = reinterpret_cast<float*>(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int k0 = blockIdx.y * p.per, n_slabs = max(0, min(p.kslabs, k0 + p.per) - k0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tg::mbar_init(&full[s], 1);
      tg::mbar_init(&empty[s], 1);
      tg::mbar_init(&xready[s], 1);
    }
    tg::mbar_init(acc_bar, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tg::s32(tmem_slot)), "r"(TCOLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tg::fence_before();
  __syncthreads();
  tg::fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();  // the successor may be scheduled once every CTA of this grid is resident

  auto load_x = [&](int i, int s) {
    char* dst = sm + s * STAGE + W_BYTES;
    tg::tma2d(dst, &tx, (k0 + i) * BK, 0, &full[s]);
    if constexpr (XM == X_SWIGLU) tg::tma2d(dst + X_BYTES, &tx, p.K + (k0 + i) * BK, 0, &full[s]);
  };

  if (warp == 0) {
    if (lane == 0) {
      int pre = 0;
      if (p.prefetch_w) {  // weight slabs do not depend on the preceding kernel
        pre = min(n_slabs, S);
        for (int i = 0; i < pre; ++i) {
          tg::expect_tx(&full[i], STAGE);
          tg::tma2d(sm + i * STAGE, &tw, (k0 + i) * BK, tile * BW, &full[i]);
        }
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) load_x(i, i);
      int i = pre;
      for (; i < n_slabs; ++i) {
        const int s = i % S;
        if (i >= S && !tg::wait(&empty[s], ((i / S) - 1) & 1, abort, p.err, 31)) break;
        tg::expect_tx(&full[s], STAGE);
        tg::tma2d(sm + s * STAGE, &tw, (k0 + i) * BK, tile * BW, &full[s]);
        load_x(i, s);
      }
      if (*abort) {  // let the copies in flight land before the ring is reused or released
        int zero = 0;
        for (int k = max(0, i - S); k < i; ++k) tg::wait(&full[k % S], (k / S) & 1, (volatile int*)&zero, p.err, 31);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < n_slabs; ++i) {
        const int s = i % S;
        if (!tg::wait(XM == X_PLAIN ? &full[s] : &xready[s], (i / S) & 1, abort, p.err, 32)) break;
        tg::fence_after();
        const uint32_t sw = tg::s32(sm + s * STAGE), sx = sw + W_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) tg::mma(tmem, tg::desc_k128(sw + kk * 32), tg::desc_k128(sx + kk * 32), IDS, (i | kk) ? 1u : 0u);
        tg::commit(&empty[s]);
      }
      tg::commit(acc_bar);  // arrives once every MMA issued above has completed
    }
  } else {
    const int tt = threadIdx.x - 64;  // 0..127
    const int q = warp & 3, wq = warp - 2;  // TMEM lane quarter; transform warp index 0..3
    constexpr int CPL = NTOK / 4;            // 16-byte chunks per lane of one slab
    if constexpr (XM != X_PLAIN) {
      // Warp wq transforms, in place, the slabs of the ring stages s with s % 4 == wq (up to four
      // slabs in flight hide each one's load / compute / store latency).  A stage always belongs to
      // the same warp, which waits on its barrier phase by phase: a parity wait issued before the
      // previous phase completed would return at once.  Lane l covers 16-byte chunk j = l % 8 of rows
      // l / 8 + 4m of the 128-byte-swizzled slab; that chunk holds logical columns
      // 8 * (j ^ (row % 8)) .. +7, and row % 8 is l / 8 + 4 (m % 2).  X_RMS: each warp adds its slabs'
      // per-token sums of squares into its own row of ssq_w, in slab order.
      const int j = lane & 7, rb = lane >> 3;
      const int c0a = (j ^ rb) * 8, c0b = (j ^ (rb + 4)) * 8;
      if constexpr (XM == X_RMS) {
        for (int t = lane; t < NTOK; t += 32) ssq_w[wq * NTOK + t] = 0.f;
        __syncwarp();
      }
      for (int i = 0; i < n_slabs; ++i) {
        const int s = i % S;
        if ((s & 3) != wq) continue;
        float ga[8], gb[8];
        if constexpr (XM == X_RMS) {  // the norm weights of this slab, requested before the wait
          load8(p.g + (long)(k0 + i) * BK + c0a, ga);
          load8(p.g + (long)(k0 + i) * BK + c0b, gb);
        }
        if (!tg::wait(&full[s], (i / S) & 1, abort, p.err, 34)) break;
        char* xs = sm + s * STAGE + W_BYTES;
#pragma unroll 2
        for (int m = 0; m < CPL; ++m) {
          const int off = (rb + 4 * m) * 128 + j * 16;
          float f[8], o[8];
          load8(reinterpret_cast<const bf16*>(xs + off), f);
          if constexpr (XM == X_RMS) {
            float v = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              v += f[e] * f[e];
              o[e] = f[e] * ((m & 1) ? gb[e] : ga[e]);
            }
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            if (j == 0) ssq_w[wq * NTOK + rb + 4 * m] += v;
          } else {
            float u[8];
            load8(reinterpret_cast<const bf16*>(xs + X_BYTES + off), u);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = silu_f(f[e]) * u[e];
          }
          store8(reinterpret_cast<bf16*>(xs + off), o);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) tg::arrive(&xready[s]);
      }
    }
    const int n = q * 32 + lane;
    const bool ok = __all_sync(0xffffffffu, tg::wait(acc_bar, 0, abort, p.err, 33)) && n_slabs > 0;
    tg::fence_after();
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll
    for (int c0 = 0; c0 < NTOK; c0 += 32) {
      uint32_t v[32];
      tg::tmem_ld32(lane_base + c0, v);
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (c0 + e < NTOK) part[(c0 + e) * BW + n] = ok ? __uint_as_float(v[e]) : 0.f;
    }
    tg::fence_before();
    if constexpr (XM == X_RMS) {  // per-token sums of the 4 warps, in order
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (tt < NTOK) ssq[tt] = ((ssq_w[tt] + ssq_w[NTOK + tt]) + ssq_w[2 * NTOK + tt]) + ssq_w[3 * NTOK + tt];
    }
  }
  __syncwarp();
  cluster_sync();  // every rank's partial is complete and visible

  pdl_wait();  // R may be written and Y read by earlier kernels
  {
    const uint32_t rank = cluster_rank(), ranks = cluster_size();
    const int groups = p.M * (BW / 4), share = (groups + (int)ranks - 1) / (int)ranks;
    const int g0 = (int)rank * share, g1 = min(groups, g0 + share);
    const uint32_t pbase = tg::s32(part), sbase = tg::s32(ssq);
    for (int g = g0 + threadIdx.x; g < g1; g += THREADS) {
      const int t = g / (BW / 4), c = (g % (BW / 4)) * 4, n = tile * BW + c;
      if (n >= p.N) continue;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      float ss = 0.f;
      for (uint32_t r = 0; r < ranks; ++r) {
        const float4 b = ld_cluster4(pbase + (uint32_t)((t * BW + c) * 4), r);
        a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
        if constexpr (XM == X_RMS) ss += ld_cluster1(sbase + (uint32_t)(t * 4), r);
      }
      if constexpr (XM == X_RMS) {
        const float rs = rsqrtf(ss / (float)p.K + p.eps);
        a.x *= rs, a.y *= rs, a.z *= rs, a.w *= rs;
      }
      const long at = (long)t * p.N + n;
      if (p.r) {
        const uint2 rr = *reinterpret_cast<const uint2*>(p.r + at);
        const float2 r0 = __bfloat1622float2(*reinterpret_cast<const bf162*>(&rr.x));
        const float2 r1 = __bfloat1622float2(*reinterpret_cast<const bf162*>(&rr.y));
        a.x += r0.x, a.y += r0.y, a.z += r1.x, a.w += r1.y;
      }
      bf162 o0 = __floats2bfloat162_rn(a.x, a.y), o1 = __floats2bfloat162_rn(a.z, a.w);
      uint2 ov;
      ov.x = *reinterpret_cast<uint32_t*>(&o0);
      ov.y = *reinterpret_cast<uint32_t*>(&o1);
      *reinterpret_cast<uint2*>(p.y + at) = ov;
    }
  }
  cluster_sync();  // no partial is released while another rank may still read it
  if (warp == 1) {
    tg::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
  }
}
}  // namespace cs

// ---------------------------------------------------------------------------------- host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                              CUtensorMapFloatOOBfill);

static EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    AX_REQUIRE(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess && ptr,
               "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}

// rows x cols bf16, K-major box {64, box_rows}, 128-byte swizzle; out-of-range rows read as zero
static CUtensorMap kmajor_map(const void* base, long rows, long cols, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AX_REQUIRE(r == CUDA_SUCCESS, "tensor map encode failed (", (int)r, ")");
  return m;
}

static int smem_bytes() { return STAGES * STAGE_BYTES + NBAR * 8 + 32 + 1024; }

// K x MN matrix stored row-major (MN contiguous), box 64 x 64, 128-byte swizzle; out-of-range rows
// and columns read as zero
static CUtensorMap mnmajor_map(const void* base, long k_rows, long mn_cols) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)mn_cols, (cuuint64_t)k_rows};
  cuuint64_t strides[1] = {(cuuint64_t)mn_cols * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AX_REQUIRE(r == CUDA_SUCCESS, "tensor map encode failed (", (int)r, ")");
  return m;
}

// A: K-major (M x K) or MN-major (K x M); B: K-major (N x K) or MN-major (K x N)
template <int MODE, bool A_MN = false, bool B_MN = false>
static void launch(const void* A, const void* B, Params p, cudaStream_t st) {
  AX_REQUIRE((A_MN || B_MN) ? true : p.K % 8 == 0, "tcgemm: K must be a multiple of 8, got ", p.K);
  AX_REQUIRE(p.N % 32 == 0, "tcgemm: N must be a multiple of 32, got ", p.N);
  AX_REQUIRE(!A_MN || p.M % 8 == 0, "tcgemm: M must be a multiple of 8 for an MN-major A");
  AX_REQUIRE(reinterpret_cast<uintptr_t>(A) % 16 == 0 && reinterpret_cast<uintptr_t>(B) % 16 == 0, "tcgemm: 16-byte aligned operands");
  if (p.M == 0 || p.N == 0 || p.K == 0) return;
  const CUtensorMap ta = A_MN ? mnmajor_map(A, p.K, p.M) : kmajor_map(A, p.M, p.K, BM);
  const CUtensorMap tb = B_MN ? mnmajor_map(B, p.K, p.N) : kmajor_map(B, p.N, p.K, BN);
  p.tiles_m = (p.M + BM - 1) / BM;
  p.tiles_n = (p.N + BN - 1) / BN;
  static bool attr[64] = {false};  // one flag set per instantiation
  int dev = 0;
  AX_CUDA_OK(cudaGetDevice(&dev));
  if (!attr[dev]) {
    AX_CUDA_OK(cudaFuncSetAttribute(gemm_k<MODE, A_MN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes()));
    attr[dev] = true;
  }
  const int grid = MODE == AGATHER ? num_sms() : std::min(p.tiles_m * p.tiles_n, num_sms());
  if (MODE == AGATHER) p.ag_target *= grid;  // every CTA copies a share of every chunk
  launch_pdl(gemm_k<MODE, A_MN, B_MN>, dim3(grid), dim3(threads_of(MODE)), (size_t)smem_bytes(), st, ta, tb, p);
}

template <int NTOK>
static void launch_stream(const void* X, const void* W, const void* R, void* Y, int M, int N, int K, float* ws, int* cnt, int* err,
                          bool prefetch_w, cudaStream_t st) {
  constexpr int STAGE = sk::BW * sk::BK * 2 + NTOK * sk::BK * 2;
  const int smem = sk::STAGES * STAGE + sk::NBAR * 8 + 16 + 1024;
  static bool attr[64] = {false};
  int dev = 0;
  AX_CUDA_OK(cudaGetDevice(&dev));
  if (!attr[dev]) {
    AX_CUDA_OK(cudaFuncSetAttribute(sk::stream_k<NTOK>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  const CUtensorMap tw = kmajor_map(W, N, K, sk::BW);
  const CUtensorMap tx = kmajor_map(X, M, K, NTOK);
  sk::Params p{};
  p.M = M, p.N = N, p.K = K, p.kslabs = K / sk::BK;
  p.units = ((N + sk::BW - 1) / sk::BW) * p.kslabs;
  const int grid = std::min(num_sms(), p.units);
  p.per = (p.units + grid - 1) / grid;
  p.r = static_cast<const bf16*>(R), p.y = static_cast<bf16*>(Y), p.ws = ws, p.cnt = cnt, p.err = err, p.prefetch_w = prefetch_w ? 1 : 0;
  launch_pdl(sk::stream_k<NTOK>, dim3((p.units + p.per - 1) / p.per), dim3(sk::THREADS), (size_t)smem, st, tw, tx, p);
}


// Clusters of s CTAs (1 <= s <= 16) of this kernel that can be resident at once on the current device.
template <int NTOK, int XM>
static int cluster_fit(int s) {
  static std::mutex mu;
  static int fit[64][cs::MAX_SPLITS + 1] = {};
  int dev = 0;
  AX_CUDA_OK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> g(mu);
  if (!fit[dev][s]) {
    const void* kern = reinterpret_cast<const void*>(cs::stream_cluster_k<NTOK, XM>);
    smem_attr(kern, cs::smem_bytes<NTOK, XM>());
    if (s > 8) AX_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1, attr[0].val.clusterDim.y = s, attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, s, 1);
    cfg.blockDim = dim3(cs::THREADS);
    cfg.dynamicSmemBytes = cs::smem_bytes<NTOK, XM>();
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    AX_CUDA_OK(cudaOccupancyMaxActiveClusters(&n, cs::stream_cluster_k<NTOK, XM>, &cfg));
    fit[dev][s] = std::max(n, 1);
  }
  return fit[dev][s];
}

// Split count forced by AXRL_CLUSTER_SPLITS (1..16), 0 when unset.
static int forced_cluster_splits() {
  static int v = [] {
    const char* e = std::getenv("AXRL_CLUSTER_SPLITS");
    const int n = e ? std::atoi(e) : 0;
    return (n >= 1 && n <= cs::MAX_SPLITS) ? n : 0;
  }();
  return v;
}

// Largest split count (<= 8, <= K slabs) for which the occupancy query (cluster_fit) reports every
// cluster of the (tiles x splits) grid resident at once; 1 when even single-CTA tiles need several
// waves (large matrices).  The query counts one CTA per SM for this cluster launch although two fit
// by shared memory, so the grids are small (2 splits for the 48-tile qkv matrix, 4 for the 32-tile o
// / down matrices).  Larger grids (4 / 8 splits) are faster in isolated chains of one projection
// (qkv 13.3 vs 15.2 us, down 20.0 vs 22.2 at 8 rows) but made the whole Qwen3-8B decode step slower
// (batch 8: 4.68 vs 4.30 ms), so the choice stays; AXRL_CLUSTER_SPLITS forces a count for tuning.
template <int NTOK, int XM>
static int cluster_splits(int n_tiles, int kslabs) {
  if (const int f = forced_cluster_splits()) {
    if (f > 8) cluster_fit<NTOK, XM>(f);  // sets the non-portable cluster size attribute
    return std::min(f, kslabs);
  }
  for (int s = std::min(8, kslabs); s >= 1; --s)
    if (n_tiles <= cluster_fit<NTOK, XM>(s)) return s;
  return 1;
}

template <int NTOK, int XM>
static void launch_stream_cluster(const void* X, const void* W, const void* R, void* Y, int M, int N, int K, int* err, bool prefetch_w,
                                  const void* g, float eps, cudaStream_t st) {
  const int smem = cs::smem_bytes<NTOK, XM>();
  smem_attr(reinterpret_cast<const void*>(cs::stream_cluster_k<NTOK, XM>), smem);
  const CUtensorMap tw = kmajor_map(W, N, K, cs::BW);
  const CUtensorMap tx = kmajor_map(X, M, XM == cs::X_SWIGLU ? 2L * K : (long)K, NTOK);
  cs::Params p{};
  p.M = M, p.N = N, p.K = K, p.kslabs = K / cs::BK;
  const int n_tiles = (N + cs::BW - 1) / cs::BW;
  int splits = cluster_splits<NTOK, XM>(n_tiles, p.kslabs);
  p.per = (p.kslabs + splits - 1) / splits;
  splits = (p.kslabs + p.per - 1) / p.per;  // every split covers at least one slab
  p.r = static_cast<const bf16*>(R), p.y = static_cast<bf16*>(Y), p.err = err, p.prefetch_w = prefetch_w ? 1 : 0;
  p.g = static_cast<const bf16*>(g), p.eps = eps;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1, attr[0].val.clusterDim.y = splits, attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_tiles, splits, 1);
  cfg.blockDim = dim3(cs::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  AX_CUDA_OK(cudaLaunchKernelEx(&cfg, cs::stream_cluster_k<NTOK, XM>, tw, tx, p));
}

template <int XM>
static void stream_cluster_rows(const void* X, const void* W, const void* R, void* Y, int M, int N, int K, int* err, bool prefetch_w,
                                const void* g, float eps, cudaStream_t st) {
  if (M <= 16) launch_stream_cluster<16, XM>(X, W, R, Y, M, N, K, err, prefetch_w, g, eps, st);
  else if (M <= 32) launch_stream_cluster<32, XM>(X, W, R, Y, M, N, K, err, prefetch_w, g, eps, st);
  else if (M <= 64) launch_stream_cluster<64, XM>(X, W, R, Y, M, N, K, err, prefetch_w, g, eps, st);
  else launch_stream_cluster<128, XM>(X, W, R, Y, M, N, K, err, prefetch_w, g, eps, st);
}

}  // namespace tg

// Decode-size GEMM (M <= 64 rows) streaming the weights on the tensor cores.  ws: M x N fp32 and
// cnt: 4 * ceil(N / 128) ints, both zero and left zero; calls sharing them must be stream-ordered.
void tcgemm_stream(const void* X, const void* W, const void* R, void* Y, int M, int N, int K, float* ws, int* cnt, int* err, bool prefetch_w,
                   cudaStream_t st) {
  AX_REQUIRE(M >= 1 && M <= 64, "tcgemm_stream: 1..64 rows, got ", M);
  AX_REQUIRE(K % 64 == 0 && N % 8 == 0, "tcgemm_stream: K multiple of 64, N multiple of 8");
  if (M <= 32) tg::launch_stream<32>(X, W, R, Y, M, N, K, ws, cnt, err, prefetch_w, st);
  else tg::launch_stream<64>(X, W, R, Y, M, N, K, ws, cnt, err, prefetch_w, st);
}

// Resident clusters of 1..16 CTAs of the streaming kernel for `ntok` token rows (plain input).
std::vector<int64_t> tcgemm_stream_cluster_fit(int ntok) {
  std::vector<int64_t> out;
  for (int s = 1; s <= tg::cs::MAX_SPLITS; ++s)
    out.push_back(ntok <= 16   ? tg::cluster_fit<16, 0>(s)
                  : ntok <= 32 ? tg::cluster_fit<32, 0>(s)
                  : ntok <= 64 ? tg::cluster_fit<64, 0>(s)
                               : tg::cluster_fit<128, 0>(s));
  return out;
}

// Decode-size GEMM (M <= 128 rows) streaming the weights on the tensor cores, split-K partials
// reduced inside a thread-block cluster (deterministic; no workspace).  xmode 0: Y = X @ W^T (+ R);
// 1: Y = RMSNorm(X; g, eps) @ W^T (+ R); 2: Y = (silu(X[:, :K]) * X[:, K:]) @ W^T (+ R) with X of
// width 2K.  Y and R: 8-byte aligned.
void tcgemm_stream_cluster(const void* X, const void* W, const void* R, void* Y, int M, int N, int K, int* err, bool prefetch_w,
                           cudaStream_t st, int xmode, const void* g, float eps) {
  AX_REQUIRE(M >= 1 && M <= 128, "tcgemm_stream_cluster: 1..128 rows, got ", M);
  AX_REQUIRE(K % 64 == 0 && N % 8 == 0, "tcgemm_stream_cluster: K multiple of 64, N multiple of 8");
  AX_REQUIRE(reinterpret_cast<uintptr_t>(X) % 16 == 0 && reinterpret_cast<uintptr_t>(W) % 16 == 0 && reinterpret_cast<uintptr_t>(Y) % 8 == 0 &&
                 reinterpret_cast<uintptr_t>(R) % 8 == 0 && reinterpret_cast<uintptr_t>(g) % 16 == 0,
             "tcgemm_stream_cluster: operand alignment");
  AX_REQUIRE(xmode >= 0 && xmode <= 2 && (xmode != 1 || g != nullptr), "tcgemm_stream_cluster: input transform");
  if (xmode == 1) tg::stream_cluster_rows<tg::cs::X_RMS>(X, W, R, Y, M, N, K, err, prefetch_w, g, eps, st);
  else if (xmode == 2) tg::stream_cluster_rows<tg::cs::X_SWIGLU>(X, W, R, Y, M, N, K, err, prefetch_w, g, eps, st);
  else tg::stream_cluster_rows<tg::cs::X_PLAIN>(X, W, R, Y, M, N, K, err, prefetch_w, g, eps, st);
}

// D[M,N] (+)= A[M,K] @ B[N,K]^T (+ C), bf16; err: device int that records a wait timeout.
void tcgemm_tn(const void* A, const void* B, const void* C, void* D, int M, int N, int K, int* err, cudaStream_t st) {
  tg::Params p{};
  p.M = M, p.N = N, p.K = K, p.d = static_cast<bf16*>(D), p.c = static_cast<const bf16*>(C), p.rows_per_rank = 1, p.err = err;
  tg::launch<tg::LOCAL>(A, B, p, st);
}

// Data gradient: dX[M, Ko] = dY[M, Nr] @ W[Nr, Ko] (W read MN-major), bf16.
void tcgemm_nn(const void* dY, const void* W, void* dX, int M, int Ko, int Nr, int* err, cudaStream_t st) {
  tg::Params p{};
  p.M = M, p.N = Ko, p.K = Nr, p.d = static_cast<bf16*>(dX), p.rows_per_rank = 1, p.err = err;
  tg::launch<tg::LOCAL, false, true>(dY, W, p, st);
}

// Weight gradient in bf16: G[Nw, Kw] = dY[T, Nw]^T @ X[T, Kw] (both read MN-major).
void tcgemm_wgrad_bf16(const void* dY, const void* X, void* G, int Nw, int Kw, int T, int* err, cudaStream_t st) {
  tg::Params p{};
  p.M = Nw, p.N = Kw, p.K = T, p.d = static_cast<bf16*>(G), p.rows_per_rank = 1, p.err = err;
  tg::launch<tg::LOCAL, true, true>(dY, X, p, st);
}

// Weight gradient: G[Nw, Kw] (fp32) (+)= dY[T, Nw]^T @ X[T, Kw] (both read MN-major).
void tcgemm_wgrad(const void* dY, const void* X, float* G, int Nw, int Kw, int T, bool accumulate, int* err, cudaStream_t st) {
  tg::Params p{};
  p.M = Nw, p.N = Kw, p.K = T, p.d32 = G, p.accumulate = accumulate ? 1 : 0, p.rows_per_rank = 1, p.err = err;
  tg::launch<tg::F32ACC, true, true>(dY, X, p, st);
}

// Row-parallel GEMM whose output rows are reduce-scattered: row r of A @ B^T goes to rank
// r / rows_per_rank's receive buffer (peers[owner], device pointers), slot `rank`; channel `ch`
// of the TP flag arrays carries the free / data handshakes of epoch `epoch`.
void tcgemm_tn_to_slots(const void* A, const void* B, const int64_t* peers, int rank, int world, int rows_per_rank, int M, int N, int K,
                        const int64_t* flag_peers, const int* my_flags, int ch, int epoch, unsigned* ticket, uint64_t timeout_ns,
                        int* status, int* err, cudaStream_t st) {
  AX_REQUIRE(world >= 1 && world <= tg::kMaxTP && rank < world && ch >= 0 && ch < tg::kFreeBase, "tcgemm slots: TP layout");
  tg::Params p{};
  p.M = M, p.N = N, p.K = K, p.peers = peers, p.rank = rank, p.rows_per_rank = rows_per_rank, p.err = err;
  p.flag_peers = flag_peers, p.my_flags = my_flags, p.ch = ch, p.epoch = epoch, p.world = world, p.ticket = ticket;
  p.timeout_ns = timeout_ns, p.status = status;
  tg::launch<tg::SLOTS>(A, B, p, st);
}

// All-gather -> GEMM: D[world * rows_per_rank, N] = gather(A) @ B^T, where this rank's rows are already
// at rows [rank * rows_per_rank, ...) of its gather buffer src_peers[rank] (the A operand) and the
// other ranks' rows are pulled from src_peers[s] by the kernel.  ag_cnt: world zeroed ints, kept
// across calls (call index `call` >= 1, consecutive); channel `ch` of the TP flags carries the
// data / free handshakes of epoch `epoch`.
void tcgemm_ag(const int64_t* src_peers, const void* B, void* D, int rank, int world, int rows_per_rank, int N, int K,
               const int64_t* flag_peers, const int* my_flags, int ch, int epoch, int* ag_cnt, int call, uint64_t timeout_ns, int* status,
               int* err, const void* A_local_buffer, cudaStream_t st) {
  AX_REQUIRE(world >= 1 && world <= tg::kMaxTP && rank < world && ch >= 0 && ch < tg::kFreeBase, "tcgemm ag: TP layout");
  AX_REQUIRE(rows_per_rank % tg::BM == 0 && K % 8 == 0, "tcgemm ag: rows per rank a multiple of 128, K a multiple of 8");
  AX_REQUIRE(((long)K * 2) % 16 == 0 && world <= 32, "tcgemm ag: 16-byte rows");
  tg::Params p{};
  p.M = world * rows_per_rank, p.N = N, p.K = K, p.d = static_cast<bf16*>(D), p.rank = rank, p.rows_per_rank = rows_per_rank;
  p.err = err, p.flag_peers = flag_peers, p.my_flags = my_flags, p.ch = ch, p.epoch = epoch, p.world = world;
  p.timeout_ns = timeout_ns, p.status = status, p.src_peers = src_peers, p.ag_cnt = ag_cnt, p.ag_target = call;
  tg::launch<tg::AGATHER>(A_local_buffer, B, p, st);
}

}  // namespace ax
