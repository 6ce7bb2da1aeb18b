// Range-list flash attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
// Reference counterpart: MagiAttention's calc_attn called from the packed forward
// (axrl/utils/megatron/magi_forward.py:439-466).
//
// Same problem and outputs as attn_fwd_k in attention.cu (packed tokens, (q-range, k-range, type)
// triples, head_dim 128, GQA; O bf16 and the base-2 log-sum-exp of the scaled scores), computed
// with one CTA per (128-row q tile, q head):
//
//   warp 4      TMA producer: the Q tile once, then K/V tiles of 128 keys into a 2-stage ring
//               (cp.async.bulk.tensor, 128-byte swizzle, no multicast).
//   warp 5      MMA issuer (one thread) and TMEM owner: S_j = Q K_j^T into one of two S buffers
//               in TMEM (128 x 128 fp32 each), then O += P_{j-1} V_{j-1} into the O accumulator
//               (TMEM, 128 x 128 fp32), so the QK product of a tile overlaps the softmax of the
//               previous one.  A = Q / P and B = K are K-major, B = V is MN-major (V tiles are
//               used as loaded, no transpose).
//   warps 0-3   softmax, one query row per thread (TMEM lane = row): read S with tcgen05.ld,
//               mask (range ends, causal diagonal), online softmax in base 2, write P (bf16) to
//               shared memory in the UMMA K-major layout; the epilogue reads O back, divides by
//               the row sum and stores O and the log-sum-exp.
//
// The running maximum used for the exponentials is only raised when a tile's maximum exceeds it
// by more than 8 (log2 units): P then stays below 2^8, and O in TMEM is rescaled only on those
// rare steps instead of after every tile.  The result is exact (the final division uses the same
// maximum as the exponentials).
//
// Every mbarrier wait is bounded; on expiry the CTA records an error code, drains its own copies
// and tensor-core work, frees its TMEM and exits.
#include <cuda.h>

#include "common.cuh"
#include "tcgen05.cuh"

namespace ax {
namespace atc {

using namespace tc;

constexpr int D = 128;
constexpr int BM = 128;
constexpr int BN = 128;
constexpr int THREADS = 192;
constexpr int TILE = BN * D * 2;   // 32 KB: one 128 x 128 bf16 tile (two 64-column boxes of 16 KB)
constexpr int HALF = TILE / 2;
constexpr uint32_t TMEM_COLS = 512;  // S0 [0,128), S1 [128,256), O [256,384)
constexpr float RESCALE_THRESHOLD = 8.f;

// barrier slots
constexpr int B_Q = 0, B_KV_FULL = 1, B_KV_EMPTY = 3, B_S_FULL = 5, B_S_FREE = 7, B_P_FULL = 9, B_O_DONE = 10, B_DRAIN = 11,
              B_P_FREE = 12, NBAR = 14;

struct Params {
  bf16* o;
  float* lse2;
  const int* qseg;
  const int* kr;
  const int* tiles;
  int Hq, Hkv, T;
  float scale_log2;
  int* err;
};

// Key tiles of a q tile: every k-range of the q segment, BN keys at a time from the range start,
// up to the range end (for causal ranges, the last key any row of the tile may see).
struct KeyTiles {
  const int* kr;
  int r, r_last, q0, qe, ka, k0, rend, ty;
  __device__ void load_range() {
    while (r < r_last) {
      k0 = kr[r * 3];
      const int k1 = kr[r * 3 + 1];
      ty = kr[r * 3 + 2];
      rend = ty == 1 ? min(k1, k0 + (qe - q0)) : k1;
      if (rend > k0) {
        ka = k0;
        return;
      }
      ++r;
    }
  }
  __device__ bool valid() const { return r < r_last; }
  __device__ void next() {
    ka += BN;
    if (ka >= rend) {
      ++r;
      load_range();
    }
  }
};

// DOUBLE_P: two P buffers, so the softmax of tile j does not wait for PV_{j-1} (only for PV_{j-2},
// whose buffer it reuses, and for PV_{j-1} on the rare O rescale).
template <bool DOUBLE_P>
__global__ void __launch_bounds__(THREADS, 1) attn_fwd_tc_k(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                                                          const __grid_constant__ CUtensorMap tv, Params p) {
  constexpr int NP = DOUBLE_P ? 2 : 1;
  extern __shared__ char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  char* sQ = sm;
  char* sK = sm + TILE;          // 2 stages
  char* sV = sm + 3 * TILE;      // 2 stages
  char* sP = sm + 5 * TILE;  // NP buffers
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + (5 + NP) * TILE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBAR);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = p.tiles[blockIdx.y * 2], qs = p.tiles[blockIdx.y * 2 + 1];
  const int h = blockIdx.x, hk = h / (p.Hq / p.Hkv);
  const int q0 = p.qseg[seg * 4], q1 = p.qseg[seg * 4 + 1], r_first = p.qseg[seg * 4 + 2], r_last = p.qseg[seg * 4 + 3];
  const int qe = min(qs + BM, q1);

  if (tid == 0) {
    mbar_init(&bar[B_Q], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar[B_KV_FULL + s], 1);
      mbar_init(&bar[B_KV_EMPTY + s], 1);
      mbar_init(&bar[B_S_FULL + s], 1);
      mbar_init(&bar[B_S_FREE + s], 4);
    }
    mbar_init(&bar[B_P_FULL], 4);
    mbar_init(&bar[B_O_DONE], 1);
    mbar_init(&bar[B_P_FREE], 1);
    mbar_init(&bar[B_P_FREE + 1], 1);
    mbar_init(&bar[B_DRAIN], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tq)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tv)) : "memory");
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  KeyTiles kt{p.kr, r_first, r_last, q0, qe, 0, 0, 0, 0};
  kt.load_range();

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_expect_tx(&bar[B_Q], TILE);
      tma_2d(sQ, &tq, h * D, qs, &bar[B_Q]);
      tma_2d(sQ + HALF, &tq, h * D + 64, qs, &bar[B_Q]);
      int j = 0;
      for (; kt.valid(); kt.next(), ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&bar[B_KV_EMPTY + s], ((j - 2) >> 1) & 1, abort, p.err, 1)) break;
        mbar_expect_tx(&bar[B_KV_FULL + s], 2 * TILE);
        tma_2d(sK + s * TILE, &tk, hk * D, kt.ka, &bar[B_KV_FULL + s]);
        tma_2d(sK + s * TILE + HALF, &tk, hk * D + 64, kt.ka, &bar[B_KV_FULL + s]);
        tma_2d(sV + s * TILE, &tv, hk * D, kt.ka, &bar[B_KV_FULL + s]);
        tma_2d(sV + s * TILE + HALF, &tv, hk * D + 64, kt.ka, &bar[B_KV_FULL + s]);
      }
      if (*abort) {  // let every copy this CTA started land before its shared memory is released
        int zero = 0;
        mbar_wait(&bar[B_Q], 0, (volatile int*)&zero, p.err, 1);
        for (int i = max(0, j - 2); i < j; ++i) mbar_wait(&bar[B_KV_FULL + (i & 1)], (i >> 1) & 1, (volatile int*)&zero, p.err, 1);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_QK = idesc_bf16(BN, false), ID_PV = idesc_bf16(D, true);
      const uint32_t q_base = s32(sQ), k_base = s32(sK), v_base = s32(sV), p_base = s32(sP);
      bool ok = mbar_wait(&bar[B_Q], 0, abort, p.err, 2);
      tc_fence_after();
      int j = 0;
      auto pv = [&](int t) {  // O += P_t V_t
        if (!mbar_wait(&bar[B_P_FULL], t & 1, abort, p.err, 4)) return false;
        tc_fence_after();
        const uint32_t vb = v_base + (t & 1) * TILE;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t a = sdesc(p_base + (DOUBLE_P ? (t & 1) * TILE : 0) + (kk >> 2) * HALF + (kk & 3) * 32, 16, 1024);
          const uint64_t b = sdesc(vb + kk * 2048, HALF, 1024);
          tc_mma(tmem + 256, a, b, ID_PV, (t > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&bar[B_O_DONE]);
        tc_commit(&bar[B_KV_EMPTY + (t & 1)]);
        if constexpr (DOUBLE_P) tc_commit(&bar[B_P_FREE + (t & 1)]);
        return true;
      };
      for (; ok && kt.valid(); kt.next(), ++j) {
        const int b = j & 1;
        if (!mbar_wait(&bar[B_KV_FULL + b], (j >> 1) & 1, abort, p.err, 3)) break;
        if (j >= 2 && !mbar_wait(&bar[B_S_FREE + b], ((j - 2) >> 1) & 1, abort, p.err, 3)) break;
        tc_fence_after();
        const uint32_t kb = k_base + b * TILE;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
          tc_mma(tmem + b * BN, sdesc(q_base + off, 16, 1024), sdesc(kb + off, 16, 1024), ID_QK, kk > 0 ? 1u : 0u);
        }
        tc_commit(&bar[B_S_FULL + b]);
        if (j >= 1 && !pv(j - 1)) break;
      }
      if (!*abort && j >= 1) pv(j - 1);
      // nothing this thread issued may still run when TMEM is freed
      tc_commit(&bar[B_DRAIN]);
      int zero = 0;
      mbar_wait(&bar[B_DRAIN], 0, (volatile int*)&zero, p.err, 5);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (warps 0-3)
    const int row = qs + tid;  // this thread's query row (TMEM lane tid)
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
    float m_used = -INFINITY, l = 0.f;
    int j = 0;
    char* prow0 = sP + (tid >> 3) * 1024 + (tid & 7) * 128;  // row tid of the first 64-key block
    for (; kt.valid(); kt.next(), ++j) {
      const int b = j & 1;
      // tcgen05.ld / st are warp-collective (.sync.aligned): every decision in front of one is
      // made warp-uniform, so no lane can leave the loop or skip a TMEM access alone
      if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_S_FULL + b], (j >> 1) & 1, abort, p.err, 6))) break;
      tc_fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        float t[32];
        tmem_ld32(lane_addr + b * BN + c * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = t[i];
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_S_FREE + b]);
      // mask + scale (log2 units)
      const int kend = min(kt.ka + BN, kt.rend);
      const int climit = row < qe ? (kt.ty == 1 ? min(kend - kt.ka, row - q0 + kt.k0 - kt.ka + 1) : kend - kt.ka) : 0;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        s[c] = c < climit ? s[c] * p.scale_log2 : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      if constexpr (DOUBLE_P) {
        // P buffer j&1 is free once PV_{j-2} finished (which also bounds how far O_DONE can lag,
        // so its parity below is unambiguous)
        if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait(&bar[B_P_FREE + (j & 1)], ((j - 2) >> 1) & 1, abort, p.err, 7))) break;
      } else {
        // P_j may only overwrite P_{j-1} (and O may only be rescaled) once PV_{j-1} has finished
        if (j >= 1 && !__all_sync(0xffffffffu, mbar_wait(&bar[B_O_DONE], (j - 1) & 1, abort, p.err, 7))) break;
        tc_fence_after();
      }
      const float m_new = fmaxf(m_used, mt);
      const bool raise = m_new > m_used + RESCALE_THRESHOLD;
      const bool rescale = raise && j >= 1 && m_used != -INFINITY;  // O holds earlier tiles' sum: scale it down
      if (__any_sync(0xffffffffu, rescale)) {  // the whole warp touches its O rows; others scale by 1
        if constexpr (DOUBLE_P) {  // O may only be rescaled once PV_{j-1} has finished (rare)
          if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_O_DONE], (j - 1) & 1, abort, p.err, 9))) break;
          tc_fence_after();
        }
        const float alpha = rescale ? exp2f(m_used - m_new) : 1.f;
        l *= alpha;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(lane_addr + 256 + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(lane_addr + 256 + c * 32, o);
        }
        tmem_st_wait();
      }
      if (raise) m_used = m_new;
      // P = exp2(s - m), bf16, K-major 128-byte-swizzled rows
      float rs = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < BN / 8; ++c8) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float a = m_used == -INFINITY ? 0.f : exp2f(s[c8 * 8 + 2 * i] - m_used);
          const float bb = m_used == -INFINITY ? 0.f : exp2f(s[c8 * 8 + 2 * i + 1] - m_used);
          rs += a + bb;
          bf162 v2 = __floats2bfloat162_rn(a, bb);
          w[i] = *reinterpret_cast<uint32_t*>(&v2);
        }
        char* dst = prow0 + (DOUBLE_P ? (j & 1) * TILE : 0) + (c8 >> 3) * HALF + (((c8 & 7) ^ (tid & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l += rs;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P visible to the tensor cores
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_P_FULL]);
    }
    // epilogue: wait for the last PV, normalise, store
    const int n = j;
    bool ok = __all_sync(0xffffffffu, !*abort);
    if (ok && n >= 1) {
      if constexpr (DOUBLE_P)  // PV_{n-1} done (PV products complete in issue order), on its P buffer's barrier
        ok = __all_sync(0xffffffffu, mbar_wait(&bar[B_P_FREE + ((n - 1) & 1)], ((n - 1) >> 1) & 1, abort, p.err, 8));
      else
        ok = __all_sync(0xffffffffu, mbar_wait(&bar[B_O_DONE], (n - 1) & 1, abort, p.err, 8));
    }
    if (ok && n >= 1) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = p.o + ((long)row * p.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        tmem_ld32(lane_addr + 256 + c * 32, o);
        tmem_ld_wait();
        if (row < qe) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = o[i + e] * inv;
            store8(orow + c * 32 + i, f);
          }
        }
      }
      if (row < qe) p.lse2[(long)h * p.T + row] = l > 0.f ? m_used + log2f(l) : INFINITY;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------------------------- 8-warp softmax
// Same pipeline with the softmax of every query row split over two warps (warps w and w + 4 own
// TMEM lanes 32 (w % 4) .. +31; warp w < 4 takes key columns 0-63 of each tile, warp w + 4 columns
// 64-127).  The two threads of a row exchange their partial maxima through shared memory once per
// tile (a per-pair mbarrier with bounded waits; the exchange buffer alternates with the tile
// parity), so both raise the running maximum identically, and they add their partial row sums
// once at the end.  P is exponentiated in fp32 (ex2.approx.ftz.f32) and rounded to bf16 pairs for
// the PV product, with the row sum taken in fp32; exponentiating bf16x2 pairs instead
// (ex2.approx.ftz.bf16x2, half the special-function work) rounds the exponent's input to bf16 and
// moved the log-sum-exp by up to 6e-3 (log2 units) against fp32, so it is not used.
//
// TMEM_P: P goes to tensor memory instead of shared memory (two buffers, TMEM columns [384, 448)
// and [448, 512), written with tcgen05.st) and the PV product takes its A operand from there.
// The softmax of tile j + 1 then no longer waits for PV(j): P buffer j % 2 is reused by tile j + 2,
// and S(j + 2) completes only after every earlier MMA, PV(j) included, has.  Only the rare O
// rescale waits for PV(j).
constexpr int THREADS8 = 320;  // warps 0-7 softmax, 8 TMA producer, 9 MMA issuer
constexpr int B8_Q = 0, B8_KV_FULL = 1, B8_KV_EMPTY = 3, B8_S_FULL = 5, B8_S_FREE = 7, B8_P_FULL = 9, B8_O_DONE = 10, B8_DRAIN = 11,
              B8_XCH = 12, NBAR8 = 16;

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool TMEM_P>
__global__ void __launch_bounds__(THREADS8, 1) attn_fwd_tc8_k(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                                                            const __grid_constant__ CUtensorMap tv, Params p) {
  extern __shared__ char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  char* sQ = sm;
  char* sK = sm + TILE;      // 2 stages
  char* sV = sm + 3 * TILE;  // 2 stages
  char* sP = sm + 5 * TILE;
  float* xmax = reinterpret_cast<float*>(sm + 6 * TILE);  // [tile parity][half][row]
  float* xsum = xmax + 2 * 2 * BM;                         // [half][row]
  uint64_t* bar = reinterpret_cast<uint64_t*>(xsum + 2 * BM);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBAR8);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = p.tiles[blockIdx.y * 2], qs = p.tiles[blockIdx.y * 2 + 1];
  const int h = blockIdx.x, hk = h / (p.Hq / p.Hkv);
  const int q0 = p.qseg[seg * 4], q1 = p.qseg[seg * 4 + 1], r_first = p.qseg[seg * 4 + 2], r_last = p.qseg[seg * 4 + 3];
  const int qe = min(qs + BM, q1);

  if (tid == 0) {
    mbar_init(&bar[B8_Q], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar[B8_KV_FULL + s], 1);
      mbar_init(&bar[B8_KV_EMPTY + s], 1);
      mbar_init(&bar[B8_S_FULL + s], 1);
      mbar_init(&bar[B8_S_FREE + s], 8);
    }
    mbar_init(&bar[B8_P_FULL], 8);
    mbar_init(&bar[B8_O_DONE], 1);
    mbar_init(&bar[B8_DRAIN], 1);
    for (int w = 0; w < 4; ++w) mbar_init(&bar[B8_XCH + w], 64);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tq)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tv)) : "memory");
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  KeyTiles kt{p.kr, r_first, r_last, q0, qe, 0, 0, 0, 0};
  kt.load_range();

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_expect_tx(&bar[B8_Q], TILE);
      tma_2d(sQ, &tq, h * D, qs, &bar[B8_Q]);
      tma_2d(sQ + HALF, &tq, h * D + 64, qs, &bar[B8_Q]);
      int j = 0;
      for (; kt.valid(); kt.next(), ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&bar[B8_KV_EMPTY + s], ((j - 2) >> 1) & 1, abort, p.err, 1)) break;
        mbar_expect_tx(&bar[B8_KV_FULL + s], 2 * TILE);
        tma_2d(sK + s * TILE, &tk, hk * D, kt.ka, &bar[B8_KV_FULL + s]);
        tma_2d(sK + s * TILE + HALF, &tk, hk * D + 64, kt.ka, &bar[B8_KV_FULL + s]);
        tma_2d(sV + s * TILE, &tv, hk * D, kt.ka, &bar[B8_KV_FULL + s]);
        tma_2d(sV + s * TILE + HALF, &tv, hk * D + 64, kt.ka, &bar[B8_KV_FULL + s]);
      }
      if (*abort) {  // let every copy this CTA started land before its shared memory is released
        int zero = 0;
        mbar_wait(&bar[B8_Q], 0, (volatile int*)&zero, p.err, 1);
        for (int i = max(0, j - 2); i < j; ++i) mbar_wait(&bar[B8_KV_FULL + (i & 1)], (i >> 1) & 1, (volatile int*)&zero, p.err, 1);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_QK = idesc_bf16(BN, false), ID_PV = idesc_bf16(D, true);
      const uint32_t q_base = s32(sQ), k_base = s32(sK), v_base = s32(sV), p_base = s32(sP);
      bool ok = mbar_wait(&bar[B8_Q], 0, abort, p.err, 2);
      tc_fence_after();
      int j = 0;
      auto pv = [&](int t) {  // O += P_t V_t
        if (!mbar_wait(&bar[B8_P_FULL], t & 1, abort, p.err, 4)) return false;
        tc_fence_after();
        const uint32_t vb = v_base + (t & 1) * TILE;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t b = sdesc(vb + kk * 2048, HALF, 1024);
          if constexpr (TMEM_P) {
            tc_mma_ts(tmem + 256, tmem + 384 + (t & 1) * 64 + kk * 8, b, ID_PV, (t > 0 || kk > 0) ? 1u : 0u);
          } else {
            const uint64_t a = sdesc(p_base + (kk >> 2) * HALF + (kk & 3) * 32, 16, 1024);
            tc_mma(tmem + 256, a, b, ID_PV, (t > 0 || kk > 0) ? 1u : 0u);
          }
        }
        tc_commit(&bar[B8_O_DONE]);
        tc_commit(&bar[B8_KV_EMPTY + (t & 1)]);
        return true;
      };
      for (; ok && kt.valid(); kt.next(), ++j) {
        const int b = j & 1;
        if (!mbar_wait(&bar[B8_KV_FULL + b], (j >> 1) & 1, abort, p.err, 3)) break;
        if (j >= 2 && !mbar_wait(&bar[B8_S_FREE + b], ((j - 2) >> 1) & 1, abort, p.err, 3)) break;
        tc_fence_after();
        const uint32_t kb = k_base + b * TILE;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
          tc_mma(tmem + b * BN, sdesc(q_base + off, 16, 1024), sdesc(kb + off, 16, 1024), ID_QK, kk > 0 ? 1u : 0u);
        }
        tc_commit(&bar[B8_S_FULL + b]);
        if (j >= 1 && !pv(j - 1)) break;
      }
      if (!*abort && j >= 1) pv(j - 1);
      tc_commit(&bar[B8_DRAIN]);
      int zero = 0;
      mbar_wait(&bar[B8_DRAIN], 0, (volatile int*)&zero, p.err, 5);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (warps 0-7)
    const int wq = warp & 3, half = warp >> 2;
    const int r = wq * 32 + lane;  // row within the tile == TMEM lane
    const int row = qs + r;
    const int col0 = half * (BN / 2);
    const uint32_t lane_addr = tmem + ((uint32_t)(wq * 32) << 16);
    uint64_t* xbar = &bar[B8_XCH + wq];
    float m_used = -INFINITY, l = 0.f;
    int j = 0;
    char* prow = sP + half * HALF + (r >> 3) * 1024 + (r & 7) * 128;  // this row in this half's 64-key box
    for (; kt.valid(); kt.next(), ++j) {
      const int b = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&bar[B8_S_FULL + b], (j >> 1) & 1, abort, p.err, 6))) break;
      tc_fence_after();
      float s[BN / 2];
      {
        float t[32];
        tmem_ld32(lane_addr + b * BN + col0, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[i] = t[i];
        tmem_ld32(lane_addr + b * BN + col0 + 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[32 + i] = t[i];
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B8_S_FREE + b]);
      const int kend = min(kt.ka + BN, kt.rend);
      const int climit = row < qe ? (kt.ty == 1 ? min(kend - kt.ka, row - q0 + kt.k0 - kt.ka + 1) : kend - kt.ka) : 0;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN / 2; ++c) {
        s[c] = col0 + c < climit ? s[c] * p.scale_log2 : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      // exchange the partial maximum with the row's other half
      xmax[((j & 1) * 2 + half) * BM + r] = mt;
      mbar_arrive(xbar);
      if (!__all_sync(0xffffffffu, mbar_wait(xbar, j & 1, abort, p.err, 10))) break;
      mt = fmaxf(mt, xmax[((j & 1) * 2 + (half ^ 1)) * BM + r]);
      if constexpr (!TMEM_P) {
        // P_j overwrites P_{j-1} (and O may be rescaled) only once PV_{j-1} has finished
        if (j >= 1 && !__all_sync(0xffffffffu, mbar_wait(&bar[B8_O_DONE], (j - 1) & 1, abort, p.err, 7))) break;
        tc_fence_after();
      }
      const float m_new = fmaxf(m_used, mt);
      const bool raise = m_new > m_used + RESCALE_THRESHOLD;
      const bool rescale = raise && j >= 1 && m_used != -INFINITY;
      if (__any_sync(0xffffffffu, rescale)) {  // both halves of these rows decide alike
        if constexpr (TMEM_P) {  // O may only be rescaled once PV_{j-1} has finished (its phase is the
                                 // latest O_DONE can have reached: PV_j needs this tile's P)
          if (!__all_sync(0xffffffffu, mbar_wait(&bar[B8_O_DONE], (j - 1) & 1, abort, p.err, 7))) break;
          tc_fence_after();
        }
        const float alpha = rescale ? exp2f(m_used - m_new) : 1.f;
        l *= alpha;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float o[32];
          tmem_ld32(lane_addr + 256 + col0 + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(lane_addr + 256 + col0 + c * 32, o);
        }
        tmem_st_wait();
      }
      if (raise) m_used = m_new;
      float rs = 0.f;
      const bool live = m_used != -INFINITY;
      if constexpr (TMEM_P) {
        uint32_t w[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float e0 = live ? ex2f(s[2 * i] - m_used) : 0.f, e1 = live ? ex2f(s[2 * i + 1] - m_used) : 0.f;
          rs += e0 + e1;
          w[i] = pack_bf16x2(e0, e1);
        }
        tmem_st32u(lane_addr + 384 + (j & 1) * 64 + half * 32, w);
        tmem_st_wait();
      } else {
#pragma unroll
        for (int c8 = 0; c8 < BN / 16; ++c8) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float e0 = live ? ex2f(s[c8 * 8 + 2 * i] - m_used) : 0.f, e1 = live ? ex2f(s[c8 * 8 + 2 * i + 1] - m_used) : 0.f;
            rs += e0 + e1;
            w[i] = pack_bf16x2(e0, e1);
          }
          *reinterpret_cast<uint4*>(prow + ((c8 ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P visible to the tensor cores
      }
      l += rs;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B8_P_FULL]);
    }
    // epilogue: last PV done, add the two halves' row sums, normalise, store this half's columns
    const int n = j;
    bool ok = __all_sync(0xffffffffu, !*abort);
    if (ok && n >= 1) ok = __all_sync(0xffffffffu, mbar_wait(&bar[B8_O_DONE], (n - 1) & 1, abort, p.err, 8));
    if (ok && n >= 1) {
      xsum[half * BM + r] = l;
      mbar_arrive(xbar);
      ok = __all_sync(0xffffffffu, mbar_wait(xbar, n & 1, abort, p.err, 11));
    }
    if (ok && n >= 1) {
      tc_fence_after();
      const float L = xsum[r] + xsum[BM + r];
      const float inv = L > 0.f ? 1.f / L : 0.f;
      bf16* orow = p.o + ((long)row * p.Hq + h) * D + col0;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float o[32];
        tmem_ld32(lane_addr + 256 + col0 + c * 32, o);
        tmem_ld_wait();
        if (row < qe) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = o[i + e] * inv;
            store8(orow + c * 32 + i, f);
          }
        }
      }
      if (row < qe && half == 0) p.lse2[(long)h * p.T + row] = L > 0.f ? m_used + log2f(L) : INFINITY;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------------------------- paired heads
// Two q heads of one GQA group per CTA (heads 2hp and 2hp + 1 read the same K/V rows, so every K/V
// tile feeds twice the tensor-core work):
//   warps 0-3   softmax of head A, one query row per thread over all 128 key columns (no exchange
//               between warps);
//   warps 4-7   softmax of head B;
//   warp 8      TMA producer: both Q tiles, then K and V tiles through one 4-slot ring (K(j) in
//               slot 2j % 4, V(j) in slot (2j + 1) % 4);
//   warp 9      MMA issuer and TMEM owner.
// TMEM: S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512).  P_X (bf16 pairs) overwrites the
// first 64 columns of S_X and is the A operand of PV_X straight from tensor memory.  Per key tile j
// the issue order is PV_A(j-1), QK_A(j), PV_B(j-1), QK_B(j): while one head's softmax runs, the
// tensor cores work for the other.  S_X(j) may overwrite P_X(j-1) because the tensor pipe executes
// one thread's MMAs in issue order, and the commit that signals S_X(j) also covers PV_X(j-1), so
// the softmax may rescale O_X without another wait.  A K slot is released once both QK products of
// its tile are done, a V slot once both PV products are.
constexpr int THREADS_P = 320;
constexpr int NSLOT = 4;
constexpr int BP_Q = 0, BP_FULL = 1, BP_EMPTY = BP_FULL + NSLOT, BP_S = BP_EMPTY + NSLOT, BP_P = BP_S + 2, BP_O = BP_P + 2,
              BP_DRAIN = BP_O + 1, NBARP = BP_DRAIN + 1;

__global__ void __launch_bounds__(THREADS_P, 1) attn_fwd_tcp_k(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                                                              const __grid_constant__ CUtensorMap tv, Params p) {
  extern __shared__ char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  char* sQ = sm;              // head A, then head B
  char* ring = sm + 2 * TILE;  // NSLOT tiles
  uint64_t* bar = reinterpret_cast<uint64_t*>(ring + NSLOT * TILE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBARP);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = p.tiles[blockIdx.y * 2], qs = p.tiles[blockIdx.y * 2 + 1];
  const int hA = blockIdx.x * 2, hk = hA / (p.Hq / p.Hkv);
  const int q0 = p.qseg[seg * 4], q1 = p.qseg[seg * 4 + 1], r_first = p.qseg[seg * 4 + 2], r_last = p.qseg[seg * 4 + 3];
  const int qe = min(qs + BM, q1);

  if (tid == 0) {
    mbar_init(&bar[BP_Q], 1);
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&bar[BP_FULL + s], 1);
      mbar_init(&bar[BP_EMPTY + s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bar[BP_S + x], 1);
      mbar_init(&bar[BP_P + x], 4);
    }
    mbar_init(&bar[BP_O], 1);
    mbar_init(&bar[BP_DRAIN], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tq)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tv)) : "memory");
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  KeyTiles kt{p.kr, r_first, r_last, q0, qe, 0, 0, 0, 0};
  kt.load_range();

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_expect_tx(&bar[BP_Q], 2 * TILE);
      tma_2d(sQ, &tq, hA * D, qs, &bar[BP_Q]);
      tma_2d(sQ + HALF, &tq, hA * D + 64, qs, &bar[BP_Q]);
      tma_2d(sQ + TILE, &tq, (hA + 1) * D, qs, &bar[BP_Q]);
      tma_2d(sQ + TILE + HALF, &tq, (hA + 1) * D + 64, qs, &bar[BP_Q]);
      int u = 0;  // slot uses issued
      for (bool go = true; go && kt.valid(); kt.next()) {
        for (int kv = 0; kv < 2; ++kv, ++u) {
          const int s = u % NSLOT;
          if (u >= NSLOT && !mbar_wait(&bar[BP_EMPTY + s], ((u / NSLOT) - 1) & 1, abort, p.err, 41)) {
            go = false;
            break;
          }
          mbar_expect_tx(&bar[BP_FULL + s], TILE);
          const CUtensorMap* m = kv ? &tv : &tk;
          tma_2d(ring + s * TILE, m, hk * D, kt.ka, &bar[BP_FULL + s]);
          tma_2d(ring + s * TILE + HALF, m, hk * D + 64, kt.ka, &bar[BP_FULL + s]);
        }
      }
      if (*abort) {  // let every copy this CTA started land before its shared memory is released
        int zero = 0;
        mbar_wait(&bar[BP_Q], 0, (volatile int*)&zero, p.err, 41);
        for (int i = max(0, u - NSLOT); i < u; ++i) mbar_wait(&bar[BP_FULL + i % NSLOT], (i / NSLOT) & 1, (volatile int*)&zero, p.err, 41);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_QK = idesc_bf16(BN, false), ID_PV = idesc_bf16(D, true);
      const uint32_t qa = s32(sQ), qb = qa + TILE, rb = s32(ring);
      auto slot = [&](int u) { return rb + (uint32_t)(u % NSLOT) * TILE; };
      auto full = [&](int u) { return mbar_wait(&bar[BP_FULL + u % NSLOT], (u / NSLOT) & 1, abort, p.err, 42); };
      auto qk = [&](uint32_t d, uint32_t qbase, uint32_t kbase) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
          tc_mma(d, sdesc(qbase + off, 16, 1024), sdesc(kbase + off, 16, 1024), ID_QK, kk > 0 ? 1u : 0u);
        }
      };
      auto pv = [&](uint32_t o, uint32_t pcol, uint32_t vbase, bool acc) {
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          tc_mma_ts(o, pcol + kk * 8, sdesc(vbase + kk * 2048, HALF, 1024), ID_PV, (acc || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(&bar[BP_Q], 0, abort, p.err, 43);
      tc_fence_after();
      int j = 0;
      for (; ok && kt.valid(); kt.next(), ++j) {
        const int uk = 2 * j, uv = 2 * j - 1;  // K(j); V(j - 1)
        if (!(ok = full(uk))) break;
        if (j > 0 && !(ok = full(uv) && mbar_wait(&bar[BP_P], (j - 1) & 1, abort, p.err, 44))) break;
        tc_fence_after();
        if (j > 0) pv(tmem + 256, tmem, slot(uv), j > 1);
        qk(tmem, qa, slot(uk));
        tc_commit(&bar[BP_S]);
        if (j > 0) {
          if (!(ok = mbar_wait(&bar[BP_P + 1], (j - 1) & 1, abort, p.err, 45))) break;
          tc_fence_after();
          pv(tmem + 384, tmem + 128, slot(uv), j > 1);
          tc_commit(&bar[BP_EMPTY + uv % NSLOT]);
        }
        qk(tmem + 128, qb, slot(uk));
        tc_commit(&bar[BP_S + 1]);
        tc_commit(&bar[BP_EMPTY + uk % NSLOT]);
      }
      if (ok && j >= 1) {
        const int uv = 2 * j - 1;
        ok = full(uv) && mbar_wait(&bar[BP_P], (j - 1) & 1, abort, p.err, 46);
        if (ok) {
          tc_fence_after();
          pv(tmem + 256, tmem, slot(uv), j > 1);
          ok = mbar_wait(&bar[BP_P + 1], (j - 1) & 1, abort, p.err, 47);
        }
        if (ok) {
          tc_fence_after();
          pv(tmem + 384, tmem + 128, slot(uv), j > 1);
          tc_commit(&bar[BP_EMPTY + uv % NSLOT]);
          tc_commit(&bar[BP_O]);
        }
      }
      tc_commit(&bar[BP_DRAIN]);
      int zero = 0;
      mbar_wait(&bar[BP_DRAIN], 0, (volatile int*)&zero, p.err, 48);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (warps 0-7)
    const int hx = warp >> 2, wq = warp & 3;
    const int r = wq * 32 + lane;  // row within the tile == TMEM lane
    const int row = qs + r;
    const uint32_t lane_addr = tmem + ((uint32_t)(wq * 32) << 16);
    const uint32_t s_col = hx * 128, o_col = 256 + hx * 128;
    float m_used = -INFINITY, l = 0.f;
    int j = 0;
    for (; kt.valid(); kt.next(), ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&bar[BP_S + hx], j & 1, abort, p.err, 50 + hx))) break;
      tc_fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        float t[32];
        tmem_ld32(lane_addr + s_col + c * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = t[i];
      }
      const int kend = min(kt.ka + BN, kt.rend);
      const int climit = row < qe ? (kt.ty == 1 ? min(kend - kt.ka, row - q0 + kt.k0 - kt.ka + 1) : kend - kt.ka) : 0;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        s[c] = c < climit ? s[c] * p.scale_log2 : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      const float m_new = fmaxf(m_used, mt);
      const bool raise = m_new > m_used + RESCALE_THRESHOLD;
      const bool rescale = raise && j >= 1 && m_used != -INFINITY;
      if (__any_sync(0xffffffffu, rescale)) {  // PV_X(j-1) is complete: S_X(j)'s commit covers it
        const float alpha = rescale ? exp2f(m_used - m_new) : 1.f;
        l *= alpha;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(lane_addr + o_col + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(lane_addr + o_col + c * 32, o);
        }
        tmem_st_wait();
      }
      if (raise) m_used = m_new;
      const bool live = m_used != -INFINITY;
      float rs = 0.f;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t w[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float e0 = live ? ex2f(s[h2 * 64 + 2 * i] - m_used) : 0.f, e1 = live ? ex2f(s[h2 * 64 + 2 * i + 1] - m_used) : 0.f;
          rs += e0 + e1;
          w[i] = pack_bf16x2(e0, e1);
        }
        tmem_st32u(lane_addr + s_col + h2 * 32, w);
      }
      tmem_st_wait();
      l += rs;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[BP_P + hx]);
    }
    const int n = j;
    bool ok = __all_sync(0xffffffffu, !*abort);
    if (ok && n >= 1) ok = __all_sync(0xffffffffu, mbar_wait(&bar[BP_O], 0, abort, p.err, 52));
    if (ok && n >= 1) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = p.o + ((long)row * p.Hq + hA + hx) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        tmem_ld32(lane_addr + o_col + c * 32, o);
        if (row < qe) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = o[i + e] * inv;
            store8(orow + c * 32 + i, f);
          }
        }
      }
      if (row < qe) p.lse2[(long)(hA + hx) * p.T + row] = l > 0.f ? m_used + log2f(l) : INFINITY;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------------------------- host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                              CUtensorMapFloatOOBfill);

static EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    AX_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess && ptr, "cuTensorMapEncodeTiled");
    fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}

// rows x width bf16 matrix (row stride = width), box 64 columns x 128 rows, 128-byte swizzle.
static CUtensorMap map_rows(const void* base, long rows, long width) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)width * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AX_CHECK(r == CUDA_SUCCESS, "tensor map encode failed (", (int)r, ")");
  return m;
}

static at::Tensor& err_flag(int dev) {
  static at::Tensor e[16];
  if (!e[dev].defined()) e[dev] = at::zeros({1}, at::TensorOptions().device(at::kCUDA, dev).dtype(at::kInt));
  return e[dev];
}

}  // namespace atc

// q (T,Hq,128), k/v (Tk,Hkv,128) -> o (T,Hq,128) bf16, lse2 (Hq,T) fp32 (base-2, +inf for rows without keys)
// variant: 0 = 4 softmax warps, 1 = 4 softmax warps with double-buffered P, 2 = 8 softmax warps,
// 3 = 8 softmax warps with P in tensor memory, 4 = two heads of a GQA group per CTA (variant 3 when
// the group size is odd)
std::vector<at::Tensor> attn_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor qseg, at::Tensor kr, at::Tensor tiles, double scale,
                                    int64_t variant) {
  using namespace atc;
  AX_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.size(2) == D, "q bf16 (T,Hq,128)");
  AX_CHECK(k.is_contiguous() && v.is_contiguous() && k.sizes() == v.sizes() && k.size(2) == D, "k/v layout");
  const int T = q.size(0), Hq = q.size(1), Tk = k.size(0), Hkv = k.size(1);
  AX_CHECK(Hq % Hkv == 0, "GQA");
  auto o = at::zeros_like(q);
  auto lse2 = at::full({Hq, T}, INFINITY, q.options().dtype(at::kFloat));
  const int nt = tiles.size(0);
  // grid (heads, tiles): blocks start in index order, so the heaviest tiles (first in the table) of
  // every head start first
  AX_CHECK(nt <= 65535, "attention: at most 65535 tiles per launch");
  if (nt == 0 || T == 0 || Tk == 0) return {o, lse2};
  AX_CHECK(qseg.is_cuda() && kr.is_cuda() && tiles.is_cuda(), "attention tables on the device");
  const CUtensorMap tq = map_rows(q.data_ptr(), T, (long)Hq * D);
  const CUtensorMap tk = map_rows(k.data_ptr(), Tk, (long)Hkv * D);
  const CUtensorMap tv = map_rows(v.data_ptr(), Tk, (long)Hkv * D);
  Params p{(bf16*)o.data_ptr(), lse2.data_ptr<float>(), qseg.data_ptr<int>(), kr.data_ptr<int>(), tiles.data_ptr<int>(), Hq, Hkv, T,
           (float)(scale * 1.4426950408889634), err_flag(q.get_device()).data_ptr<int>()};
  if (variant == 4 && (Hq / Hkv) % 2 == 0) {
    const int smemp = (2 + NSLOT) * TILE + NBARP * 8 + 16 + 1024;
    smem_attr(reinterpret_cast<const void*>(attn_fwd_tcp_k), smemp);
    attn_fwd_tcp_k<<<dim3(Hq / 2, nt), THREADS_P, smemp, stream()>>>(tq, tk, tv, p);
    AX_LAUNCH_OK();
    return {o, lse2};
  }
  if (variant == 2 || variant == 3 || variant == 4) {
    if (variant == 4) variant = 3;  // odd GQA group: one head per CTA
    const int smem8 = 6 * TILE + 3 * 2 * BM * 4 + NBAR8 * 8 + 16 + 1024;
    auto* kern = variant == 3 ? attn_fwd_tc8_k<true> : attn_fwd_tc8_k<false>;
    smem_attr(reinterpret_cast<const void*>(kern), smem8);
    kern<<<dim3(Hq, nt), THREADS8, smem8, stream()>>>(tq, tk, tv, p);
    AX_LAUNCH_OK();
    return {o, lse2};
  }
  const bool dbl = variant == 1;
  const int smem = (dbl ? 7 : 6) * TILE + NBAR * 8 + 16 + 1024;
  smem_attr(dbl ? reinterpret_cast<const void*>(attn_fwd_tc_k<true>) : reinterpret_cast<const void*>(attn_fwd_tc_k<false>), smem);
  if (dbl) attn_fwd_tc_k<true><<<dim3(Hq, nt), THREADS, smem, stream()>>>(tq, tk, tv, p);
  else attn_fwd_tc_k<false><<<dim3(Hq, nt), THREADS, smem, stream()>>>(tq, tk, tv, p);
  AX_LAUNCH_OK();
  return {o, lse2};
}

// Error code of the last failed wait of the tcgen05 attention (0 = none); reading it synchronises.
int64_t attn_tc_error() { return atc::err_flag(c10::cuda::current_device()).item<int>(); }

}  // namespace ax
