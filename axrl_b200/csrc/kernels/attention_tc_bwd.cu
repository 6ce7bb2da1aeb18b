// Range-list flash attention backward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
// Reference counterpart: the backward of MagiAttention's calc_attn
// (axrl/utils/megatron/magi_forward.py:439-466).
//
// Same problem, inputs and outputs as attn_bwd_k in attention.cu (dQ accumulated in fp32 through
// atomics, dK / dV in bf16), computed with one CTA per (128-key tile, kv head).  For every q head of
// the GQA group and every 128-row q tile that sees the key tile:
//
//   S^T  = K Q^T          (TMEM cols [0,128); keys are the MMA's M, so TMEM lane = key)
//   dP^T = V dO^T         (TMEM cols [128,256))
//   P^T  = exp2(S^T * scale*log2e - lse2),  dS^T = scale * P^T o (dP^T - Dsum)   (softmax warps)
//   dV  += P^T dO         (TMEM cols [256,384), accumulated over all q tiles and heads)
//   dK  += dS^T Q         (TMEM cols [384,512))
//   dQ   = dS K           (TMEM cols [0,128) again; added to the fp32 dQ accumulator by the softmax
//                          warps, TMEM lane = q row)
//
// Operand layouts: Q, dO, K, V tiles are loaded once each by TMA as 128 rows x 128 columns in two
// 64-column boxes with 128-byte swizzle and serve both as K-major operands (Q, dO, K, V on the
// first two products) and as MN-major ones (dO, Q, K on the last three).  P^T and dS^T are written
// by the softmax warps in the same swizzled layout: K-major A for dV / dK, MN-major A for dQ.
//
// Warp roles: warp 8 TMA producer, warp 9 MMA issuer (one thread) and TMEM owner, warps 0-7 the
// element-wise gradient and the dQ / dK / dV read-out: warps w and w + 4 share TMEM lanes
// 32 (w % 4) (one key row for the key-major products, one q row for dQ) and split the 128 columns
// in halves, so there is no cross-thread reduction.  The q tile's lse and Dsum values are staged
// once in shared memory (alternating buffers by tile parity, a bounded mbarrier among the 256
// threads), and dQ is added to the fp32 accumulator with 16-byte vector reductions
// (red.global.add.v4.f32).  Every mbarrier wait is bounded; on expiry the CTA records an error
// code, drains its copies and tensor-core work, frees TMEM and exits.
#include <cuda.h>

#include <string>

#include "common.cuh"
#include "tcgen05.cuh"

namespace ax {
namespace atb {

using namespace tc;

constexpr int D = 128;
constexpr int BK = 128;  // keys per CTA
constexpr int BQ = 128;  // q rows per tile
constexpr int THREADS = 320;  // warps 0-7 element-wise, 8 TMA producer, 9 MMA issuer
constexpr int TILE = 128 * 128 * 2;
constexpr int HALF = TILE / 2;
constexpr uint32_t TMEM_COLS = 512;
constexpr int C_S = 0, C_DP = 128, C_DV = 256, C_DK = 384;

constexpr int B_KV = 0, B_QD = 1, B_S = 2, B_P = 3, B_MM = 4, B_DQF = 5, B_DRAIN = 6, B_LD = 7, B_QD1 = 8, B_EM = 9, NBAR = 11;

// 2^x with the hardware approximation (flushes denormal results to zero; P is rounded to bf16 anyway)
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void red_add_f32(float* p, float a) { asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory"); }
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

struct Params {
  const float* lse2;  // (Hq, T)
  const float* dsum;  // (Hq, T)
  float* dq_acc;      // (T, Hq, D)
  bf16* dk;           // (Tk, Hkv, D)
  bf16* dv;
  const int* kseg;   // (Nk, 4): k0, k1, first, last
  const int* qr;     // (Nitems, 3): q0, q1, type
  const int* tiles;  // (Ntiles, 2): kseg index, 128-key tile start
  int Hq, Hkv, T;
  float scale_log2, scale;
  int* err;
};

// q tiles seen by one key tile: every q head of the group, every q-range of the key segment, from
// the first row that can see a key of the tile (causal ranges) to the range end.
struct QTiles {
  const int* qr;
  int it0, it1, G, ks, k0s;
  int g, it, q0, q1, ty, qs;
  int step = BQ;  // q rows per tile
  __device__ void seek() {
    while (g < G) {
      while (it < it1) {
        q0 = qr[it * 3];
        q1 = qr[it * 3 + 1];
        ty = qr[it * 3 + 2];
        qs = q0 + (ty == 1 ? max(0, ks - k0s) : 0);
        if (qs < q1) return;
        ++it;
      }
      ++g;
      it = it0;
    }
  }
  __device__ bool valid() const { return g < G; }
  __device__ void next() {
    qs += step;
    if (qs >= q1) {
      ++it;
      seek();
    }
  }
};

// DBL: Q and dO double-buffered (the next q tile loads while this one is in the products); P^T goes
// back into tensor memory over the consumed S^T columns (each half-row warp inside its own half:
// q columns [0, 64) -> TMEM columns [0, 32), [64, 128) -> [64, 96)) and is the A operand of dV from
// there, which frees the shared-memory P^T tile for the second buffers.  Shared memory is then
// 7 tiles + the lse / Dsum stages, so the dynamic shared memory base must be 1024-byte aligned
// (checked; a misaligned base records an error and the CTA exits).
template <bool DBL>
__global__ void __launch_bounds__(THREADS, 1) attn_bwd_tc_k(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                                                          const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                                                          Params p) {
  extern __shared__ __align__(1024) char smem_raw[];
  if constexpr (DBL) {
    if (reinterpret_cast<uintptr_t>(smem_raw) & 1023) {
      if (threadIdx.x == 0) atomicCAS(p.err, 0, 19);
      return;
    }
  }
  char* sm = DBL ? smem_raw : reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  char* sK = sm;
  char* sV = sm + TILE;
  char* sQ = sm + 2 * TILE;                  // DBL: two buffers (2, 3)
  char* sdO = sm + (DBL ? 4 : 3) * TILE;     // DBL: two buffers (4, 5)
  char* sP = sm + 4 * TILE;                  // P^T  [key][q] (not DBL)
  char* sdS = sm + (DBL ? 6 : 5) * TILE;     // dS^T [key][q]
  float* sL = reinterpret_cast<float*>(sm + (DBL ? 7 : 6) * TILE);  // [tile parity][q column]: lse2
  float* sDs = sL + 2 * BQ;                              // [tile parity][q column]: Dsum
  uint64_t* bar = reinterpret_cast<uint64_t*>(sDs + 2 * BQ);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBAR);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = p.tiles[blockIdx.y * 2], ks = p.tiles[blockIdx.y * 2 + 1];
  const int hk = blockIdx.x, G = p.Hq / p.Hkv;
  const int k0s = p.kseg[seg * 4], k1s = p.kseg[seg * 4 + 1], it0 = p.kseg[seg * 4 + 2], it1 = p.kseg[seg * 4 + 3];
  const int ke = min(ks + BK, k1s);

  if (tid == 0) {
    mbar_init(&bar[B_KV], 1);
    mbar_init(&bar[B_QD], 1);
    mbar_init(&bar[B_S], 1);
    mbar_init(&bar[B_P], 8);
    mbar_init(&bar[B_MM], 1);
    mbar_init(&bar[B_DQF], 8);
    mbar_init(&bar[B_DRAIN], 1);
    mbar_init(&bar[B_LD], 256);
    mbar_init(&bar[B_QD1], 1);
    mbar_init(&bar[B_EM], 1);
    mbar_init(&bar[B_EM + 1], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  QTiles qt{p.qr, it0, it1, G, ks, k0s, 0, it0, 0, 0, 0, 0};
  qt.seek();

  if (warp == 8 && DBL) {
    // ------------------------------------------------------------ producer (DBL): K/V once, then per q tile
    // its lse2 / Dsum (the warp's lanes) and Q / dO (TMA) into buffer i & 1
    if (lane == 0) {
      mbar_expect_tx(&bar[B_KV], 2 * TILE);
      tma_2d(sK, &tk, hk * D, ks, &bar[B_KV]);
      tma_2d(sK + HALF, &tk, hk * D + 64, ks, &bar[B_KV]);
      tma_2d(sV, &tv, hk * D, ks, &bar[B_KV]);
      tma_2d(sV + HALF, &tv, hk * D + 64, ks, &bar[B_KV]);
    }
    int i = 0;
    for (; qt.valid(); qt.next(), ++i) {
      const int b = i & 1;
      int ok = 1;
      if (lane == 0 && i >= 2) ok = mbar_wait(&bar[B_EM + b], ((i - 2) >> 1) & 1, abort, p.err, 11);  // buffer b consumed
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      const int h = hk * G + qt.g, qe = min(qt.qs + BQ, qt.q1);
      float* L = sL + b * BQ;
      float* Ds = sDs + b * BQ;
      for (int c = lane; c < BQ; c += 32) {
        const bool in = qt.qs + c < qe;
        L[c] = in ? p.lse2[(long)h * p.T + qt.qs + c] : 0.f;
        Ds[c] = in ? p.dsum[(long)h * p.T + qt.qs + c] : 0.f;
      }
      __syncwarp();  // the stores are ordered before lane 0's arrival on this buffer's barrier
      if (lane == 0) {
        uint64_t* qd = &bar[b ? B_QD1 : B_QD];
        mbar_expect_tx(qd, 2 * TILE);
        tma_2d(sQ + b * TILE, &tq, h * D, qt.qs, qd);
        tma_2d(sQ + b * TILE + HALF, &tq, h * D + 64, qt.qs, qd);
        tma_2d(sdO + b * TILE, &tdo, h * D, qt.qs, qd);
        tma_2d(sdO + b * TILE + HALF, &tdo, h * D + 64, qt.qs, qd);
      }
      __syncwarp();
    }
    if (lane == 0 && *abort) {  // every copy this CTA started lands before its shared memory is released
      int zero = 0;
      mbar_wait(&bar[B_KV], 0, (volatile int*)&zero, p.err, 11);
      for (int j = max(0, i - 2); j < i; ++j) mbar_wait(&bar[(j & 1) ? B_QD1 : B_QD], (j >> 1) & 1, (volatile int*)&zero, p.err, 11);
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_expect_tx(&bar[B_KV], 2 * TILE);
      tma_2d(sK, &tk, hk * D, ks, &bar[B_KV]);
      tma_2d(sK + HALF, &tk, hk * D + 64, ks, &bar[B_KV]);
      tma_2d(sV, &tv, hk * D, ks, &bar[B_KV]);
      tma_2d(sV + HALF, &tv, hk * D + 64, ks, &bar[B_KV]);
      int i = 0;
      for (; qt.valid(); qt.next(), ++i) {
        const int b = DBL ? (i & 1) : 0;
        if constexpr (DBL) {  // this buffer's previous tile (i - 2) consumed
          if (i >= 2 && !mbar_wait(&bar[B_EM + b], ((i - 2) >> 1) & 1, abort, p.err, 11)) break;
        } else {
          if (i >= 1 && !mbar_wait(&bar[B_MM], (i - 1) & 1, abort, p.err, 11)) break;  // Q / dO of the previous tile consumed
        }
        const int h = hk * G + qt.g;
        uint64_t* qd = &bar[b ? B_QD1 : B_QD];
        char* q_dst = sQ + b * TILE;
        char* do_dst = sdO + b * TILE;
        mbar_expect_tx(qd, 2 * TILE);
        tma_2d(q_dst, &tq, h * D, qt.qs, qd);
        tma_2d(q_dst + HALF, &tq, h * D + 64, qt.qs, qd);
        tma_2d(do_dst, &tdo, h * D, qt.qs, qd);
        tma_2d(do_dst + HALF, &tdo, h * D + 64, qt.qs, qd);
      }
      if (*abort) {  // every copy this CTA started lands before its shared memory is released
        int zero = 0;
        mbar_wait(&bar[B_KV], 0, (volatile int*)&zero, p.err, 11);
        for (int j = max(0, i - (DBL ? 2 : 1)); j < i; ++j) {
          const int b = DBL ? (j & 1) : 0;
          mbar_wait(&bar[b ? B_QD1 : B_QD], (DBL ? (j >> 1) : j) & 1, (volatile int*)&zero, p.err, 11);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_KMAJ = idesc_bf16(128, false), ID_BMN = idesc_bf16(128, true), ID_ABMN = idesc_bf16(128, true, true);
      const uint32_t k_b = s32(sK), v_b = s32(sV), p_b = s32(sP), ds_b = s32(sdS);
      bool ok = mbar_wait(&bar[B_KV], 0, abort, p.err, 12);
      int i = 0;
      for (; ok && qt.valid(); qt.next(), ++i) {
        const int b = DBL ? (i & 1) : 0;
        const uint32_t q_b = s32(sQ + b * TILE), do_b = s32(sdO + b * TILE);
        if (!mbar_wait(&bar[b ? B_QD1 : B_QD], (DBL ? (i >> 1) : i) & 1, abort, p.err, 12)) break;
        if (i >= 1 && !mbar_wait(&bar[B_DQF], (i - 1) & 1, abort, p.err, 12)) break;  // dQ of the previous tile read out
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {  // S^T = K Q^T, dP^T = V dO^T (K = head dim)
          const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
          tc_mma(tmem + C_S, sdesc(k_b + off, 16, 1024), sdesc(q_b + off, 16, 1024), ID_KMAJ, kk > 0);
          tc_mma(tmem + C_DP, sdesc(v_b + off, 16, 1024), sdesc(do_b + off, 16, 1024), ID_KMAJ, kk > 0);
        }
        tc_commit(&bar[B_S]);
        if (!mbar_wait(&bar[B_P], i & 1, abort, p.err, 13)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {  // dV += P^T dO, dK += dS^T Q (K = q rows)
          const uint32_t a_off = (kk >> 2) * HALF + (kk & 3) * 32;
          if constexpr (DBL)  // P^T from TMEM: q 16 kk .. +15 at column (kk < 4 ? 0 : 64) + (kk % 4) * 8
            tc_mma_ts(tmem + C_DV, tmem + C_S + (kk >> 2) * 64 + (kk & 3) * 8, sdesc(do_b + kk * 2048, HALF, 1024), ID_BMN, (i > 0 || kk > 0));
          else
            tc_mma(tmem + C_DV, sdesc(p_b + a_off, 16, 1024), sdesc(do_b + kk * 2048, HALF, 1024), ID_BMN, (i > 0 || kk > 0));
          tc_mma(tmem + C_DK, sdesc(ds_b + a_off, 16, 1024), sdesc(q_b + kk * 2048, HALF, 1024), ID_BMN, (i > 0 || kk > 0));
        }
        if constexpr (DBL) tc_commit(&bar[B_EM + b]);  // Q / dO of this buffer consumed
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)  // dQ = dS K (K = keys; dS read MN-major from dS^T)
          tc_mma(tmem + C_S, sdesc(ds_b + kk * 2048, HALF, 1024), sdesc(k_b + kk * 2048, HALF, 1024), ID_ABMN, kk > 0);
        tc_commit(&bar[B_MM]);
      }
      tc_commit(&bar[B_DRAIN]);
      int zero = 0;
      mbar_wait(&bar[B_DRAIN], 0, (volatile int*)&zero, p.err, 14);
    }
  } else {
    // ------------------------------------------------------------ gradient element-wise + read-out (warps 0-7)
    const int wq = warp & 3, half = warp >> 2;
    const int r = wq * 32 + lane;  // TMEM lane: key row of the key-major products, q row of dQ
    const int col0 = half * (BQ / 2);
    const int key = ks + r;
    const uint32_t lane_addr = tmem + ((uint32_t)(wq * 32) << 16);
    char* prow = sP + (r >> 3) * 1024 + (r & 7) * 128 + half * HALF;
    char* dsrow = sdS + (r >> 3) * 1024 + (r & 7) * 128 + half * HALF;
    int i = 0;
    for (; qt.valid(); qt.next(), ++i) {
      const int h = hk * G + qt.g;
      const int qs = qt.qs, qe = min(qs + BQ, qt.q1);
      // q columns cfirst <= c < climit see this key: rows of the tile, and for causal ranges only
      // rows with (q - q0) >= (key - k0s)
      const int climit = key < ke ? qe - qs : 0;
      const int cfirst = qt.ty == 1 ? max(0, (key - k0s) - (qs - qt.q0)) : 0;
      if constexpr (!DBL) {  // stage the tile's lse2 / Dsum once (thread (half, r) loads column r of its half's copy)
        float* L = sL + (i & 1) * BQ;
        float* Ds = sDs + (i & 1) * BQ;
        if (half == 0) L[r] = qs + r < qe ? p.lse2[(long)h * p.T + qs + r] : 0.f;
        else Ds[r] = qs + r < qe ? p.dsum[(long)h * p.T + qs + r] : 0.f;
        mbar_arrive(&bar[B_LD]);
        if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_LD], i & 1, abort, p.err, 17))) break;
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_S], i & 1, abort, p.err, 15))) break;
      if constexpr (DBL)  // the producer staged this tile's lse2 / Dsum with buffer i & 1
        if (!__all_sync(0xffffffffu, mbar_wait(&bar[(i & 1) ? B_QD1 : B_QD], (i >> 1) & 1, abort, p.err, 17))) break;
      tc_fence_after();
      const float* L = sL + (i & 1) * BQ;
      const float* Ds = sDs + (i & 1) * BQ;
#pragma unroll 1
      for (int cc = 0; cc < BQ / 2; cc += 32) {
        const int c0 = col0 + cc;
        float s[32], dp[32];
        tmem_ld32(lane_addr + C_S + c0, s);
        tmem_ld32(lane_addr + C_DP + c0, dp);
        uint32_t pw[16], dw[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float pv[2], dv2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int c = c0 + e + u;
            const bool vis = c >= cfirst && c < climit;
            const float pr = vis ? ex2_fast(fmaf(s[e + u], p.scale_log2, -L[c])) : 0.f;
            pv[u] = pr;
            dv2[u] = vis ? pr * (dp[e + u] - Ds[c]) * p.scale : 0.f;
          }
          bf162 a = __floats2bfloat162_rn(pv[0], pv[1]), b = __floats2bfloat162_rn(dv2[0], dv2[1]);
          pw[e / 2] = *reinterpret_cast<uint32_t*>(&a);
          dw[e / 2] = *reinterpret_cast<uint32_t*>(&b);
        }
        if constexpr (DBL) tmem_st16u(lane_addr + C_S + half * 64 + (cc >> 1), pw);  // over S^T columns this warp has read
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {  // 4 chunks of 8 q columns, 128-byte swizzled rows of this half's box
          const int ch = (cc >> 3) + q8;  // 16-byte chunk index within the 64-column box
          const int off = ((ch ^ (r & 7)) << 4);
          if constexpr (!DBL)
            *reinterpret_cast<uint4*>(prow + off) = make_uint4(pw[q8 * 4], pw[q8 * 4 + 1], pw[q8 * 4 + 2], pw[q8 * 4 + 3]);
          *reinterpret_cast<uint4*>(dsrow + off) = make_uint4(dw[q8 * 4], dw[q8 * 4 + 1], dw[q8 * 4 + 2], dw[q8 * 4 + 3]);
        }
      }
      if constexpr (DBL) tmem_st_wait();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P^T / dS^T visible to the tensor cores
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_P]);
      // dQ of this tile: TMEM lane = q row, this half's 64 head-dim columns
      if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_MM], i & 1, abort, p.err, 16))) break;
      tc_fence_after();
      const int qrow = qs + r;
      float* dq = p.dq_acc + ((long)qrow * p.Hq + h) * D + col0;
#pragma unroll 1
      for (int cc = 0; cc < D / 2; cc += 32) {
        float v[32];
        tmem_ld32(lane_addr + C_S + col0 + cc, v);
        if (qrow < qe) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) red_add_v4(dq + cc + e, v[e], v[e + 1], v[e + 2], v[e + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B_DQF]);
    }
    // dK / dV of this key tile (accumulated over every q tile and head), this half's columns
    const bool ok = __all_sync(0xffffffffu, !*abort) && i > 0;
    if (ok) {
      tc_fence_after();
      bf16* dkr = p.dk + ((long)key * p.Hkv + hk) * D + col0;
      bf16* dvr = p.dv + ((long)key * p.Hkv + hk) * D + col0;
#pragma unroll 1
      for (int cc = 0; cc < D / 2; cc += 32) {
        float a[32], b[32];
        tmem_ld32(lane_addr + C_DK + col0 + cc, a);
        tmem_ld32(lane_addr + C_DV + col0 + cc, b);
        if (key < ke) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            float fa[8], fb[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              fa[u] = a[e + u];
              fb[u] = b[e + u];
            }
            store8(dkr + cc + e, fa);
            store8(dvr + cc + e, fb);
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------------------------- 64-row q blocks
// Second backward kernel, one CTA per (128-key tile, kv head) as above, reorganised so that loads,
// the element-wise work and the dQ read-out overlap the tensor-core products:
//   * q rows come in blocks of 64 through a 3-stage ring (Q, dO: 16 KB each, plus the block's lse2
//     and Dsum, loaded by the producer warp's lanes);
//   * S^T = K Q^T and dP^T = V dO^T (128 x 64 each) go to one of two TMEM buffers ([0,128) or
//     [128,256): S^T in the first 64 columns, dP^T in the next 64), so the products of block i + 1
//     run while the element-wise warps work on block i;
//   * the element-wise warps write P^T and dS^T back over the first 32 columns of S^T and dP^T as
//     bf16 pairs, where dV += P^T dO and dK += dS^T Q (TMEM cols [256,384) and [384,512)) take them
//     as the A operand; dS^T also goes to shared memory (two buffers) as the B operand of
//     dQ^T = K^T dS^T (M = head dim, N = 64 q rows), which lands on the S^T columns of its buffer;
//   * four separate warps read dQ^T out (TMEM lane = head dim, so each fp32 reduction instruction
//     covers 128 consecutive bytes of the dQ accumulator) and store dK / dV at the end.
// The tensor pipe executes one thread's products in issue order, which makes the reuse of TMEM
// columns by a later product safe once the earlier one has been issued.
// Warps 0-7 element-wise (warps w and w + 4 share TMEM lanes 32 (w % 4) = key rows and split the 64
// q columns), 8-11 dQ read-out and the final dK / dV store, 12 TMA, 13 MMA issuer and TMEM owner.
// Every mbarrier wait is bounded.
namespace atb2 {
using namespace tc;
constexpr int BQ2 = 64, NST = 3, THREADS2 = 448;
constexpr int QT = BQ2 * D * 2;  // 16 KB: 64 rows x 128 head dims (two 64-column boxes of 8 KB)
constexpr int QHALF = QT / 2;
constexpr int DST = 128 * BQ2 * 2;  // 16 KB: dS^T [128 keys][64 q], one 128-byte swizzled box
constexpr uint32_t C2_BUF = 128, C2_DP = 64, C2_DV = 256, C2_DK = 384;  // buffer b: S^T / dQ^T at 128 b, dP^T at 128 b + 64
constexpr int B2_KV = 0, B2_FULL = 1, B2_EMPTY = B2_FULL + NST, B2_S = B2_EMPTY + NST, B2_P = B2_S + 2, B2_DQF = B2_P + 2,
              B2_DQE = B2_DQF + 2, B2_DONE = B2_DQE + 2, B2_DRAIN = B2_DONE + 1, NBAR2 = B2_DRAIN + 1;
}  // namespace atb2

__global__ void __launch_bounds__(atb2::THREADS2, 1) attn_bwd_tc2_k(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                                                                     const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                                                                     Params p) {
  using namespace atb2;
  extern __shared__ char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  char* sK = sm;
  char* sV = sm + TILE;
  char* sSt = sm + 2 * TILE;       // NST stages of (Q, dO), 32 KB each
  char* sDS = sSt + NST * 2 * QT;  // two dS^T buffers
  float* sLD = reinterpret_cast<float*>(sDS + 2 * DST);  // [stage][lse2 64 | Dsum 64]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sLD + NST * 2 * BQ2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBAR2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = p.tiles[blockIdx.y * 2], ks = p.tiles[blockIdx.y * 2 + 1];
  const int hk = blockIdx.x, G = p.Hq / p.Hkv;
  const int k0s = p.kseg[seg * 4], k1s = p.kseg[seg * 4 + 1], it0 = p.kseg[seg * 4 + 2], it1 = p.kseg[seg * 4 + 3];
  const int ke = min(ks + BK, k1s);

  if (tid == 0) {
    mbar_init(&bar[B2_KV], 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(&bar[B2_FULL + s], 1);
      mbar_init(&bar[B2_EMPTY + s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar[B2_S + b], 1);
      mbar_init(&bar[B2_P + b], 8);
      mbar_init(&bar[B2_DQF + b], 1);
      mbar_init(&bar[B2_DQE + b], 4);
    }
    mbar_init(&bar[B2_DONE], 1);
    mbar_init(&bar[B2_DRAIN], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 13) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  QTiles qt{p.qr, it0, it1, G, ks, k0s, 0, it0, 0, 0, 0, 0, BQ2};
  qt.seek();
  auto q_at = [&](int s) { return sSt + s * 2 * QT; };    // Q of stage s (dO at + QT)
  auto ld_at = [&](int s) { return sLD + s * 2 * BQ2; };  // lse2 of stage s (Dsum at + BQ2)

  if (warp == 12) {
    // ------------------------------------------------------------ producer: K/V once, then (Q, dO, lse2, Dsum) per block
    if (lane == 0) {
      mbar_expect_tx(&bar[B2_KV], 2 * TILE);
      tma_2d(sK, &tk, hk * D, ks, &bar[B2_KV]);
      tma_2d(sK + HALF, &tk, hk * D + 64, ks, &bar[B2_KV]);
      tma_2d(sV, &tv, hk * D, ks, &bar[B2_KV]);
      tma_2d(sV + HALF, &tv, hk * D + 64, ks, &bar[B2_KV]);
    }
    int i = 0;
    for (; qt.valid(); qt.next(), ++i) {
      const int s = i % NST;
      if (i >= NST && !__all_sync(0xffffffffu, mbar_wait(&bar[B2_EMPTY + s], ((i / NST) - 1) & 1, abort, p.err, 61))) break;
      const int h = hk * G + qt.g, qe = min(qt.qs + BQ2, qt.q1);
      float* L = ld_at(s);
      for (int c = lane; c < BQ2; c += 32) {
        const bool in = qt.qs + c < qe;
        L[c] = in ? p.lse2[(long)h * p.T + qt.qs + c] : INFINITY;
        L[BQ2 + c] = in ? p.dsum[(long)h * p.T + qt.qs + c] : 0.f;
      }
      __syncwarp();
      if (lane == 0) {
        char* dst = q_at(s);
        mbar_expect_tx(&bar[B2_FULL + s], 2 * QT);
        tma_2d(dst, &tq, h * D, qt.qs, &bar[B2_FULL + s]);
        tma_2d(dst + QHALF, &tq, h * D + 64, qt.qs, &bar[B2_FULL + s]);
        tma_2d(dst + QT, &tdo, h * D, qt.qs, &bar[B2_FULL + s]);
        tma_2d(dst + QT + QHALF, &tdo, h * D + 64, qt.qs, &bar[B2_FULL + s]);
      }
      __syncwarp();
    }
    if (lane == 0 && *abort) {  // every copy this CTA started lands before its shared memory is released
      int zero = 0;
      mbar_wait(&bar[B2_KV], 0, (volatile int*)&zero, p.err, 61);
      for (int j = max(0, i - NST); j < i; ++j) mbar_wait(&bar[B2_FULL + j % NST], (j / NST) & 1, (volatile int*)&zero, p.err, 61);
    }
  } else if (warp == 13) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(BQ2, false);       // A = K / V, B = Q / dO, both K-major, N = 64
      constexpr uint32_t ID_G = idesc_bf16(D, true);          // A from TMEM, B = dO / Q MN-major, N = 128
      constexpr uint32_t ID_Q = idesc_bf16(BQ2, true, true);  // A = K^T and B = dS^T, both MN-major, N = 64
      const uint32_t k_b = s32(sK), v_b = s32(sV), ds_b = s32(sDS);
      // S^T / dP^T of block j into buffer j & 1, once its Q / dO landed and dQ^T of block j - 2
      // (same columns) has been read out
      auto sp = [&](int j) -> bool {
        const int s = j % NST, b = j & 1;
        if (!mbar_wait(&bar[B2_FULL + s], (j / NST) & 1, abort, p.err, 63)) return false;
        if (j >= 2 && !mbar_wait(&bar[B2_DQE + b], ((j - 2) >> 1) & 1, abort, p.err, 65)) return false;
        tc_fence_after();
        const uint32_t q_b = s32(q_at(s)), do_b = q_b + QT, cs = tmem + b * C2_BUF;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {  // K = head dim
          const uint32_t ak = (kk >> 2) * HALF + (kk & 3) * 32, bk = (kk >> 2) * QHALF + (kk & 3) * 32;
          tc_mma(cs, sdesc(k_b + ak, 16, 1024), sdesc(q_b + bk, 16, 1024), ID_S, kk > 0);
          tc_mma(cs + C2_DP, sdesc(v_b + ak, 16, 1024), sdesc(do_b + bk, 16, 1024), ID_S, kk > 0);
        }
        tc_commit(&bar[B2_S + b]);
        return true;
      };
      bool ok = mbar_wait(&bar[B2_KV], 0, abort, p.err, 62);
      int n = 0;  // blocks of this CTA
      for (QTiles c = qt; c.valid(); c.next()) ++n;
      if (ok && n > 0) ok = sp(0);
      for (int i = 0; ok && i < n; ++i) {
        const int s = i % NST, b = i & 1;
        if (i + 1 < n && !(ok = sp(i + 1))) break;
        if (!(ok = mbar_wait(&bar[B2_P + b], (i >> 1) & 1, abort, p.err, 64))) break;
        tc_fence_after();
        const uint32_t q_b = s32(q_at(s)), do_b = q_b + QT, cs = tmem + b * C2_BUF;
#pragma unroll
        for (int kk = 0; kk < BQ2 / 16; ++kk) {  // dV += P^T dO, dK += dS^T Q (K = q rows; P^T, dS^T from TMEM)
          tc_mma_ts(tmem + C2_DV, cs + kk * 8, sdesc(do_b + kk * 2048, QHALF, 1024), ID_G, (i > 0 || kk > 0));
          tc_mma_ts(tmem + C2_DK, cs + C2_DP + kk * 8, sdesc(q_b + kk * 2048, QHALF, 1024), ID_G, (i > 0 || kk > 0));
        }
        tc_commit(&bar[B2_EMPTY + s]);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)  // dQ^T = K^T dS^T (K = keys), over S^T of this buffer
          tc_mma(cs, sdesc(k_b + kk * 2048, HALF, 1024), sdesc(ds_b + b * DST + kk * 2048, DST, 1024), ID_Q, kk > 0);
        tc_commit(&bar[B2_DQF + b]);
      }
      if (ok) tc_commit(&bar[B2_DONE]);
      tc_commit(&bar[B2_DRAIN]);
      int zero = 0;
      mbar_wait(&bar[B2_DRAIN], 0, (volatile int*)&zero, p.err, 66);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ element-wise gradient (TMEM lane = key)
    const int wq = warp & 3, half = warp >> 2;
    const int r = wq * 32 + lane;
    const int key = ks + r;
    const uint32_t lane_addr = tmem + ((uint32_t)(wq * 32) << 16);
    const int c0 = half * 32;  // this warp's q columns
    int i = 0;
    for (; qt.valid(); qt.next(), ++i) {
      const int s = i % NST, b = i & 1;
      const int qs = qt.qs, qe = min(qs + BQ2, qt.q1);
      const int climit = key < ke ? qe - qs : 0;
      const int cfirst = qt.ty == 1 ? max(0, (key - k0s) - (qs - qt.q0)) : 0;
      if (!__all_sync(0xffffffffu, mbar_wait(&bar[B2_S + b], (i >> 1) & 1, abort, p.err, 67))) break;
      // the stage's lse2 / Dsum were stored by the producer's lanes before its arrival on FULL
      if (!__all_sync(0xffffffffu, mbar_wait(&bar[B2_FULL + s], (i / NST) & 1, abort, p.err, 67))) break;
      // dS^T buffer b is free once dQ of block i - 2 has been computed
      if (i >= 2 && !__all_sync(0xffffffffu, mbar_wait(&bar[B2_DQF + b], ((i - 2) >> 1) & 1, abort, p.err, 68))) break;
      tc_fence_after();
      const float* L = ld_at(s);
      const float* Ds = L + BQ2;
      const uint32_t cs = lane_addr + b * C2_BUF;
      char* dsrow = sDS + b * DST + (r >> 3) * 1024 + (r & 7) * 128;
      float sv[32], dp[32];
      tmem_ld32(cs + c0, sv);
      tmem_ld32(cs + C2_DP + c0, dp);
      uint32_t pw[16], dw[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float pv[2], dv2[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = c0 + e + u;
          const bool vis = c >= cfirst && c < climit;
          const float pr = vis ? ex2_fast(fmaf(sv[e + u], p.scale_log2, -L[c])) : 0.f;
          pv[u] = pr;
          dv2[u] = vis ? pr * (dp[e + u] - Ds[c]) * p.scale : 0.f;
        }
        bf162 a2 = __floats2bfloat162_rn(pv[0], pv[1]), d2 = __floats2bfloat162_rn(dv2[0], dv2[1]);
        pw[e / 2] = *reinterpret_cast<uint32_t*>(&a2);
        dw[e / 2] = *reinterpret_cast<uint32_t*>(&d2);
      }
      tmem_st16u(cs + half * 16, pw);          // P^T (bf16 pairs) over the consumed S^T columns
      tmem_st16u(cs + C2_DP + half * 16, dw);  // dS^T over dP^T
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {  // dS^T row r, q columns c0 + 8 q8 .. +7: 16-byte chunk (half*4 + q8) of the 128-byte row
        const int ch = half * 4 + q8;
        *reinterpret_cast<uint4*>(dsrow + ((ch ^ (r & 7)) << 4)) = make_uint4(dw[q8 * 4], dw[q8 * 4 + 1], dw[q8 * 4 + 2], dw[q8 * 4 + 3]);
      }
      tmem_st_wait();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // dS^T visible to the tensor cores
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B2_P + b]);
    }
  } else {
    // ------------------------------------------------------------ dQ read-out (TMEM lane = head dim), then dK / dV
    const int wq = warp - 8;
    const int d = wq * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(wq * 32) << 16);
    int i = 0;
    bool ok = true;
    for (; qt.valid(); qt.next(), ++i) {
      const int b = i & 1;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&bar[B2_DQF + b], (i >> 1) & 1, abort, p.err, 69)))) break;
      tc_fence_after();
      const int h = hk * G + qt.g, qs = qt.qs, n = min(qs + BQ2, qt.q1) - qs;
      float* dq = p.dq_acc + ((long)qs * p.Hq + h) * D + d;
      const long rstride = (long)p.Hq * D;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        float v[32];
        tmem_ld32(lane_addr + b * C2_BUF + hh * 32, v);
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (hh * 32 + c < n) red_add_f32(dq + (hh * 32 + c) * rstride, v[c]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[B2_DQE + b]);
    }
    ok = ok && __all_sync(0xffffffffu, !*abort) && i > 0;
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar[B2_DONE], 0, abort, p.err, 70));
    if (ok) {  // TMEM lane = key for dK / dV
      tc_fence_after();
      const int key = ks + d;
      bf16* dkr = p.dk + ((long)key * p.Hkv + hk) * D;
      bf16* dvr = p.dv + ((long)key * p.Hkv + hk) * D;
#pragma unroll 1
      for (int cc = 0; cc < D; cc += 32) {
        float a[32], bb[32];
        tmem_ld32(lane_addr + C2_DK + cc, a);
        tmem_ld32(lane_addr + C2_DV + cc, bb);
        if (key < ke) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            float fa[8], fb[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              fa[u] = a[e + u];
              fb[u] = bb[e + u];
            }
            store8(dkr + cc + e, fa);
            store8(dvr + cc + e, fb);
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 13) {
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

static CUtensorMap map_rows(const void* base, long rows, long width, int box_rows = 128) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)width * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
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

}  // namespace atb

// The key-tile part of the backward: dq_acc (fp32, zeroed by the caller) += dQ, dk / dv (zeroed) = dK / dV.
// tiles: (n, 2) int32 (kseg index, 128-key tile start); dsum = rowsum(dO o O) (Hq, T).
// AXRL_ATTN_BWD_BLOCKS=64 selects attn_bwd_tc2_k (64-row q blocks through a 3-stage ring, dQ read out
// by separate warps); set_attn_bwd_blocks64 switches it at run time.
static int& bwd_blocks64_flag() {
  static int on = [] {
    const char* e = std::getenv("AXRL_ATTN_BWD_BLOCKS");
    return (e && std::string(e) == "64") ? 1 : 0;
  }();
  return on;
}
static bool bwd_blocks64() { return bwd_blocks64_flag() != 0; }
void set_attn_bwd_blocks64(bool on) { bwd_blocks64_flag() = on ? 1 : 0; }
// The 128-row kernel runs with Q / dO double-buffered and P^T in tensor memory (468 against 434
// TFLOP/s single-buffered on the 15 872-token Qwen3-8B pack); AXRL_ATTN_BWD_DBL=0 selects the latter.
static int& bwd_dbl_flag() {
  static int on = [] {
    const char* e = std::getenv("AXRL_ATTN_BWD_DBL");
    return (e && std::string(e) == "0") ? 0 : 1;
  }();
  return on;
}
static bool bwd_dbl() { return bwd_dbl_flag() != 0; }
void set_attn_bwd_dbl(bool on) { bwd_dbl_flag() = on ? 1 : 0; }

void attn_bwd_tc_tiles(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor lse2, at::Tensor dsum, at::Tensor dq_acc,
                       at::Tensor dk, at::Tensor dv, at::Tensor kseg, at::Tensor qr, at::Tensor tiles, double scale) {
  using namespace atb;
  const int T = q.size(0), Hq = q.size(1), Tk = k.size(0), Hkv = k.size(1);
  const int nt = tiles.size(0);
  // grid (heads, tiles): blocks start in index order, so the heaviest tiles (first in the table) of
  // every head start first
  AX_CHECK(nt <= 65535, "attention: at most 65535 tiles per launch");
  if (nt == 0 || T == 0 || Tk == 0) return;
  AX_CHECK(q.size(2) == D && k.size(2) == D && dout.sizes() == q.sizes() && k.sizes() == v.sizes(), "attention backward shapes");
  const CUtensorMap tq = map_rows(q.data_ptr(), T, (long)Hq * D);
  const CUtensorMap tdo = map_rows(dout.data_ptr(), T, (long)Hq * D);
  const CUtensorMap tk = map_rows(k.data_ptr(), Tk, (long)Hkv * D);
  const CUtensorMap tv = map_rows(v.data_ptr(), Tk, (long)Hkv * D);
  Params p{lse2.data_ptr<float>(), dsum.data_ptr<float>(), dq_acc.data_ptr<float>(), (bf16*)dk.data_ptr(), (bf16*)dv.data_ptr(),
           kseg.data_ptr<int>(), qr.data_ptr<int>(), tiles.data_ptr<int>(), Hq, Hkv, T, (float)(scale * 1.4426950408889634), (float)scale,
           err_flag(q.get_device()).data_ptr<int>()};
  if (bwd_blocks64()) {
    using namespace atb2;
    const CUtensorMap tq64 = map_rows(q.data_ptr(), T, (long)Hq * D, BQ2);
    const CUtensorMap tdo64 = map_rows(dout.data_ptr(), T, (long)Hq * D, BQ2);
    const int smem2 = 2 * TILE + NST * 2 * QT + 2 * DST + NST * 2 * BQ2 * 4 + NBAR2 * 8 + 16 + 1024;
    smem_attr(reinterpret_cast<const void*>(attn_bwd_tc2_k), smem2);
    attn_bwd_tc2_k<<<dim3(Hkv, nt), THREADS2, smem2, stream()>>>(tq64, tk, tv, tdo64, p);
    AX_LAUNCH_OK();
    return;
  }
  if (bwd_dbl()) {
    const int smem_d = 7 * TILE + 4 * BQ * 4 + NBAR * 8 + 16;  // the base is 1024-byte aligned (checked in the kernel)
    smem_attr(reinterpret_cast<const void*>(attn_bwd_tc_k<true>), smem_d);
    attn_bwd_tc_k<true><<<dim3(Hkv, nt), THREADS, smem_d, stream()>>>(tq, tk, tv, tdo, p);
    AX_LAUNCH_OK();
    return;
  }
  const int smem = 6 * TILE + 4 * BQ * 4 + NBAR * 8 + 16 + 1024;
  smem_attr(reinterpret_cast<const void*>(attn_bwd_tc_k<false>), smem);
  attn_bwd_tc_k<false><<<dim3(Hkv, nt), THREADS, smem, stream()>>>(tq, tk, tv, tdo, p);
  AX_LAUNCH_OK();
}

int64_t attn_bwd_tc_error() { return atb::err_flag(c10::cuda::current_device()).item<int>(); }

}  // namespace ax
