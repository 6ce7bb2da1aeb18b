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

constexpr int B_KV = 0, B_QD = 1, B_S = 2, B_P = 3, B_MM = 4, B_DQF = 5, B_DRAIN = 6, B_LD = 7, NBAR = 8;

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
    qs += BQ;
    if (qs >= q1) {
      ++it;
      seek();
    }
  }
};

__global__ void __launch_bounds__(THREADS, 1) attn_bwd_tc_k(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                                                          const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                                                          Params p) {
  extern __shared__ char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  char* sK = sm;
  char* sV = sm + TILE;
  char* sQ = sm + 2 * TILE;
  char* sdO = sm + 3 * TILE;
  char* sP = sm + 4 * TILE;   // P^T  [key][q]
  char* sdS = sm + 5 * TILE;  // dS^T [key][q]
  float* sL = reinterpret_cast<float*>(sm + 6 * TILE);  // [tile parity][q column]: lse2
  float* sDs = sL + 2 * BQ;                              // [tile parity][q column]: Dsum
  uint64_t* bar = reinterpret_cast<uint64_t*>(sDs + 2 * BQ);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBAR);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = p.tiles[blockIdx.x * 2], ks = p.tiles[blockIdx.x * 2 + 1];
  const int hk = blockIdx.y, G = p.Hq / p.Hkv;
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

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_expect_tx(&bar[B_KV], 2 * TILE);
      tma_2d(sK, &tk, hk * D, ks, &bar[B_KV]);
      tma_2d(sK + HALF, &tk, hk * D + 64, ks, &bar[B_KV]);
      tma_2d(sV, &tv, hk * D, ks, &bar[B_KV]);
      tma_2d(sV + HALF, &tv, hk * D + 64, ks, &bar[B_KV]);
      int i = 0;
      for (; qt.valid(); qt.next(), ++i) {
        if (i >= 1 && !mbar_wait(&bar[B_MM], (i - 1) & 1, abort, p.err, 11)) break;  // Q / dO of the previous tile consumed
        const int h = hk * G + qt.g;
        mbar_expect_tx(&bar[B_QD], 2 * TILE);
        tma_2d(sQ, &tq, h * D, qt.qs, &bar[B_QD]);
        tma_2d(sQ + HALF, &tq, h * D + 64, qt.qs, &bar[B_QD]);
        tma_2d(sdO, &tdo, h * D, qt.qs, &bar[B_QD]);
        tma_2d(sdO + HALF, &tdo, h * D + 64, qt.qs, &bar[B_QD]);
      }
      if (*abort) {  // every copy this CTA started lands before its shared memory is released
        int zero = 0;
        mbar_wait(&bar[B_KV], 0, (volatile int*)&zero, p.err, 11);
        if (i >= 1) mbar_wait(&bar[B_QD], (i - 1) & 1, (volatile int*)&zero, p.err, 11);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_KMAJ = idesc_bf16(128, false), ID_BMN = idesc_bf16(128, true), ID_ABMN = idesc_bf16(128, true, true);
      const uint32_t k_b = s32(sK), v_b = s32(sV), q_b = s32(sQ), do_b = s32(sdO), p_b = s32(sP), ds_b = s32(sdS);
      bool ok = mbar_wait(&bar[B_KV], 0, abort, p.err, 12);
      int i = 0;
      for (; ok && qt.valid(); qt.next(), ++i) {
        if (!mbar_wait(&bar[B_QD], i & 1, abort, p.err, 12)) break;
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
          tc_mma(tmem + C_DV, sdesc(p_b + a_off, 16, 1024), sdesc(do_b + kk * 2048, HALF, 1024), ID_BMN, (i > 0 || kk > 0));
          tc_mma(tmem + C_DK, sdesc(ds_b + a_off, 16, 1024), sdesc(q_b + kk * 2048, HALF, 1024), ID_BMN, (i > 0 || kk > 0));
        }
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
      // stage the tile's lse2 / Dsum once (thread (half, r) loads column r of its half's copy)
      {
        float* L = sL + (i & 1) * BQ;
        float* Ds = sDs + (i & 1) * BQ;
        if (half == 0) L[r] = qs + r < qe ? p.lse2[(long)h * p.T + qs + r] : 0.f;
        else Ds[r] = qs + r < qe ? p.dsum[(long)h * p.T + qs + r] : 0.f;
        mbar_arrive(&bar[B_LD]);
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_LD], i & 1, abort, p.err, 17))) break;
      if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_S], i & 1, abort, p.err, 15))) break;
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
            const float pr = vis ? exp2f(s[e + u] * p.scale_log2 - L[c]) : 0.f;
            pv[u] = pr;
            dv2[u] = vis ? pr * (dp[e + u] - Ds[c]) * p.scale : 0.f;
          }
          bf162 a = __floats2bfloat162_rn(pv[0], pv[1]), b = __floats2bfloat162_rn(dv2[0], dv2[1]);
          pw[e / 2] = *reinterpret_cast<uint32_t*>(&a);
          dw[e / 2] = *reinterpret_cast<uint32_t*>(&b);
        }
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {  // 4 chunks of 8 q columns, 128-byte swizzled rows of this half's box
          const int ch = (cc >> 3) + q8;  // 16-byte chunk index within the 64-column box
          const int off = ((ch ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(prow + off) = make_uint4(pw[q8 * 4], pw[q8 * 4 + 1], pw[q8 * 4 + 2], pw[q8 * 4 + 3]);
          *reinterpret_cast<uint4*>(dsrow + off) = make_uint4(dw[q8 * 4], dw[q8 * 4 + 1], dw[q8 * 4 + 2], dw[q8 * 4 + 3]);
        }
      }
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

}  // namespace atb

// The key-tile part of the backward: dq_acc (fp32, zeroed by the caller) += dQ, dk / dv (zeroed) = dK / dV.
// tiles: (n, 2) int32 (kseg index, 128-key tile start); dsum = rowsum(dO o O) (Hq, T).
void attn_bwd_tc_tiles(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor lse2, at::Tensor dsum, at::Tensor dq_acc,
                       at::Tensor dk, at::Tensor dv, at::Tensor kseg, at::Tensor qr, at::Tensor tiles, double scale) {
  using namespace atb;
  const int T = q.size(0), Hq = q.size(1), Tk = k.size(0), Hkv = k.size(1);
  const int nt = tiles.size(0);
  if (nt == 0 || T == 0 || Tk == 0) return;
  AX_CHECK(q.size(2) == D && k.size(2) == D && dout.sizes() == q.sizes() && k.sizes() == v.sizes(), "attention backward shapes");
  const CUtensorMap tq = map_rows(q.data_ptr(), T, (long)Hq * D);
  const CUtensorMap tdo = map_rows(dout.data_ptr(), T, (long)Hq * D);
  const CUtensorMap tk = map_rows(k.data_ptr(), Tk, (long)Hkv * D);
  const CUtensorMap tv = map_rows(v.data_ptr(), Tk, (long)Hkv * D);
  Params p{lse2.data_ptr<float>(), dsum.data_ptr<float>(), dq_acc.data_ptr<float>(), (bf16*)dk.data_ptr(), (bf16*)dv.data_ptr(),
           kseg.data_ptr<int>(), qr.data_ptr<int>(), tiles.data_ptr<int>(), Hq, Hkv, T, (float)(scale * 1.4426950408889634), (float)scale,
           err_flag(q.get_device()).data_ptr<int>()};
  const int smem = 6 * TILE + 4 * BQ * 4 + NBAR * 8 + 16 + 1024;
  smem_attr(reinterpret_cast<const void*>(attn_bwd_tc_k), smem);
  attn_bwd_tc_k<<<dim3(nt, Hkv), THREADS, smem, stream()>>>(tq, tk, tv, tdo, p);
  AX_LAUNCH_OK();
}

int64_t attn_bwd_tc_error() { return atb::err_flag(c10::cuda::current_device()).item<int>(); }

}  // namespace ax
