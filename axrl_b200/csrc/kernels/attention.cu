// Range-list flash attention, forward and backward, head_dim 128, bf16 in / fp32 accumulate.
//
// The problem is a set of (q-range, k-range, type) triples over one packed token buffer
// (type 0 = full, 1 = causal relative to the range starts) — the vocabulary of the
// reference's MagiAttention calls (axrl/utils/megatron/magi_forward.py:445-466) and of TE
// THD varlen attention (axrl/utils/megatron/model_forward.py:89-94).  Flat causal packing,
// prefix trees and CP-local shards are all expressed this way.
//
// Forward: one CTA per (128-row q tile, q head); 8 warps x 16 rows; online softmax across
// every k-range of the tile's q-segment; K/V tiles of 64 keys double-buffered with cp.async.
// Backward: one CTA per (64-key k tile, kv head); 4 warps x 16 keys; loops over every q head
// of the GQA group and every q tile that sees the k tile; dK/dV in registers, dQ through
// fp32 atomics.  Scores use exp2 with the softmax scale folded into log2(e).
//
// Tensor-core path: mma.sync m16n8k16 (bf16).  Shared memory rows of 128 bf16 are stored
// with a 16-byte-chunk XOR swizzle (chunk ^ row%8) so ldmatrix is conflict-free.
#include <string>

#include "common.cuh"

namespace ax {
namespace attn {

constexpr int D = 128;
constexpr int FWD_BM = 128;
constexpr int FWD_BN = 64;
constexpr int BWD_BN = 64;
constexpr int BWD_BM = 64;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Swizzled byte offset of element (row, col) in a [rows][128] bf16 tile.
__device__ __forceinline__ int swz(int row, int col) {
  int chunk = (col >> 3) ^ (row & 7);
  return row * (D * 2) + chunk * 16 + (col & 7) * 2;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  uint32_t s = smem_u32(smem);
  int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  bf162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Load `rows` x 128 bf16 rows (global row stride `gstride` elements) into a swizzled tile.
// Rows with index >= valid_rows are zero-filled.
__device__ __forceinline__ void load_tile(char* sm, const bf16* g, long gstride, int rows, int valid_rows, int tid, int nthr) {
  for (int i = tid; i < rows * 16; i += nthr) {
    int r = i >> 4, c = (i & 15) * 8;
    bool ok = r < valid_rows;
    const bf16* src = ok ? g + (long)r * gstride + c : g;
    cp_async16(sm + swz(r, c), src, ok);
  }
}

// ------------------------------------------------------------------------------------ forward
struct FwdParams {
  const bf16* q;  // (T, Hq, D)
  const bf16* k;  // (T, Hkv, D)
  const bf16* v;
  bf16* o;
  float* lse2;  // (Hq, T): log2-domain log-sum-exp of scaled scores (+inf for rows with no keys)
  const int* qseg;   // (Nq, 4): q0, q1, first, last
  const int* kr;     // (Nk, 3): k0, k1, type
  const int* tiles;  // (Ntiles, 2): qseg index, q tile start
  int Hq, Hkv, T;
  float scale_log2;
};

__global__ void __launch_bounds__(256, 1) attn_fwd_k(FwdParams p) {
  extern __shared__ __align__(128) char smem[];
  char* sQ = smem;
  char* sK = smem + FWD_BM * D * 2;
  char* sV = sK + 2 * FWD_BN * D * 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = p.tiles[blockIdx.x * 2], qs = p.tiles[blockIdx.x * 2 + 1];
  const int h = blockIdx.y, hk = h / (p.Hq / p.Hkv);
  const int q0 = p.qseg[seg * 4], q1 = p.qseg[seg * 4 + 1], r_first = p.qseg[seg * 4 + 2], r_last = p.qseg[seg * 4 + 3];
  const int qe = min(qs + FWD_BM, q1);
  const long qstride = (long)p.Hq * D, kstride = (long)p.Hkv * D;

  load_tile(sQ, p.q + (long)qs * qstride + (long)h * D, qstride, FWD_BM, qe - qs, tid, 256);
  cp_commit();

  // Tile iterator over all k-ranges of this q segment.
  auto range_end = [&](int r) {
    int k0 = p.kr[r * 3], k1 = p.kr[r * 3 + 1], ty = p.kr[r * 3 + 2];
    return ty == 1 ? min(k1, k0 + (qe - q0)) : k1;
  };
  int lr = r_first, lks = lr < r_last ? p.kr[lr * 3] : 0;  // loader position
  auto advance = [&](int& r, int& ks) {
    ks += FWD_BN;
    while (r < r_last && ks >= range_end(r)) {
      ++r;
      if (r < r_last) ks = p.kr[r * 3];
    }
  };
  // skip empty leading ranges
  while (lr < r_last && lks >= range_end(lr)) {
    ++lr;
    if (lr < r_last) lks = p.kr[lr * 3];
  }
  int stage = 0;
  if (lr < r_last) {
    int kend = range_end(lr);
    load_tile(sK, p.k + (long)lks * kstride + (long)hk * D, kstride, FWD_BN, kend - lks, tid, 256);
    load_tile(sV, p.v + (long)lks * kstride + (long)hk * D, kstride, FWD_BN, kend - lks, tid, 256);
  }
  cp_commit();

  // Q fragments (16 rows per warp)
  cp_wait<1>();
  __syncthreads();
  uint32_t qf[8][4];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    int row = warp * 16 + (lane & 15), col = kk * 16 + (lane >> 4) * 8;
    ldsm_x4(smem_u32(sQ + swz(row, col)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }

  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const int row_a = qs + warp * 16 + (lane >> 2);  // absolute q index of c0/c1; c2/c3 is +8

  int cr = lr, cks = lks;
  while (cr < r_last) {
    // prefetch next tile
    int nr = cr, nks = cks;
    advance(nr, nks);
    if (nr < r_last) {
      int kend = range_end(nr);
      char* dK = sK + (stage ^ 1) * FWD_BN * D * 2;
      char* dV = sV + (stage ^ 1) * FWD_BN * D * 2;
      load_tile(dK, p.k + (long)nks * kstride + (long)hk * D, kstride, FWD_BN, kend - nks, tid, 256);
      load_tile(dV, p.v + (long)nks * kstride + (long)hk * D, kstride, FWD_BN, kend - nks, tid, 256);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();

    const char* cK = sK + stage * FWD_BN * D * 2;
    const char* cV = sV + stage * FWD_BN * D * 2;
    const int k0 = p.kr[cr * 3], k1 = p.kr[cr * 3 + 1], ty = p.kr[cr * 3 + 2];
    // S = Q K^T  (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < 4; ++n2) {  // pairs of n-tiles (16 keys)
        uint32_t b0, b1, b2, b3;
        int key = n2 * 16 + (lane & 7) + (lane >> 4) * 8, col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(smem_u32(cK + swz(key, col)), b0, b1, b2, b3);
        mma16816(s[2 * n2], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma16816(s[2 * n2 + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
    // mask + scale
    const bool need_mask = (cks + FWD_BN > k1) || (ty == 1 && (cks + FWD_BN - 1 - k0) > (qs - q0)) || (qe - qs < FWD_BM);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[n][e] * p.scale_log2;
        if (need_mask) {
          int qi = row_a + (e >> 1) * 8;
          int kj = cks + n * 8 + (lane & 3) * 2 + (e & 1);
          bool ok = kj < k1 && qi < qe && (ty == 0 || (kj - k0) <= (qi - q0));
          x = ok ? x : -INFINITY;
        }
        s[n][e] = x;
      }
    }
    // online softmax (rows r and r+8)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * hh], s[n][2 * hh + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      float mnew = fmaxf(m[hh], mx);
      float corr = (mnew == -INFINITY) ? 1.f : exp2f(m[hh] - mnew);
      float msub = (mnew == -INFINITY) ? 0.f : mnew;
      float rs = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        float a = exp2f(s[n][2 * hh] - msub), b = exp2f(s[n][2 * hh + 1] - msub);
        s[n][2 * hh] = a;
        s[n][2 * hh + 1] = b;
        rs += a + b;
      }
      l[hh] = l[hh] * corr + rs;
      m[hh] = mnew;
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        acc[d][2 * hh] *= corr;
        acc[d][2 * hh + 1] *= corr;
      }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step
      uint32_t a0 = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      uint32_t a1 = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      uint32_t a2 = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      uint32_t a3 = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int d2 = 0; d2 < 8; ++d2) {  // pairs of 8-dim n-tiles
        uint32_t b0, b1, b2, b3;
        int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, col = d2 * 16 + (lane >> 4) * 8;
        ldsm_x4_t(smem_u32(cV + swz(key, col)), b0, b1, b2, b3);
        mma16816(acc[2 * d2], a0, a1, a2, a3, b0, b1);
        mma16816(acc[2 * d2 + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // everyone done with this stage before it is overwritten
    stage ^= 1;
    cr = nr;
    cks = nks;
  }
  cp_wait<0>();

  // finalize
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float ls = l[hh];
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    int qi = row_a + hh * 8;
    float inv = ls > 0.f ? 1.f / ls : 0.f;
    if (qi < qe) {
      bf16* orow = p.o + (long)qi * qstride + (long)h * D;
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        int col = d * 8 + (lane & 3) * 2;
        *reinterpret_cast<bf162*>(orow + col) = __floats2bfloat162_rn(acc[d][2 * hh] * inv, acc[d][2 * hh + 1] * inv);
      }
      if ((lane & 3) == 0) p.lse2[(long)h * p.T + qi] = ls > 0.f ? m[hh] + log2f(ls) : INFINITY;
    }
  }
}

// ------------------------------------------------------------------------------------ backward
// Dsum[h, i] = sum_d dO[i,h,d] * O[i,h,d]
__global__ void attn_bwd_pre_k(const bf16* __restrict__ o, const bf16* __restrict__ dout, float* __restrict__ dsum, int T, int Hq) {
  int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= T * Hq) return;
  int t = w / Hq, h = w % Hq;
  const bf16* a = o + ((long)t * Hq + h) * D + lane * 4;
  const bf16* b = dout + ((long)t * Hq + h) * D + lane * 4;
  float2 a0 = __bfloat1622float2(*reinterpret_cast<const bf162*>(a));
  float2 a1 = __bfloat1622float2(*reinterpret_cast<const bf162*>(a + 2));
  float2 b0 = __bfloat1622float2(*reinterpret_cast<const bf162*>(b));
  float2 b1 = __bfloat1622float2(*reinterpret_cast<const bf162*>(b + 2));
  float s = warp_sum(a0.x * b0.x + a0.y * b0.y + a1.x * b1.x + a1.y * b1.y);
  if (lane == 0) dsum[(long)h * T + t] = s;
}

struct BwdParams {
  const bf16 *q, *k, *v, *dout;
  const float *lse2, *dsum;
  float* dq_acc;  // (T, Hq, D) fp32
  bf16 *dk, *dv;  // (T, Hkv, D)
  const int* kseg;   // (Nk, 4): k0, k1, first, last
  const int* qr;     // (Nitems, 3): q0, q1, type
  const int* tiles;  // (Ntiles, 2): kseg index, k tile start
  int Hq, Hkv, T;
  float scale_log2, scale;
  int skip_dq;  // dQ computed by attn_bwd_dq_k instead (deterministic mode)
};

__global__ void __launch_bounds__(128, 2) attn_bwd_k(BwdParams p) {
  extern __shared__ __align__(128) char smem[];
  char* sK = smem;                      // 64 x 128
  char* sV = sK + BWD_BN * D * 2;       // 64 x 128
  char* sQ = sV + BWD_BN * D * 2;       // 64 x 128
  char* sdO = sQ + BWD_BM * D * 2;      // 64 x 128
  bf16* sdS = reinterpret_cast<bf16*>(sdO + BWD_BM * D * 2);  // [key 64][q 64 + 8 pad]
  float* sL = reinterpret_cast<float*>(sdS + BWD_BN * (BWD_BM + 8));  // 64
  float* sDs = sL + BWD_BM;                                            // 64
  constexpr int DS_LD = BWD_BM + 8;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = p.tiles[blockIdx.x * 2], ks = p.tiles[blockIdx.x * 2 + 1];
  const int hk = blockIdx.y, G = p.Hq / p.Hkv;
  const int k0s = p.kseg[seg * 4], k1s = p.kseg[seg * 4 + 1], it0 = p.kseg[seg * 4 + 2], it1 = p.kseg[seg * 4 + 3];
  const int ke = min(ks + BWD_BN, k1s);
  const long qstride = (long)p.Hq * D, kstride = (long)p.Hkv * D;

  load_tile(sK, p.k + (long)ks * kstride + (long)hk * D, kstride, BWD_BN, ke - ks, tid, 128);
  load_tile(sV, p.v + (long)ks * kstride + (long)hk * D, kstride, BWD_BN, ke - ks, tid, 128);
  cp_commit();
  cp_wait<0>();
  __syncthreads();

  float dk[16][4], dv[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  const int key_a = ks + warp * 16 + (lane >> 2);  // absolute key of c0/c1 rows (S^T rows are keys)

  for (int g = 0; g < G; ++g) {
    const int h = hk * G + g;
    for (int it = it0; it < it1; ++it) {
      const int q0 = p.qr[it * 3], q1 = p.qr[it * 3 + 1], ty = p.qr[it * 3 + 2];
      // first q row that can see any key of this tile
      int qstart = q0;
      if (ty == 1) qstart = q0 + max(0, ks - k0s);
      if (qstart >= q1) continue;
      for (int qs = qstart; qs < q1; qs += BWD_BM) {
        const int qe = min(qs + BWD_BM, q1);
        __syncthreads();
        load_tile(sQ, p.q + (long)qs * qstride + (long)h * D, qstride, BWD_BM, qe - qs, tid, 128);
        load_tile(sdO, p.dout + (long)qs * qstride + (long)h * D, qstride, BWD_BM, qe - qs, tid, 128);
        cp_commit();
        for (int i = tid; i < BWD_BM; i += 128) {
          int qi = qs + i;
          sL[i] = qi < qe ? p.lse2[(long)h * p.T + qi] : INFINITY;
          sDs[i] = qi < qe ? p.dsum[(long)h * p.T + qi] : 0.f;
        }
        cp_wait<0>();
        __syncthreads();

        // S^T = K Q^T : (16 keys x 64 q) per warp
        float st[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) st[n][0] = st[n][1] = st[n][2] = st[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t a0, a1, a2, a3;
          {
            int row = warp * 16 + (lane & 15), col = kk * 16 + (lane >> 4) * 8;
            ldsm_x4(smem_u32(sK + swz(row, col)), a0, a1, a2, a3);
          }
#pragma unroll
          for (int n2 = 0; n2 < 4; ++n2) {
            uint32_t b0, b1, b2, b3;
            int qrow = n2 * 16 + (lane & 7) + (lane >> 4) * 8, col = kk * 16 + ((lane >> 3) & 1) * 8;
            ldsm_x4(smem_u32(sQ + swz(qrow, col)), b0, b1, b2, b3);
            mma16816(st[2 * n2], a0, a1, a2, a3, b0, b1);
            mma16816(st[2 * n2 + 1], a0, a1, a2, a3, b2, b3);
          }
        }
        // P^T = exp2(S^T * scale_log2 - lse2[q]) with mask
        const bool need_mask = (ke - ks < BWD_BN) || (qe - qs < BWD_BM) ||
                               (ty == 1 && (ks + BWD_BN - 1 - k0s) > (qs - q0));
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            int ql = n * 8 + (lane & 3) * 2 + (e & 1);
            int kj = key_a + (e >> 1) * 8;
            float x = st[n][e] * p.scale_log2 - sL[ql];
            bool ok = true;
            if (need_mask) {
              int qi = qs + ql;
              ok = kj < ke && qi < qe && (ty == 0 || (kj - k0s) <= (qi - q0));
            }
            st[n][e] = ok ? exp2f(x) : 0.f;
          }
        }
        // dV += P^T dO   (A = P^T from regs, B = dO [q][d] via ldmatrix.trans)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          uint32_t a0 = pack_bf16(st[2 * kk][0], st[2 * kk][1]);
          uint32_t a1 = pack_bf16(st[2 * kk][2], st[2 * kk][3]);
          uint32_t a2 = pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]);
          uint32_t a3 = pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
          for (int d2 = 0; d2 < 8; ++d2) {
            uint32_t b0, b1, b2, b3;
            int qrow = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, col = d2 * 16 + (lane >> 4) * 8;
            ldsm_x4_t(smem_u32(sdO + swz(qrow, col)), b0, b1, b2, b3);
            mma16816(dv[2 * d2], a0, a1, a2, a3, b0, b1);
            mma16816(dv[2 * d2 + 1], a0, a1, a2, a3, b2, b3);
          }
        }
        // dP^T = V dO^T  (16 keys x 64 q)
        float dpt[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) dpt[n][0] = dpt[n][1] = dpt[n][2] = dpt[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t a0, a1, a2, a3;
          {
            int row = warp * 16 + (lane & 15), col = kk * 16 + (lane >> 4) * 8;
            ldsm_x4(smem_u32(sV + swz(row, col)), a0, a1, a2, a3);
          }
#pragma unroll
          for (int n2 = 0; n2 < 4; ++n2) {
            uint32_t b0, b1, b2, b3;
            int qrow = n2 * 16 + (lane & 7) + (lane >> 4) * 8, col = kk * 16 + ((lane >> 3) & 1) * 8;
            ldsm_x4(smem_u32(sdO + swz(qrow, col)), b0, b1, b2, b3);
            mma16816(dpt[2 * n2], a0, a1, a2, a3, b0, b1);
            mma16816(dpt[2 * n2 + 1], a0, a1, a2, a3, b2, b3);
          }
        }
        // dS^T = P^T * (dP^T - Dsum[q]) * scale ; stash to smem for dQ
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            int ql = n * 8 + (lane & 3) * 2 + (e & 1);
            st[n][e] = st[n][e] * (dpt[n][e] - sDs[ql]) * p.scale;
          }
          int kr0 = warp * 16 + (lane >> 2);
          int qc = n * 8 + (lane & 3) * 2;
          *reinterpret_cast<bf162*>(&sdS[kr0 * DS_LD + qc]) = __floats2bfloat162_rn(st[n][0], st[n][1]);
          *reinterpret_cast<bf162*>(&sdS[(kr0 + 8) * DS_LD + qc]) = __floats2bfloat162_rn(st[n][2], st[n][3]);
        }
        // dK += dS^T Q   (A = dS^T regs, B = Q [q][d] via ldmatrix.trans)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          uint32_t a0 = pack_bf16(st[2 * kk][0], st[2 * kk][1]);
          uint32_t a1 = pack_bf16(st[2 * kk][2], st[2 * kk][3]);
          uint32_t a2 = pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]);
          uint32_t a3 = pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
          for (int d2 = 0; d2 < 8; ++d2) {
            uint32_t b0, b1, b2, b3;
            int qrow = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, col = d2 * 16 + (lane >> 4) * 8;
            ldsm_x4_t(smem_u32(sQ + swz(qrow, col)), b0, b1, b2, b3);
            mma16816(dk[2 * d2], a0, a1, a2, a3, b0, b1);
            mma16816(dk[2 * d2 + 1], a0, a1, a2, a3, b2, b3);
          }
        }
        __syncthreads();
        // dQ[q, d] += sum_key dS[q, key] K[key, d]: warp w takes q rows [16w, 16w+16)
        if (!p.skip_dq) {
          float dqa[16][4];
#pragma unroll
          for (int i = 0; i < 16; ++i) dqa[i][0] = dqa[i][1] = dqa[i][2] = dqa[i][3] = 0.f;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step
            // A = dS (q rows x keys): stored transposed [key][q] -> ldmatrix.trans
            uint32_t a0, a1, a2, a3;
            {
              int key = kk * 16 + (lane & 7) + (lane >> 4) * 8;
              int qc = warp * 16 + ((lane >> 3) & 1) * 8;
              ldsm_x4_t(smem_u32(&sdS[key * DS_LD + qc]), a0, a1, a2, a3);
            }
#pragma unroll
            for (int d2 = 0; d2 < 8; ++d2) {
              uint32_t b0, b1, b2, b3;
              int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, col = d2 * 16 + (lane >> 4) * 8;
              ldsm_x4_t(smem_u32(sK + swz(key, col)), b0, b1, b2, b3);
              mma16816(dqa[2 * d2], a0, a1, a2, a3, b0, b1);
              mma16816(dqa[2 * d2 + 1], a0, a1, a2, a3, b2, b3);
            }
          }
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            int qi = qs + warp * 16 + (lane >> 2) + hh * 8;
            if (qi < qe) {
              float* dst = p.dq_acc + (long)qi * qstride + (long)h * D;
#pragma unroll
              for (int d = 0; d < 16; ++d) {
                int col = d * 8 + (lane & 3) * 2;
                atomicAdd(dst + col, dqa[d][2 * hh]);
                atomicAdd(dst + col + 1, dqa[d][2 * hh + 1]);
              }
            }
          }
        }
      }
    }
  }
  // write dK, dV for this kv head
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    int kj = key_a + hh * 8;
    if (kj < ke) {
      bf16* dkr = p.dk + (long)kj * kstride + (long)hk * D;
      bf16* dvr = p.dv + (long)kj * kstride + (long)hk * D;
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        int col = d * 8 + (lane & 3) * 2;
        *reinterpret_cast<bf162*>(dkr + col) = __floats2bfloat162_rn(dk[d][2 * hh], dk[d][2 * hh + 1]);
        *reinterpret_cast<bf162*>(dvr + col) = __floats2bfloat162_rn(dv[d][2 * hh], dv[d][2 * hh + 1]);
      }
    }
  }
}

__global__ void f32_to_bf16_k(const float* __restrict__ a, bf16* __restrict__ b, long n) {
  for (long i = (blockIdx.x * (long)blockDim.x + threadIdx.x) * 4; i < n; i += (long)gridDim.x * blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4*>(a + i);
    *reinterpret_cast<bf162*>(b + i) = __floats2bfloat162_rn(v.x, v.y);
    *reinterpret_cast<bf162*>(b + i + 2) = __floats2bfloat162_rn(v.z, v.w);
  }
}

// Merge of split-key partials (o_s, lse2_s), s < P, of the same queries: lse2 = log2(sum 2^lse2_s)
// over the sources that saw keys (lse2_s = +inf marks a row with no keys in source s), o = sum
// o_s * 2^(lse2_s - lse2).  One warp per (token, head) row, four bf16 per lane.
constexpr int MERGE_MAX = 16;
struct MergeParams {
  const bf16* o[MERGE_MAX];
  const float* lse[MERGE_MAX];
  bf16* out;
  float* lse_out;
  int P, T, Hq;
};

__global__ void attn_merge_k(MergeParams p) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= p.T * p.Hq) return;
  const int t = w / p.Hq, h = w % p.Hq;
  const long li = (long)h * p.T + t, oi = ((long)t * p.Hq + h) * D + lane * 4;
  float m = -INFINITY;
  for (int s = 0; s < p.P; ++s) {
    const float l = p.lse[s][li];
    if (l != INFINITY) m = fmaxf(m, l);
  }
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, den = 0.f;
  if (m != -INFINITY) {
    for (int s = 0; s < p.P; ++s) {
      const float l = p.lse[s][li];
      if (l == INFINITY) continue;
      const float wgt = exp2f(l - m);
      den += wgt;
      const uint2 raw = *reinterpret_cast<const uint2*>(p.o[s] + oi);
      const float2 a = __bfloat1622float2(*reinterpret_cast<const bf162*>(&raw.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const bf162*>(&raw.y));
      acc[0] += wgt * a.x, acc[1] += wgt * a.y, acc[2] += wgt * b.x, acc[3] += wgt * b.y;
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  uint2 o;
  o.x = pack_bf16(acc[0] * inv, acc[1] * inv);
  o.y = pack_bf16(acc[2] * inv, acc[3] * inv);
  *reinterpret_cast<uint2*>(p.out + oi) = o;
  if (lane == 0) p.lse_out[li] = den > 0.f ? m + log2f(den) : INFINITY;
}

}  // namespace attn

std::vector<at::Tensor> attn_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor qseg, at::Tensor kr, at::Tensor tiles,
                                    double scale, int64_t variant);

// Forward implementation: the tcgen05 kernel (attention_tc.cu) with two q heads of a GQA group per
// CTA (588 TFLOP/s on the 15 872-token Qwen3-8B pack, against 479 for one head per CTA with 8
// softmax warps and P in tensor memory, AXRL_ATTN_FWD=tc8p, and 257 for the 4-warp variant);
// AXRL_ATTN_FWD=tc4 selects the 4-warp variant, =tc8 8 warps with P in shared memory, =tc2 the
// 4-warp double-buffered-P variant, =mma the mma.sync kernel below.
static int tc_forward_mode() {  // -1: mma.sync, else the attn_fwd_tc variant
  static int mode = [] {
    const char* e = std::getenv("AXRL_ATTN_FWD");
    const std::string v = e ? e : "";
    return v == "mma" ? -1 : v == "tc2" ? 1 : v == "tc8" ? 2 : v == "tc4" ? 0 : v == "tc8p" ? 3 : 4;
  }();
  return mode;
}
static bool use_tc_forward() { return tc_forward_mode() >= 0; }

std::vector<at::Tensor> attn_fwd_mma(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor qseg, at::Tensor kr, at::Tensor tiles,
                                     double scale);

// q: (T,Hq,128) k,v: (Tk,Hkv,128) -> o (T,Hq,128), lse2 (Hq,T)
std::vector<at::Tensor> attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor qseg, at::Tensor kr, at::Tensor tiles,
                                 double scale) {
  if (use_tc_forward()) return attn_fwd_tc(q, k, v, qseg, kr, tiles, scale, tc_forward_mode());
  return attn_fwd_mma(q, k, v, qseg, kr, tiles, scale);
}

// mma.sync forward (the pre-tcgen05 tensor-core path)
std::vector<at::Tensor> attn_fwd_mma(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor qseg, at::Tensor kr, at::Tensor tiles,
                                     double scale) {
  using namespace attn;
  AX_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.size(2) == D, "q bf16 (T,Hq,128)");
  AX_CHECK(k.is_contiguous() && v.is_contiguous() && k.sizes() == v.sizes(), "k/v layout");
  int T = q.size(0), Hq = q.size(1), Hkv = k.size(1);
  AX_CHECK(Hq % Hkv == 0, "GQA");
  auto o = at::zeros_like(q);
  auto lse2 = at::full({Hq, T}, INFINITY, q.options().dtype(at::kFloat));
  int nt = tiles.size(0);
  if (nt == 0 || T == 0) return {o, lse2};
  AX_CHECK(qseg.is_cuda() && kr.is_cuda() && tiles.is_cuda() && qseg.scalar_type() == at::kInt && kr.scalar_type() == at::kInt &&
               tiles.scalar_type() == at::kInt, "attention tables: int32 device tensors");
  auto& qseg_d = qseg;
  auto& kr_d = kr;
  FwdParams p{(const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(), (const bf16*)v.data_ptr(), (bf16*)o.data_ptr(),
              lse2.data_ptr<float>(), qseg_d.data_ptr<int>(), kr_d.data_ptr<int>(), tiles.data_ptr<int>(), Hq, Hkv, T,
              (float)(scale * 1.4426950408889634)};
  int smem = (FWD_BM + 4 * FWD_BN) * D * 2;
  smem_attr(reinterpret_cast<const void*>(attn_fwd_k), smem);
  attn_fwd_k<<<dim3(nt, Hq), 256, smem, stream()>>>(p);
  AX_LAUNCH_OK();
  return {o, lse2};
}

namespace attn {
// Deterministic dQ: one CTA per (128-row q tile, q head) walks every key tile of its q segment
// (the forward's iteration) and accumulates dQ = sum_j dS_j K_j in registers, so no two CTAs add
// into the same dQ row.  Per 64-key tile: S = Q K^T and dP = dO V^T (mma.sync), P = exp2(S *
// scale*log2e - lse2) (the forward's log-sum-exp; no running maximum needed), dS = P (dP - Dsum) *
// scale, dQ += dS K.  Writes bf16 dQ directly.
struct DqParams {
  const bf16 *q, *k, *v, *dout;
  const float *lse2, *dsum;
  bf16* dq;
  const int* qseg;
  const int* kr;
  const int* tiles;
  int Hq, Hkv, T;
  float scale_log2, scale;
};

__global__ void __launch_bounds__(256, 1) attn_bwd_dq_k(DqParams p) {
  extern __shared__ __align__(128) char smem[];
  char* sQ = smem;
  char* sdO = sQ + FWD_BM * D * 2;
  char* sK = sdO + FWD_BM * D * 2;
  char* sV = sK + 2 * FWD_BN * D * 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = p.tiles[blockIdx.x * 2], qs = p.tiles[blockIdx.x * 2 + 1];
  const int h = blockIdx.y, hk = h / (p.Hq / p.Hkv);
  const int q0 = p.qseg[seg * 4], q1 = p.qseg[seg * 4 + 1], r_first = p.qseg[seg * 4 + 2], r_last = p.qseg[seg * 4 + 3];
  const int qe = min(qs + FWD_BM, q1);
  const long qstride = (long)p.Hq * D, kstride = (long)p.Hkv * D;

  load_tile(sQ, p.q + (long)qs * qstride + (long)h * D, qstride, FWD_BM, qe - qs, tid, 256);
  load_tile(sdO, p.dout + (long)qs * qstride + (long)h * D, qstride, FWD_BM, qe - qs, tid, 256);
  cp_commit();

  auto range_end = [&](int r) {
    int k0 = p.kr[r * 3], k1 = p.kr[r * 3 + 1], ty = p.kr[r * 3 + 2];
    return ty == 1 ? min(k1, k0 + (qe - q0)) : k1;
  };
  int lr = r_first, lks = lr < r_last ? p.kr[lr * 3] : 0;
  auto advance = [&](int& r, int& ks) {
    ks += FWD_BN;
    while (r < r_last && ks >= range_end(r)) {
      ++r;
      if (r < r_last) ks = p.kr[r * 3];
    }
  };
  while (lr < r_last && lks >= range_end(lr)) {
    ++lr;
    if (lr < r_last) lks = p.kr[lr * 3];
  }
  int stage = 0;
  if (lr < r_last) {
    int kend = range_end(lr);
    load_tile(sK, p.k + (long)lks * kstride + (long)hk * D, kstride, FWD_BN, kend - lks, tid, 256);
    load_tile(sV, p.v + (long)lks * kstride + (long)hk * D, kstride, FWD_BN, kend - lks, tid, 256);
  }
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  uint32_t qf[8][4], of[8][4];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    int row = warp * 16 + (lane & 15), col = kk * 16 + (lane >> 4) * 8;
    ldsm_x4(smem_u32(sQ + swz(row, col)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    ldsm_x4(smem_u32(sdO + swz(row, col)), of[kk][0], of[kk][1], of[kk][2], of[kk][3]);
  }
  const int row_a = qs + warp * 16 + (lane >> 2);  // rows of c0/c1; c2/c3 are +8
  float lse[2], dsm[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int qi = row_a + hh * 8;
    lse[hh] = qi < qe ? p.lse2[(long)h * p.T + qi] : INFINITY;
    dsm[hh] = qi < qe ? p.dsum[(long)h * p.T + qi] : 0.f;
  }
  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  int cr = lr, cks = lks;
  while (cr < r_last) {
    int nr = cr, nks = cks;
    advance(nr, nks);
    if (nr < r_last) {
      int kend = range_end(nr);
      load_tile(sK + (stage ^ 1) * FWD_BN * D * 2, p.k + (long)nks * kstride + (long)hk * D, kstride, FWD_BN, kend - nks, tid, 256);
      load_tile(sV + (stage ^ 1) * FWD_BN * D * 2, p.v + (long)nks * kstride + (long)hk * D, kstride, FWD_BN, kend - nks, tid, 256);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const char* cK = sK + stage * FWD_BN * D * 2;
    const char* cV = sV + stage * FWD_BN * D * 2;
    const int k0 = p.kr[cr * 3], k1 = p.kr[cr * 3 + 1], ty = p.kr[cr * 3 + 2];
    float sc[8][4], dp[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[n][e] = dp[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < 4; ++n2) {
        uint32_t b0, b1, b2, b3, c0, c1, c2, c3;
        int key = n2 * 16 + (lane & 7) + (lane >> 4) * 8, col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(smem_u32(cK + swz(key, col)), b0, b1, b2, b3);
        ldsm_x4(smem_u32(cV + swz(key, col)), c0, c1, c2, c3);
        mma16816(sc[2 * n2], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma16816(sc[2 * n2 + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
        mma16816(dp[2 * n2], of[kk][0], of[kk][1], of[kk][2], of[kk][3], c0, c1);
        mma16816(dp[2 * n2 + 1], of[kk][0], of[kk][1], of[kk][2], of[kk][3], c2, c3);
      }
    }
    // dS = P (dP - Dsum) * scale, masked like the forward
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hh = e >> 1;
        const int qi = row_a + hh * 8;
        const int kj = cks + n * 8 + (lane & 3) * 2 + (e & 1);
        const bool ok = kj < k1 && qi < qe && (ty == 0 || (kj - k0) <= (qi - q0));
        const float pr = ok ? exp2f(sc[n][e] * p.scale_log2 - lse[hh]) : 0.f;
        sc[n][e] = pr * (dp[n][e] - dsm[hh]) * p.scale;
      }
    }
    // dQ += dS K   (A = dS from registers, B = K [key][d] via ldmatrix.trans)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a0 = pack_bf16(sc[2 * kk][0], sc[2 * kk][1]);
      uint32_t a1 = pack_bf16(sc[2 * kk][2], sc[2 * kk][3]);
      uint32_t a2 = pack_bf16(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
      uint32_t a3 = pack_bf16(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
      for (int d2 = 0; d2 < 8; ++d2) {
        uint32_t b0, b1, b2, b3;
        int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, col = d2 * 16 + (lane >> 4) * 8;
        ldsm_x4_t(smem_u32(cK + swz(key, col)), b0, b1, b2, b3);
        mma16816(acc[2 * d2], a0, a1, a2, a3, b0, b1);
        mma16816(acc[2 * d2 + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
    stage ^= 1;
    cr = nr;
    cks = nks;
  }
  cp_wait<0>();
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int qi = row_a + hh * 8;
    if (qi < qe) {
      bf16* orow = p.dq + (long)qi * qstride + (long)h * D;
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        int col = d * 8 + (lane & 3) * 2;
        *reinterpret_cast<bf162*>(orow + col) = __floats2bfloat162_rn(acc[d][2 * hh], acc[d][2 * hh + 1]);
      }
    }
  }
}
}  // namespace attn

// Deterministic mode (AXRL_DETERMINISTIC_ATTN=1 or set_attn_deterministic): dK / dV from the
// key-tile kernel without its dQ atomics, dQ from attn_bwd_dq_k.
static int& deterministic_flag() {
  static int on = [] {
    const char* e = std::getenv("AXRL_DETERMINISTIC_ATTN");
    return (e && e[0] == '1') ? 1 : 0;
  }();
  return on;
}
void set_attn_deterministic(bool on) { deterministic_flag() = on ? 1 : 0; }
bool attn_deterministic() { return deterministic_flag() != 0; }

void attn_bwd_tc_tiles(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor lse2, at::Tensor dsum, at::Tensor dq_acc,
                       at::Tensor dk, at::Tensor dv, at::Tensor kseg, at::Tensor qr, at::Tensor tiles, double scale);

// Backward implementation: the tcgen05 kernel (attention_tc_bwd.cu, 128-key tiles from
// ``tiles_tc``; 307 TFLOP/s against 157 for the mma.sync kernel on the 15 872-token Qwen3-8B
// pack); AXRL_ATTN_BWD=mma selects the mma.sync kernel below.  Deterministic mode always runs the
// mma.sync key-tile kernel without dQ atomics plus the separate dQ pass.
static int& tc_backward_flag() {
  static int on = [] {
    const char* e = std::getenv("AXRL_ATTN_BWD");
    return (e && std::string(e) == "mma") ? 0 : 1;
  }();
  return on;
}
static bool use_tc_backward() { return tc_backward_flag() != 0; }
void set_attn_bwd_tc(bool on) { tc_backward_flag() = on ? 1 : 0; }

// dK/dV of one key set and dQ added into `dq_acc` (fp32), given the softmax statistics of the whole
// row: `lse2` and `dsum` = rowsum(dO * O) of the final output.  Exact for a split over key sources,
// since every source's probabilities are 2^(S * scale * log2e - lse2) with the final lse2.
static void attn_bwd_core(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                          const at::Tensor& lse2, const at::Tensor& dsum, at::Tensor& dq_acc, at::Tensor& dk, at::Tensor& dv,
                          const at::Tensor& kseg, const at::Tensor& qr, const at::Tensor& tiles, double scale,
                          const c10::optional<at::Tensor>& tiles_tc) {
  using namespace attn;
  const int T = q.size(0), Hq = q.size(1), Hkv = k.size(1);
  if (use_tc_backward() && tiles_tc.has_value()) {
    attn_bwd_tc_tiles(dout, q, k, v, lse2, dsum, dq_acc, dk, dv, kseg, qr, *tiles_tc, scale);
    return;
  }
  const int nt = tiles.size(0);
  if (nt == 0) return;
  AX_CHECK(kseg.is_cuda() && qr.is_cuda() && tiles.is_cuda(), "attention tables must be on the device");
  BwdParams p{(const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(), (const bf16*)v.data_ptr(), (const bf16*)dout.data_ptr(),
              lse2.data_ptr<float>(), dsum.data_ptr<float>(), dq_acc.data_ptr<float>(), (bf16*)dk.data_ptr(),
              (bf16*)dv.data_ptr(), kseg.data_ptr<int>(), qr.data_ptr<int>(), tiles.data_ptr<int>(), Hq, Hkv, T,
              (float)(scale * 1.4426950408889634), (float)scale, 0};
  const int smem = (2 * BWD_BN + 2 * BWD_BM) * D * 2 + BWD_BN * (BWD_BM + 8) * 2 + 2 * BWD_BM * 4;
  smem_attr(reinterpret_cast<const void*>(attn_bwd_k), smem);
  attn_bwd_k<<<dim3(nt, Hkv), 128, smem, stream()>>>(p);
  AX_LAUNCH_OK();
}

// rowsum(dO * O) per (head, token): (Hq, T) fp32.
at::Tensor attn_bwd_dsum(at::Tensor o, at::Tensor dout) {
  using namespace attn;
  AX_CHECK(o.is_contiguous() && dout.is_contiguous() && o.sizes() == dout.sizes() && o.size(2) == D, "attn_bwd_dsum: o/dout shape");
  const int T = o.size(0), Hq = o.size(1);
  auto dsum = at::empty({Hq, T}, o.options().dtype(at::kFloat));
  const long w = (long)T * Hq;
  if (w == 0) return dsum;
  attn_bwd_pre_k<<<(w * 32 + 255) / 256, 256, 0, stream()>>>((const bf16*)o.data_ptr(), (const bf16*)dout.data_ptr(),
                                                            dsum.data_ptr<float>(), T, Hq);
  AX_LAUNCH_OK();
  return dsum;
}

// One key source of a split attention: returns (dK, dV) of that source's keys and adds its share
// of dQ into `dq_acc` ((T, Hq, 128) fp32).
std::vector<at::Tensor> attn_bwd_partial(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor lse2, at::Tensor dsum,
                                         at::Tensor dq_acc, at::Tensor kseg, at::Tensor qr, at::Tensor tiles, double scale,
                                         c10::optional<at::Tensor> tiles_tc) {
  AX_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.is_contiguous() && dq_acc.sizes() == q.sizes(), "attn_bwd_partial: dq_acc");
  AX_CHECK(lse2.size(0) == q.size(1) && lse2.size(1) == q.size(0) && dsum.sizes() == lse2.sizes(), "attn_bwd_partial: lse2/dsum");
  auto dk = at::zeros_like(k), dv = at::zeros_like(v);
  if (q.size(0) > 0 && k.size(0) > 0) attn_bwd_core(dout, q, k, v, lse2, dsum, dq_acc, dk, dv, kseg, qr, tiles, scale, tiles_tc);
  return {dk, dv};
}

// Merge the per-source partial outputs of a split attention (see attn_merge_k).
std::vector<at::Tensor> attn_merge(std::vector<at::Tensor> os, std::vector<at::Tensor> lses) {
  using namespace attn;
  const int P = (int)os.size();
  AX_CHECK(P >= 1 && P <= MERGE_MAX && (int)lses.size() == P, "attn_merge: 1..16 partials");
  const int T = os[0].size(0), Hq = os[0].size(1);
  MergeParams mp{};
  for (int s = 0; s < P; ++s) {
    AX_CHECK(os[s].is_contiguous() && os[s].sizes() == os[0].sizes() && os[s].size(2) == D && os[s].scalar_type() == at::kBFloat16,
             "attn_merge: partial outputs (T, Hq, 128) bf16");
    AX_CHECK(lses[s].is_contiguous() && lses[s].size(0) == Hq && lses[s].size(1) == T, "attn_merge: lse2 (Hq, T)");
    mp.o[s] = (const bf16*)os[s].data_ptr();
    mp.lse[s] = lses[s].data_ptr<float>();
  }
  auto out = at::empty_like(os[0]);
  auto lse = at::empty({Hq, T}, os[0].options().dtype(at::kFloat));
  mp.out = (bf16*)out.data_ptr();
  mp.lse_out = lse.data_ptr<float>();
  mp.P = P, mp.T = T, mp.Hq = Hq;
  const long w = (long)T * Hq;
  if (w == 0) return {out, lse};
  attn_merge_k<<<(w * 32 + 255) / 256, 256, 0, stream()>>>(mp);
  AX_LAUNCH_OK();
  return {out, lse};
}

std::vector<at::Tensor> attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse2,
                                 at::Tensor kseg, at::Tensor qr, at::Tensor tiles, double scale, c10::optional<at::Tensor> tiles_tc,
                                 c10::optional<at::Tensor> qseg, c10::optional<at::Tensor> kr, c10::optional<at::Tensor> fwd_tiles) {
  using namespace attn;
  int T = q.size(0), Hq = q.size(1), Hkv = k.size(1);
  auto dq_acc = at::zeros({T, Hq, D}, q.options().dtype(at::kFloat));
  auto dk = at::zeros_like(k), dv = at::zeros_like(v);
  auto dq = at::empty_like(q);
  if (T == 0) return {dq, dk, dv};
  auto dsum = at::empty({Hq, T}, q.options().dtype(at::kFloat));
  long w = (long)T * Hq;
  attn_bwd_pre_k<<<(w * 32 + 255) / 256, 256, 0, stream()>>>((const bf16*)o.data_ptr(), (const bf16*)dout.data_ptr(),
                                                            dsum.data_ptr<float>(), T, Hq);
  AX_LAUNCH_OK();
  const bool det = deterministic_flag() != 0 && fwd_tiles.has_value() && qseg.has_value() && kr.has_value();
  if (!det) attn_bwd_core(dout, q, k, v, lse2, dsum, dq_acc, dk, dv, kseg, qr, tiles, scale, tiles_tc);
  else if (tiles.size(0) > 0) {  // dK/dV by the mma.sync kernel without its dQ atomics
    AX_CHECK(kseg.is_cuda() && qr.is_cuda() && tiles.is_cuda(), "attention tables must be on the device");
    BwdParams p{(const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(), (const bf16*)v.data_ptr(), (const bf16*)dout.data_ptr(),
                lse2.data_ptr<float>(), dsum.data_ptr<float>(), dq_acc.data_ptr<float>(), (bf16*)dk.data_ptr(),
                (bf16*)dv.data_ptr(), kseg.data_ptr<int>(), qr.data_ptr<int>(), tiles.data_ptr<int>(), Hq, Hkv, T,
                (float)(scale * 1.4426950408889634), (float)scale, 1};
    const int smem = (2 * BWD_BN + 2 * BWD_BM) * D * 2 + BWD_BN * (BWD_BM + 8) * 2 + 2 * BWD_BM * 4;
    smem_attr(reinterpret_cast<const void*>(attn_bwd_k), smem);
    attn_bwd_k<<<dim3(tiles.size(0), Hkv), 128, smem, stream()>>>(p);
    AX_LAUNCH_OK();
  }
  if (det) {  // dQ owned by one CTA per q tile: no atomics, fixed summation order
    DqParams dp{(const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(), (const bf16*)v.data_ptr(), (const bf16*)dout.data_ptr(),
                lse2.data_ptr<float>(), dsum.data_ptr<float>(), (bf16*)dq.data_ptr(), qseg->data_ptr<int>(), kr->data_ptr<int>(),
                fwd_tiles->data_ptr<int>(), Hq, Hkv, T, (float)(scale * 1.4426950408889634), (float)scale};
    const int ntq = fwd_tiles->size(0);
    dq.zero_();
    if (ntq > 0) {
      const int smem = (2 * FWD_BM + 4 * FWD_BN) * D * 2;
      smem_attr(reinterpret_cast<const void*>(attn_bwd_dq_k), smem);
      attn_bwd_dq_k<<<dim3(ntq, Hq), 256, smem, stream()>>>(dp);
      AX_LAUNCH_OK();
    }
    return {dq, dk, dv};
  }
  long n = (long)T * Hq * D;
  f32_to_bf16_k<<<std::min<long>((n / 4 + 255) / 256, num_sms() * 8), 256, 0, stream()>>>(dq_acc.data_ptr<float>(),
                                                                                         (bf16*)dq.data_ptr(), n);
  AX_LAUNCH_OK();
  return {dq, dk, dv};
}

}  // namespace ax
