// Paged decode attention with a TMA page pipeline (one new query token per sequence, split-KV).
//
// Same partial buffers and combine kernel as decode_attn.cu, with larger work items: an item is a
// 512-token chunk of one sequence for one kv head (the second, chunk-granular work list that
// decode_plan writes after the 128-token one).  Every CTA of the persistent grid (one per SM)
// streams the K / V pages of ALL its items through one ring, so loads never stop at an item
// boundary:
//
//   warp 4      producer (one thread): per item the GQA group's q rows (one 2-D TMA load of
//               16 rows), then per 64-token page four 2-D TMA loads (K and V, two 64-column
//               boxes each, 128-byte swizzle; the cache viewed as (pages * Hkv * 64) rows of 128
//               values) into a 4-stage ring of 32 KB slots.
//   warps 0-3   one item at a time: the group's q heads (<= 16) are the M = 16 rows of mma.sync
//               m16n8k16; warp w takes token rows 32 (w % 2) .. +31 of pages w / 2, w / 2 + 2, ...
//               of the chunk with an online softmax across them, then the warps merge through
//               shared memory into the partial of the chunk's first 128-token split; the chunk's
//               other splits are marked empty (max -inf), which the combine skips.
//
// Per-item costs (q rows, merge, partial store) are paid once per 512 tokens instead of per 128.
// The page size must be 64.  Reference counterpart: the rollout engine's decode attention backends
// (SGLang FA3 / FlashInfer), reached via axrl/worker/sglang_worker.py:80-107.  Every wait is
// bounded: on expiry the CTA records an error code, lets its copies land and exits; the consumers
// decide to stop only after a barrier, so all four reach the same barriers.
#include <cuda.h>

#include "common.cuh"
#include "tcgen05.cuh"

namespace ax {
namespace dtm {

constexpr int D = 128, PAGE = 64, SPLIT = 128, CHUNK = 512, STAGES = 4, CW = 4, THREADS = 160;
constexpr int QBOX = 16 * 64 * 2;  // 16 q rows x 64 columns bf16 = 2 KB
constexpr int BOX = PAGE * 64 * 2;  // 64 rows x 64 columns bf16 = 8 KB
constexpr int SLOT = 4 * BOX;       // K lo, K hi, V lo, V hi
constexpr int RS = D + 2;           // merge buffer row: D outputs, max, sum

struct Params {
  const bf16* q;          // (B, Hq, D)
  const int* bt;          // (B, max_pages)
  const int* seq_lens;    // (B,)
  const int* prefix4;     // (B + 1,) items per sequence (512-token chunks), cumulative
  float* part_o;          // (B, Hq, splits, D)
  float* part_ml;         // (B, Hq, splits, 2)
  int B, Hq, Hkv, max_pages, splits, max_len;
  float scale_log2;
  int* err;
  bf16* out;  // (B, Hq, D); non-null: the combine is fused (the last chunk of a (sequence, kv head) merges)
  int* cnt;   // (B * Hkv) chunk arrival counters, zero between launches (self-cleaning)
};

__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
// byte offset of (row, col) in a page slot region of two 64-column 128-byte-swizzled boxes
__device__ __forceinline__ uint32_t pg_off(int row, int col) {
  return (uint32_t)((col >> 6) * BOX + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}
// byte offset of (row, col) in the q tile: two 64-column 128-byte-swizzled boxes of 16 rows
__device__ __forceinline__ uint32_t q_off(int row, int col) {
  return (uint32_t)((col >> 6) * QBOX + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}
__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n" : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n" : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3]) : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  bf162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

struct Item {
  int b, hk, sp, t0, len, npages, nsplits;
};
__device__ __forceinline__ Item item_of(const Params& p, int w) {
  Item it;
  it.hk = w % p.Hkv;
  const int j = w / p.Hkv;
  int lo = 0, hi = p.B - 1;  // last b with prefix4[b] <= j
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.prefix4[mid] <= j) lo = mid;
    else hi = mid - 1;
  }
  it.b = lo;
  const int c = j - p.prefix4[lo];
  it.len = min(p.seq_lens[lo], p.max_len);
  it.t0 = c * CHUNK;
  it.sp = c * (CHUNK / SPLIT);
  const int rem = it.len - it.t0;
  it.npages = rem <= 0 ? 0 : min(CHUNK / PAGE, (rem + PAGE - 1) / PAGE);
  it.nsplits = rem <= 0 ? 0 : min(CHUNK / SPLIT, (rem + SPLIT - 1) / SPLIT);
  return it;
}

// Merge of every chunk partial of (it.b, it.hk) into the output rows of the GQA group (consumer
// thread tid: row tid / 8, 16 columns from (tid % 8) * 16); resets the arrival counter.
__device__ void combine_group(const Params& p, const Item& it, int tid) {
  const int G = p.Hq / p.Hkv, r = tid >> 3, c0 = (tid & 7) * 16;
  const int nch = p.prefix4[it.b + 1] - p.prefix4[it.b];
  if (r < G) {
    const long row = (long)it.b * p.Hq + it.hk * G + r;
    float M = -INFINITY;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, __ldcg(p.part_ml + (row * p.splits + c * (CHUNK / SPLIT)) * 2));
    float L = 0.f, o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = 0.f;
    for (int c = 0; c < nch; ++c) {
      const long base = row * p.splits + c * (CHUNK / SPLIT);
      const float mc = __ldcg(p.part_ml + base * 2);
      const float f = mc == -INFINITY ? 0.f : exp2f(mc - M);
      if (f == 0.f) continue;  // an empty chunk
      L += f * __ldcg(p.part_ml + base * 2 + 1);
      const float* po = p.part_o + base * D + c0;
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(po + j));
        o[j] += f * v.x, o[j + 1] += f * v.y, o[j + 2] += f * v.z, o[j + 3] += f * v.w;
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    float f8[8];
#pragma unroll
    for (int h8 = 0; h8 < 16; h8 += 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j) f8[j] = o[h8 + j] * inv;
      store8(p.out + row * D + c0 + h8, f8);
    }
  }
  if (tid == 0) p.cnt[it.b * p.Hkv + it.hk] = 0;
}

__global__ void __launch_bounds__(THREADS, 1) decode_tma_k(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                                                        const __grid_constant__ CUtensorMap tq, Params p) {
  extern __shared__ char smem_raw[];
  char* sm = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  char* ring = sm;                                           // STAGES x SLOT
  char* sQ = ring + STAGES * SLOT;                           // 2 x (16 x 128 bf16), by item parity
  float* sRed = reinterpret_cast<float*>(sQ + 2 * 2 * QBOX);  // CW x 16 x RS
  uint64_t* full = reinterpret_cast<uint64_t*>(sRed + CW * 16 * RS);
  uint64_t* empty = full + STAGES;
  uint64_t* qfull = empty + STAGES;
  uint64_t* qempty = qfull + 2;
  volatile int* abort = reinterpret_cast<volatile int*>(qempty + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.Hq / p.Hkv;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 2);  // the two warps reading a page release it
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(&qfull[s], 1);
      tc::mbar_init(&qempty[s], CW);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_trigger();  // successors (the output projection) may become resident and stream weights now

  if (warp == CW) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      pdl_wait();  // the work list, block table and q come from the preceding kernels
      const int total = p.prefix4[p.B] * p.Hkv;
      const int G = p.Hq / p.Hkv;
      int pc = 0, n = 0;
      for (int w = blockIdx.x; w < total && !*abort; w += gridDim.x) {
        const Item it = item_of(p, w);
        if (it.npages == 0) continue;
        const int qs = n & 1;
        if (n >= 2 && !tc::mbar_wait(&qempty[qs], ((n >> 1) - 1) & 1, abort, p.err, 33)) break;
        tc::mbar_expect_tx(&qfull[qs], 2 * QBOX);
        tc::tma_2d(sQ + qs * 2 * QBOX, &tq, 0, it.b * p.Hq + it.hk * G, &qfull[qs]);
        tc::tma_2d(sQ + qs * 2 * QBOX + QBOX, &tq, 64, it.b * p.Hq + it.hk * G, &qfull[qs]);
        ++n;
        for (int pg = 0; pg < it.npages; ++pg, ++pc) {
          const int s = pc % STAGES;
          if (pc >= STAGES && !tc::mbar_wait(&empty[s], ((pc / STAGES) - 1) & 1, abort, p.err, 31)) break;
          const int page = p.bt[(long)it.b * p.max_pages + it.t0 / PAGE + pg];
          const int y = (page * p.Hkv + it.hk) * PAGE;
          tc::mbar_expect_tx(&full[s], SLOT);
          char* dst = ring + s * SLOT;
          tc::tma_2d(dst, &tk, 0, y, &full[s]);
          tc::tma_2d(dst + BOX, &tk, 64, y, &full[s]);
          tc::tma_2d(dst + 2 * BOX, &tv, 0, y, &full[s]);
          tc::tma_2d(dst + 3 * BOX, &tv, 64, y, &full[s]);
        }
      }
      if (*abort) {  // let every copy this CTA started land before shared memory is released
        int zero = 0;
        for (int i = max(0, pc - STAGES); i < pc; ++i) tc::mbar_wait(&full[i % STAGES], (i / STAGES) & 1, (volatile int*)&zero, p.err, 31);
        for (int i = max(0, n - 2); i < n; ++i) tc::mbar_wait(&qfull[i & 1], (i >> 1) & 1, (volatile int*)&zero, p.err, 33);
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers (warps 0-3)
  pdl_wait();
  const int total = p.prefix4[p.B] * p.Hkv;
  int pc = 0, n = 0;
  __shared__ int s_last;
  for (int w = blockIdx.x; w < total; w += gridDim.x) {
    const Item it = item_of(p, w);
    if (it.npages == 0) {  // same decision in every warp (and in the producer)
      if (p.out != nullptr) {  // an empty chunk still arrives (as an empty partial), so its (sequence, kv head) completes
        const int r = tid >> 3;
        if (r < G && (tid & 7) == 0) {
          const long base = ((long)it.b * p.Hq + it.hk * G + r) * p.splits + it.sp;
          p.part_ml[base * 2] = -INFINITY;
          p.part_ml[base * 2 + 1] = 0.f;
        }
        __threadfence();
        consumers_sync();
        if (tid == 0) s_last = atomicAdd(p.cnt + it.b * p.Hkv + it.hk, 1) + 1 == p.prefix4[it.b + 1] - p.prefix4[it.b];
        consumers_sync();
        if (s_last) combine_group(p, it, tid);
        consumers_sync();
      }
      continue;
    }
    const int qs = n & 1;
    const uint32_t qb = sa(sQ + qs * 2 * QBOX);
    const int rb = (warp & 1) * 32;  // first row of this warp's 32 tokens within each page
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float acc[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    bool ok = __all_sync(0xffffffffu, tc::mbar_wait(&qfull[qs], (n >> 1) & 1, abort, p.err, 34));
    for (int pg = warp >> 1; ok && pg < it.npages; pg += 2) {
      const int s = (pc + pg) % STAGES;
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&full[s], ((pc + pg) / STAGES) & 1, abort, p.err, 32));
      const int ws = it.t0 + pg * PAGE + rb, we = min(ws + 32, it.len);
      if (ok && ws < we) {
        const uint32_t kb = sa(ring + s * SLOT), vb = kb + 2 * BOX;
        float sc[4][4];
#pragma unroll
        for (int nn = 0; nn < 4; ++nn) sc[nn][0] = sc[nn][1] = sc[nn][2] = sc[nn][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(qb + q_off(lane & 15, kk * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
          for (int n2 = 0; n2 < 2; ++n2) {
            uint32_t b0, b1, b2, b3;
            const int key = n2 * 16 + (lane & 7) + (lane >> 4) * 8, col = kk * 16 + ((lane >> 3) & 1) * 8;
            ldsm_x4(kb + pg_off(rb + key, col), b0, b1, b2, b3);
            mma16816(sc[2 * n2], a0, a1, a2, a3, b0, b1);
            mma16816(sc[2 * n2 + 1], a0, a1, a2, a3, b2, b3);
          }
        }
        // online softmax across this warp's pages (rows hh = 0, 1 of the fragment)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float mx = -INFINITY;
#pragma unroll
          for (int nn = 0; nn < 4; ++nn)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int tok = ws + nn * 8 + (lane & 3) * 2 + e;
              const float x = tok < we ? sc[nn][2 * hh + e] * p.scale_log2 : -INFINITY;
              sc[nn][2 * hh + e] = x;
              mx = fmaxf(mx, x);
            }
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          const float m_new = fmaxf(m[hh], mx);  // finite: this slice has at least one valid token
          const float alpha = m[hh] == -INFINITY ? 0.f : exp2f(m[hh] - m_new);
          float rsum = 0.f;
#pragma unroll
          for (int nn = 0; nn < 4; ++nn)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float v = exp2f(sc[nn][2 * hh + e] - m_new);
              sc[nn][2 * hh + e] = v;
              rsum += v;
            }
          rsum += __shfl_xor_sync(0xffffffffu, rsum, 1);
          rsum += __shfl_xor_sync(0xffffffffu, rsum, 2);
          l[hh] = l[hh] * alpha + rsum;
          m[hh] = m_new;
#pragma unroll
          for (int d = 0; d < 16; ++d) {
            acc[d][2 * hh] *= alpha;
            acc[d][2 * hh + 1] *= alpha;
          }
        }
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint32_t a0 = pack_bf16(sc[2 * kk][0], sc[2 * kk][1]), a1 = pack_bf16(sc[2 * kk][2], sc[2 * kk][3]);
          const uint32_t a2 = pack_bf16(sc[2 * kk + 1][0], sc[2 * kk + 1][1]), a3 = pack_bf16(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
          for (int d2 = 0; d2 < 8; ++d2) {
            uint32_t b0, b1, b2, b3;
            const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, col = d2 * 16 + (lane >> 4) * 8;
            ldsm_x4_t(vb + pg_off(rb + key, col), b0, b1, b2, b3);
            mma16816(acc[2 * d2], a0, a1, a2, a3, b0, b1);
            mma16816(acc[2 * d2 + 1], a0, a1, a2, a3, b2, b3);
          }
        }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);  // this warp is done with the page
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&qempty[qs]);
    // cross-warp merge (rows < G only)
    const int G = p.Hq / p.Hkv;
    float* mine = sRed + warp * 16 * RS;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = (lane >> 2) + hh * 8;
      if (r < G) {
#pragma unroll
        for (int d = 0; d < 16; ++d) {
          const int c = d * 8 + (lane & 3) * 2;
          mine[r * RS + c] = acc[d][2 * hh];
          mine[r * RS + c + 1] = acc[d][2 * hh + 1];
        }
        if ((lane & 3) == 0) {
          mine[r * RS + D] = m[hh];
          mine[r * RS + D + 1] = l[hh];
        }
      }
    }
    consumers_sync();
    if (*abort) break;
    {
      const int r = tid >> 3, c0 = (tid & 7) * 16;
      if (r < G) {
        float M = -INFINITY;
        for (int w2 = 0; w2 < CW; ++w2) M = fmaxf(M, sRed[(w2 * 16 + r) * RS + D]);
        float L = 0.f, o[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = 0.f;
        for (int w2 = 0; w2 < CW; ++w2) {
          const float mw = sRed[(w2 * 16 + r) * RS + D];
          const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
          L += f * sRed[(w2 * 16 + r) * RS + D + 1];
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] += f * sRed[(w2 * 16 + r) * RS + c0 + j];
        }
        const long row = (long)it.b * p.Hq + it.hk * G + r;
        const int nch = p.prefix4[it.b + 1] - p.prefix4[it.b];
        if (p.out != nullptr && nch == 1) {  // the only chunk: this is the output
          const float inv = L > 0.f ? 1.f / L : 0.f;
          float f[8];
#pragma unroll
          for (int h8 = 0; h8 < 16; h8 += 8) {
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] = o[h8 + j] * inv;
            store8(p.out + row * D + c0 + h8, f);
          }
        } else {
          const long base = row * p.splits + it.sp;
          float* po = p.part_o + base * D + c0;
#pragma unroll
          for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(po + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
          if ((tid & 7) == 0) {
            p.part_ml[base * 2] = M;
            p.part_ml[base * 2 + 1] = L;
          } else if (p.out == nullptr && (tid & 7) < it.nsplits) {  // the chunk's other splits hold nothing
            p.part_ml[(base + (tid & 7)) * 2] = -INFINITY;
            p.part_ml[(base + (tid & 7)) * 2 + 1] = 0.f;
          }
        }
      }
    }
    if (p.out != nullptr && p.prefix4[it.b + 1] - p.prefix4[it.b] > 1) {
      // the last chunk of this (sequence, kv head) to finish merges all of them into the output
      __threadfence();
      consumers_sync();
      if (tid == 0) s_last = atomicAdd(p.cnt + it.b * p.Hkv + it.hk, 1) + 1 == p.prefix4[it.b + 1] - p.prefix4[it.b];
      consumers_sync();
      if (s_last) {
        __threadfence();
        combine_group(p, it, tid);
      }
    }
    consumers_sync();  // the merge buffer is read before the next item overwrites it
    pc += it.npages;
    ++n;
  }
}

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
// the cache (pages, Hkv, 64, 128) as (pages * Hkv * 64) rows of 128 bf16; box 64 x 64, 128-byte swizzle
static CUtensorMap rows_map(const void* base, long rows, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AX_CHECK(r == CUDA_SUCCESS, "tensor map encode failed (", (int)r, ")");
  return m;
}
static CUtensorMap cache_map(const void* base, long rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)PAGE};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AX_CHECK(r == CUDA_SUCCESS, "tensor map encode failed (", (int)r, ")");
  return m;
}
static at::Tensor& err_flag(int dev) {
  static at::Tensor e[64];
  if (!e[dev].defined()) e[dev] = at::zeros({1}, at::TensorOptions().device(at::kCUDA, dev).dtype(at::kInt));
  return e[dev];
}
}  // namespace dtm

// paged_decode_attn on the TMA-fed kernel (page size 64, planned work list).  With `out` and `cnt`
// the combine is fused (the caller launches nothing else); without them only the partials are
// written and the caller runs the combine.
void paged_decode_attn_tma_partials(at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor block_table, at::Tensor seq_lens,
                                    at::Tensor part_o, at::Tensor part_ml, int64_t splits, double scale, at::Tensor prefix, int max_len,
                                    bf16* out, int* cnt) {
  using namespace dtm;
  const int B = q.size(0), Hq = q.size(1), Hkv = kc.size(1);
  AX_CHECK(kc.size(2) == PAGE && kc.size(3) == D && kc.is_contiguous() && vc.is_contiguous(), "TMA decode: page size 64, head dim 128");
  AX_CHECK(q.is_contiguous() && prefix.numel() >= 2 * (B + 1), "contiguous q, chunk work list");
  const long rows = kc.size(0) * (long)Hkv * PAGE;
  const CUtensorMap tk = cache_map(kc.data_ptr(), rows), tv = cache_map(vc.data_ptr(), rows);
  const CUtensorMap tq = rows_map(q.data_ptr(), (long)B * Hq, 16);
  Params p{(const bf16*)q.data_ptr(), block_table.data_ptr<int>(), seq_lens.data_ptr<int>(), prefix.data_ptr<int>() + B + 1, part_o.data_ptr<float>(),
           part_ml.data_ptr<float>(), B, Hq, Hkv, (int)block_table.size(1), (int)splits, max_len, (float)(scale * 1.4426950408889634),
           err_flag(q.get_device()).data_ptr<int>(), out, cnt};
  const int smem = STAGES * SLOT + 2 * 2 * QBOX + CW * 16 * RS * 4 + (2 * STAGES + 4) * 8 + 16 + 1024;
  static bool attr[64] = {false};
  const int dev = q.get_device();
  if (!attr[dev]) {
    AX_CUDA_OK(cudaFuncSetAttribute(decode_tma_k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  launch_pdl(decode_tma_k, dim3(num_sms()), dim3(THREADS), smem, stream(), tk, tv, tq, p);
  AX_LAUNCH_OK();
}

int64_t decode_tma_error() { return dtm::err_flag(c10::cuda::current_device()).item<int>(); }

}  // namespace ax
