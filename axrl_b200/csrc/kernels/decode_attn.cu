// Paged-KV decode attention (one new query token per sequence) with split-KV partials,
// plus the paged KV-cache layout helpers.  Reference counterpart: the rollout engine's
// decode attention backends (SGLang FA3 / FlashInfer), reached via
// axrl/worker/sglang_worker.py:80-107.
//
// Cache layout (per layer): k_cache, v_cache = [num_pages, Hkv, page_size, 128] bf16, so one
// (page, head) block is a contiguous page_size x 256-byte run.
//
// Kernel: one CTA per (sequence, kv head, split of SPLIT tokens); 4 warps, each warp owns one
// 32-token slice.  The GQA group's q heads (<= 16) form the M=16 rows of mma.m16n8k16, so K/V
// are read exactly once per kv head.  The grid's split count is fixed by the cache capacity
// (graph-capture friendly); CTAs past a sequence's end exit.  A combine kernel merges splits.
#include <string>

#include "common.cuh"

namespace ax {
namespace dec {

constexpr int D = 128;
constexpr int WARPS = 4;
constexpr int SLICE = 32;                // tokens per warp (68 KB smem per CTA: 3 CTAs per SM)
constexpr int NSUB = SLICE / 8;          // n8 key tiles per warp
constexpr int SPLIT = WARPS * SLICE;     // tokens per CTA

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ int swz(int row, int col) {
  int chunk = (col >> 3) ^ (row & 7);
  return row * (D * 2) + chunk * 16 + (col & 7) * 2;
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(pred ? 16 : 0));
}
__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n" : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3]) : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  bf162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

struct Params {
  const bf16* q;          // (B, Hq, D)
  const bf16* kc;         // (pages, Hkv, P, D)
  const bf16* vc;
  const int* block_table; // (B, max_pages)
  const int* seq_lens;    // (B,)
  float* part_o;          // (B, Hq, splits, D) unnormalised partial outputs
  float* part_ml;         // (B, Hq, splits, 2): (max, sum) in log2 domain
  int Hq, Hkv, P, max_pages, splits;
  float scale_log2;
  int max_len;            // lengths are clamped to this (<= max_pages * P and <= splits * SPLIT)
};

// One (sequence b, kv head hk, split sp) work item; all threads of the CTA call it together.
__device__ __forceinline__ void decode_item(const Params& p, char* smem, int b, int hk, int sp) {
  const int len = min(p.seq_lens[b], p.max_len);  // never read block_table past max_pages
  const int t0 = sp * SPLIT;
  if (t0 >= len) return;
  const int G = p.Hq / p.Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  char* sQ = smem;                                   // 16 x 128
  char* sK = sQ + 16 * D * 2 + warp * 2 * SLICE * D * 2;
  char* sV = sK + SLICE * D * 2;
  // Cross-warp merge buffer (WARPS x 16 x (D + 2) fp32) aliases the K/V area once all warps are done.
  float* sRed = reinterpret_cast<float*>(smem + 16 * D * 2);

  // Q rows (g < G valid, rest zero)
  for (int i = tid; i < 16 * 16; i += 128) {
    int r = i >> 4, c = (i & 15) * 8;
    bool ok = r < G;
    const bf16* src = p.q + ((long)b * p.Hq + hk * G + (ok ? r : 0)) * D + c;
    cp_async16(sQ + swz(r, c), src, ok);
  }
  // This warp's token slice [ws, we)
  const int ws = t0 + warp * SLICE, we = min(ws + SLICE, len);
  for (int i = lane; i < SLICE * 16; i += 32) {
    int r = i >> 4, c = (i & 15) * 8;
    int tok = ws + r;
    bool ok = tok < we;
    long off = 0;
    if (ok) {
      int page = p.block_table[(long)b * p.max_pages + tok / p.P];
      off = (((long)page * p.Hkv + hk) * p.P + (tok % p.P)) * D + c;
    }
    cp_async16(sK + swz(r, c), p.kc + off, ok);
    cp_async16(sV + swz(r, c), p.vc + off, ok);
  }
  asm volatile("cp.async.commit_group;\n" ::);
  asm volatile("cp.async.wait_group 0;\n" ::);
  __syncthreads();

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  if (ws < we) {
    float s[NSUB][4];
#pragma unroll
    for (int n = 0; n < NSUB; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(smem_u32(sQ + swz(lane & 15, kk * 16 + (lane >> 4) * 8)), a0, a1, a2, a3);
#pragma unroll
      for (int n2 = 0; n2 < NSUB / 2; ++n2) {
        uint32_t b0, b1, b2, b3;
        int key = n2 * 16 + (lane & 7) + (lane >> 4) * 8, col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(smem_u32(sK + swz(key, col)), b0, b1, b2, b3);
        mma16816(s[2 * n2], a0, a1, a2, a3, b0, b1);
        mma16816(s[2 * n2 + 1], a0, a1, a2, a3, b2, b3);
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < NSUB; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          int tok = ws + n * 8 + (lane & 3) * 2 + e;
          float x = tok < we ? s[n][2 * hh + e] * p.scale_log2 : -INFINITY;
          s[n][2 * hh + e] = x;
          mx = fmaxf(mx, x);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      m[hh] = mx;
      float rs = 0.f;
#pragma unroll
      for (int n = 0; n < NSUB; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float v = exp2f(s[n][2 * hh + e] - mx);
          s[n][2 * hh + e] = v;
          rs += v;
        }
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
      l[hh] = rs;
    }
#pragma unroll
    for (int kk = 0; kk < NSUB / 2; ++kk) {
      uint32_t a0 = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      uint32_t a1 = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      uint32_t a2 = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      uint32_t a3 = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int d2 = 0; d2 < 8; ++d2) {
        uint32_t b0, b1, b2, b3;
        int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, col = d2 * 16 + (lane >> 4) * 8;
        ldsm_x4_t(smem_u32(sV + swz(key, col)), b0, b1, b2, b3);
        mma16816(acc[2 * d2], a0, a1, a2, a3, b0, b1);
        mma16816(acc[2 * d2 + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }
  // cross-warp merge through shared memory
  __syncthreads();
  constexpr int RS = D + 2;
  float* mine = sRed + warp * 16 * RS;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    int r = (lane >> 2) + hh * 8;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      int c = d * 8 + (lane & 3) * 2;
      mine[r * RS + c] = acc[d][2 * hh];
      mine[r * RS + c + 1] = acc[d][2 * hh + 1];
    }
    if ((lane & 3) == 0) {
      mine[r * RS + D] = m[hh];
      mine[r * RS + D + 1] = l[hh];
    }
  }
  __syncthreads();
  // thread t: row r = t / 8 (16 rows), 16 columns each
  {
    int r = tid >> 3, c0 = (tid & 7) * 16;
    if (r < G) {
      float M = -INFINITY;
      for (int w = 0; w < WARPS; ++w) M = fmaxf(M, sRed[(w * 16 + r) * RS + D]);
      float L = 0.f, o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = 0.f;
      for (int w = 0; w < WARPS; ++w) {
        float mw = sRed[(w * 16 + r) * RS + D];
        float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
        L += f * sRed[(w * 16 + r) * RS + D + 1];
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] += f * sRed[(w * 16 + r) * RS + c0 + j];
      }
      long base = (((long)b * p.Hq + hk * G + r) * p.splits + sp);
      float* po = p.part_o + base * D + c0;
#pragma unroll
      for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(po + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
      if ((tid & 7) == 0) {
        p.part_ml[base * 2] = M;
        p.part_ml[base * 2 + 1] = L;
      }
    }
  }
}

// Fixed grid: one CTA per (sequence, kv head, split of the cache capacity); CTAs past the end of
// their sequence exit at once (used by the allocation-free entry point).
__global__ void __launch_bounds__(128) decode_k(Params p) {
  extern __shared__ __align__(128) char smem[];
  decode_item(p, smem, blockIdx.x, blockIdx.y, blockIdx.z);
}

// Work list of the live (sequence, split) pairs: prefix[b] = sum over earlier sequences of
// ceil(len / SPLIT).  With `chunks` (the array holds 2 (B + 1) entries) the second half is the
// same count in 512-token chunks (the items of the TMA-fed kernel).  Computed once per decode
// step and shared by every layer.
__global__ void decode_plan_k(const int* __restrict__ seq_lens, int B, int* __restrict__ prefix, int chunks) {
  pdl_trigger();  // successors may launch now; they wait for this grid's completion
  pdl_wait();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int acc = 0, acc4 = 0;
  for (int b = 0; b < B; ++b) {
    prefix[b] = acc;
    acc += (seq_lens[b] + SPLIT - 1) / SPLIT;
    if (chunks) {
      prefix[B + 1 + b] = acc4;
      acc4 += (seq_lens[b] + 4 * SPLIT - 1) / (4 * SPLIT);
    }
  }
  prefix[B] = acc;
  if (chunks) prefix[2 * B + 1] = acc4;
}

// Persistent grid sized to the SMs: each CTA walks work items (kv head fastest), so the launch
// costs the live work only, not B x Hkv x (capacity / SPLIT) mostly-empty CTAs.
__global__ void __launch_bounds__(128) decode_persist_k(Params p, const int* __restrict__ prefix, int B) {
  pdl_trigger();  // successors may launch now; they wait for this grid's completion
  pdl_wait();
  extern __shared__ __align__(128) char smem[];
  const int total = prefix[B] * p.Hkv;
  for (int w = blockIdx.x; w < total; w += gridDim.x) {
    const int hk = w % p.Hkv, j = w / p.Hkv;
    int lo = 0, hi = B - 1;  // last b with prefix[b] <= j
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= j) lo = mid;
      else hi = mid - 1;
    }
    __syncthreads();  // the previous item's merge buffer aliases this item's K/V tiles
    decode_item(p, smem, lo, hk, j - prefix[lo]);
  }
}

// out[b, h, :] = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s ; one warp per (b, h)
__global__ void combine_k(const float* __restrict__ part_o, const float* __restrict__ part_ml, const int* __restrict__ seq_lens,
                          bf16* __restrict__ out, int B, int Hq, int splits, int max_len) {
  pdl_trigger();  // successors may launch now; they wait for this grid's completion
  pdl_wait();
  int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= B * Hq) return;
  int b = w / Hq;
  int ns = min(splits, (min(seq_lens[b], max_len) + SPLIT - 1) / SPLIT);
  const float* ml = part_ml + (long)w * splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, ml[2 * s]);
  float L = 0.f;
  float4 o = make_float4(0, 0, 0, 0);
  for (int s = 0; s < ns; ++s) {
    float f = ml[2 * s] == -INFINITY ? 0.f : exp2f(ml[2 * s] - M);
    if (f == 0.f) continue;  // an empty split (its output rows were never written) contributes nothing
    L += f * ml[2 * s + 1];
    float4 v = *reinterpret_cast<const float4*>(part_o + ((long)w * splits + s) * D + lane * 4);
    o.x += f * v.x; o.y += f * v.y; o.z += f * v.z; o.w += f * v.w;
  }
  float inv = L > 0.f ? 1.f / L : 0.f;
  bf16* dst = out + (long)w * D + lane * 4;
  *reinterpret_cast<bf162*>(dst) = __floats2bfloat162_rn(o.x * inv, o.y * inv);
  *reinterpret_cast<bf162*>(dst + 2) = __floats2bfloat162_rn(o.z * inv, o.w * inv);
}

// Scatter new k/v rows (T, Hkv, D) into the paged caches at slots (slot = page * P + offset).
__global__ void kv_store_k(const bf16* __restrict__ k, const bf16* __restrict__ v, bf16* __restrict__ kc, bf16* __restrict__ vc,
                           const int64_t* __restrict__ slots, int T, int Hkv, int P) {
  long i = blockIdx.x * (long)blockDim.x + threadIdx.x;  // one 16-byte chunk
  long n = (long)T * Hkv * 16;
  if (i >= n) return;
  int c = (i & 15) * 8;
  long th = i >> 4;
  int t = th / Hkv, h = th % Hkv;
  long slot = slots[t];
  long dst = (((slot / P) * Hkv + h) * P + slot % P) * D + c;
  long src = ((long)t * Hkv + h) * D + c;
  *reinterpret_cast<V8*>(kc + dst) = *reinterpret_cast<const V8*>(k + src);
  *reinterpret_cast<V8*>(vc + dst) = *reinterpret_cast<const V8*>(v + src);
}

// Device-side decode bookkeeping between two graph-replayed decode steps (one CTA, B <= 1024).
// For every live row (len > 0): append the sampled token to the ring, then either freeze the row
// (it reached end_total, or sampled EOS with stop_on_eos) or advance it: next input token, position,
// length, KV slot from the block table, and the token to force on the next sample (EOS when the
// next token is the row's last and force_eos is set).  Frozen rows get len 0 so decode skips them.
__global__ void decode_advance_k(int B, const int64_t* __restrict__ out_tok, const float* __restrict__ out_lp,
                                 int64_t* __restrict__ tok, int* __restrict__ pos, int* __restrict__ len,
                                 int64_t* __restrict__ slot, const int* __restrict__ bt, int max_pages, int P,
                                 const int* __restrict__ end_total, const int* __restrict__ force_eos,
                                 const int* __restrict__ stop_on_eos, int64_t eos, int64_t* __restrict__ forced,
                                 int64_t* __restrict__ ring_tok, float* __restrict__ ring_lp, int* __restrict__ ring_step,
                                 int ring_cap, int ring_ld, int64_t scratch_slot, int64_t* __restrict__ seed) {
  pdl_trigger();  // successors may launch now; they wait for this grid's completion
  pdl_wait();
  __shared__ int step;
  if (threadIdx.x == 0) step = ring_step[0];
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    int l = len[b];
    long ri = (long)(step % ring_cap) * ring_ld + b;  // ring rows are max_batch wide, not bucket wide
    if (l <= 0) {
      ring_tok[ri] = -1;
      ring_lp[ri] = 0.f;
      continue;
    }
    int64_t t = out_tok[b];
    ring_tok[ri] = t;
    ring_lp[ri] = out_lp[b];
    int n = l + 1;
    bool done = n >= end_total[b] || (stop_on_eos[b] && t == eos);
    if (done) {
      len[b] = 0;
      slot[b] = scratch_slot;
      forced[b] = -1;
      continue;
    }
    tok[b] = t;
    pos[b] = n - 1;
    len[b] = n;
    slot[b] = (int64_t)bt[(long)b * max_pages + (n - 1) / P] * P + (n - 1) % P;
    forced[b] = (force_eos[b] && n + 1 == end_total[b]) ? eos : -1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ring_step[0] = step + 1;
    seed[0] += 1;
  }
}

}  // namespace dec

void decode_advance(int64_t B, at::Tensor out_tok, at::Tensor out_lp, at::Tensor tok, at::Tensor pos, at::Tensor len, at::Tensor slot,
                    at::Tensor bt, int64_t P, at::Tensor end_total, at::Tensor force_eos, at::Tensor stop_on_eos, int64_t eos,
                    at::Tensor forced, at::Tensor ring_tok, at::Tensor ring_lp, at::Tensor ring_step, int64_t scratch_slot,
                    at::Tensor seed) {
  AX_CHECK(B <= 1024, "decode batch must be <= 1024");
  if (B == 0) return;
  launch_pdl(dec::decode_advance_k, dim3(1), dim3(256), 0, stream(),
      (int)B, out_tok.data_ptr<int64_t>(), out_lp.data_ptr<float>(), tok.data_ptr<int64_t>(), pos.data_ptr<int>(), len.data_ptr<int>(),
      slot.data_ptr<int64_t>(), bt.data_ptr<int>(), (int)bt.size(1), (int)P, end_total.data_ptr<int>(), force_eos.data_ptr<int>(),
      stop_on_eos.data_ptr<int>(), eos, forced.data_ptr<int64_t>(), ring_tok.data_ptr<int64_t>(), ring_lp.data_ptr<float>(),
      ring_step.data_ptr<int>(), (int)ring_tok.size(0), (int)ring_tok.size(1), scratch_slot, seed.data_ptr<int64_t>());
  AX_LAUNCH_OK();
}

// q (B,Hq,128); caches (pages,Hkv,P,128); block_table (B,max_pages) int32; seq_lens (B,) int32.
// `splits` is fixed by the caller (ceil(max_context / SPLIT), SPLIT = 128 tokens) so the launch
// shape is static.
void decode_plan(at::Tensor seq_lens, at::Tensor prefix) {
  int B = seq_lens.numel();
  AX_CHECK(prefix.scalar_type() == at::kInt && prefix.numel() >= B + 1, "prefix: int32 (B + 1)");
  const int chunks = prefix.numel() >= 2 * (B + 1) ? 1 : 0;
  launch_pdl(dec::decode_plan_k, dim3(1), dim3(32), 0, stream(), seq_lens.data_ptr<int>(), B, prefix.data_ptr<int>(), chunks);
  AX_LAUNCH_OK();
}

void paged_decode_attn_tma_partials(at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor block_table, at::Tensor seq_lens,
                                    at::Tensor part_o, at::Tensor part_ml, int64_t splits, double scale, at::Tensor prefix, int max_len,
                                    bf16* out, int* cnt);

// Planned launches with 64-token pages run the TMA page-pipeline kernel (decode_attn_tma.cu):
// Qwen3-8B decode at 2048-token contexts on B200, 8.75 ms per step at batch 64 and 4.72 ms at
// batch 8 against 12.0 / 5.24 ms with the cp.async persistent kernel.  AXRL_DECODE_ATTN=persist
// selects the latter.
static int& decode_tma_flag() {
  static int on = [] {
    const char* e = std::getenv("AXRL_DECODE_ATTN");
    return (e && std::string(e) == "persist") ? 0 : 1;
  }();
  return on;
}
static bool decode_tma_enabled() { return decode_tma_flag() != 0; }
void set_decode_attn_tma(bool on) { decode_tma_flag() = on ? 1 : 0; }

// chunk_cnt: optional zeroed int32 buffer of >= B * Hkv (sequence, kv head) counters; with it the
// TMA kernel merges its chunks itself (no combine launch) and leaves the counters zeroed again.
void paged_decode_attn(at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor block_table, at::Tensor seq_lens, at::Tensor out,
                       at::Tensor part_o, at::Tensor part_ml, int64_t splits, double scale, c10::optional<at::Tensor> prefix,
                       c10::optional<at::Tensor> chunk_cnt) {
  using namespace dec;
  int B = q.size(0), Hq = q.size(1), Hkv = kc.size(1), P = kc.size(2);
  AX_CHECK(q.size(2) == D && kc.size(3) == D, "head_dim 128");
  AX_CHECK(Hq % Hkv == 0 && Hq / Hkv <= 16, "GQA group must be <= 16");
  AX_CHECK(part_o.numel() >= (long)B * Hq * splits * D && part_ml.numel() >= (long)B * Hq * splits * 2, "partial buffers too small");
  if (B == 0) return;
  const int max_len = (int)std::min<long>((long)block_table.size(1) * P, (long)splits * SPLIT);
  Params p{(const bf16*)q.data_ptr(), (const bf16*)kc.data_ptr(), (const bf16*)vc.data_ptr(), block_table.data_ptr<int>(),
           seq_lens.data_ptr<int>(), part_o.data_ptr<float>(), part_ml.data_ptr<float>(), Hq, Hkv, P, (int)block_table.size(1),
           (int)splits, (float)(scale * 1.4426950408889634), max_len};
  int smem = 16 * D * 2 + WARPS * 2 * SLICE * D * 2;
  static_assert(WARPS * 16 * (D + 2) * 4 <= WARPS * 2 * SLICE * D * 2, "merge buffer must fit in the K/V area");
  // the shared-memory opt-in is a per-device function attribute
  static bool attr[64] = {false};
  const int dev = c10::cuda::current_device();
  AX_CHECK(dev >= 0 && dev < 64, "device index");
  if (!attr[dev]) {
    AX_CUDA_OK(cudaFuncSetAttribute(decode_k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    AX_CUDA_OK(cudaFuncSetAttribute(decode_persist_k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  if (prefix.has_value() && decode_tma_enabled() && P == 64 && prefix->numel() >= 2 * (B + 1)) {  // planned, TMA page pipeline
    AX_CHECK(prefix->scalar_type() == at::kInt && prefix->numel() >= B + 1, "prefix: int32 (B + 1)");
    if (chunk_cnt.has_value() && out.is_contiguous()) {  // combine fused into the TMA kernel
      AX_CHECK(chunk_cnt->is_cuda() && chunk_cnt->scalar_type() == at::kInt && chunk_cnt->numel() >= (long)B * Hkv,
               "chunk_cnt: int32 >= B * Hkv");
      paged_decode_attn_tma_partials(q, kc, vc, block_table, seq_lens, part_o, part_ml, splits, scale, *prefix, max_len,
                                     (bf16*)out.data_ptr(), chunk_cnt->data_ptr<int>());
      return;
    }
    paged_decode_attn_tma_partials(q, kc, vc, block_table, seq_lens, part_o, part_ml, splits, scale, *prefix, max_len, nullptr, nullptr);
  } else if (prefix.has_value()) {  // planned: persistent grid over the live work items
    AX_CHECK(prefix->scalar_type() == at::kInt && prefix->numel() >= B + 1, "prefix: int32 (B + 1)");
    launch_pdl(decode_persist_k, dim3(num_sms() * 3), dim3(128), smem, stream(), p, (const int*)prefix->data_ptr<int>(), B);
  } else {
    decode_k<<<dim3(B, Hkv, splits), 128, smem, stream()>>>(p);
  }
  AX_LAUNCH_OK();
  long w = (long)B * Hq;
  launch_pdl(combine_k, dim3((w * 32 + 255) / 256), dim3(256), 0, stream(), (const float*)part_o.data_ptr<float>(),
             (const float*)part_ml.data_ptr<float>(), (const int*)seq_lens.data_ptr<int>(), (bf16*)out.data_ptr(), B, Hq, (int)splits,
             max_len);
  AX_LAUNCH_OK();
}

void kv_store(at::Tensor k, at::Tensor v, at::Tensor kc, at::Tensor vc, at::Tensor slots) {
  using namespace dec;
  int T = k.size(0), Hkv = k.size(1), P = kc.size(2);
  long n = (long)T * Hkv * 16;
  if (n == 0) return;
  kv_store_k<<<(n + 255) / 256, 256, 0, stream()>>>((const bf16*)k.data_ptr(), (const bf16*)v.data_ptr(), (bf16*)kc.data_ptr(),
                                                  (bf16*)vc.data_ptr(), slots.data_ptr<int64_t>(), T, Hkv, P);
  AX_LAUNCH_OK();
}

}  // namespace ax

// ------------------------------------------------------------------------------------------------
// Allocation-free entry point (declared and documented in decode_attn_noalloc.h; no counterpart in
// the reference).  Same kernels as paged_decode_attn; the split-KV partials live in a file-scope
// device array instead of caller-provided workspace tensors.
#include <cstdio>
#include <mutex>

#include "decode_attn_noalloc.h"

static __device__ __align__(256) float g_decode_noalloc_scratch[(long)AXRL_DECODE_NOALLOC_MAX_ROWS * (ax::dec::D + 2)];

namespace {
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64] = {nullptr};  // device address of the array, per device
bool g_noalloc_attr[64] = {false};     // shared-memory opt-in of decode_k done, per device
}  // namespace

extern "C" int axrl_paged_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_table,
                                                   const int* seq_lens, void* out, int B, int Hq, int Hkv, int page_size, int max_pages,
                                                   int max_context, float scale, void* stream) {
  using namespace ax::dec;
  using ax::bf16;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || Hq / Hkv > 16 || page_size <= 0 || max_pages <= 0 || max_context <= 0 ||
      (long)max_pages * page_size < max_context || !q || !k_cache || !v_cache || !block_table || !seq_lens || !out) {
    std::fprintf(stderr, "axrl_paged_decode_attention_noalloc: invalid arguments\n");
    return 2;
  }
  if (B == 0) return 0;
  const int splits = (max_context + SPLIT - 1) / SPLIT;
  const long rows = (long)B * Hq * splits;
  if (rows > AXRL_DECODE_NOALLOC_MAX_ROWS) {
    std::fprintf(stderr,
                 "axrl_paged_decode_attention_noalloc: B*Hq*ceil(max_context/%d) = %ld rows exceeds the %d-row scratch array; "
                 "use paged_decode_attn with a workspace instead\n",
                 SPLIT, rows, AXRL_DECODE_NOALLOC_MAX_ROWS);
    return 1;
  }
  // An error left pending by earlier work on this thread (or a context already in an error state)
  // belongs to its owner: report it without launching and without clearing it.
  if (cudaPeekAtLastError() != cudaSuccess) {
    std::fprintf(stderr, "axrl_paged_decode_attention_noalloc: a CUDA error is already pending; nothing launched\n");
    return 5;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 3;
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr) {
        std::fprintf(stderr, "axrl_paged_decode_attention_noalloc: cudaGetSymbolAddress failed: %s\n", cudaGetErrorString(e));
        return 3;
      }
      g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    scratch = g_noalloc_ptr[dev];
    if (!g_noalloc_attr[dev]) {
      int smem = 16 * D * 2 + WARPS * 2 * SLICE * D * 2;
      if (cudaFuncSetAttribute(decode_k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 4;
      g_noalloc_attr[dev] = true;
    }
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Params p{static_cast<const bf16*>(q), static_cast<const bf16*>(k_cache), static_cast<const bf16*>(v_cache), block_table, seq_lens,
           scratch, scratch + rows * D, Hq, Hkv, page_size, max_pages, splits, scale * 1.4426950408889634f, max_context};
  int smem = 16 * D * 2 + WARPS * 2 * SLICE * D * 2;
  decode_k<<<dim3(B, Hkv, splits), 128, smem, st>>>(p);
  if (cudaGetLastError() != cudaSuccess) return 4;
  long w = (long)B * Hq;
  combine_k<<<(w * 32 + 255) / 256, 256, 0, st>>>(p.part_o, p.part_ml, seq_lens, static_cast<bf16*>(out), B, Hq, splits, max_context);
  if (cudaGetLastError() != cudaSuccess) return 4;
  return 0;
}
