// Vocabulary-row kernels: fused log-softmax/label-gather/entropy (fwd + in-place bwd) and
// Gumbel-max sampling with the sampled token's log-prob in the same pass.
// Reference counterparts: vocab_parallel_log_prob / vocab_parallel_entropy
// (axrl/utils/megatron/tensor_parallel.py:8-82) and the engine's sampler.
#include "common.cuh"

namespace ax {

struct LseAcc {  // running max m, sum e^(s-m), sum e^(s-m)*s
  float m, s, w;
};

__device__ __forceinline__ LseAcc lse_merge(LseAcc a, LseAcc b) {
  if (a.m == -INFINITY) return b;
  if (b.m == -INFINITY) return a;
  float m = fmaxf(a.m, b.m);
  float ea = exp2f((a.m - m) * kLog2e), eb = exp2f((b.m - m) * kLog2e);
  return {m, a.s * ea + b.s * eb, a.w * ea + b.w * eb};
}

__device__ __forceinline__ void lse_push(LseAcc& a, float x) {
  if (x > a.m) {
    float e = exp2f((a.m - x) * kLog2e);
    a.s = a.s * e + 1.f;
    a.w = a.w * e + x;
    a.m = x;
  } else {
    float e = exp2f((x - a.m) * kLog2e);
    a.s += e;
    a.w += e * x;
  }
}

__device__ LseAcc block_lse(LseAcc a) {
  __shared__ LseAcc sh[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    LseAcc b{__shfl_xor_sync(0xffffffffu, a.m, o), __shfl_xor_sync(0xffffffffu, a.s, o), __shfl_xor_sync(0xffffffffu, a.w, o)};
    a = lse_merge(a, b);
  }
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) sh[wid] = a;
  __syncthreads();
  a = lane < nw ? sh[lane] : LseAcc{-INFINITY, 0.f, 0.f};
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    LseAcc b{__shfl_xor_sync(0xffffffffu, a.m, o), __shfl_xor_sync(0xffffffffu, a.s, o), __shfl_xor_sync(0xffffffffu, a.w, o)};
    a = lse_merge(a, b);
  }
  return a;
}

// s = z / t.  lp = s[label] - lse; ent = lse - E[s].
__global__ void logprob_fwd_k(const bf16* __restrict__ logits, const int* __restrict__ labels, float inv_t, int V,
                              float* __restrict__ lp, float* __restrict__ lse_out, float* __restrict__ ent) {
  const bf16* row = logits + (size_t)blockIdx.x * V;
  LseAcc a{-INFINITY, 0.f, 0.f};
  int v8 = V / 8;
  for (int i = threadIdx.x; i < v8; i += blockDim.x) {
    float f[8];
    load8(row + i * 8, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) lse_push(a, f[j] * inv_t);
  }
  for (int i = v8 * 8 + threadIdx.x; i < V; i += blockDim.x) lse_push(a, __bfloat162float(row[i]) * inv_t);
  a = block_lse(a);
  if (threadIdx.x == 0) {
    float lse = a.m + __logf(a.s);
    int lab = labels[blockIdx.x];
    lse_out[blockIdx.x] = lse;
    // lab >= V: a trained row whose label lives in another vocabulary shard (TP)
    lp[blockIdx.x] = (lab >= 0 && lab < V) ? __bfloat162float(row[lab]) * inv_t - lse : 0.f;
    if (ent) ent[blockIdx.x] = lse - a.w / a.s;
  }
}

// In place: logits <- dL/dz = [ (1[j=label] - p_j) * g_lp  - p_j (s_j - E[s]) * g_ent ] / t
__global__ void logprob_bwd_k(bf16* __restrict__ logits, const int* __restrict__ labels, const float* __restrict__ lse,
                              const float* __restrict__ g_lp, const float* __restrict__ ent, const float* __restrict__ g_ent,
                              float inv_t, int V) {
  bf16* row = logits + (size_t)blockIdx.x * V;
  float L = lse[blockIdx.x];
  int lab = labels[blockIdx.x];
  float gl = lab >= 0 ? g_lp[blockIdx.x] : 0.f;
  float ge = g_ent ? g_ent[blockIdx.x] : 0.f;
  float Es = ent ? L - ent[blockIdx.x] : 0.f;
  int v8 = V / 8;
  for (int i = threadIdx.x; i < v8 + (V - v8 * 8); i += blockDim.x) {
    if (i < v8) {
      float f[8];
      load8(row + i * 8, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float s = f[j] * inv_t;
        float p = exp2f((s - L) * kLog2e);
        int col = i * 8 + j;
        f[j] = (((col == lab) ? gl : 0.f) - p * gl - ge * p * (s - Es)) * inv_t;
      }
      store8(row + i * 8, f);
    } else {
      int col = v8 * 8 + (i - v8);
      float s = __bfloat162float(row[col]) * inv_t;
      float p = exp2f((s - L) * kLog2e);
      row[col] = __float2bfloat16((((col == lab) ? gl : 0.f) - p * gl - ge * p * (s - Es)) * inv_t);
    }
  }
}

void logprob_fwd(at::Tensor logits, at::Tensor labels, double temperature, at::Tensor lp, at::Tensor lse, at::Tensor ent) {
  AX_CHECK(logits.scalar_type() == at::kBFloat16 && logits.is_contiguous() && logits.dim() == 2, "logits bf16 (C,V)");
  int C = logits.size(0), V = logits.size(1);
  if (C == 0) return;
  logprob_fwd_k<<<C, 512, 0, stream()>>>((const bf16*)logits.data_ptr(), labels.data_ptr<int>(), (float)(1.0 / temperature), V,
                                        lp.data_ptr<float>(), lse.data_ptr<float>(), ent.numel() ? ent.data_ptr<float>() : nullptr);
  AX_LAUNCH_OK();
}

void logprob_bwd(at::Tensor logits, at::Tensor labels, at::Tensor lse, at::Tensor g_lp, at::Tensor ent, at::Tensor g_ent,
                 double temperature) {
  int C = logits.size(0), V = logits.size(1);
  if (C == 0) return;
  bool e = ent.numel() > 0 && g_ent.numel() > 0;
  logprob_bwd_k<<<C, 512, 0, stream()>>>((bf16*)logits.data_ptr(), labels.data_ptr<int>(), lse.data_ptr<float>(),
                                        g_lp.data_ptr<float>(), e ? ent.data_ptr<float>() : nullptr,
                                        e ? g_ent.data_ptr<float>() : nullptr, (float)(1.0 / temperature), V);
  AX_LAUNCH_OK();
}

// ----------------------------------------------------------------------------- sampling
// Counter-based uniform in (0,1) from (seed, row, col) via the SplitMix64 finaliser
// (Steele, Lea & Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014).
__device__ __forceinline__ float hash_uniform(uint64_t seed, uint64_t row, uint64_t col) {
  uint64_t z = seed + 0x9E3779B97F4A7C15ull * (row * 0x100000001B3ull + col + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return ((float)(z >> 40) + 0.5f) * (1.0f / 16777216.0f);  // 24-bit mantissa, never 0 or 1
}

struct ArgMax {
  float v;
  int i;
};

__device__ __forceinline__ void argmax_merge(ArgMax& a, float v, int i) {
  if (v > a.v || (v == a.v && i < a.i)) a = {v, i};
}

// Stage 1 of exact categorical sampling at temperature t by Gumbel-max (argmax_j s_j + G_j,
// G_j = -log(-log U_j)); temperature <= 0 means greedy.  The vocabulary row is split over
// gridDim.y CTAs so small decode batches still use every SM; each CTA writes its partial
// (max, sum-exp, best key, best index).  The seed is read from device memory so the kernel can
// live inside a captured CUDA graph.
template <typename T>
__global__ void sample_part_k(const T* __restrict__ logits, int V, const float* __restrict__ temp, const int64_t* __restrict__ seed,
                              const int* __restrict__ row_ids, float4* __restrict__ part) {
  pdl_trigger();  // successors may launch now; they wait for this grid's completion
  pdl_wait();
  __shared__ ArgMax shm[32];
  int row = blockIdx.x, S = gridDim.y, sp = blockIdx.y;
  int chunk = (V + S - 1) / S, j0 = sp * chunk, j1 = min(V, j0 + chunk);
  int rid = row_ids ? row_ids[row] : row;
  const T* lr = logits + (size_t)row * V;
  float t = temp[row];
  bool greedy = t <= 0.f;
  float inv_t = greedy ? 1.f : 1.f / t;
  uint64_t sd = (uint64_t)seed[0];
  LseAcc a{-INFINITY, 0.f, 0.f};
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
    float sv = (float)lr[j] * inv_t;
    lse_push(a, sv);
    float key = greedy ? sv : sv - __logf(-__logf(hash_uniform(sd, (uint64_t)rid, (uint64_t)j)));
    argmax_merge(best, key, j);
  }
  a = block_lse(a);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) argmax_merge(best, __shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o));
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) shm[wid] = best;
  __syncthreads();
  if (wid == 0) {
    best = lane < nw ? shm[lane] : ArgMax{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) argmax_merge(best, __shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o));
    if (lane == 0) part[(size_t)row * S + sp] = make_float4(a.m, a.s, best.v, __int_as_float(best.i));
  }
}

// Stage 2: one warp per row merges the partials; a forced token (e.g. an EOS ending a response
// at a prescribed length) replaces the sample, its log-prob still taken under the same distribution.
template <typename T>
__global__ void sample_merge_k(const T* __restrict__ logits, int V, int S, const float* __restrict__ temp, const float4* __restrict__ part,
                               const int64_t* __restrict__ forced, int64_t* __restrict__ out_tok, float* __restrict__ out_lp, int B) {
  pdl_trigger();  // successors may launch now; they wait for this grid's completion
  pdl_wait();
  int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= B) return;
  LseAcc a{-INFINITY, 0.f, 0.f};
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int s = lane; s < S; s += 32) {
    float4 q = part[(size_t)row * S + s];
    a = lse_merge(a, LseAcc{q.x, q.y, 0.f});
    argmax_merge(best, q.z, __float_as_int(q.w));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a = lse_merge(a, LseAcc{__shfl_xor_sync(0xffffffffu, a.m, o), __shfl_xor_sync(0xffffffffu, a.s, o), 0.f});
    argmax_merge(best, __shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o));
  }
  if (lane == 0) {
    float t = temp[row];
    float inv_t = t <= 0.f ? 1.f : 1.f / t;
    int tok = (forced != nullptr && forced[row] >= 0) ? (int)forced[row] : best.i;
    out_tok[row] = tok;
    out_lp[row] = (float)logits[(size_t)row * V + tok] * inv_t - (a.m + __logf(a.s));
  }
}

void sample_tokens(at::Tensor logits, at::Tensor temperature, at::Tensor seed, at::Tensor out_tok, at::Tensor out_lp,
                   c10::optional<at::Tensor> row_ids, c10::optional<at::Tensor> forced) {
  AX_CHECK(logits.dim() == 2 && logits.is_contiguous(), "logits (B,V) contiguous");
  int B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  const int* rid = row_ids.has_value() ? row_ids->data_ptr<int>() : nullptr;
  const int64_t* fz = forced.has_value() ? forced->data_ptr<int64_t>() : nullptr;
  int S = std::max(1, std::min(64, (num_sms() * 4 + B - 1) / B));
  S = std::min(S, std::max(1, V / 1024));
  auto part = at::empty({(long)B * S * 4}, logits.options().dtype(at::kFloat));
  dim3 g1(B, S);
  int wb = (B * 32 + 255) / 256;
  if (logits.scalar_type() == at::kFloat) {
    launch_pdl(sample_part_k<float>, g1, dim3(256), 0, stream(), (const float*)logits.data_ptr<float>(), V, temperature.data_ptr<float>(), seed.data_ptr<int64_t>(), rid,
                                                  reinterpret_cast<float4*>(part.data_ptr<float>()));
    launch_pdl(sample_merge_k<float>, dim3(wb), dim3(256), 0, stream(), (const float*)logits.data_ptr<float>(), V, S, temperature.data_ptr<float>(),
                                                   reinterpret_cast<float4*>(part.data_ptr<float>()), fz, out_tok.data_ptr<int64_t>(),
                                                   out_lp.data_ptr<float>(), B);
  } else {
    AX_CHECK(logits.scalar_type() == at::kBFloat16, "logits bf16/fp32");
    launch_pdl(sample_part_k<bf16>, g1, dim3(256), 0, stream(), (const bf16*)logits.data_ptr(), V, temperature.data_ptr<float>(), seed.data_ptr<int64_t>(),
                                                 rid, reinterpret_cast<float4*>(part.data_ptr<float>()));
    launch_pdl(sample_merge_k<bf16>, dim3(wb), dim3(256), 0, stream(), (const bf16*)logits.data_ptr(), V, S, temperature.data_ptr<float>(),
                                                  reinterpret_cast<float4*>(part.data_ptr<float>()), fz, out_tok.data_ptr<int64_t>(),
                                                  out_lp.data_ptr<float>(), B);
  }
  AX_LAUNCH_OK();
}

}  // namespace ax
