// Gated DeltaNet decode step on the per-sequence recurrent states, in place in the engine's pool.
//
// For row b (sequence slot s = slots[b]) and value head h, with S = pool[s, h] (d_k x d_v, fp32):
//   S   <- exp(g) * S
//   u    = S^T k                         (d_v)
//   S   <- S + k (beta (v - u))^T
//   o    = S^T q                         (d_v; q is already L2-normalised and scaled)
// One CTA per (row, head); thread j owns column j of S (d_k values), so the state is read and
// written once, coalesced along j, and both reductions over d_k stay in registers.
// Reference counterpart: flash-linear-attention's fused recurrent gated delta rule used by the
// reference's Qwen3.5 / 3.6 rollouts (GDN branch of axrl/utils/megatron/magi_forward.py:790-848).
#include "common.cuh"

namespace ax {
namespace gdn {

constexpr int MAX_DK = 256;

__global__ void gdn_step_k(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, const float* __restrict__ g,
                           const float* __restrict__ beta, float* __restrict__ pool, const int64_t* __restrict__ slots, float* __restrict__ out,
                           int H, int dk, int dv) {
  __shared__ float sq[MAX_DK], sk[MAX_DK];
  const int b = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  const long row = (long)b * H + h;
  for (int i = threadIdx.x; i < dk; i += blockDim.x) {
    sq[i] = q[row * dk + i];
    sk[i] = k[row * dk + i];
  }
  __syncthreads();
  if (j >= dv) return;
  const float a = __expf(g[row]), bt = beta[row];
  float* S = pool + ((long)slots[b] * H + h) * dk * dv + j;
  float u = 0.f;
  for (int i = 0; i < dk; ++i) u += S[(long)i * dv] * a * sk[i];
  const float delta = bt * (v[row * dv + j] - u);
  float o = 0.f;
  for (int i = 0; i < dk; ++i) {
    const float s = S[(long)i * dv] * a + sk[i] * delta;
    S[(long)i * dv] = s;
    o += s * sq[i];
  }
  out[row * dv + j] = o;
}

}  // namespace gdn

// q, k (B, H, dk), v (B, H, dv), g, beta (B, H): fp32 contiguous; pool (slots, H, dk, dv) fp32 updated
// in place at rows ``slots`` (B,) int64; returns o (B, H, dv) fp32.
at::Tensor gdn_step(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta, at::Tensor pool, at::Tensor slots) {
  AX_CHECK(q.scalar_type() == at::kFloat && k.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat && pool.scalar_type() == at::kFloat,
           "fp32 inputs");
  AX_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && g.is_contiguous() && beta.is_contiguous() && pool.is_contiguous(),
           "contiguous inputs");
  const int B = q.size(0), H = q.size(1), dk = q.size(2), dv = v.size(2);
  AX_CHECK(dk <= gdn::MAX_DK && dv <= 1024 && pool.size(1) == H && pool.size(2) == dk && pool.size(3) == dv, "state shape");
  AX_CHECK(slots.scalar_type() == at::kLong && slots.numel() == B, "slots int64 (B,)");
  auto out = at::empty({B, H, dv}, q.options());
  if (B == 0) return out;
  const int threads = ((dv + 31) / 32) * 32;
  gdn::gdn_step_k<<<dim3(B, H), threads, 0, stream()>>>(q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), g.data_ptr<float>(),
                                                         beta.data_ptr<float>(), pool.data_ptr<float>(), slots.data_ptr<int64_t>(),
                                                         out.data_ptr<float>(), H, dk, dv);
  AX_LAUNCH_OK();
  return out;
}

}  // namespace ax
