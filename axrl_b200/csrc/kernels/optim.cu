// Optimizer-side kernels over flat fp32 buffers: squared-norm reduction, fused
// clip + AdamW (+ bf16 parameter write-back), and embedding gather / scatter-add.
// Reference counterpart: Megatron distributed optimizer with Apex/TE fused Adam and
// multi_tensor_l2norm grad clipping (axrl/worker/megatron_worker.py:480-509,923-930).
//
// No host synchronisation: the global grad norm stays on the device and the Adam kernel
// derives the clip coefficient from it.
#include "common.cuh"

namespace ax {

// acc[0] += sum(x^2) over n elements (fp32 partials per CTA, one atomic per CTA)
__global__ void sqnorm_k(const float* __restrict__ x, long n, float* __restrict__ acc) {
  __shared__ float sh[32];
  float s = 0.f;
  long n4 = n / 4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(x)[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long i = n4 * 4 + blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) s += x[i] * x[i];
  s = block_sum(s, sh);
  if (threadIdx.x == 0) atomicAdd(acc, s);
}

void sqnorm_accumulate(at::Tensor x, at::Tensor acc) {
  AX_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && acc.scalar_type() == at::kFloat, "fp32 inputs");
  long n = x.numel();
  if (n == 0) return;
  int ctas = (int)std::min<long>((n / 4 + 255) / 256 + 1, num_sms() * 4);
  sqnorm_k<<<ctas, 256, 0, stream()>>>(x.data_ptr<float>(), n, acc.data_ptr<float>());
  AX_LAUNCH_OK();
}

// AdamW with bias correction on elements [0, n).  Elements >= decay_end skip weight decay.
// g_scale = min(1, clip / (sqrt(sqnorm[0]) + 1e-6)) when clip > 0 (grad-norm clipping).
__global__ void adamw_k(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                        bf16* __restrict__ p_bf16, long n, long decay_end, float lr, float b1, float b2, float eps, float wd,
                        float bc1, float bc2, const float* __restrict__ sqnorm, float clip, float extra_scale) {
  float gs = extra_scale;
  if (clip > 0.f && sqnorm != nullptr) {
    float norm = sqrtf(sqnorm[0]) * extra_scale;
    gs *= fminf(1.f, clip / (norm + 1e-6f));
  }
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float gi = g[i] * gs;
    float mi = b1 * m[i] + (1.f - b1) * gi;
    float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float upd = (mi / bc1) / (sqrtf(vi / bc2) + eps);
    float pi = p[i];
    if (i < decay_end) upd += wd * pi;
    pi -= lr * upd;
    p[i] = pi;
    if (p_bf16) p_bf16[i] = __float2bfloat16(pi);
  }
}

void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> p_bf16, int64_t decay_end,
                double lr, double b1, double b2, double eps, double wd, int64_t step, c10::optional<at::Tensor> sqnorm, double clip,
                double extra_scale) {
  long n = p.numel();
  AX_CHECK(g.numel() == n && m.numel() == n && v.numel() == n, "buffer sizes");
  if (n == 0) return;
  float bc1 = 1.f - (float)std::pow(b1, (double)step), bc2 = 1.f - (float)std::pow(b2, (double)step);
  int ctas = (int)std::min<long>((n + 255) / 256, num_sms() * 8);
  adamw_k<<<ctas, 256, 0, stream()>>>(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                                     p_bf16.has_value() ? (bf16*)p_bf16->data_ptr() : nullptr, n, decay_end, (float)lr, (float)b1,
                                     (float)b2, (float)eps, (float)wd, bc1, bc2,
                                     sqnorm.has_value() ? sqnorm->data_ptr<float>() : nullptr, (float)clip, (float)extra_scale);
  AX_LAUNCH_OK();
}

// Partitioned AdamW fused with the parameter all-gather of the distributed optimizer: this rank's
// shard [s0, s0 + n) of the flat parameters is updated from its reduced gradient and the new bf16
// values are stored straight into every rank's parameter buffer (P2P stores through `ptrs`, this
// rank's own buffer included), replacing an AdamW pass followed by a broadcast pass that re-read
// the fp32 master.  8 elements per thread step (n % 8 == 0).
__global__ void adamw_p2p_k(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                            const int64_t* __restrict__ ptrs, int world, long s0, long n, long decay_end, float lr, float b1, float b2,
                            float eps, float wd, float bc1, float bc2, const float* __restrict__ sqnorm, float clip, float extra_scale) {
  float gs = extra_scale;
  if (clip > 0.f && sqnorm != nullptr) {
    const float norm = sqrtf(sqnorm[0]) * extra_scale;
    gs *= fminf(1.f, clip / (norm + 1e-6f));
  }
  const long n8 = n / 8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    float pv[8], gv[8], mv[8], vv[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4 a = reinterpret_cast<const float4*>(p)[2 * i + h], b = reinterpret_cast<const float4*>(g)[2 * i + h];
      const float4 c = reinterpret_cast<const float4*>(m)[2 * i + h], d = reinterpret_cast<const float4*>(v)[2 * i + h];
      pv[4 * h] = a.x, pv[4 * h + 1] = a.y, pv[4 * h + 2] = a.z, pv[4 * h + 3] = a.w;
      gv[4 * h] = b.x, gv[4 * h + 1] = b.y, gv[4 * h + 2] = b.z, gv[4 * h + 3] = b.w;
      mv[4 * h] = c.x, mv[4 * h + 1] = c.y, mv[4 * h + 2] = c.z, mv[4 * h + 3] = c.w;
      vv[4 * h] = d.x, vv[4 * h + 1] = d.y, vv[4 * h + 2] = d.z, vv[4 * h + 3] = d.w;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float gi = gv[j] * gs;
      mv[j] = b1 * mv[j] + (1.f - b1) * gi;
      vv[j] = b2 * vv[j] + (1.f - b2) * gi * gi;
      float upd = (mv[j] / bc1) / (sqrtf(vv[j] / bc2) + eps);
      if (8 * i + j < decay_end) upd += wd * pv[j];
      pv[j] -= lr * upd;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      reinterpret_cast<float4*>(p)[2 * i + h] = make_float4(pv[4 * h], pv[4 * h + 1], pv[4 * h + 2], pv[4 * h + 3]);
      reinterpret_cast<float4*>(m)[2 * i + h] = make_float4(mv[4 * h], mv[4 * h + 1], mv[4 * h + 2], mv[4 * h + 3]);
      reinterpret_cast<float4*>(v)[2 * i + h] = make_float4(vv[4 * h], vv[4 * h + 1], vv[4 * h + 2], vv[4 * h + 3]);
    }
    V8 out;
#pragma unroll
    for (int j = 0; j < 4; ++j) out.h[j] = __floats2bfloat162_rn(pv[2 * j], pv[2 * j + 1]);
    for (int r = 0; r < world; ++r) reinterpret_cast<V8*>(reinterpret_cast<bf16*>(ptrs[r]) + s0)[i] = out;
  }
}

void adamw_p2p_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, at::Tensor ptrs, int64_t s0, int64_t decay_end, double lr,
                    double b1, double b2, double eps, double wd, int64_t step, at::Tensor sqnorm, double clip, double extra_scale) {
  const long n = p.numel();
  AX_CHECK(g.numel() == n && m.numel() == n && v.numel() == n && n % 8 == 0 && s0 % 8 == 0, "buffer sizes (multiples of 8)");
  AX_CHECK(ptrs.is_cuda() && ptrs.scalar_type() == at::kLong, "ptrs: int64 device tensor of parameter buffers");
  if (n == 0) return;
  const float bc1 = 1.f - (float)std::pow(b1, (double)step), bc2 = 1.f - (float)std::pow(b2, (double)step);
  const int ctas = (int)std::min<long>((n / 8 + 255) / 256, num_sms() * 8);
  adamw_p2p_k<<<ctas, 256, 0, stream()>>>(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                                         ptrs.data_ptr<int64_t>(), (int)ptrs.numel(), s0, n, decay_end, (float)lr, (float)b1, (float)b2,
                                         (float)eps, (float)wd, bc1, bc2, sqnorm.data_ptr<float>(), (float)clip, (float)extra_scale);
  AX_LAUNCH_OK();
}

// out[t, :] = table[ids[t], :]   (bf16 rows, H % 8 == 0)
__global__ void embed_fwd_k(const int64_t* __restrict__ ids, const bf16* __restrict__ table, bf16* __restrict__ out, int T, int H) {
  pdl_wait();
  pdl_trigger();
  long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  int per = H / 8;
  if (i >= (long)T * per) return;
  int t = i / per, c = (i % per) * 8;
  *reinterpret_cast<V8*>(out + (long)t * H + c) = *reinterpret_cast<const V8*>(table + ids[t] * (long)H + c);
}

// grad[ids[t], :] += dout[t, :]  (fp32 accumulation, one warp per token)
__global__ void embed_bwd_k(const int64_t* __restrict__ ids, const bf16* __restrict__ dout, float* __restrict__ grad, int T, int H) {
  int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= T) return;
  const bf16* src = dout + (long)w * H;
  float* dst = grad + ids[w] * (long)H;
  for (int c = lane * 8; c < H; c += 256) {
    float f[8];
    load8(src + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(dst + c + j, f[j]);
  }
}

at::Tensor embed_fwd(at::Tensor ids, at::Tensor table) {
  AX_CHECK(ids.scalar_type() == at::kLong && table.scalar_type() == at::kBFloat16 && table.is_contiguous(), "ids int64, table bf16");
  int T = ids.numel(), H = table.size(1);
  auto out = at::empty({T, H}, table.options());
  long n = (long)T * (H / 8);
  if (n == 0) return out;
  launch_pdl(embed_fwd_k, dim3((n + 255) / 256), dim3(256), 0, stream(), (const int64_t*)ids.data_ptr<int64_t>(), (const bf16*)table.data_ptr(), (bf16*)out.data_ptr(), T, H);
  AX_LAUNCH_OK();
  return out;
}

void embed_bwd(at::Tensor ids, at::Tensor dout, at::Tensor grad) {
  AX_CHECK(grad.scalar_type() == at::kFloat && grad.is_contiguous(), "grad fp32");
  int T = ids.numel(), H = grad.size(1);
  if (T == 0) return;
  embed_bwd_k<<<((long)T * 32 + 255) / 256, 256, 0, stream()>>>(ids.data_ptr<int64_t>(), (const bf16*)dout.data_ptr(),
                                                               grad.data_ptr<float>(), T, H);
  AX_LAUNCH_OK();
}

}  // namespace ax
