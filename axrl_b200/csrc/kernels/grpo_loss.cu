// Fused per-token GRPO / PPO clipped policy objective and its gradient.
//
// For every token (fp32):
//   r     = exp(clamp(lp - base, -20, 20))
//   ppo   = max(-A r, -A clamp(r, 1 - lo, 1 + hi))
//   pg    = A < 0 && dual > 0 ? min(-dual A, ppo) : ppo           (dual clip on negative advantages)
//   out   = pg * w                                                  (w: truncated IS weight x masks)
//   dout/dlp = w * dpg/dlp, with max/min/clamp following autograd's conventions (ties split the
//   gradient in half; clamp passes it on the closed interval; the log-ratio clamp stops it).
// Also written: r, and the effective clipped ratio pg / (-A) (1 where |A| < 1e-4) for the metrics.
// One launch replaces the ~15 elementwise kernels (forward and backward) of the PyTorch objective.
//
// Reference semantics: grpo_loss / ppo_loss of axrl/trainer/grpo_trainer.py:197-803.
#include "common.cuh"

namespace ax {

__global__ void grpo_pg_k(const float* __restrict__ lp, const float* __restrict__ base, const float* __restrict__ adv,
                          const float* __restrict__ w, long n, float lo, float hi, float dual, float* __restrict__ out,
                          float* __restrict__ grad, float* __restrict__ ratio_out, float* __restrict__ eff_out) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float A = adv[i];
    const float d = lp[i] - base[i];
    const float dc = fminf(fmaxf(d, -20.f), 20.f);
    const float dr_dlp_scale = (d >= -20.f && d <= 20.f) ? 1.f : 0.f;  // clamp gradient (closed interval)
    const float r = expf(dc);
    const float dr = r * dr_dlp_scale;                                   // d r / d lp
    const float rc = fminf(fmaxf(r, 1.f - lo), 1.f + hi);
    const float dclip = (r >= 1.f - lo && r <= 1.f + hi) ? 1.f : 0.f;
    const float u = -A * r, c = -A * rc;
    const float du = -A * dr, dcl = -A * dclip * dr;
    float ppo, dppo;
    if (u > c) { ppo = u; dppo = du; }
    else if (u < c) { ppo = c; dppo = dcl; }
    else { ppo = u; dppo = 0.5f * (du + dcl); }
    float pg = ppo, dpg = dppo;
    if (dual > 0.f && A < 0.f) {
      const float cap = -dual * A;
      if (cap < ppo) { pg = cap; dpg = 0.f; }
      else if (cap == ppo) { dpg = 0.5f * dppo; }
    }
    const float wi = w[i];
    out[i] = pg * wi;
    grad[i] = dpg * wi;
    ratio_out[i] = r;
    eff_out[i] = fabsf(A) < 1e-4f ? 1.f : pg / (-A);
  }
}

// out = g_scalar_or_tensor * grad (elementwise backward)
__global__ void scale_by_k(const float* __restrict__ g, const float* __restrict__ grad, long n, float* __restrict__ out) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) out[i] = g[i] * grad[i];
}

std::vector<at::Tensor> grpo_pg_fwd(at::Tensor lp, at::Tensor base, at::Tensor adv, at::Tensor w, double lo, double hi, double dual) {
  for (auto* t : {&lp, &base, &adv, &w})
    AX_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == lp.numel(), "fp32 contiguous inputs");
  auto out = at::empty_like(lp), grad = at::empty_like(lp), ratio = at::empty_like(lp), eff = at::empty_like(lp);
  long n = lp.numel();
  if (n) {
    int ctas = (int)std::min<long>((n + 255) / 256, (long)num_sms() * 8);
    grpo_pg_k<<<ctas, 256, 0, stream()>>>(lp.data_ptr<float>(), base.data_ptr<float>(), adv.data_ptr<float>(), w.data_ptr<float>(), n,
                                         (float)lo, (float)hi, (float)dual, out.data_ptr<float>(), grad.data_ptr<float>(),
                                         ratio.data_ptr<float>(), eff.data_ptr<float>());
    AX_LAUNCH_OK();
  }
  return {out, grad, ratio, eff};
}

at::Tensor grpo_pg_bwd(at::Tensor g, at::Tensor grad) {
  auto gc = g.contiguous();
  AX_CHECK(gc.scalar_type() == at::kFloat && gc.numel() == grad.numel(), "grad shape");
  auto out = at::empty_like(grad);
  long n = grad.numel();
  if (n) {
    int ctas = (int)std::min<long>((n + 255) / 256, (long)num_sms() * 8);
    scale_by_k<<<ctas, 256, 0, stream()>>>(gc.data_ptr<float>(), grad.data_ptr<float>(), n, out.data_ptr<float>());
    AX_LAUNCH_OK();
  }
  return out;
}

}  // namespace ax
