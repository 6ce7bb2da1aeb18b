// RMSNorm, fused Qwen3 q/k-norm + RoPE (+ optional paged-KV write), SwiGLU.
// All math in fp32, one rounding to bf16 on output.  Reference semantics:
// TE fused RMSNorm / RoPE and Megatron SwiGLU (axrl/utils/megatron/magi_forward.py:405-430).
#include "common.cuh"

namespace ax {

// ----------------------------------------------------------------------------- RMSNorm
// One CTA per row; row re-read from L1/L2 on the second pass.
__global__ void rmsnorm_fwd_k(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ y,
                              float* __restrict__ rstd, int H, float eps) {
  pdl_trigger();  // successors may launch now; they wait for this grid's completion
  pdl_wait();
  __shared__ float sh[32];
  const bf16* xr = x + (size_t)blockIdx.x * H;
  bf16* yr = y + (size_t)blockIdx.x * H;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = block_sum(ss, sh);
  float r = rsqrtf(ss / H + eps);
  if (threadIdx.x == 0) rstd[blockIdx.x] = r;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float f[8], g[8];
    load8(xr + c, f);
    load8(w + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = f[i] * r * g[i];
    store8(yr + c, f);
  }
}

// dx = r * (w*dy - xhat * mean(xhat * w * dy)),  dw partials per CTA.
__global__ void rmsnorm_bwd_k(const bf16* __restrict__ dy, const bf16* __restrict__ x, const bf16* __restrict__ w,
                              const float* __restrict__ rstd, bf16* __restrict__ dx, float* __restrict__ dw_part,
                              int T, int H, int rows_per_cta) {
  __shared__ float sh[32];
  extern __shared__ float dw_acc[];  // H floats
  for (int c = threadIdx.x; c < H; c += blockDim.x) dw_acc[c] = 0.f;
  __syncthreads();
  int r0 = blockIdx.x * rows_per_cta, r1 = min(T, r0 + rows_per_cta);
  for (int row = r0; row < r1; ++row) {
    const bf16* xr = x + (size_t)row * H;
    const bf16* dyr = dy + (size_t)row * H;
    float r = rstd[row];
    float dot = 0.f;
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
      float a[8], g[8], d[8];
      load8(xr + c, a);
      load8(w + c, g);
      load8(dyr + c, d);
#pragma unroll
      for (int i = 0; i < 8; ++i) dot += a[i] * r * g[i] * d[i];
    }
    dot = block_sum(dot, sh) / H;
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
      float a[8], g[8], d[8], o[8];
      load8(xr + c, a);
      load8(w + c, g);
      load8(dyr + c, d);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float xh = a[i] * r;
        o[i] = r * (g[i] * d[i] - xh * dot);
        dw_acc[c + i] += d[i] * xh;  // each thread owns its columns: no race
      }
      store8(dx + (size_t)row * H + c, o);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < H; c += blockDim.x) dw_part[(size_t)blockIdx.x * H + c] = dw_acc[c];
}

std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, at::Tensor w, double eps) {
  AX_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(), "x: contiguous bf16 (T,H)");
  int T = x.size(0), H = x.size(1);
  AX_CHECK(H % 8 == 0, "H % 8");
  at::Tensor wb = w.scalar_type() == at::kBFloat16 ? w.contiguous() : w.to(at::kBFloat16).contiguous();
  auto y = at::empty_like(x);
  auto rstd = at::empty({T}, x.options().dtype(at::kFloat));
  if (T == 0) return {y, rstd};
  int thr = H >= 2048 ? 256 : 128;
  launch_pdl(rmsnorm_fwd_k, dim3(T), dim3(thr), 0, stream(), (const bf16*)x.data_ptr(), (const bf16*)wb.data_ptr(), (bf16*)y.data_ptr(),
                                        rstd.data_ptr<float>(), H, (float)eps);
  AX_LAUNCH_OK();
  return {y, rstd};
}

std::vector<at::Tensor> rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd) {
  int T = x.size(0), H = x.size(1);
  at::Tensor wb = w.scalar_type() == at::kBFloat16 ? w.contiguous() : w.to(at::kBFloat16).contiguous();
  auto dx = at::empty_like(x);
  int ctas = std::min(T, num_sms() * 4);
  if (ctas == 0) return {dx, at::zeros({H}, x.options().dtype(at::kFloat))};
  int rows = (T + ctas - 1) / ctas;
  ctas = (T + rows - 1) / rows;
  auto part = at::empty({ctas, H}, x.options().dtype(at::kFloat));
  int thr = H >= 2048 ? 256 : 128;
  rmsnorm_bwd_k<<<ctas, thr, H * sizeof(float), stream()>>>((const bf16*)dy.data_ptr(), (const bf16*)x.data_ptr(),
                                                           (const bf16*)wb.data_ptr(), rstd.data_ptr<float>(),
                                                           (bf16*)dx.data_ptr(), part.data_ptr<float>(), T, H, rows);
  AX_LAUNCH_OK();
  return {dx, part.sum(0)};
}

// ----------------------------------------------------------------------------- q/k norm + RoPE
// One warp per (token, head), D = 128: lane l owns elements {2l, 2l+1} of each half.
// heads [0, nq) are q, [nq, nq+nkv) are k, [nq+nkv, nq+2nkv) are v (copied).
// If kc/vc (paged caches, [slots, nkv, D]) are given, k/v are also written at slot[t].
template <bool kWriteCache>
__global__ void qknorm_rope_fwd_k(const bf16* __restrict__ qkv, const bf16* __restrict__ qw, const bf16* __restrict__ kw,
                                  const int* __restrict__ pos, const float* __restrict__ inv_freq,
                                  bf16* __restrict__ q, bf16* __restrict__ k, bf16* __restrict__ v,
                                  float* __restrict__ rstd, int T, int nq, int nkv, float eps,
                                  bf16* __restrict__ kc, bf16* __restrict__ vc, const int64_t* __restrict__ slots, int P) {
  pdl_trigger();  // successors may launch now; they wait for this grid's completion
  pdl_wait();
  constexpr int D = 128;
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  int nh = nq + 2 * nkv;
  if (warp >= T * nh) return;
  int t = warp / nh, h = warp % nh;
  const bf16* src = qkv + ((size_t)t * nh + h) * D;
  int i0 = 2 * lane, i1 = D / 2 + 2 * lane;
  float2 a = __bfloat1622float2(*reinterpret_cast<const bf162*>(src + i0));
  float2 b = __bfloat1622float2(*reinterpret_cast<const bf162*>(src + i1));
  if (h >= nq + nkv) {  // v: copy
    int hv = h - nq - nkv;
    bf16* dst = v + ((size_t)t * nkv + hv) * D;
    *reinterpret_cast<bf162*>(dst + i0) = __floats2bfloat162_rn(a.x, a.y);
    *reinterpret_cast<bf162*>(dst + i1) = __floats2bfloat162_rn(b.x, b.y);
    if (kWriteCache) {
      long sl = slots[t];
      bf16* cd = vc + (((sl / P) * nkv + hv) * P + sl % P) * D;
      *reinterpret_cast<bf162*>(cd + i0) = __floats2bfloat162_rn(a.x, a.y);
      *reinterpret_cast<bf162*>(cd + i1) = __floats2bfloat162_rn(b.x, b.y);
    }
    return;
  }
  float ss = warp_sum(a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y);
  float r = rsqrtf(ss / D + eps);
  bool isq = h < nq;
  const bf16* wv = isq ? qw : kw;
  float2 wa = __bfloat1622float2(*reinterpret_cast<const bf162*>(wv + i0));
  float2 wb = __bfloat1622float2(*reinterpret_cast<const bf162*>(wv + i1));
  a.x *= r * wa.x; a.y *= r * wa.y; b.x *= r * wb.x; b.y *= r * wb.y;
  float p = (float)pos[t];
  float s0, c0, s1, c1;
  sincosf(p * inv_freq[2 * lane], &s0, &c0);
  sincosf(p * inv_freq[2 * lane + 1], &s1, &c1);
  float2 oa = make_float2(a.x * c0 - b.x * s0, a.y * c1 - b.y * s1);
  float2 ob = make_float2(b.x * c0 + a.x * s0, b.y * c1 + a.y * s1);
  bf16* dst = isq ? q + ((size_t)t * nq + h) * D : k + ((size_t)t * nkv + (h - nq)) * D;
  *reinterpret_cast<bf162*>(dst + i0) = __floats2bfloat162_rn(oa.x, oa.y);
  *reinterpret_cast<bf162*>(dst + i1) = __floats2bfloat162_rn(ob.x, ob.y);
  if (kWriteCache && !isq) {
    long sl = slots[t];
    bf16* cd = kc + (((sl / P) * nkv + (h - nq)) * P + sl % P) * D;
    *reinterpret_cast<bf162*>(cd + i0) = __floats2bfloat162_rn(oa.x, oa.y);
    *reinterpret_cast<bf162*>(cd + i1) = __floats2bfloat162_rn(ob.x, ob.y);
  }
  if (lane == 0 && rstd) rstd[(size_t)t * (nq + nkv) + h] = r;
}

// Backward: inverse rotation, through weight, through RMSNorm.  dw accumulated per CTA in smem.
__global__ void qknorm_rope_bwd_k(const bf16* __restrict__ dq, const bf16* __restrict__ dk, const bf16* __restrict__ dv,
                                  const bf16* __restrict__ qkv, const bf16* __restrict__ qw, const bf16* __restrict__ kw,
                                  const int* __restrict__ pos, const float* __restrict__ inv_freq,
                                  const float* __restrict__ rstd, bf16* __restrict__ dqkv, float* __restrict__ dqw,
                                  float* __restrict__ dkw, int T, int nq, int nkv) {
  constexpr int D = 128;
  __shared__ float acc[2][D];
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) (&acc[0][0])[i] = 0.f;
  __syncthreads();
  int lane = threadIdx.x & 31;
  int nh = nq + 2 * nkv;
  int i0 = 2 * lane, i1 = D / 2 + 2 * lane;
  float aq[4] = {0, 0, 0, 0}, ak[4] = {0, 0, 0, 0};
  int warps_total = gridDim.x * (blockDim.x >> 5);
  for (int item = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; item < T * nh; item += warps_total) {
    int t = item / nh, h = item % nh;
    bf16* out = dqkv + ((size_t)t * nh + h) * D;
    if (h >= nq + nkv) {
      const bf16* g = dv + ((size_t)t * nkv + (h - nq - nkv)) * D;
      *reinterpret_cast<bf162*>(out + i0) = *reinterpret_cast<const bf162*>(g + i0);
      *reinterpret_cast<bf162*>(out + i1) = *reinterpret_cast<const bf162*>(g + i1);
      continue;
    }
    bool isq = h < nq;
    const bf16* g = isq ? dq + ((size_t)t * nq + h) * D : dk + ((size_t)t * nkv + (h - nq)) * D;
    float2 ga = __bfloat1622float2(*reinterpret_cast<const bf162*>(g + i0));
    float2 gb = __bfloat1622float2(*reinterpret_cast<const bf162*>(g + i1));
    float p = (float)pos[t];
    float s0, c0, s1, c1;
    sincosf(p * inv_freq[2 * lane], &s0, &c0);
    sincosf(p * inv_freq[2 * lane + 1], &s1, &c1);
    // d(normed) = R^T g
    float2 na = make_float2(ga.x * c0 + gb.x * s0, ga.y * c1 + gb.y * s1);
    float2 nb = make_float2(gb.x * c0 - ga.x * s0, gb.y * c1 - ga.y * s1);
    const bf16* src = qkv + ((size_t)t * nh + h) * D;
    float2 xa = __bfloat1622float2(*reinterpret_cast<const bf162*>(src + i0));
    float2 xb = __bfloat1622float2(*reinterpret_cast<const bf162*>(src + i1));
    float r = rstd[(size_t)t * (nq + nkv) + h];
    const bf16* wv = isq ? qw : kw;
    float2 wa = __bfloat1622float2(*reinterpret_cast<const bf162*>(wv + i0));
    float2 wb = __bfloat1622float2(*reinterpret_cast<const bf162*>(wv + i1));
    float xh[4] = {xa.x * r, xa.y * r, xb.x * r, xb.y * r};
    float dn[4] = {na.x, na.y, nb.x, nb.y};
    float wf[4] = {wa.x, wa.y, wb.x, wb.y};
    float* accp = isq ? aq : ak;
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      accp[j] += dn[j] * xh[j];
      dot += xh[j] * wf[j] * dn[j];
    }
    dot = warp_sum(dot) / D;
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = r * (wf[j] * dn[j] - xh[j] * dot);
    *reinterpret_cast<bf162*>(out + i0) = __floats2bfloat162_rn(o[0], o[1]);
    *reinterpret_cast<bf162*>(out + i1) = __floats2bfloat162_rn(o[2], o[3]);
  }
  atomicAdd(&acc[0][i0], aq[0]); atomicAdd(&acc[0][i0 + 1], aq[1]);
  atomicAdd(&acc[0][i1], aq[2]); atomicAdd(&acc[0][i1 + 1], aq[3]);
  atomicAdd(&acc[1][i0], ak[0]); atomicAdd(&acc[1][i0 + 1], ak[1]);
  atomicAdd(&acc[1][i1], ak[2]); atomicAdd(&acc[1][i1 + 1], ak[3]);
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    atomicAdd(dqw + i, acc[0][i]);
    atomicAdd(dkw + i, acc[1][i]);
  }
}

static at::Tensor as_bf16(const at::Tensor& t) { return t.scalar_type() == at::kBFloat16 ? t.contiguous() : t.to(at::kBFloat16).contiguous(); }

std::vector<at::Tensor> qknorm_rope_fwd(at::Tensor qkv, at::Tensor qw, at::Tensor kw, at::Tensor pos, at::Tensor inv_freq,
                                        int64_t nq, int64_t nkv, double eps) {
  AX_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous(), "qkv bf16 contiguous");
  int T = qkv.size(0);
  int D = inv_freq.numel() * 2;
  AX_CHECK(D == 128, "head_dim 128 supported");
  AX_CHECK(qkv.size(1) == (nq + 2 * nkv) * D, "qkv width");
  auto opt = qkv.options();
  auto q = at::empty({T, nq, D}, opt), k = at::empty({T, nkv, D}, opt), v = at::empty({T, nkv, D}, opt);
  auto rstd = at::empty({T, nq + nkv}, opt.dtype(at::kFloat));
  long warps = (long)T * (nq + 2 * nkv);
  if (warps == 0) return {q, k, v, rstd};
  auto qwb = as_bf16(qw), kwb = as_bf16(kw);
  auto p32 = pos.scalar_type() == at::kInt ? pos.contiguous() : pos.to(at::kInt).contiguous();
  auto inv = inv_freq.to(at::kFloat).contiguous();
  launch_pdl(qknorm_rope_fwd_k<false>, dim3((warps * 32 + 255) / 256), dim3(256), 0, stream(),
      (const bf16*)qkv.data_ptr(), (const bf16*)qwb.data_ptr(), (const bf16*)kwb.data_ptr(), p32.data_ptr<int>(),
      inv.data_ptr<float>(), (bf16*)q.data_ptr(), (bf16*)k.data_ptr(), (bf16*)v.data_ptr(), rstd.data_ptr<float>(), T, nq,
      nkv, (float)eps, nullptr, nullptr, nullptr, 1);
  AX_LAUNCH_OK();
  return {q, k, v, rstd};
}

// Inference variant: also scatters k/v into paged caches k_cache/v_cache ([pages, nkv, P, D]) at slots[t]
// (slot = page * P + offset).
std::vector<at::Tensor> qknorm_rope_cache(at::Tensor qkv, at::Tensor qw, at::Tensor kw, at::Tensor pos, at::Tensor inv_freq,
                                          int64_t nq, int64_t nkv, double eps, at::Tensor k_cache, at::Tensor v_cache,
                                          at::Tensor slots) {
  int T = qkv.size(0);
  int D = inv_freq.numel() * 2;
  AX_CHECK(D == 128, "head_dim 128 supported");
  AX_CHECK(slots.scalar_type() == at::kLong && slots.numel() == T, "slots int64 (T,)");
  auto opt = qkv.options();
  auto q = at::empty({T, nq, D}, opt), k = at::empty({T, nkv, D}, opt), v = at::empty({T, nkv, D}, opt);
  long warps = (long)T * (nq + 2 * nkv);
  if (warps == 0) return {q, k, v};
  launch_pdl(qknorm_rope_fwd_k<true>, dim3((warps * 32 + 255) / 256), dim3(256), 0, stream(),
      (const bf16*)qkv.data_ptr(), (const bf16*)qw.data_ptr(), (const bf16*)kw.data_ptr(), pos.data_ptr<int>(),
      inv_freq.data_ptr<float>(), (bf16*)q.data_ptr(), (bf16*)k.data_ptr(), (bf16*)v.data_ptr(), nullptr, T, nq, nkv,
      (float)eps, (bf16*)k_cache.data_ptr(), (bf16*)v_cache.data_ptr(), slots.data_ptr<int64_t>(), (int)k_cache.size(2));
  AX_LAUNCH_OK();
  return {q, k, v};
}

std::vector<at::Tensor> qknorm_rope_bwd(at::Tensor dq, at::Tensor dk, at::Tensor dv, at::Tensor qkv, at::Tensor qw,
                                        at::Tensor kw, at::Tensor pos, at::Tensor inv_freq, at::Tensor rstd, int64_t nq,
                                        int64_t nkv) {
  int T = qkv.size(0);
  auto dqkv = at::empty_like(qkv);
  auto dqw = at::zeros({128}, qkv.options().dtype(at::kFloat));
  auto dkw = at::zeros({128}, qkv.options().dtype(at::kFloat));
  long items = (long)T * (nq + 2 * nkv);
  if (items == 0) return {dqkv, dqw, dkw};
  auto qwb = as_bf16(qw), kwb = as_bf16(kw);
  auto p32 = pos.scalar_type() == at::kInt ? pos.contiguous() : pos.to(at::kInt).contiguous();
  auto inv = inv_freq.to(at::kFloat).contiguous();
  int ctas = std::min<long>((items + 7) / 8, num_sms() * 8);
  qknorm_rope_bwd_k<<<ctas, 256, 0, stream()>>>((const bf16*)dq.data_ptr(), (const bf16*)dk.data_ptr(), (const bf16*)dv.data_ptr(),
                                               (const bf16*)qkv.data_ptr(), (const bf16*)qwb.data_ptr(),
                                               (const bf16*)kwb.data_ptr(), p32.data_ptr<int>(), inv.data_ptr<float>(),
                                               rstd.data_ptr<float>(), (bf16*)dqkv.data_ptr(), dqw.data_ptr<float>(),
                                               dkw.data_ptr<float>(), T, nq, nkv);
  AX_LAUNCH_OK();
  return {dqkv, dqw, dkw};
}

// ----------------------------------------------------------------------------- SwiGLU
__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }

__global__ void swiglu_fwd_k(const bf16* __restrict__ gu, bf16* __restrict__ y, long T, int F) {
  pdl_trigger();  // successors may launch now; they wait for this grid's completion
  pdl_wait();
  long n8 = T * (F / 8);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    long t = i / (F / 8);
    int c = (int)(i % (F / 8)) * 8;
    float g[8], u[8], o[8];
    load8(gu + t * 2 * F + c, g);
    load8(gu + t * 2 * F + F + c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = g[j] * sigm(g[j]) * u[j];
    store8(y + t * F + c, o);
  }
}

__global__ void swiglu_bwd_k(const bf16* __restrict__ dy, const bf16* __restrict__ gu, bf16* __restrict__ dgu, long T, int F) {
  long n8 = T * (F / 8);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    long t = i / (F / 8);
    int c = (int)(i % (F / 8)) * 8;
    float g[8], u[8], d[8], dg[8], du[8];
    load8(gu + t * 2 * F + c, g);
    load8(gu + t * 2 * F + F + c, u);
    load8(dy + t * F + c, d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float s = sigm(g[j]);
      du[j] = d[j] * g[j] * s;
      dg[j] = d[j] * u[j] * s * (1.f + g[j] * (1.f - s));
    }
    store8(dgu + t * 2 * F + c, dg);
    store8(dgu + t * 2 * F + F + c, du);
  }
}

at::Tensor swiglu_fwd(at::Tensor gu) {
  AX_CHECK(gu.scalar_type() == at::kBFloat16 && gu.is_contiguous(), "gate_up bf16 contiguous");
  long T = gu.numel() / gu.size(-1);
  int F = gu.size(-1) / 2;
  AX_CHECK(F % 8 == 0, "F % 8");
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto y = at::empty(sizes, gu.options());
  long n8 = T * (F / 8);
  if (n8 == 0) return y;
  int ctas = (int)std::min<long>((n8 + 255) / 256, num_sms() * 16);
  launch_pdl(swiglu_fwd_k, dim3(ctas), dim3(256), 0, stream(), (const bf16*)gu.data_ptr(), (bf16*)y.data_ptr(), T, F);
  AX_LAUNCH_OK();
  return y;
}

at::Tensor swiglu_bwd(at::Tensor dy, at::Tensor gu) {
  long T = gu.numel() / gu.size(-1);
  int F = gu.size(-1) / 2;
  auto dgu = at::empty_like(gu);
  long n8 = T * (F / 8);
  if (n8 == 0) return dgu;
  int ctas = (int)std::min<long>((n8 + 255) / 256, num_sms() * 16);
  swiglu_bwd_k<<<ctas, 256, 0, stream()>>>((const bf16*)dy.data_ptr(), (const bf16*)gu.data_ptr(), (bf16*)dgu.data_ptr(), T, F);
  AX_LAUNCH_OK();
  return dgu;
}

}  // namespace ax
