// Fused MoE router: softmax over the expert logits, top-k selection, optional replay of recorded
// expert ids (R3), optional renormalisation of the selected probabilities — one warp per token.
//
// Reference semantics: the Megatron router with fp32 scores and RouterReplay
// (axrl/utils/megatron/router_replay.py:67-108): weights are the softmax probabilities of the
// chosen experts (replayed ids where the replay mask is set, the live top-k elsewhere), divided by
// their sum when norm_topk_prob is set.  Ties in top-k prefer the lower expert id.
#include "common.cuh"

namespace ax {

template <int EPL>  // experts per lane (E <= 32 * EPL)
__global__ void router_topk_k(const float* __restrict__ logits, int T, int E, int k, int renorm, const int64_t* __restrict__ replay,
                              const bool* __restrict__ replay_mask, float* __restrict__ probs, float* __restrict__ w_out,
                              int64_t* __restrict__ id_out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* row = logits + (long)warp * E;
  float v[EPL];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    int e = lane + 32 * j;
    v[j] = e < E ? row[e] : -INFINITY;
    m = fmaxf(m, v[j]);
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    v[j] = (lane + 32 * j) < E ? expf(v[j] - m) : 0.f;
    s += v[j];
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float inv = 1.f / s;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    v[j] *= inv;
    int e = lane + 32 * j;
    if (e < E) probs[(long)warp * E + e] = v[j];
  }
  const bool use_replay = replay != nullptr && (replay_mask == nullptr || replay_mask[warp]);
  float sel_sum = 0.f;
  float chosen[8];
  int chosen_id[8];
  float taken[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) taken[j] = v[j];
  for (int r = 0; r < k; ++r) {
    int id;
    float p;
    if (use_replay) {
      id = (int)replay[(long)warp * k + r];
      p = __shfl_sync(0xffffffffu, v[(id >> 5) < EPL ? (id >> 5) : 0], id & 31);
    } else {
      // warp argmax over the not-yet-taken probabilities (lower id wins ties)
      float best = -1.f;
      int bid = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        int e = lane + 32 * j;
        if (e < E && (taken[j] > best || (taken[j] == best && e < bid))) {
          best = taken[j];
          bid = e;
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        float ob = __shfl_xor_sync(0xffffffffu, best, o);
        int oid = __shfl_xor_sync(0xffffffffu, bid, o);
        if (ob > best || (ob == best && oid < bid)) {
          best = ob;
          bid = oid;
        }
      }
      id = bid;
      p = best;
      if ((id & 31) == lane) taken[id >> 5] = -2.f;  // remove from further rounds
    }
    if (r < 8) {
      chosen[r] = p;
      chosen_id[r] = id;
    }
    sel_sum += p;
  }
  if (lane == 0) {
    const float scale = renorm ? 1.f / fmaxf(sel_sum, 1e-20f) : 1.f;
    for (int r = 0; r < k; ++r) {
      w_out[(long)warp * k + r] = chosen[r] * scale;
      id_out[(long)warp * k + r] = chosen_id[r];
    }
  }
}

std::vector<at::Tensor> router_topk(at::Tensor logits, int64_t k, bool renorm, c10::optional<at::Tensor> replay,
                                    c10::optional<at::Tensor> replay_mask) {
  AX_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.is_contiguous() && logits.dim() == 2, "logits: fp32 (T, E)");
  int T = logits.size(0), E = logits.size(1);
  AX_CHECK(k >= 1 && k <= 8 && k <= E && E <= 256, "router: k <= 8, E <= 256");
  if (replay) AX_CHECK(replay->scalar_type() == at::kLong && replay->is_contiguous() && replay->size(0) == T && replay->size(1) == k, "replay ids");
  if (replay_mask) AX_CHECK(replay_mask->scalar_type() == at::kBool && replay_mask->numel() == T, "replay mask");
  auto probs = at::empty({T, E}, logits.options());
  auto w = at::empty({T, k}, logits.options());
  auto ids = at::empty({T, k}, logits.options().dtype(at::kLong));
  if (T == 0) return {w, ids, probs};
  int blocks = (T * 32 + 255) / 256;
  const int64_t* rp = replay ? replay->data_ptr<int64_t>() : nullptr;
  const bool* rm = replay_mask ? replay_mask->data_ptr<bool>() : nullptr;
  if (E <= 128)
    router_topk_k<4><<<blocks, 256, 0, stream()>>>(logits.data_ptr<float>(), T, E, (int)k, renorm, rp, rm, probs.data_ptr<float>(),
                                                   w.data_ptr<float>(), ids.data_ptr<int64_t>());
  else
    router_topk_k<8><<<blocks, 256, 0, stream()>>>(logits.data_ptr<float>(), T, E, (int)k, renorm, rp, rm, probs.data_ptr<float>(),
                                                   w.data_ptr<float>(), ids.data_ptr<int64_t>());
  AX_LAUNCH_OK();
  return {w, ids, probs};
}

// Weighted top-k combine of expert outputs: out[t] = sum_j w[t, j] * y[pos[t k + j]], summed in
// fp32 and stored as bf16 (one gather per token instead of scattering every (token, expert) row
// into an fp32 buffer with atomics).  One warp per token, 8 bf16 per lane per step, k <= 8.
__global__ void moe_combine_fwd_k(const bf16* __restrict__ y, const float* __restrict__ w, const int* __restrict__ pos,
                                  bf16* __restrict__ out, int T, int k, int H) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (t >= T) return;
  int p[8];
  float wt[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    p[j] = j < k ? pos[(long)t * k + j] : 0;
    wt[j] = j < k ? w[(long)t * k + j] : 0.f;
  }
  for (int c = lane * 8; c < H; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= k) break;
      float v[8];
      load8(y + (long)p[j] * H + c, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += wt[j] * v[e];
    }
    store8(out + (long)t * H + c, acc);
  }
}

// Its backward: dy[pos[t k + j]] = w[t, j] * dout[t] (bf16), dw[t, j] = <y[pos[t k + j]], dout[t]> (fp32).
__global__ void moe_combine_bwd_k(const bf16* __restrict__ y, const float* __restrict__ w, const int* __restrict__ pos,
                                  const bf16* __restrict__ dout, bf16* __restrict__ dy, float* __restrict__ dw, int T, int k, int H) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (t >= T) return;
  int p[8];
  float wt[8], dot[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    p[j] = j < k ? pos[(long)t * k + j] : 0;
    wt[j] = j < k ? w[(long)t * k + j] : 0.f;
    dot[j] = 0.f;
  }
  for (int c = lane * 8; c < H; c += 256) {
    float g[8];
    load8(dout + (long)t * H + c, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= k) break;
      float v[8], d[8];
      load8(y + (long)p[j] * H + c, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        dot[j] += v[e] * g[e];
        d[e] = wt[j] * g[e];
      }
      store8(dy + (long)p[j] * H + c, d);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j >= k) break;
    const float s = warp_sum(dot[j]);
    if (lane == 0) dw[(long)t * k + j] = s;
  }
}

// y (R, H) bf16 rows, w (T, k) fp32, pos (T k) int32 row of y for each (token, slot) -> (T, H) bf16
at::Tensor moe_combine(at::Tensor y, at::Tensor w, at::Tensor pos) {
  AX_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.dim() == 2 && y.size(1) % 8 == 0, "y: (R, H) bf16, H % 8 == 0");
  AX_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.dim() == 2 && w.size(1) <= 8, "w: (T, k <= 8) fp32");
  AX_CHECK(pos.scalar_type() == at::kInt && pos.is_contiguous() && pos.numel() == w.numel(), "pos: (T k) int32");
  const int T = w.size(0), k = w.size(1), H = y.size(1);
  auto out = at::empty({T, H}, y.options());
  if (T == 0) return out;
  moe_combine_fwd_k<<<(T * 32 + 255) / 256, 256, 0, stream()>>>((const bf16*)y.data_ptr(), w.data_ptr<float>(), pos.data_ptr<int>(),
                                                                (bf16*)out.data_ptr(), T, k, H);
  AX_LAUNCH_OK();
  return out;
}

std::vector<at::Tensor> moe_combine_bwd(at::Tensor y, at::Tensor w, at::Tensor pos, at::Tensor dout) {
  AX_CHECK(dout.scalar_type() == at::kBFloat16 && dout.is_contiguous() && dout.size(0) == w.size(0) && dout.size(1) == y.size(1),
           "dout: (T, H) bf16");
  const int T = w.size(0), k = w.size(1), H = y.size(1);
  auto dy = at::zeros_like(y);  // rows no token points at (dropped or padding) get zero gradient
  auto dw = at::empty_like(w);
  if (T == 0) return {dy, dw};
  moe_combine_bwd_k<<<(T * 32 + 255) / 256, 256, 0, stream()>>>((const bf16*)y.data_ptr(), w.data_ptr<float>(), pos.data_ptr<int>(),
                                                                (const bf16*)dout.data_ptr(), (bf16*)dy.data_ptr(), dw.data_ptr<float>(),
                                                                T, k, H);
  AX_LAUNCH_OK();
  return {dy, dw};
}

}  // namespace ax
