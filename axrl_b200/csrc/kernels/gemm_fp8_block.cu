// Block-scaled fp8 (e4m3) GEMM for rollout serving, on 5th-gen tensor cores:
//   Y[M,N] (bf16) = sum_kb (Xq[M, kb] @ Wq[N, kb]^T) * sx[m, kb] * sw[n/128, kb]
// X is quantised per token and 128-wide K group (1x128 scales), W per 128x128 block — the layout
// the trainer->rollout weight sync produces (e4m3 values + fp32 dequantisation scales).  Built from
// the CUTLASS sm100 blockwise-scaling collective (tcgen05.mma kind::f8f6f4, TMEM accumulators, TMA,
// cluster 1x1x1: no multicast) inside our own wrapper; scales are K-major ([m][kb], [nb][kb]).
//
// quant_fp8_rows: x (bf16) -> e4m3 values + per (row, 128-group) scales amax/448, one warp per group.
//
// Reference counterpart: the blockwise-fp8 rollout of the MoE model (SGLang fp8 checkpoints,
// tests/moe/test_fp8_mismatch_results.py:22-23) and Megatron fp8_recipe="blockwise"
// (axrl/configs.py:391).
#include <cuda_fp8.h>

#include "common.cuh"
#include "cutlass/detail/blockwise_scale_layout.hpp"
#include "gemm_sm100.cuh"

namespace ax {
namespace fp8 {

using namespace cute;
using ElemA = cutlass::float_e4m3_t;
using ElemB = cutlass::float_e4m3_t;
using Tile = Shape<_128, _128, _128>;
using Cluster = Shape<_1, _1, _1>;
using ScaleConfig = cutlass::detail::Sm100BlockwiseScaleConfig<1, 128, 128, cute::UMMA::Major::K, cute::UMMA::Major::K>;
using LayoutSFA = decltype(ScaleConfig::deduce_layoutSFA());
using LayoutSFB = decltype(ScaleConfig::deduce_layoutSFB());

using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, Tile, Cluster, cutlass::epilogue::collective::EpilogueTileAuto, float, float,
    cutlass::bfloat16_t, cutlass::layout::RowMajor, 8, cutlass::bfloat16_t, cutlass::layout::RowMajor, 8,
    cutlass::epilogue::TmaWarpSpecialized1Sm>::CollectiveOp;
using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, ElemA, cute::tuple<cutlass::layout::RowMajor, LayoutSFA>, 16, ElemB,
    cute::tuple<cutlass::layout::ColumnMajor, LayoutSFB>, 16, float, Tile, Cluster,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
    cutlass::gemm::KernelTmaWarpSpecializedBlockwise1SmSm100>::CollectiveOp;
using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop, Epilogue, void>;
using Op = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;

__global__ void quant_rows_k(const bf16* __restrict__ x, long M, int K, __nv_fp8_e4m3* __restrict__ q, float* __restrict__ s) {
  const int groups = K / 128;
  const long warp = (blockIdx.x * (long)blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (warp >= M * groups) return;
  const long row = warp / groups;
  const int g = (int)(warp % groups);
  const bf16* src = x + row * K + g * 128 + lane * 4;
  float v[4];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = __bfloat162float(src[j]);
    amax = fmaxf(amax, fabsf(v[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = fmaxf(amax, 1e-12f) / 448.f;
  const float inv = 1.f / scale;
  __nv_fp8_e4m3* dst = q + row * K + g * 128 + lane * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) dst[j] = __nv_fp8_e4m3(v[j] * inv);
  if (lane == 0) s[row * groups + g] = scale;
}

}  // namespace fp8

// x (M,K) bf16 -> (q (M,K) e4m3, s (M, K/128) fp32)
std::vector<at::Tensor> quant_fp8_rows(at::Tensor x) {
  AX_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x: contiguous bf16 (M, K)");
  long M = x.size(0);
  int K = x.size(1);
  AX_CHECK(K % 128 == 0, "K must be a multiple of 128");
  auto q = at::empty({M, K}, x.options().dtype(at::kFloat8_e4m3fn));
  auto s = at::empty({M, K / 128}, x.options().dtype(at::kFloat));
  long warps = M * (K / 128);
  if (warps) {
    fp8::quant_rows_k<<<(int)((warps * 32 + 255) / 256), 256, 0, stream()>>>((const bf16*)x.data_ptr(), M, K,
                                                                             (__nv_fp8_e4m3*)q.data_ptr(), s.data_ptr<float>());
    AX_LAUNCH_OK();
  }
  return {q, s};
}

// y (M,N) bf16 = blockwise-scaled xq @ wq^T
at::Tensor fp8_block_linear(at::Tensor xq, at::Tensor xs, at::Tensor wq, at::Tensor ws) {
  AX_CHECK(xq.is_cuda() && xq.scalar_type() == at::kFloat8_e4m3fn && xq.is_contiguous() && xq.dim() == 2, "xq: e4m3 (M,K)");
  AX_CHECK(wq.is_cuda() && wq.scalar_type() == at::kFloat8_e4m3fn && wq.is_contiguous() && wq.dim() == 2, "wq: e4m3 (N,K)");
  int M = xq.size(0), K = xq.size(1), N = wq.size(0);
  AX_CHECK(wq.size(1) == K && K % 128 == 0 && N % 128 == 0, "shapes: K and N multiples of 128");
  AX_CHECK(xs.scalar_type() == at::kFloat && xs.is_contiguous() && xs.size(0) == M && xs.size(1) == K / 128, "xs: (M, K/128) fp32");
  AX_CHECK(ws.scalar_type() == at::kFloat && ws.is_contiguous() && ws.size(0) == N / 128 && ws.size(1) == K / 128, "ws: (N/128, K/128) fp32");
  auto y = at::empty({M, N}, xq.options().dtype(at::kBFloat16));
  if (M == 0) return y;
  using namespace fp8;
  using SA = typename Kernel::StrideA;
  using SB = typename Kernel::StrideB;
  using SC = typename Kernel::StrideC;
  using SD = typename Kernel::StrideD;
  auto shape = make_shape(M, N, K, 1);
  typename Op::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                              {M, N, K, 1},
                              {(const ElemA*)xq.data_ptr(), cutlass::make_cute_packed_stride(SA{}, make_shape(M, K, 1)),
                               (const ElemB*)wq.data_ptr(), cutlass::make_cute_packed_stride(SB{}, make_shape(N, K, 1)),
                               xs.data_ptr<float>(), ScaleConfig::tile_atom_to_shape_SFA(shape), ws.data_ptr<float>(),
                               ScaleConfig::tile_atom_to_shape_SFB(shape)},
                              {{1.f, 0.f}, nullptr, cutlass::make_cute_packed_stride(SC{}, make_shape(M, N, 1)),
                               (cutlass::bfloat16_t*)y.data_ptr(), cutlass::make_cute_packed_stride(SD{}, make_shape(M, N, 1))}};
  cudaGetDevice(&args.hw_info.device_id);
  args.hw_info.sm_count = num_sms();
  Op op;
  AX_CHECK(op.can_implement(args) == cutlass::Status::kSuccess, "fp8 block GEMM cannot implement M=", M, " N=", N, " K=", K);
  size_t wsz = Op::get_workspace_size(args);
  at::Tensor wst;
  if (wsz) wst = at::empty({(int64_t)wsz}, xq.options().dtype(at::kByte));
  AX_CHECK(op.initialize(args, wsz ? wst.data_ptr() : nullptr, stream()) == cutlass::Status::kSuccess, "fp8 GEMM init");
  AX_CHECK(op.run(stream()) == cutlass::Status::kSuccess, "fp8 GEMM run");
  return y;
}

}  // namespace ax
