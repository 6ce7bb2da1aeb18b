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

void quant_rows(const void* x, long M, int K, void* q, float* s, cudaStream_t st) {
  long warps = M * (K / 128);
  if (!warps) return;
  quant_rows_k<<<(int)((warps * 32 + 255) / 256), 256, 0, st>>>((const bf16*)x, M, K, (__nv_fp8_e4m3*)q, s);
  AX_LAUNCH_OK();
}

// y (M,N) bf16 = blockwise-scaled xq @ wq^T; xs (M, K/128), ws (N/128, K/128) fp32, K-major.
void block_linear(const void* xq, const float* xs, const void* wq, const float* ws, void* y, int M, int N, int K, cudaStream_t st) {
  using SA = typename Kernel::StrideA;
  using SB = typename Kernel::StrideB;
  using SC = typename Kernel::StrideC;
  using SD = typename Kernel::StrideD;
  auto shape = make_shape(M, N, K, 1);
  typename Op::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                              {M, N, K, 1},
                              {(const ElemA*)xq, cutlass::make_cute_packed_stride(SA{}, make_shape(M, K, 1)), (const ElemB*)wq,
                               cutlass::make_cute_packed_stride(SB{}, make_shape(N, K, 1)), xs, ScaleConfig::tile_atom_to_shape_SFA(shape), ws,
                               ScaleConfig::tile_atom_to_shape_SFB(shape)},
                              {{1.f, 0.f}, nullptr, cutlass::make_cute_packed_stride(SC{}, make_shape(M, N, 1)), (cutlass::bfloat16_t*)y,
                               cutlass::make_cute_packed_stride(SD{}, make_shape(M, N, 1))}};
  cudaGetDevice(&args.hw_info.device_id);
  args.hw_info.sm_count = num_sms();
  Op op;
  AX_REQUIRE(op.can_implement(args) == cutlass::Status::kSuccess, "fp8 block GEMM cannot implement M=", M, " N=", N, " K=", K);
  Scratch wsp(Op::get_workspace_size(args), st);
  AX_REQUIRE(op.initialize(args, wsp.ptr, st) == cutlass::Status::kSuccess, "fp8 GEMM init");
  AX_REQUIRE(op.run(st) == cutlass::Status::kSuccess, "fp8 GEMM run");
}

}  // namespace fp8
}  // namespace ax
