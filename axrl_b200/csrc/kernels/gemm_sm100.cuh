// bf16 GEMMs on 5th-gen tensor cores (tcgen05.mma, TMEM accumulators, TMA operand loads),
// composed from CUTLASS sm100 collectives.  Every configuration is a 1-SM kernel without a
// thread-block cluster, so each CTA loads its own operand tiles.
//
// Convention: D[M,N] = alpha * A[M,K] @ B[K,N] + beta * C[M,N], row-major D/C.
//   LayoutA RowMajor    -> A stored M x K (K contiguous)
//   LayoutA ColumnMajor -> A stored K x M (M contiguous)
//   LayoutB ColumnMajor -> B stored N x K (K contiguous)   (x @ W^T with W [N,K])
//   LayoutB RowMajor    -> B stored K x N (N contiguous)
#pragma once
#include "../cuda_common.cuh"
#include "gemm_api.h"

#include "cute/tensor.hpp"
#include "cutlass/cutlass.h"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/dispatch_policy.hpp"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

namespace ax {
namespace gemm {

using namespace cute;

struct Sm1 {
  using Tile = Shape<_128, _128, _64>;
  using Cluster = Shape<_1, _1, _1>;
  using Kernel = cutlass::gemm::KernelTmaWarpSpecialized1SmSm100;
  using Epi = cutlass::epilogue::TmaWarpSpecialized1Sm;
};
struct Sm1Narrow {
  using Tile = Shape<_128, _64, _64>;
  using Cluster = Shape<_1, _1, _1>;
  using Kernel = cutlass::gemm::KernelTmaWarpSpecialized1SmSm100;
  using Epi = cutlass::epilogue::TmaWarpSpecialized1Sm;
};
// Large problems: 1-SM 128x256 tiles.  Every configuration runs without a thread-block cluster
// (cluster 1x1x1), so no operand tile is ever loaded with cluster multicast: each CTA loads its
// own copy (this code also runs in multi-GPU processes).
struct Sm2 {
  using Tile = Shape<_128, _256, _64>;
  using Cluster = Shape<_1, _1, _1>;
  using Kernel = cutlass::gemm::KernelTmaWarpSpecialized1SmSm100;
  using Epi = cutlass::epilogue::TmaWarpSpecialized1Sm;
};

template <class LayoutA, class LayoutB, class ElemD, class Cfg, class Sched = void, class LayoutD = cutlass::layout::RowMajor>
struct Gemm {
  using ElemA = cutlass::bfloat16_t;
  using ElemB = cutlass::bfloat16_t;
  using ElemAcc = float;
  using LayoutC = LayoutD;
  static constexpr int kAlignD = 128 / cutlass::sizeof_bits<ElemD>::value;

  using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, typename Cfg::Tile, typename Cfg::Cluster,
      cutlass::epilogue::collective::EpilogueTileAuto, ElemAcc, ElemAcc, ElemD, LayoutC, kAlignD, ElemD, LayoutC, kAlignD,
      typename Cfg::Epi>::CollectiveOp;

  using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, ElemA, LayoutA, 8, ElemB, LayoutB, 8, ElemAcc,
      typename Cfg::Tile, typename Cfg::Cluster,
      cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
      typename Cfg::Kernel>::CollectiveOp;

  using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop, Epilogue, Sched>;
  using Op = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;

  static void run(const void* A, const void* B, const void* C, void* D, int M, int N, int K, float alpha, float beta,
                  cudaStream_t st) {
    using SA = typename Kernel::StrideA;
    using SB = typename Kernel::StrideB;
    using SC = typename Kernel::StrideC;
    using SD = typename Kernel::StrideD;
    SA sa = cutlass::make_cute_packed_stride(SA{}, cute::make_shape(M, K, 1));
    SB sb = cutlass::make_cute_packed_stride(SB{}, cute::make_shape(N, K, 1));
    SC sc = cutlass::make_cute_packed_stride(SC{}, cute::make_shape(M, N, 1));
    SD sd = cutlass::make_cute_packed_stride(SD{}, cute::make_shape(M, N, 1));
    typename Op::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                {M, N, K, 1},
                                {static_cast<const ElemA*>(A), sa, static_cast<const ElemB*>(B), sb},
                                {{alpha, beta}, static_cast<const ElemD*>(C), sc, static_cast<ElemD*>(D), sd}};
    cudaGetDevice(&args.hw_info.device_id);
    args.hw_info.sm_count = num_sms();
    if constexpr (std::is_same_v<Sched, cutlass::gemm::StreamKScheduler>) {
      // Skinny problems (decode) have too few output tiles to fill 148 SMs: let the scheduler
      // split K (stream-K) so every SM streams weights.  The decomposition can be overridden at
      // run time (set_streamk_decomposition) for tuning sweeps.
      using DM = cutlass::gemm::kernel::detail::DecompositionMode;
      const DecompOverride& o = decomp_override();
      args.scheduler.decomposition_mode = o.mode == 1 ? DM::DataParallel : o.mode == 2 ? DM::SplitK : o.mode == 3 ? DM::StreamK
                                                                                                             : DM::Heuristic;
      if (o.mode == 2 && o.splits > 0) args.scheduler.splits = o.splits;
    }
    Op op;
    auto st_impl = op.can_implement(args);
    AX_REQUIRE(st_impl == cutlass::Status::kSuccess, "GEMM cannot implement M=", M, " N=", N, " K=", K);
    Scratch ws(Op::get_workspace_size(args), st);
    auto s1 = op.initialize(args, ws.ptr, st);
    AX_REQUIRE(s1 == cutlass::Status::kSuccess, "GEMM init failed");
    // programmatic dependent launch: the kernel's load warps wait for the predecessor grid
    // (CUTLASS_ENABLE_GDC_FOR_SM100), so its prologue overlaps the predecessor's tail
    auto s2 = op.run(st, nullptr, pdl_enabled());
    AX_REQUIRE(s2 == cutlass::Status::kSuccess, "GEMM run failed");
  }
};

using RM = cutlass::layout::RowMajor;
using CM = cutlass::layout::ColumnMajor;
using SK = cutlass::gemm::StreamKScheduler;

}  // namespace gemm
}  // namespace ax

