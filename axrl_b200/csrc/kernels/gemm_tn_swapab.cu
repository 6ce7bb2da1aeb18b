// Forward GEMM for skinny activations (decode, M <= 64), swap-AB on tcgen05: compute
// Y^T[N, M] = W[N, K] @ X[M, K]^T so the weight matrix fills the 128-row MMA dimension and the
// few activation rows become a narrow N tile (32 or 64 columns in TMEM).  D (and the optional
// residual C) are column-major in this orientation, i.e. exactly row-major Y[M, N].  Stream-K
// spreads the K loop of the N/128 weight tiles over every SM, so the kernel streams weights
// at HBM rate through TMA.
#include "gemm_sm100.cuh"

namespace ax {
namespace gemm {

struct SwapN32 {
  using Tile = Shape<_128, _32, _64>;
  using Cluster = Shape<_1, _1, _1>;
  using Kernel = cutlass::gemm::KernelTmaWarpSpecialized1SmSm100;
  using Epi = cutlass::epilogue::TmaWarpSpecialized1Sm;
};
struct SwapN64 {
  using Tile = Shape<_128, _64, _64>;
  using Cluster = Shape<_1, _1, _1>;
  using Kernel = cutlass::gemm::KernelTmaWarpSpecialized1SmSm100;
  using Epi = cutlass::epilogue::TmaWarpSpecialized1Sm;
};

// A = W (N x K, K contiguous), B = X (M x K, K contiguous), D = Y viewed as N x M column-major.
// (128/256-row swap-AB tiles were measured slower than the 1-SM 128x128 stream-K GEMM from 96
// rows on, so swap-AB stops at 64 rows.)
void tn_swapab(const void* X, const void* W, const void* C, void* D, int M, int N, int K, cudaStream_t st) {
  if (M <= 32) Gemm<RM, CM, cutlass::bfloat16_t, SwapN32, SK, CM>::run(W, X, C, D, N, M, K, 1.f, C ? 1.f : 0.f, st);
  else Gemm<RM, CM, cutlass::bfloat16_t, SwapN64, SK, CM>::run(W, X, C, D, N, M, K, 1.f, C ? 1.f : 0.f, st);
}

}  // namespace gemm
}  // namespace ax
