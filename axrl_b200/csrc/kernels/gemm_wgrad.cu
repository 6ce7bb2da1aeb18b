// Weight-gradient GEMM family: D[M,N] (+)= A^T @ B with A stored [K,M] (dY), B stored [K,N] (X).
// fp32 D with beta = 1 accumulates straight into the optimizer's main_grad buffer.
#include "gemm_sm100.cuh"

namespace ax {
namespace gemm {
using RM = cutlass::layout::RowMajor;
using CM = cutlass::layout::ColumnMajor;

void run_wgrad(const void* A, const void* B, void* D, int M, int N, int K, bool accumulate, bool d_fp32, cudaStream_t st) {
  float beta = accumulate ? 1.f : 0.f;
  if (d_fp32) {
    if (M >= 512 && N >= 512) Gemm<CM, RM, float, Sm2>::run(A, B, accumulate ? D : nullptr, D, M, N, K, 1.f, beta, st);
    else Gemm<CM, RM, float, Sm1>::run(A, B, accumulate ? D : nullptr, D, M, N, K, 1.f, beta, st);
    return;
  }
  if (M >= 512 && N >= 512) Gemm<CM, RM, cutlass::bfloat16_t, Sm2>::run(A, B, accumulate ? D : nullptr, D, M, N, K, 1.f, beta, st);
  else Gemm<CM, RM, cutlass::bfloat16_t, Sm1>::run(A, B, accumulate ? D : nullptr, D, M, N, K, 1.f, beta, st);
}
}  // namespace gemm
}  // namespace ax
