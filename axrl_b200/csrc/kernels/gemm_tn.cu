// Forward GEMM family: D[M,N] = A[M,K] @ B[N,K]^T  (activations x weights^T).
#include "gemm_sm100.cuh"

namespace ax {
namespace gemm {
using RM = cutlass::layout::RowMajor;
using CM = cutlass::layout::ColumnMajor;

void run_tn(const void* A, const void* B, void* D, int M, int N, int K, bool d_fp32, cudaStream_t st) {
  if (d_fp32) {
    if (M >= 512) Gemm<RM, CM, float, Sm2>::run(A, B, nullptr, D, M, N, K, 1.f, 0.f, st);
    else Gemm<RM, CM, float, Sm1>::run(A, B, nullptr, D, M, N, K, 1.f, 0.f, st);
    return;
  }
  if (M >= 512) Gemm<RM, CM, cutlass::bfloat16_t, Sm2>::run(A, B, nullptr, D, M, N, K, 1.f, 0.f, st);
  else if (M > 64) Gemm<RM, CM, cutlass::bfloat16_t, Sm1>::run(A, B, nullptr, D, M, N, K, 1.f, 0.f, st);
  else Gemm<RM, CM, cutlass::bfloat16_t, Sm1Narrow>::run(A, B, nullptr, D, M, N, K, 1.f, 0.f, st);
}
}  // namespace gemm
}  // namespace ax
