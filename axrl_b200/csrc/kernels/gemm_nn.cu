// Data-gradient GEMM family: D[M,N] = A[M,K] @ B[K,N]  (dY @ W).
#include "gemm_sm100.cuh"

namespace ax {
namespace gemm {
using RM = cutlass::layout::RowMajor;

void run_nn(const void* A, const void* B, void* D, int M, int N, int K, cudaStream_t st) {
  if (M >= 512) Gemm<RM, RM, cutlass::bfloat16_t, Sm2>::run(A, B, nullptr, D, M, N, K, 1.f, 0.f, st);
  else Gemm<RM, RM, cutlass::bfloat16_t, Sm1>::run(A, B, nullptr, D, M, N, K, 1.f, 0.f, st);
}
}  // namespace gemm
}  // namespace ax
