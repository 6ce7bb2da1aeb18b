// Data-gradient GEMM (dY @ W), small M, stream-K.
#include "gemm_sm100.cuh"

namespace ax {
namespace gemm {
void nn_sm1_sk(const void* A, const void* B, void* D, int M, int N, int K, cudaStream_t st) {
  Gemm<RM, RM, cutlass::bfloat16_t, Sm1, SK>::run(A, B, nullptr, D, M, N, K, 1.f, 0.f, st);
}
}  // namespace gemm
}  // namespace ax
