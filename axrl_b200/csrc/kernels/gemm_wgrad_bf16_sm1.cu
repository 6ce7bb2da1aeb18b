// Weight-gradient GEMM with a bf16 result (no accumulation).
#include "gemm_sm100.cuh"

namespace ax {
namespace gemm {
void wgrad_bf16_sm1(const void* A, const void* B, void* D, int M, int N, int K, cudaStream_t st) {
  Gemm<CM, RM, cutlass::bfloat16_t, Sm1>::run(A, B, nullptr, D, M, N, K, 1.f, 0.f, st);
}
}  // namespace gemm
}  // namespace ax
