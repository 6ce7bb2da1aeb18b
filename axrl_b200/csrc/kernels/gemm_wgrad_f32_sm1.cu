// Weight-gradient GEMM accumulating into fp32 main_grad, small shapes.
#include "gemm_sm100.cuh"

namespace ax {
namespace gemm {
void wgrad_f32_sm1(const void* A, const void* B, void* D, int M, int N, int K, bool acc, cudaStream_t st) {
  Gemm<CM, RM, float, Sm1, SK>::run(A, B, acc ? D : nullptr, D, M, N, K, 1.f, acc ? 1.f : 0.f, st);
}
}  // namespace gemm
}  // namespace ax
