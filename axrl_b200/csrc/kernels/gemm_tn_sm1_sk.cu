// Forward GEMM, medium M (decode batches 65-511): 1-SM 128x128 tiles, stream-K.
#include "gemm_sm100.cuh"

namespace ax {
namespace gemm {
void tn_sm1_sk(const void* A, const void* B, const void* C, void* D, int M, int N, int K, cudaStream_t st) {
  Gemm<RM, CM, cutlass::bfloat16_t, Sm1, SK>::run(A, B, C, D, M, N, K, 1.f, C ? 1.f : 0.f, st);
}
}  // namespace gemm
}  // namespace ax
