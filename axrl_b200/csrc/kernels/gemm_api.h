// Raw-pointer entry points of the tcgen05 GEMMs (CUTLASS sm100 collectives instantiated in
// gemm_*.cu, grouped_gemm.cu and gemm_fp8_block.cu).  No CUTLASS or torch types, so the torch
// wrappers can call them without parsing either.
#pragma once
#include <cuda_runtime.h>

namespace ax {
namespace gemm {

// Stream-K decomposition override for tuning: mode 0 heuristic, 1 data-parallel, 2 split-K
// (``splits`` ways), 3 stream-K.  Process-wide; read at each launch.
struct DecompOverride {
  int mode = 0;
  int splits = 0;
};
inline DecompOverride& decomp_override() {
  static DecompOverride o;
  return o;
}

// One translation unit per instantiation (parallel builds).  C (optional, beta = 1) is a
// residual added in the epilogue.
//   tn: D = A[M,K] @ B[N,K]^T (+ C)      nn: D = A[M,K] @ B[K,N]      wgrad: D (+)= A^T @ B, A stored [K,M]
void tn_sm2(const void* A, const void* B, const void* C, void* D, int M, int N, int K, cudaStream_t st);
void tn_sm1_sk(const void* A, const void* B, const void* C, void* D, int M, int N, int K, cudaStream_t st);
void tn_narrow_sk(const void* A, const void* B, const void* C, void* D, int M, int N, int K, cudaStream_t st);
void nn_sm2(const void* A, const void* B, void* D, int M, int N, int K, cudaStream_t st);
void nn_sm1_sk(const void* A, const void* B, void* D, int M, int N, int K, cudaStream_t st);
void wgrad_f32_sm2(const void* A, const void* B, void* D, int M, int N, int K, bool acc, cudaStream_t st);
void wgrad_f32_sm1(const void* A, const void* B, void* D, int M, int N, int K, bool acc, cudaStream_t st);
void wgrad_bf16_sm1(const void* A, const void* B, void* D, int M, int N, int K, cudaStream_t st);
// skinny (M <= 64): Y[M,N] = X[M,K] @ W[N,K]^T (+ C) computed as Y^T = W @ X^T (swap-AB)
void tn_swapab(const void* X, const void* W, const void* C, void* D, int M, int N, int K, cudaStream_t st);

}  // namespace gemm

// Grouped (per-expert) GEMMs, grouped_gemm.cu.  off: E+1 int32 expert row offsets on the device.
namespace grouped {
void fwd(const int* off, int E, int N, int K, const void* X, const void* W, void* Y, cudaStream_t st);
void dgrad(const int* off, int E, int N, int K, const void* dY, const void* W, void* dX, cudaStream_t st);
void wgrad_acc(const int* off, int E, int N, int K, const void* dY, const void* X, float* acc, const void* zeros, cudaStream_t st);
}  // namespace grouped

// Block-scaled fp8 GEMM and row quantiser, gemm_fp8_block.cu.
namespace fp8 {
void quant_rows(const void* x, long M, int K, void* q, float* s, cudaStream_t st);
void block_linear(const void* xq, const float* xs, const void* wq, const float* ws, void* y, int M, int N, int K, cudaStream_t st);
}  // namespace fp8
}  // namespace ax
