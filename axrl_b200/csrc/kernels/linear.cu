// torch-facing GEMM wrappers used by ops.linear / ops.logprob.
#include "common.cuh"
#include "gemm_sm100.cuh"

namespace ax {

static void check_bf16_2d(const at::Tensor& t, const char* n) {
  AX_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 && t.stride(0) == t.size(1),
           n, ": contiguous bf16 matrix required");
  AX_CHECK(t.size(1) % 8 == 0, n, ": inner dimension must be a multiple of 8 (16-byte TMA rows)");
  AX_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, n, ": 16-byte aligned base required");
}

// y[M,N] = x[M,K] @ w[N,K]^T
at::Tensor linear_fwd(at::Tensor x, at::Tensor w) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  AX_CHECK(x.size(1) == w.size(1), "K mismatch");
  int M = x.size(0), N = w.size(0), K = x.size(1);
  auto y = at::empty({M, N}, x.options());
  if (M == 0 || N == 0) return y;
  if (K == 0) return y.zero_();
  gemm::run_tn(x.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K, false, stream());
  return y;
}

// dx[M,K] = dy[M,N] @ w[N,K]
at::Tensor linear_dgrad(at::Tensor dy, at::Tensor w) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(w, "w");
  int M = dy.size(0), N = dy.size(1), K = w.size(1);
  AX_CHECK(w.size(0) == N, "N mismatch");
  auto dx = at::empty({M, K}, dy.options());
  if (M == 0 || K == 0) return dx;
  if (N == 0) return dx.zero_();
  gemm::run_nn(dy.data_ptr(), w.data_ptr(), dx.data_ptr(), M, K, N, stream());
  return dx;
}

// dw[N,K] = dy[M,N]^T @ x[M,K]   (bf16 result)
at::Tensor linear_wgrad(at::Tensor dy, at::Tensor x) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(x, "x");
  int M = dy.size(0), N = dy.size(1), K = x.size(1);
  auto dw = at::empty({N, K}, dy.options());
  if (M == 0) return dw.zero_();
  gemm::run_wgrad(dy.data_ptr(), x.data_ptr(), dw.data_ptr(), N, K, M, false, false, stream());
  return dw;
}

// acc[N,K] (fp32) += dy[M,N]^T @ x[M,K]
void linear_wgrad_acc(at::Tensor dy, at::Tensor x, at::Tensor acc) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(x, "x");
  int M = dy.size(0), N = dy.size(1), K = x.size(1);
  AX_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.size(0) == N && acc.size(1) == K, "acc fp32 [N,K]");
  if (M == 0) return;
  gemm::run_wgrad(dy.data_ptr(), x.data_ptr(), acc.data_ptr(), N, K, M, true, true, stream());
}

// Generic: trans_b ? a @ b^T : a @ b   (bf16 out)
at::Tensor gemm_bf16(at::Tensor a, at::Tensor b, bool trans_b) {
  return trans_b ? linear_fwd(a, b) : linear_dgrad(a, b);
}

}  // namespace ax
