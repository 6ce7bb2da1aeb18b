// torch-facing GEMM wrappers used by ops.linear / ops.logprob / the rollout engine.
// Tile-config choice by M (tokens): >= 512 -> 1-SM 128x256 data-parallel tiles;
// 65..511 -> 1-SM 128x128 stream-K; <= 64 -> 1-SM 128x64 stream-K (decode: weight streaming).
#include <string>
#include <vector>

#include <c10/cuda/CUDACachingAllocator.h>

#include "common.cuh"
#include "gemm_api.h"

namespace ax {

void* scratch_alloc(size_t bytes, cudaStream_t st) { return c10::cuda::CUDACachingAllocator::raw_alloc_with_stream(bytes, st); }
void scratch_free(void* p) { c10::cuda::CUDACachingAllocator::raw_delete(p); }

static void check_bf16_2d(const at::Tensor& t, const char* n) {
  AX_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 && t.stride(0) == t.size(1),
           n, ": contiguous bf16 matrix required");
  AX_CHECK(t.size(1) % 8 == 0, n, ": inner dimension must be a multiple of 8 (16-byte TMA rows)");
  AX_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, n, ": 16-byte aligned base required");
}

at::Tensor skinny_linear(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual);
at::Tensor skinny_tma_linear(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual);
at::Tensor skinny_linear_out(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual, c10::optional<at::Tensor> out);
at::Tensor skinny_tma_linear_out(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual, c10::optional<at::Tensor> out);

void tcgemm_tn(const void* A, const void* B, const void* C, void* D, int M, int N, int K, int* err, cudaStream_t st);

static at::Tensor& tcgemm_err(int dev) {
  static at::Tensor e[64];
  if (!e[dev].defined()) e[dev] = at::zeros({1}, at::TensorOptions().device(at::kCUDA, dev).dtype(at::kInt));
  return e[dev];
}

// Training-size forward GEMMs (>= 512 rows) run on the hand-written persistent tcgen05 kernel
// (tcgemm.cu), measured at or above the CUTLASS 128x256 configuration on every Qwen3-8B shape
// (gate/up +21 %, down +9 %); AXRL_TRAIN_GEMM=cutlass selects CUTLASS.
static bool use_tcgemm() {
  static bool on = [] {
    const char* e = std::getenv("AXRL_TRAIN_GEMM");
    return !(e && std::string(e) == "cutlass");
  }();
  return on;
}

void tcgemm_nn(const void* dY, const void* W, void* dX, int M, int Ko, int Nr, int* err, cudaStream_t st);
void tcgemm_wgrad(const void* dY, const void* X, float* G, int Nw, int Kw, int T, bool accumulate, int* err, cudaStream_t st);
void tcgemm_wgrad_bf16(const void* dY, const void* X, void* G, int Nw, int Kw, int T, int* err, cudaStream_t st);

// Backward GEMMs (data and weight gradients) run on the hand-written kernel unless
// AXRL_TRAIN_GEMM_BWD=cutlass (Qwen3-8B shapes at 16k tokens on B200: 10.2 ms against 10.9 ms
// for the CUTLASS pair, summed over qkv/o/gate_up/down dgrad + wgrad).
static bool use_tcgemm_bwd() {
  static bool on = [] {
    const char* e = std::getenv("AXRL_TRAIN_GEMM_BWD");
    return !(e && std::string(e) == "cutlass");
  }();
  return on;
}
static bool tc_ok(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

static void tn(const void* A, const void* B, const void* C, void* D, int M, int N, int K) {
  int dev = 0;
  if (M >= 512 && use_tcgemm() && K % 64 == 0 && N % 32 == 0 && reinterpret_cast<uintptr_t>(A) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(B) % 16 == 0 && reinterpret_cast<uintptr_t>(D) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(C) % 16 == 0 && cudaGetDevice(&dev) == cudaSuccess) {
    tcgemm_tn(A, B, C, D, M, N, K, tcgemm_err(dev).data_ptr<int>(), stream());
    return;
  }
  if (M >= 512) gemm::tn_sm2(A, B, C, D, M, N, K, stream());
  else if (M > 64) gemm::tn_sm1_sk(A, B, C, D, M, N, K, stream());
  else gemm::tn_narrow_sk(A, B, C, D, M, N, K, stream());
}

// Decode-size GEMMs are reads of the weight matrix.  Kernels for <= 64 activation rows: the
// cluster split-K tcgen05 streaming kernel (tcgemm.cu, stream_cluster_k), the persistent tcgen05
// streaming kernel (tcgemm.cu, stream_k), the cp.async / TMA mma.sync streaming kernels for <= 16
// rows (skinny_gemm.cu, skinny_tma.cu) and CUTLASS swap-AB (gemm_tn_swapab.cu).
// AXRL_DECODE_GEMM = skinny | tma | tcgen05 | tcstream | tccluster (or set_decode_gemm) forces one.
enum DecodeGemm { kTcgen05 = 0, kSkinny = 1, kTma = 2, kTcStream = 3, kTcCluster = 4 };

void tcgemm_stream(const void* X, const void* W, const void* R, void* Y, int M, int N, int K, float* ws, int* cnt, int* err, bool prefetch_w,
                   cudaStream_t st);
void tcgemm_stream_cluster(const void* X, const void* W, const void* R, void* Y, int M, int N, int K, int* err, bool prefetch_w,
                           cudaStream_t st, int xmode, const void* g, float eps);

// Zero-initialised, self-cleaning workspace of the streaming kernel, one per device.
struct StreamWorkspace {
  at::Tensor ws, cnt, err;
};
static StreamWorkspace& stream_workspace(int dev) {
  static StreamWorkspace w[64];
  if (!w[dev].ws.defined()) {
    auto o = at::TensorOptions().device(at::kCUDA, dev);
    w[dev].ws = at::zeros({64L * 262144}, o.dtype(at::kFloat));
    w[dev].cnt = at::zeros({4 * 2048}, o.dtype(at::kInt));
    w[dev].err = at::zeros({1}, o.dtype(at::kInt));
  }
  return w[dev];
}

static void tc_stream_into(const at::Tensor& x, const at::Tensor& w, const bf16* r, at::Tensor& y) {
  const int M = x.size(0), N = w.size(0), K = x.size(1);
  AX_CHECK(N <= 262144, "tcstream: N <= 262144");
  auto& ws = stream_workspace(x.get_device());
  tcgemm_stream(x.data_ptr(), w.data_ptr(), r, y.data_ptr(), M, N, K, ws.ws.data_ptr<float>(), ws.cnt.data_ptr<int>(),
                ws.err.data_ptr<int>(), weights_static(), stream());
}

static void tc_cluster_into(const at::Tensor& x, const at::Tensor& w, const bf16* r, at::Tensor& y) {
  const int M = x.size(0), N = w.size(0), K = x.size(1);
  auto& ws = stream_workspace(x.get_device());
  tcgemm_stream_cluster(x.data_ptr(), w.data_ptr(), r, y.data_ptr(), M, N, K, ws.err.data_ptr<int>(), weights_static(), stream(), 0, nullptr,
                        0.f);
}

// Decode projections with the preceding element-wise step folded into the weight-streaming GEMM
// (<= 128 rows): y = RMSNorm(h; g, eps) @ w^T (+ residual), and y = SwiGLU(gu) @ w^T (+ residual)
// with gu = [gate | up] of width 2K.  The normalised / activated rows are never written to memory.
at::Tensor linear_rms_stream(at::Tensor h, at::Tensor g, double eps, at::Tensor w, c10::optional<at::Tensor> residual) {
  check_bf16_2d(h, "h");
  check_bf16_2d(w, "w");
  const int M = h.size(0), K = h.size(1), N = w.size(0);
  AX_CHECK(w.size(1) == K && g.numel() == K && g.scalar_type() == at::kBFloat16 && g.is_contiguous(), "linear_rms_stream: shapes");
  AX_CHECK(g.is_cuda() && g.get_device() == h.get_device() && w.get_device() == h.get_device(),
           "linear_rms_stream: h, g and w must be on the same CUDA device");
  AX_CHECK(M >= 1 && M <= 128 && K % 64 == 0 && N % 8 == 0, "linear_rms_stream: 1..128 rows, K % 64 == 0, N % 8 == 0");
  const bf16* r = nullptr;
  if (residual.has_value()) {
    check_bf16_2d(*residual, "residual");
    AX_CHECK(residual->size(0) == M && residual->size(1) == N && residual->get_device() == h.get_device(), "residual shape / device");
    r = (const bf16*)residual->data_ptr();
  }
  auto y = at::empty({M, N}, h.options());
  auto& ws = stream_workspace(h.get_device());
  tcgemm_stream_cluster(h.data_ptr(), w.data_ptr(), r, y.data_ptr(), M, N, K, ws.err.data_ptr<int>(), weights_static(), stream(), 1,
                        g.data_ptr(), (float)eps);
  return y;
}

at::Tensor linear_swiglu_stream(at::Tensor gu, at::Tensor w, c10::optional<at::Tensor> residual) {
  check_bf16_2d(gu, "gu");
  check_bf16_2d(w, "w");
  const int M = gu.size(0), K = gu.size(1) / 2, N = w.size(0);
  AX_CHECK(gu.size(1) == 2 * K && w.size(1) == K, "linear_swiglu_stream: gu is [M, 2K], w is [N, K]");
  AX_CHECK(w.get_device() == gu.get_device(), "linear_swiglu_stream: gu and w must be on the same CUDA device");
  AX_CHECK(M >= 1 && M <= 128 && K % 64 == 0 && N % 8 == 0, "linear_swiglu_stream: 1..128 rows, K % 64 == 0, N % 8 == 0");
  const bf16* r = nullptr;
  if (residual.has_value()) {
    check_bf16_2d(*residual, "residual");
    AX_CHECK(residual->size(0) == M && residual->size(1) == N && residual->get_device() == gu.get_device(), "residual shape / device");
    r = (const bf16*)residual->data_ptr();
  }
  auto y = at::empty({M, N}, gu.options());
  auto& ws = stream_workspace(gu.get_device());
  tcgemm_stream_cluster(gu.data_ptr(), w.data_ptr(), r, y.data_ptr(), M, N, K, ws.err.data_ptr<int>(), weights_static(), stream(), 2,
                        nullptr, 0.f);
  return y;
}

static int parse_decode_gemm(const std::string& v) {
    return v == "skinny"     ? (int)kSkinny
           : v == "tma"       ? (int)kTma
           : v == "tcgen05"   ? (int)kTcgen05
           : v == "tcstream"  ? (int)kTcStream
           : v == "tccluster" ? (int)kTcCluster
                              : -1;
}

static int& decode_gemm_forced() {
  static int mode = [] {
    const char* e = std::getenv("AXRL_DECODE_GEMM");
    return e ? parse_decode_gemm(e) : -1;
  }();
  return mode;
}
static int decode_gemm_mode() { return decode_gemm_forced(); }

// Force one decode GEMM for M <= 64 ("" or "auto": choose by shape); tests and benchmarks.
void set_decode_gemm(std::string mode) { decode_gemm_forced() = parse_decode_gemm(mode); }

// Default (in-stream chains of 48 distinct weight matrices, Qwen3-8B projections): the cluster
// split-K tcgen05 kernel for every matrix up to 128M elements at 1..128 rows (at 48 rows qkv 17.7,
// o 12.0, gate/up 42.3, down 24.6 us against 23.0 / 23.0 / 44.2 / 34.2 for CUTLASS swap-AB; at 8
// rows 15.1 / 10.6 / 37.9 / 21.8 against the skinny kernel's 16.4 / 9.5 / 40.1 / 24.7), the skinny
// kernel for matrices up to 16M elements at <= 16 rows, CUTLASS swap-AB for the vocabulary
// projection (151936 x 4096: 195-203 us against 199-223).
static DecodeGemm decode_gemm(int M, int N, int K) {
  const int forced = decode_gemm_mode();
  const bool aligned = K % 64 == 0 && N % 8 == 0;
  const bool stream_ok = M <= 64 && aligned && N <= 262144 && (long)M * N <= 64L * 262144;
  if (forced == kTcStream && stream_ok) return kTcStream;
  if (forced == kTcCluster && M <= 128 && aligned) return kTcCluster;
  if (forced == kTcgen05) return kTcgen05;
  if ((forced == kSkinny || forced == kTma) && M <= 16 && aligned && (long)N * K <= (64L << 20)) return (DecodeGemm)forced;
  if (M <= 16 && aligned && (long)N * K <= (16L << 20)) return kSkinny;
  if (M <= 128 && aligned && (long)N * K <= (128L << 20)) return kTcCluster;
  return kTcgen05;
}

static bool streaming_into(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& r, at::Tensor& y) {
  const int M = x.size(0), N = w.size(0), K = x.size(1);
  const DecodeGemm g = decode_gemm(M, N, K);
  if (g == kTcgen05) return false;
  if (g == kTcStream) tc_stream_into(x, w, r ? (const bf16*)r->data_ptr() : nullptr, y);
  else if (g == kTcCluster) tc_cluster_into(x, w, r ? (const bf16*)r->data_ptr() : nullptr, y);
  else if (g == kSkinny) skinny_linear_out(x, w, r, y);
  else skinny_tma_linear_out(x, w, r, y);
  return true;
}

void set_pdl(bool on) { pdl_enabled() = on; }
bool get_pdl() { return pdl_enabled(); }
void set_weights_static(bool on) { weights_static() = on; }

void set_streamk_decomposition(int64_t mode, int64_t splits) {
  AX_CHECK(mode >= 0 && mode <= 3 && splits >= 0, "mode 0..3, splits >= 0");
  gemm::decomp_override().mode = (int)mode;
  gemm::decomp_override().splits = (int)splits;
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
  if (M <= 128 && M > 64 && decode_gemm(M, N, K) == kTcCluster) {  // decode at 65..128 rows
    tc_cluster_into(x, w, nullptr, y);
    return y;
  }
  if (M <= 64) {  // decode: weight streaming
    if (decode_gemm(M, N, K) == kTcStream) {
      tc_stream_into(x, w, nullptr, y);
      return y;
    }
    if (decode_gemm(M, N, K) == kTcCluster) {
      tc_cluster_into(x, w, nullptr, y);
      return y;
    }
    if (decode_gemm(M, N, K) == kSkinny) return skinny_linear(x, w, c10::nullopt);
    if (decode_gemm(M, N, K) == kTma) return skinny_tma_linear(x, w, c10::nullopt);
    gemm::tn_swapab(x.data_ptr(), w.data_ptr(), nullptr, y.data_ptr(), M, N, K, stream());
  } else {
    tn(x.data_ptr(), w.data_ptr(), nullptr, y.data_ptr(), M, N, K);
  }
  return y;
}

// y[M,N] = x[M,K] @ w[N,K]^T + residual[M,N]   (residual add fused into the epilogue)
at::Tensor linear_residual(at::Tensor x, at::Tensor w, at::Tensor residual) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  check_bf16_2d(residual, "residual");
  int M = x.size(0), N = w.size(0), K = x.size(1);
  AX_CHECK(residual.size(0) == M && residual.size(1) == N, "residual shape");
  auto y = at::empty({M, N}, x.options());
  if (M == 0 || N == 0) return y;
  if (M <= 128 && M > 64 && decode_gemm(M, N, K) == kTcCluster) {
    tc_cluster_into(x, w, (const bf16*)residual.data_ptr(), y);
    return y;
  }
  if (M <= 64) {
    if (decode_gemm(M, N, K) == kTcStream) {
      tc_stream_into(x, w, (const bf16*)residual.data_ptr(), y);
      return y;
    }
    if (decode_gemm(M, N, K) == kTcCluster) {
      tc_cluster_into(x, w, (const bf16*)residual.data_ptr(), y);
      return y;
    }
    if (decode_gemm(M, N, K) == kSkinny) return skinny_linear(x, w, residual);
    if (decode_gemm(M, N, K) == kTma) return skinny_tma_linear(x, w, residual);
    gemm::tn_swapab(x.data_ptr(), w.data_ptr(), residual.data_ptr(), y.data_ptr(), M, N, K, stream());
  } else {
    tn(x.data_ptr(), w.data_ptr(), residual.data_ptr(), y.data_ptr(), M, N, K);
  }
  return y;
}

// out[M,N] = x[M,K] @ w[N,K]^T into a caller-provided contiguous block of rows (chunked TP GEMMs)
void linear_fwd_into(at::Tensor x, at::Tensor w, at::Tensor out) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  check_bf16_2d(out, "out");
  int M = x.size(0), N = w.size(0), K = x.size(1);
  AX_CHECK(out.size(0) == M && out.size(1) == N && w.size(1) == K, "shapes");
  if (M == 0 || N == 0) return;
  if (M <= 128 && M > 64 && decode_gemm(M, N, K) == kTcCluster) {
    tc_cluster_into(x, w, nullptr, out);
    return;
  }
  if (M <= 64) {
    if (streaming_into(x, w, c10::nullopt, out)) return;
    gemm::tn_swapab(x.data_ptr(), w.data_ptr(), nullptr, out.data_ptr(), M, N, K, stream());
  } else {
    tn(x.data_ptr(), w.data_ptr(), nullptr, out.data_ptr(), M, N, K);
  }
}

// out[M,K] = dy[M,N] @ w[N,K] into caller-provided rows
void linear_dgrad_into(at::Tensor dy, at::Tensor w, at::Tensor out) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(w, "w");
  check_bf16_2d(out, "out");
  int M = dy.size(0), N = dy.size(1), K = w.size(1);
  AX_CHECK(w.size(0) == N && out.size(0) == M && out.size(1) == K, "shapes");
  if (M == 0 || K == 0) return;
  if (M >= 512 && use_tcgemm_bwd() && K % 32 == 0 && N % 8 == 0 && tc_ok(dy.data_ptr()) && tc_ok(w.data_ptr()) && tc_ok(out.data_ptr())) {
    tcgemm_nn(dy.data_ptr(), w.data_ptr(), out.data_ptr(), M, K, N, tcgemm_err(dy.get_device()).data_ptr<int>(), stream());
    return;
  }
  if (M >= 512) gemm::nn_sm2(dy.data_ptr(), w.data_ptr(), out.data_ptr(), M, K, N, stream());
  else gemm::nn_sm1_sk(dy.data_ptr(), w.data_ptr(), out.data_ptr(), M, K, N, stream());
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
  if (M >= 512 && use_tcgemm_bwd() && K % 32 == 0 && N % 8 == 0 && tc_ok(dy.data_ptr()) && tc_ok(w.data_ptr())) {
    tcgemm_nn(dy.data_ptr(), w.data_ptr(), dx.data_ptr(), M, K, N, tcgemm_err(dy.get_device()).data_ptr<int>(), stream());
    return dx;
  }
  if (M >= 512) gemm::nn_sm2(dy.data_ptr(), w.data_ptr(), dx.data_ptr(), M, K, N, stream());
  else gemm::nn_sm1_sk(dy.data_ptr(), w.data_ptr(), dx.data_ptr(), M, K, N, stream());
  return dx;
}

// dw[N,K] = dy[M,N]^T @ x[M,K]   (bf16 result)
at::Tensor linear_wgrad(at::Tensor dy, at::Tensor x) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(x, "x");
  int M = dy.size(0), N = dy.size(1), K = x.size(1);
  auto dw = at::empty({N, K}, dy.options());
  if (M == 0) return dw.zero_();
  if (use_tcgemm_bwd() && M >= 64 && N % 8 == 0 && K % 32 == 0 && tc_ok(dy.data_ptr()) && tc_ok(x.data_ptr())) {
    tcgemm_wgrad_bf16(dy.data_ptr(), x.data_ptr(), dw.data_ptr(), N, K, M, tcgemm_err(dy.get_device()).data_ptr<int>(), stream());
    return dw;
  }
  gemm::wgrad_bf16_sm1(dy.data_ptr(), x.data_ptr(), dw.data_ptr(), N, K, M, stream());
  return dw;
}

// acc[N,K] (fp32) += dy[M,N]^T @ x[M,K]
void linear_wgrad_acc(at::Tensor dy, at::Tensor x, at::Tensor acc) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(x, "x");
  int M = dy.size(0), N = dy.size(1), K = x.size(1);
  AX_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.size(0) == N && acc.size(1) == K, "acc fp32 [N,K]");
  if (M == 0) return;
  if (use_tcgemm_bwd() && M >= 64 && N % 8 == 0 && K % 32 == 0 && tc_ok(dy.data_ptr()) && tc_ok(x.data_ptr()) && tc_ok(acc.data_ptr())) {
    tcgemm_wgrad(dy.data_ptr(), x.data_ptr(), acc.data_ptr<float>(), N, K, M, true, tcgemm_err(dy.get_device()).data_ptr<int>(), stream());
    return;
  }
  if (N >= 512 && K >= 512) gemm::wgrad_f32_sm2(dy.data_ptr(), x.data_ptr(), acc.data_ptr(), N, K, M, true, stream());
  else gemm::wgrad_f32_sm1(dy.data_ptr(), x.data_ptr(), acc.data_ptr(), N, K, M, true, stream());
}

// Benchmark / test entry: force one implementation ("skinny", "swapab", "cutlass").
at::Tensor linear_variant(at::Tensor x, at::Tensor w, std::string variant) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  int M = x.size(0), N = w.size(0), K = x.size(1);
  if (variant == "skinny") return skinny_linear(x, w, c10::nullopt);
  if (variant == "tma") return skinny_tma_linear(x, w, c10::nullopt);
  auto y = at::empty({M, N}, x.options());
  if (M == 0) return y;
  if (variant == "tcstream") {
    AX_CHECK(M <= 64, "tcstream needs M <= 64");
    tc_stream_into(x, w, nullptr, y);
    return y;
  }
  if (variant == "tccluster") {
    AX_CHECK(M <= 128, "tccluster needs M <= 128");
    tc_cluster_into(x, w, nullptr, y);
    return y;
  }
  if (variant == "swapab") {
    AX_CHECK(M <= 64, "swapab needs M <= 64");
    gemm::tn_swapab(x.data_ptr(), w.data_ptr(), nullptr, y.data_ptr(), M, N, K, stream());
  } else if (variant == "cutlass") {
    tn(x.data_ptr(), w.data_ptr(), nullptr, y.data_ptr(), M, N, K);
  } else {
    AX_CHECK(false, "unknown GEMM variant ", variant);
  }
  return y;
}

// Generic: trans_b ? a @ b^T : a @ b   (bf16 out)
at::Tensor gemm_bf16(at::Tensor a, at::Tensor b, bool trans_b) { return trans_b ? linear_fwd(a, b) : linear_dgrad(a, b); }

// ---------------------------------------------------------------- grouped (per-expert) GEMMs
static void check_rows(const at::Tensor& t, const char* n) {
  AX_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous() && t.dim() == 2, n, ": contiguous bf16 (rows, C)");
  AX_CHECK(t.size(1) % 8 == 0, n, ": row length must be a multiple of 8");
}

// Y (rows, N) = per-expert X rows @ W[e]^T; offsets (E+1) int32 on the device.
at::Tensor grouped_linear_fwd(at::Tensor x, at::Tensor w, at::Tensor offsets) {
  check_rows(x, "x");
  AX_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.dim() == 3, "w: (E, N, K) bf16");
  AX_CHECK(offsets.scalar_type() == at::kInt && offsets.numel() == w.size(0) + 1, "offsets: E+1 int32");
  int E = w.size(0), N = w.size(1), K = w.size(2);
  AX_CHECK(x.size(1) == K, "K mismatch");
  auto y = at::empty({x.size(0), N}, x.options());
  if (x.size(0) == 0) return y;
  grouped::fwd(offsets.data_ptr<int>(), E, N, K, x.data_ptr(), w.data_ptr(), y.data_ptr(), stream());
  return y;
}

// dX (rows, K) = per-expert dY rows @ W[e]
at::Tensor grouped_linear_dgrad(at::Tensor dy, at::Tensor w, at::Tensor offsets) {
  check_rows(dy, "dy");
  AX_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.dim() == 3, "w: (E, N, K) bf16");
  AX_CHECK(offsets.scalar_type() == at::kInt && offsets.numel() == w.size(0) + 1, "offsets: E+1 int32");
  int E = w.size(0), N = w.size(1), K = w.size(2);
  AX_CHECK(dy.size(1) == N, "N mismatch");
  auto dx = at::empty({dy.size(0), K}, dy.options());
  if (dy.size(0) == 0) return dx;
  grouped::dgrad(offsets.data_ptr<int>(), E, N, K, dy.data_ptr(), w.data_ptr(), dx.data_ptr(), stream());
  return dx;
}

// acc (E, N, K) fp32 += per-expert dY rows^T @ X rows
void grouped_linear_wgrad_acc(at::Tensor dy, at::Tensor x, at::Tensor offsets, at::Tensor acc) {
  check_rows(dy, "dy");
  check_rows(x, "x");
  AX_CHECK(acc.is_cuda() && acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.dim() == 3, "acc: (E, N, K) fp32");
  int E = acc.size(0), N = acc.size(1), K = acc.size(2);
  AX_CHECK(offsets.scalar_type() == at::kInt && offsets.numel() == E + 1, "offsets: E+1 int32");
  AX_CHECK(dy.size(1) == N && x.size(1) == K && dy.size(0) == x.size(0), "shapes");
  auto zeros = at::zeros({8, std::max(N, K)}, dy.options());
  grouped::wgrad_acc(offsets.data_ptr<int>(), E, N, K, dy.data_ptr(), x.data_ptr(), acc.data_ptr<float>(), zeros.data_ptr(), stream());
}

// ---------------------------------------------------------------- block-scaled fp8
// x (M,K) bf16 -> (q (M,K) e4m3, s (M, K/128) fp32)
std::vector<at::Tensor> quant_fp8_rows(at::Tensor x) {
  AX_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x: contiguous bf16 (M, K)");
  long M = x.size(0);
  int K = x.size(1);
  AX_CHECK(K % 128 == 0, "K must be a multiple of 128");
  auto q = at::empty({M, K}, x.options().dtype(at::kFloat8_e4m3fn));
  auto s = at::empty({M, K / 128}, x.options().dtype(at::kFloat));
  fp8::quant_rows(x.data_ptr(), M, K, q.data_ptr(), s.data_ptr<float>(), stream());
  return {q, s};
}

// y (M,N) bf16 = blockwise-scaled xq @ wq^T
at::Tensor fp8_block_linear(at::Tensor xq, at::Tensor xs, at::Tensor wq, at::Tensor ws) {
  AX_CHECK(xq.is_cuda() && xq.scalar_type() == at::kFloat8_e4m3fn && xq.is_contiguous() && xq.dim() == 2, "xq: e4m3 (M,K)");
  AX_CHECK(wq.is_cuda() && wq.scalar_type() == at::kFloat8_e4m3fn && wq.is_contiguous() && wq.dim() == 2, "wq: e4m3 (N,K)");
  int M = xq.size(0), K = xq.size(1), N = wq.size(0);
  AX_CHECK(wq.size(1) == K && K % 128 == 0 && N % 128 == 0, "shapes: K and N multiples of 128");
  AX_CHECK(xs.scalar_type() == at::kFloat && xs.is_contiguous() && xs.size(0) == M && xs.size(1) == K / 128, "xs: (M, K/128) fp32");
  AX_CHECK(ws.scalar_type() == at::kFloat && ws.is_contiguous() && ws.size(0) == N / 128 && ws.size(1) == K / 128, "ws: (N/128, K/128) fp32");
  auto y = at::empty({M, N}, xq.options().dtype(at::kBFloat16));
  if (M == 0) return y;
  fp8::block_linear(xq.data_ptr(), xs.data_ptr<float>(), wq.data_ptr(), ws.data_ptr<float>(), y.data_ptr(), M, N, K, stream());
  return y;
}

// ---------------------------------------------------------------- hand-written tcgen05 GEMM (tcgemm.cu)
void tcgemm_ag(const int64_t* src_peers, const void* B, void* D, int rank, int world, int rows_per_rank, int N, int K,
               const int64_t* flag_peers, const int* my_flags, int ch, int epoch, int* ag_cnt, int call, uint64_t timeout_ns, int* status,
               int* err, const void* A_local_buffer, cudaStream_t st);
void tcgemm_tn_to_slots(const void* A, const void* B, const int64_t* peers, int rank, int world, int rows_per_rank, int M, int N, int K,
                        const int64_t* flag_peers, const int* my_flags, int ch, int epoch, unsigned* ticket, uint64_t timeout_ns,
                        int* status, int* err, cudaStream_t st);

// y (M, N) = x (M, K) @ w (N, K)^T (+ residual), on the hand-written persistent tcgen05 kernel
at::Tensor tc_linear(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  AX_CHECK(x.size(1) == w.size(1), "K mismatch");
  const int M = x.size(0), N = w.size(0), K = x.size(1);
  auto y = at::empty({M, N}, x.options());
  const void* c = nullptr;
  if (residual.has_value()) {
    check_bf16_2d(*residual, "residual");
    AX_CHECK(residual->size(0) == M && residual->size(1) == N, "residual shape");
    c = residual->data_ptr();
  }
  tcgemm_tn(x.data_ptr(), w.data_ptr(), c, y.data_ptr(), M, N, K, tcgemm_err(x.get_device()).data_ptr<int>(), stream());
  return y;
}

// Fused GEMM -> reduce-scatter producer: rows of x @ w^T go straight into their owner's receive
// buffer (peer_ptrs[owner], int64 device pointers of (world * rows_per_rank, N) bf16 buffers),
// slot `rank`; flag_ptrs (int64 device pointers of every rank's TP flag array), my_flags, ticket
// and status follow the TP channel protocol of tp_comm.cu.
void tc_linear_to_slots(at::Tensor x, at::Tensor w, at::Tensor peer_ptrs, int64_t rank, int64_t rows_per_rank, at::Tensor flag_ptrs,
                        at::Tensor my_flags, int64_t ch, int64_t epoch, at::Tensor ticket, int64_t timeout_ns, at::Tensor status) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  AX_CHECK(peer_ptrs.is_cuda() && peer_ptrs.scalar_type() == at::kLong, "peer_ptrs: int64 device tensor");
  AX_CHECK(flag_ptrs.is_cuda() && flag_ptrs.scalar_type() == at::kLong && flag_ptrs.numel() == peer_ptrs.numel(), "flag_ptrs");
  AX_CHECK(my_flags.scalar_type() == at::kInt && ticket.scalar_type() == at::kInt && status.scalar_type() == at::kInt, "int32 flags");
  const int M = x.size(0), N = w.size(0), K = x.size(1);
  const int world = peer_ptrs.numel();
  AX_CHECK(M % rows_per_rank == 0 && M / rows_per_rank == world, "rows must split evenly over the ranks");
  tcgemm_tn_to_slots(x.data_ptr(), w.data_ptr(), peer_ptrs.data_ptr<int64_t>(), (int)rank, world, (int)rows_per_rank, M, N, K,
                     flag_ptrs.data_ptr<int64_t>(), my_flags.data_ptr<int>(), (int)ch, (int)epoch,
                     reinterpret_cast<unsigned*>(ticket.data_ptr<int>()) + ch, (uint64_t)timeout_ns, status.data_ptr<int>(),
                     tcgemm_err(x.get_device()).data_ptr<int>(), stream());
}

// All-gather -> GEMM in one kernel: out (world * rows_per_rank, N) = gather(x) @ w^T, where `gather`
// is this rank's symmetric gather buffer with its own rows already at rank * rows_per_rank and
// src_ptrs (int64 device pointers) every rank's gather buffer; the kernel pulls the other ranks'
// rows over NVLink.  ag_cnt: world ints, zero before the first call and kept (call = 1, 2, ...).
void tc_linear_ag(at::Tensor gather, at::Tensor w, at::Tensor out, at::Tensor src_ptrs, int64_t rank, int64_t rows_per_rank,
                  at::Tensor flag_ptrs, at::Tensor my_flags, int64_t ch, int64_t epoch, at::Tensor ag_cnt, int64_t call, int64_t timeout_ns,
                  at::Tensor status) {
  check_bf16_2d(w, "w");
  AX_CHECK(gather.is_cuda() && gather.scalar_type() == at::kBFloat16 && gather.is_contiguous(), "gather: bf16 buffer");
  AX_CHECK(src_ptrs.is_cuda() && src_ptrs.scalar_type() == at::kLong && flag_ptrs.is_cuda() && flag_ptrs.numel() == src_ptrs.numel(),
           "src_ptrs / flag_ptrs: int64 device tensors");
  AX_CHECK(ag_cnt.is_cuda() && ag_cnt.scalar_type() == at::kInt && ag_cnt.numel() >= src_ptrs.numel(), "ag_cnt: int32 per rank");
  const int world = src_ptrs.numel(), N = w.size(0), K = w.size(1);
  AX_CHECK(out.is_contiguous() && out.size(0) == world * rows_per_rank && out.size(1) == N, "out: (world * rows_per_rank, N)");
  AX_CHECK(gather.numel() >= (long)world * rows_per_rank * K, "gather buffer too small");
  tcgemm_ag(src_ptrs.data_ptr<int64_t>(), w.data_ptr(), out.data_ptr(), (int)rank, world, (int)rows_per_rank, N, K, flag_ptrs.data_ptr<int64_t>(),
            my_flags.data_ptr<int>(), (int)ch, (int)epoch, ag_cnt.data_ptr<int>(), (int)call, (uint64_t)timeout_ns, status.data_ptr<int>(),
            tcgemm_err(w.get_device()).data_ptr<int>(), gather.data_ptr(), stream());
}

// Decode-size GEMM on the tcgen05 weight-streaming kernel (1..64 rows), for tests and benchmarks.
at::Tensor tc_stream_linear(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  const int M = x.size(0), N = w.size(0);
  AX_CHECK(M >= 1 && M <= 64 && x.size(1) == w.size(1), "1..64 rows, K match");
  auto y = at::empty({M, N}, x.options());
  const bf16* r = nullptr;
  if (residual.has_value()) {
    check_bf16_2d(*residual, "residual");
    r = (const bf16*)residual->data_ptr();
  }
  tc_stream_into(x, w, r, y);
  return y;
}

std::vector<int64_t> tcgemm_stream_cluster_fit(int ntok);
std::vector<int64_t> stream_cluster_fit(int64_t ntok) { return tcgemm_stream_cluster_fit((int)ntok); }
int64_t tc_stream_error() { return stream_workspace(c10::cuda::current_device()).err.item<int>(); }

// Test / benchmark entries of the hand-written backward GEMMs.
at::Tensor tc_linear_dgrad(at::Tensor dy, at::Tensor w) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(w, "w");
  const int M = dy.size(0), N = dy.size(1), K = w.size(1);
  AX_CHECK(w.size(0) == N, "N mismatch");
  auto dx = at::empty({M, K}, dy.options());
  tcgemm_nn(dy.data_ptr(), w.data_ptr(), dx.data_ptr(), M, K, N, tcgemm_err(dy.get_device()).data_ptr<int>(), stream());
  return dx;
}
void tc_linear_wgrad_acc(at::Tensor dy, at::Tensor x, at::Tensor acc, bool accumulate) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(x, "x");
  const int M = dy.size(0), N = dy.size(1), K = x.size(1);
  AX_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.size(0) == N && acc.size(1) == K, "acc fp32 [N,K]");
  tcgemm_wgrad(dy.data_ptr(), x.data_ptr(), acc.data_ptr<float>(), N, K, M, accumulate, tcgemm_err(dy.get_device()).data_ptr<int>(), stream());
}

int64_t tc_linear_error() { return tcgemm_err(c10::cuda::current_device()).item<int>(); }

}  // namespace ax
