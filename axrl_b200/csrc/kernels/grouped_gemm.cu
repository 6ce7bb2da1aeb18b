// Grouped (per-expert) bf16 GEMMs for MoE on 5th-gen tensor cores: one launch covers every
// expert, each group with its own row count taken from DEVICE offsets (no host sync).  Built from
// the CUTLASS sm100 pointer-array collectives (tcgen05.mma + TMEM accumulators, TMA loads with
// per-group tensor maps, cluster 1x1x1: no multicast); a small setup kernel turns the expert row
// offsets into the per-group problem shapes, pointers and strides.
//
//   fwd   : Y[r0:r1]  = X[r0:r1] @ W[e]^T            (W: E x N x K)
//   dgrad : dX[r0:r1] = dY[r0:r1] @ W[e]
//   wgrad : dW[e]    += dY[r0:r1]^T @ X[r0:r1]       (fp32 accumulate into the expert's main_grad)
// with rows r0 = offsets[e], r1 = offsets[e+1] of the expert-sorted token buffer.
//
// Groups with no rows: fwd/dgrad give them M = 0 (no tiles); wgrad points them at a zero block of
// 8 rows so no tensor map ever has an empty extent and the accumulated gradient is unchanged.
//
// Reference counterpart: the grouped expert GEMM of Megatron's MoE layer (TE grouped GEMM /
// sequential MLP) behind moe_token_dispatcher_type="alltoall" (axrl/worker/megatron_worker.py:833).
#include "gemm_sm100.cuh"

namespace ax {
namespace grouped {

using namespace cute;
using Problem = cutlass::gemm::GroupProblemShape<Shape<int, int, int>>;
using UShape = Problem::UnderlyingProblemShape;

template <class LayoutA, class LayoutB, class ElemD, class TileShape>
struct Grouped {
  static constexpr int kAlignD = 128 / cutlass::sizeof_bits<ElemD>::value;
  using Cluster = Shape<_1, _1, _1>;
  using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, TileShape, Cluster, cutlass::epilogue::collective::EpilogueTileAuto,
      float, float, ElemD, cutlass::layout::RowMajor*, kAlignD, ElemD, cutlass::layout::RowMajor*, kAlignD,
      cutlass::epilogue::PtrArrayTmaWarpSpecialized1Sm>::CollectiveOp;
  using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, cutlass::bfloat16_t, LayoutA*, 8, cutlass::bfloat16_t, LayoutB*, 8, float,
      TileShape, Cluster, cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
      cutlass::gemm::KernelPtrArrayTmaWarpSpecialized1SmSm100>::CollectiveOp;
  using Kernel = cutlass::gemm::kernel::GemmUniversal<Problem, Mainloop, Epilogue>;
  using Op = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;
  using SA = typename Kernel::InternalStrideA;
  using SB = typename Kernel::InternalStrideB;
  using SC = typename Kernel::InternalStrideC;
  using SD = typename Kernel::InternalStrideD;
};

using Tile = Shape<_128, _128, _64>;
using Fwd = Grouped<cutlass::layout::RowMajor, cutlass::layout::ColumnMajor, cutlass::bfloat16_t, Tile>;
using Dgrad = Grouped<cutlass::layout::RowMajor, cutlass::layout::RowMajor, cutlass::bfloat16_t, Tile>;
using Wgrad = Grouped<cutlass::layout::ColumnMajor, cutlass::layout::RowMajor, float, Tile>;

// Per-group argument arrays, carved out of one device buffer.
template <class G, class ElemD>
struct Arrays {
  UShape* shape;
  const cutlass::bfloat16_t** a;
  const cutlass::bfloat16_t** b;
  const ElemD** c;
  ElemD** d;
  typename G::SA* sa;
  typename G::SB* sb;
  typename G::SC* sc;
  typename G::SD* sd;
};

template <class G, class ElemD>
static size_t carve_bytes(int E) {
  auto align = [](size_t x) { return (x + 255) & ~size_t(255); };
  size_t sizes[9] = {sizeof(UShape), sizeof(void*), sizeof(void*), sizeof(void*), sizeof(void*), sizeof(typename G::SA),
                     sizeof(typename G::SB), sizeof(typename G::SC), sizeof(typename G::SD)};
  size_t total = 0;
  for (size_t s : sizes) total += align(s * E);
  return total;
}

template <class G, class ElemD>
static Arrays<G, ElemD> carve(void* base, int E) {
  auto align = [](size_t x) { return (x + 255) & ~size_t(255); };
  size_t sizes[9] = {sizeof(UShape), sizeof(void*), sizeof(void*), sizeof(void*), sizeof(void*), sizeof(typename G::SA),
                     sizeof(typename G::SB), sizeof(typename G::SC), sizeof(typename G::SD)};
  char* p = static_cast<char*>(base);
  Arrays<G, ElemD> r;
  size_t off = 0;
  auto take = [&](size_t s) { char* q = p + off; off += align(s * E); return q; };
  r.shape = reinterpret_cast<UShape*>(take(sizes[0]));
  r.a = reinterpret_cast<const cutlass::bfloat16_t**>(take(sizes[1]));
  r.b = reinterpret_cast<const cutlass::bfloat16_t**>(take(sizes[2]));
  r.c = reinterpret_cast<const ElemD**>(take(sizes[3]));
  r.d = reinterpret_cast<ElemD**>(take(sizes[4]));
  r.sa = reinterpret_cast<typename G::SA*>(take(sizes[5]));
  r.sb = reinterpret_cast<typename G::SB*>(take(sizes[6]));
  r.sc = reinterpret_cast<typename G::SC*>(take(sizes[7]));
  r.sd = reinterpret_cast<typename G::SD*>(take(sizes[8]));
  return r;
}

// fwd: group e: (M_e, N, K), A = X rows, B = W[e] (N x K), D = Y rows (N wide)
__global__ void setup_fwd_k(const int* __restrict__ off, int E, int N, int K, const cutlass::bfloat16_t* X, const cutlass::bfloat16_t* W,
                            cutlass::bfloat16_t* Y, Arrays<Fwd, cutlass::bfloat16_t> r) {
  int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  int r0 = off[e], m = off[e + 1] - r0;
  r.shape[e] = UShape{m, N, K};
  r.a[e] = X + (long)r0 * K;
  r.b[e] = W + (long)e * N * K;
  r.c[e] = nullptr;
  r.d[e] = Y + (long)r0 * N;
  r.sa[e] = cutlass::make_cute_packed_stride(typename Fwd::SA{}, make_shape(m, K, 1));
  r.sb[e] = cutlass::make_cute_packed_stride(typename Fwd::SB{}, make_shape(N, K, 1));
  r.sc[e] = cutlass::make_cute_packed_stride(typename Fwd::SC{}, make_shape(m, N, 1));
  r.sd[e] = cutlass::make_cute_packed_stride(typename Fwd::SD{}, make_shape(m, N, 1));
}

// dgrad: group e: (M_e, K, N): A = dY rows (M_e x N), B = W[e] stored N x K (K contiguous), D = dX rows
__global__ void setup_dgrad_k(const int* __restrict__ off, int E, int N, int K, const cutlass::bfloat16_t* dY, const cutlass::bfloat16_t* W,
                              cutlass::bfloat16_t* dX, Arrays<Dgrad, cutlass::bfloat16_t> r) {
  int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  int r0 = off[e], m = off[e + 1] - r0;
  r.shape[e] = UShape{m, K, N};
  r.a[e] = dY + (long)r0 * N;
  r.b[e] = W + (long)e * N * K;
  r.c[e] = nullptr;
  r.d[e] = dX + (long)r0 * K;
  r.sa[e] = cutlass::make_cute_packed_stride(typename Dgrad::SA{}, make_shape(m, N, 1));
  r.sb[e] = cutlass::make_cute_packed_stride(typename Dgrad::SB{}, make_shape(K, N, 1));
  r.sc[e] = cutlass::make_cute_packed_stride(typename Dgrad::SC{}, make_shape(m, K, 1));
  r.sd[e] = cutlass::make_cute_packed_stride(typename Dgrad::SD{}, make_shape(m, K, 1));
}

// wgrad: group e: (N, K, M_e): A = dY rows viewed N x M_e (N contiguous), B = X rows (M_e x K),
// C = D = dW[e] (fp32, N x K), beta = 1.  Empty experts read an 8-row zero block instead.
__global__ void setup_wgrad_k(const int* __restrict__ off, int E, int N, int K, const cutlass::bfloat16_t* dY, const cutlass::bfloat16_t* X,
                              float* dW, const cutlass::bfloat16_t* zeros, Arrays<Wgrad, float> r) {
  int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  int r0 = off[e], m = off[e + 1] - r0;
  bool empty = m == 0;
  int mk = empty ? 8 : m;
  r.shape[e] = UShape{N, K, mk};
  r.a[e] = empty ? zeros : dY + (long)r0 * N;
  r.b[e] = empty ? zeros : X + (long)r0 * K;
  r.c[e] = dW + (long)e * N * K;
  r.d[e] = dW + (long)e * N * K;
  r.sa[e] = cutlass::make_cute_packed_stride(typename Wgrad::SA{}, make_shape(N, mk, 1));
  r.sb[e] = cutlass::make_cute_packed_stride(typename Wgrad::SB{}, make_shape(K, mk, 1));
  r.sc[e] = cutlass::make_cute_packed_stride(typename Wgrad::SC{}, make_shape(N, K, 1));
  r.sd[e] = cutlass::make_cute_packed_stride(typename Wgrad::SD{}, make_shape(N, K, 1));
}

template <class G, class ElemD>
static void run(const Arrays<G, ElemD>& r, int E, float beta, cudaStream_t st) {
  typename G::Op::Arguments args;
  args.mode = cutlass::gemm::GemmUniversalMode::kGrouped;
  args.problem_shape = Problem{E, r.shape, nullptr};
  args.mainloop.ptr_A = r.a;
  args.mainloop.dA = r.sa;
  args.mainloop.ptr_B = r.b;
  args.mainloop.dB = r.sb;
  args.epilogue.thread.alpha = 1.f;
  args.epilogue.thread.beta = beta;
  args.epilogue.ptr_C = beta != 0.f ? r.c : nullptr;  // no source tensor maps when nothing is read
  args.epilogue.dC = r.sc;
  args.epilogue.ptr_D = r.d;
  args.epilogue.dD = r.sd;
  cudaGetDevice(&args.hw_info.device_id);
  args.hw_info.sm_count = num_sms();
  typename G::Op op;
  AX_REQUIRE(op.can_implement(args) == cutlass::Status::kSuccess, "grouped GEMM cannot implement");
  Scratch ws(G::Op::get_workspace_size(args), st);
  AX_REQUIRE(op.initialize(args, ws.ptr, st) == cutlass::Status::kSuccess, "grouped GEMM init");
  AX_REQUIRE(op.run(st) == cutlass::Status::kSuccess, "grouped GEMM run");
}

using B16 = cutlass::bfloat16_t;

// Y (rows, N) = per-expert X rows @ W[e]^T; off (E+1) int32 on the device.
void fwd(const int* off, int E, int N, int K, const void* X, const void* W, void* Y, cudaStream_t st) {
  Scratch buf(carve_bytes<Fwd, B16>(E), st);
  auto r = carve<Fwd, B16>(buf.ptr, E);
  setup_fwd_k<<<(E + 127) / 128, 128, 0, st>>>(off, E, N, K, (const B16*)X, (const B16*)W, (B16*)Y, r);
  AX_LAUNCH_OK();
  run<Fwd, B16>(r, E, 0.f, st);
}

// dX (rows, K) = per-expert dY rows @ W[e]
void dgrad(const int* off, int E, int N, int K, const void* dY, const void* W, void* dX, cudaStream_t st) {
  Scratch buf(carve_bytes<Dgrad, B16>(E), st);
  auto r = carve<Dgrad, B16>(buf.ptr, E);
  setup_dgrad_k<<<(E + 127) / 128, 128, 0, st>>>(off, E, N, K, (const B16*)dY, (const B16*)W, (B16*)dX, r);
  AX_LAUNCH_OK();
  run<Dgrad, B16>(r, E, 0.f, st);
}

// acc (E, N, K) fp32 += per-expert dY rows^T @ X rows; zeros: 8 x max(N, K) bf16 zeros.
void wgrad_acc(const int* off, int E, int N, int K, const void* dY, const void* X, float* acc, const void* zeros, cudaStream_t st) {
  Scratch buf(carve_bytes<Wgrad, float>(E), st);
  auto r = carve<Wgrad, float>(buf.ptr, E);
  setup_wgrad_k<<<(E + 127) / 128, 128, 0, st>>>(off, E, N, K, (const B16*)dY, (const B16*)X, acc, (const B16*)zeros, r);
  AX_LAUNCH_OK();
  run<Wgrad, float>(r, E, 1.f, st);
}

}  // namespace grouped
}  // namespace ax
