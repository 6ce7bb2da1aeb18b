// Weight-streaming GEMM for skinny activations (decode): Y[M,N] = X[M,K] @ W[N,K]^T (+ R), M <= 64.
//
// At decode batch sizes the GEMM is a read of W at HBM speed; the 128-row MMA tiles of the
// general GEMM waste most of their operand traffic on padding rows and leave SMs idle when
// N/tile is small.  Here:
//   * a CTA owns 64 rows of W and a K range; the grid is (N/64) x splits with `splits` chosen so
//     that ~3 CTAs are resident per SM (every SM streams weights);
//   * 6-stage cp.async pipeline of 64-element K slabs (W 8 KB + X MT*128 B per stage), 128-byte
//     rows XOR-swizzled so ldmatrix is conflict-free;
//   * each of the 8 warps owns 8 W rows and all MT rows of X (mma.m16n8k16, fp32 accumulate);
//   * splits > 1: partial sums go to an fp32 workspace with red.global.add; the last CTA of an
//     output tile (atomic arrival counter) adds the residual, writes bf16 and zeroes its workspace
//     tile and counter, so the workspace is clean for the next call without a memset (safe inside
//     a CUDA graph; calls must be stream-ordered because they share the workspace).
#include "common.cuh"

namespace ax {
namespace sk {

constexpr int NT = 64;
constexpr int KT = 64;
constexpr int STAGES = 6;
constexpr int THREADS = 256;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ int swz(int row, int col) { return row * 128 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2; }
__device__ __forceinline__ void cp16(void* s, const void* g, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(s)), "l"(g), "r"(pred ? 16 : 0));
}

struct Params {
  const bf16* x;
  const bf16* w;
  const bf16* r;
  bf16* y;
  float* ws;
  int* cnt;
  int M, N, K, kc, splits;
  int prefetch_w;  // weights are read-only for this launch: stream them before the predecessor ends
};

template <int MT>
__global__ void __launch_bounds__(THREADS) skinny_k(Params p) {
  extern __shared__ __align__(128) char smem[];
  constexpr int WB = NT * KT * 2;
  constexpr int XB = MT * KT * 2;
  constexpr int SB = WB + XB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * NT;
  const int kb0 = blockIdx.y * p.kc;
  const int kb1 = min(p.K, kb0 + p.kc);
  const int nk = (kb1 - kb0) / KT;

  auto load_w = [&](int kb, int slot) {
    char* sw = smem + slot * SB;
    const int k = kb0 + kb * KT;
#pragma unroll
    for (int i = tid; i < NT * 8; i += THREADS) {
      int row = i >> 3, c = (i & 7) * 8;
      int g = n0 + row;
      bool ok = g < p.N;
      cp16(sw + swz(row, c), p.w + (long)(ok ? g : 0) * p.K + k + c, ok);
    }
  };
  auto load_x = [&](int kb, int slot) {
    char* sx = smem + slot * SB + WB;
    const int k = kb0 + kb * KT;
    for (int i = tid; i < MT * 8; i += THREADS) {
      int row = i >> 3, c = (i & 7) * 8;
      bool ok = row < p.M;
      cp16(sx + swz(row, c), p.x + (long)(ok ? row : 0) * p.K + k + c, ok);
    }
  };

  // Weight slabs of the first stages may be in flight before the predecessor kernel finishes
  // (programmatic dependent launch); activations, the residual and every write wait for it.  The
  // early loads join the first commit group, so the pipeline accounting below is unchanged.
  if (p.prefetch_w) {
#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s)
      if (s < nk) load_w(s, s);
  }
  pdl_trigger();  // successors may launch now; they wait for this grid's completion
  pdl_wait();
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < nk) {
      if (!p.prefetch_w) load_w(s, s);
      load_x(s, s);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  }

  float acc[MT / 16][4];
#pragma unroll
  for (int i = 0; i < MT / 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  for (int kb = 0; kb < nk; ++kb) {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(STAGES - 2));
    __syncthreads();
    if (kb + STAGES - 1 < nk) {
      load_w(kb + STAGES - 1, (kb + STAGES - 1) % STAGES);
      load_x(kb + STAGES - 1, (kb + STAGES - 1) % STAGES);
    }
    asm volatile("cp.async.commit_group;\n" ::);
    const char* sw = smem + (kb % STAGES) * SB;
    const char* sx = sw + WB;
#pragma unroll
    for (int k16 = 0; k16 < KT / 16; ++k16) {
      uint32_t b0, b1;
      {
        int row = warp * 8 + (lane & 7), col = k16 * 16 + ((lane >> 3) & 1) * 8;
        asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(b0), "=r"(b1) : "r"(smem_u32(sw + swz(row, col))));
      }
#pragma unroll
      for (int mt = 0; mt < MT / 16; ++mt) {
        uint32_t a0, a1, a2, a3;
        int row = mt * 16 + (lane & 15), col = k16 * 16 + (lane >> 4) * 8;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3) : "r"(smem_u32(sx + swz(row, col))));
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                     : "+f"(acc[mt][0]), "+f"(acc[mt][1]), "+f"(acc[mt][2]), "+f"(acc[mt][3])
                     : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
      }
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::);

  const int col = n0 + warp * 8 + (lane & 3) * 2;
  if (p.splits == 1) {
    if (col < p.N) {
#pragma unroll
      for (int mt = 0; mt < MT / 16; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int row = mt * 16 + (lane >> 2) + h * 8;
          if (row < p.M) {
            float v0 = acc[mt][2 * h], v1 = acc[mt][2 * h + 1];
            if (p.r) {
              float2 rr = __bfloat1622float2(*reinterpret_cast<const bf162*>(p.r + (long)row * p.N + col));
              v0 += rr.x;
              v1 += rr.y;
            }
            *reinterpret_cast<bf162*>(p.y + (long)row * p.N + col) = __floats2bfloat162_rn(v0, v1);
          }
        }
    }
    return;
  }
  // split-K: accumulate partials, last arriver finalises and cleans the tile
  if (col < p.N) {
#pragma unroll
    for (int mt = 0; mt < MT / 16; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        int row = mt * 16 + (lane >> 2) + h * 8;
        if (row < p.M) {
          atomicAdd(p.ws + (long)row * p.N + col, acc[mt][2 * h]);
          atomicAdd(p.ws + (long)row * p.N + col + 1, acc[mt][2 * h + 1]);
        }
      }
  }
  __threadfence();
  __syncthreads();
  __shared__ int last;
  if (tid == 0) last = atomicAdd(p.cnt + blockIdx.x, 1) == p.splits - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int cols = min(NT, p.N - n0);
  for (int i = tid; i < p.M * (cols / 2); i += THREADS) {
    int row = i / (cols / 2), c = n0 + (i % (cols / 2)) * 2;
    float* src = p.ws + (long)row * p.N + c;
    float v0 = __ldcg(src), v1 = __ldcg(src + 1);
    if (p.r) {
      float2 rr = __bfloat1622float2(*reinterpret_cast<const bf162*>(p.r + (long)row * p.N + c));
      v0 += rr.x;
      v1 += rr.y;
    }
    *reinterpret_cast<bf162*>(p.y + (long)row * p.N + c) = __floats2bfloat162_rn(v0, v1);
    __stcg(src, 0.f);
    __stcg(src + 1, 0.f);
  }
  if (tid == 0) p.cnt[blockIdx.x] = 0;
}

// Persistent, self-cleaning split-K workspace per device (zero between calls).
constexpr long WS_FLOATS = 64L * 65536;
constexpr int WS_TILES = 8192;

struct Workspace {
  at::Tensor ws, cnt;
};

static Workspace& workspace(int dev) {
  static Workspace w[16];
  if (!w[dev].ws.defined()) {
    auto o = at::TensorOptions().device(at::kCUDA, dev);
    w[dev].ws = at::zeros({WS_FLOATS}, o.dtype(at::kFloat));
    w[dev].cnt = at::zeros({WS_TILES}, o.dtype(at::kInt));
  }
  return w[dev];
}

}  // namespace sk

// Y = X @ W^T (+ R) for X with at most 64 rows.
at::Tensor skinny_linear_out(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual, c10::optional<at::Tensor> out) {
  using namespace sk;
  AX_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && x.is_contiguous() && w.is_contiguous(), "bf16 contiguous");
  int M = x.size(0), K = x.size(1), N = w.size(0);
  AX_CHECK(M <= 64 && w.size(1) == K && K % KT == 0 && N % 8 == 0, "skinny_linear: M<=64, K%64==0, N%8==0");
  auto y = out.has_value() ? *out : at::empty({M, N}, x.options());
  AX_CHECK(y.is_contiguous() && y.size(0) == M && y.size(1) == N, "output shape");
  if (M == 0) return y;
  const bf16* r = nullptr;
  if (residual.has_value()) {
    AX_CHECK(residual->is_contiguous() && residual->size(0) == M && residual->size(1) == N, "residual shape");
    r = (const bf16*)residual->data_ptr();
  }
  int n_tiles = (N + NT - 1) / NT;
  int target = num_sms() * 3;
  int splits = std::max(1, std::min((target + n_tiles - 1) / n_tiles, K / (4 * KT)));
  int kc = ((K / splits + KT - 1) / KT) * KT;
  splits = (K + kc - 1) / kc;
  int dev = x.get_device();
  float* ws = nullptr;
  int* cnt = nullptr;
  if (splits > 1) {
    if ((long)M * N <= WS_FLOATS && n_tiles <= WS_TILES) {
      auto& W = workspace(dev);
      ws = W.ws.data_ptr<float>();
      cnt = W.cnt.data_ptr<int>();
    } else {
      splits = 1;
      kc = K;
    }
  }
  Params p{(const bf16*)x.data_ptr(), (const bf16*)w.data_ptr(), r, (bf16*)y.data_ptr(), ws, cnt, M, N, K, kc, splits,
           (int)(weights_static() && pdl_enabled())};
  dim3 grid(n_tiles, splits);
  auto launch = [&](auto kern, int mt, int which) {
    (void)which;
    int smem = STAGES * (NT * KT * 2 + mt * KT * 2);
    smem_attr(reinterpret_cast<const void*>(kern), smem);
    launch_pdl(kern, grid, dim3(THREADS), smem, stream(), p);
  };
  if (M <= 16) launch(skinny_k<16>, 16, 0);
  else if (M <= 32) launch(skinny_k<32>, 32, 1);
  else launch(skinny_k<64>, 64, 2);
  AX_LAUNCH_OK();
  return y;
}

at::Tensor skinny_linear(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual) {
  return skinny_linear_out(x, w, residual, c10::nullopt);
}

}  // namespace ax
