// Weight-streaming GEMM for skinny activations (decode): Y[M,N] = X[M,K] @ W[N,K]^T (+ R), M <= 64.
//
// At decode batch sizes the GEMM is a read of W at HBM speed, so what matters is that every SM
// streams the same number of bytes from the first microsecond to the last:
//   * the work is a list of units (64-row W tile, 64-wide K slab), tile-major; one wave of CTAs
//     (as many as fit on the SMs, ~3 per SM) each takes an equal contiguous range of units, so no
//     CTA waits for a second wave whatever N and K are (a (N/64) x splits grid left 4 to 36 CTAs of
//     a second wave on most Qwen3-8B projections);
//   * 6-stage cp.async pipeline of W slabs (8 KB) and the matching X slab (MT x 128 B), 128-byte
//     rows XOR-swizzled so ldmatrix is conflict-free;
//   * each of the 8 warps owns 8 W rows and all MT rows of X (mma.m16n8k16, fp32 accumulate);
//   * a tile whose K range lies entirely in one CTA is written directly (with the residual); a
//     tile split between CTAs accumulates in an fp32 workspace with red.global.add, and the CTA
//     whose slabs complete the tile's K range (arrival counter of slabs) adds the residual, writes
//     bf16 and zeroes its workspace tile and counter, so the workspace is clean for the next call
//     without a memset (safe inside a CUDA graph; calls must be stream-ordered because they share
//     the workspace).
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
  float* ws;  // M x N fp32, zero between calls (only touched by tiles split between CTAs)
  int* cnt;   // one slab counter per W tile, zero between calls
  int M, N, K;
  int kslabs, units, per;  // per: units per CTA
  int prefetch_w;          // weights are read-only for this launch: stream them before the predecessor ends
};

template <int MT>
__device__ __forceinline__ void flush_tile(const Params& p, int tile, int slabs, float (&acc)[MT / 16][4], int tid, int warp, int lane,
                                           int* s_last) {
  const int n0 = tile * NT;
  const int col = n0 + warp * 8 + (lane & 3) * 2;
  if (slabs == p.kslabs) {  // the whole K range was here: write the tile
    if (col < p.N) {
#pragma unroll
      for (int mt = 0; mt < MT / 16; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = mt * 16 + (lane >> 2) + h * 8;
          if (row < p.M) {
            float v0 = acc[mt][2 * h], v1 = acc[mt][2 * h + 1];
            if (p.r) {
              const float2 rr = __bfloat1622float2(*reinterpret_cast<const bf162*>(p.r + (long)row * p.N + col));
              v0 += rr.x;
              v1 += rr.y;
            }
            *reinterpret_cast<bf162*>(p.y + (long)row * p.N + col) = __floats2bfloat162_rn(v0, v1);
          }
        }
    }
    return;
  }
  if (col < p.N) {
#pragma unroll
    for (int mt = 0; mt < MT / 16; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = mt * 16 + (lane >> 2) + h * 8;
        if (row < p.M) {
          atomicAdd(p.ws + (long)row * p.N + col, acc[mt][2 * h]);
          atomicAdd(p.ws + (long)row * p.N + col + 1, acc[mt][2 * h + 1]);
        }
      }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) *s_last = atomicAdd(p.cnt + tile, slabs) + slabs == p.kslabs;
  __syncthreads();
  if (!*s_last) return;
  __threadfence();
  const int half_cols = min(NT, p.N - n0) / 2;
  for (int i = tid; i < p.M * half_cols; i += THREADS) {
    const int row = i / half_cols, c = n0 + (i % half_cols) * 2;
    float* src = p.ws + (long)row * p.N + c;
    float v0 = __ldcg(src), v1 = __ldcg(src + 1);
    if (p.r) {
      const float2 rr = __bfloat1622float2(*reinterpret_cast<const bf162*>(p.r + (long)row * p.N + c));
      v0 += rr.x;
      v1 += rr.y;
    }
    *reinterpret_cast<bf162*>(p.y + (long)row * p.N + c) = __floats2bfloat162_rn(v0, v1);
    __stcg(src, 0.f);
    __stcg(src + 1, 0.f);
  }
  if (tid == 0) p.cnt[tile] = 0;
}

template <int MT>
__global__ void __launch_bounds__(THREADS) skinny_k(Params p) {
  extern __shared__ __align__(128) char smem[];
  __shared__ int s_last;
  constexpr int WB = NT * KT * 2;
  constexpr int XB = MT * KT * 2;
  constexpr int SB = WB + XB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int u0 = blockIdx.x * p.per;
  const int n_units = max(0, min(p.units, u0 + p.per) - u0);

  auto load_w = [&](int i, int slot) {
    char* sw = smem + slot * SB;
    const int u = u0 + i, n0 = (u / p.kslabs) * NT, k = (u % p.kslabs) * KT;
#pragma unroll
    for (int e = tid; e < NT * 8; e += THREADS) {
      const int row = e >> 3, c = (e & 7) * 8;
      const int g = n0 + row;
      const bool ok = g < p.N;
      cp16(sw + swz(row, c), p.w + (long)(ok ? g : 0) * p.K + k + c, ok);
    }
  };
  auto load_x = [&](int i, int slot) {
    char* sx = smem + slot * SB + WB;
    const int k = ((u0 + i) % p.kslabs) * KT;
    for (int e = tid; e < MT * 8; e += THREADS) {
      const int row = e >> 3, c = (e & 7) * 8;
      const bool ok = row < p.M;
      cp16(sx + swz(row, c), p.x + (long)(ok ? row : 0) * p.K + k + c, ok);
    }
  };

  // Weight slabs of the first stages may be in flight before the predecessor kernel finishes
  // (programmatic dependent launch); activations, the residual and every write wait for it.  The
  // early loads join the first commit group, so the pipeline accounting below is unchanged.
  if (p.prefetch_w) {
#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s)
      if (s < n_units) load_w(s, s);
  }
  pdl_wait();
  pdl_trigger();
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < n_units) {
      if (!p.prefetch_w) load_w(s, s);
      load_x(s, s);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  }

  float acc[MT / 16][4];
#pragma unroll
  for (int i = 0; i < MT / 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  int tile = u0 / p.kslabs, slabs = 0;

  for (int i = 0; i < n_units; ++i) {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(STAGES - 2));
    __syncthreads();
    if (i + STAGES - 1 < n_units) {
      load_w(i + STAGES - 1, (i + STAGES - 1) % STAGES);
      load_x(i + STAGES - 1, (i + STAGES - 1) % STAGES);
    }
    asm volatile("cp.async.commit_group;\n" ::);
    const char* sw = smem + (i % STAGES) * SB;
    const char* sx = sw + WB;
#pragma unroll
    for (int k16 = 0; k16 < KT / 16; ++k16) {
      uint32_t b0, b1;
      {
        const int row = warp * 8 + (lane & 7), col = k16 * 16 + ((lane >> 3) & 1) * 8;
        asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(b0), "=r"(b1) : "r"(smem_u32(sw + swz(row, col))));
      }
#pragma unroll
      for (int mt = 0; mt < MT / 16; ++mt) {
        uint32_t a0, a1, a2, a3;
        const int row = mt * 16 + (lane & 15), col = k16 * 16 + (lane >> 4) * 8;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3) : "r"(smem_u32(sx + swz(row, col))));
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                     : "+f"(acc[mt][0]), "+f"(acc[mt][1]), "+f"(acc[mt][2]), "+f"(acc[mt][3])
                     : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
      }
    }
    ++slabs;
    const bool last_unit = i + 1 == n_units;
    if (last_unit || (u0 + i + 1) / p.kslabs != tile) {  // CTA-uniform
      flush_tile<MT>(p, tile, slabs, acc, tid, warp, lane, &s_last);
#pragma unroll
      for (int j = 0; j < MT / 16; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
      slabs = 0;
      ++tile;
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
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
  const int n_tiles = (N + NT - 1) / NT;
  const int kslabs = K / KT;
  const int units = n_tiles * kslabs;
  const int mt = M <= 16 ? 16 : M <= 32 ? 32 : 64;
  const int smem = STAGES * (NT * KT * 2 + mt * KT * 2);
  auto* kern = mt == 16 ? skinny_k<16> : mt == 32 ? skinny_k<32> : skinny_k<64>;
  const int which = mt == 16 ? 0 : mt == 32 ? 1 : 2;
  const int dev = x.get_device();
  static bool attr_set[16][3] = {{false}};
  static int occ[16][3] = {{0}};
  if (!attr_set[dev][which]) {
    AX_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    AX_CUDA_OK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ[dev][which], kern, THREADS, smem));
    attr_set[dev][which] = true;
  }
  // one wave: every resident CTA streams an equal share of the units
  const int slots = num_sms() * std::max(1, occ[dev][which]);
  int per = (units + slots - 1) / slots;
  float* ws = nullptr;
  int* cnt = nullptr;
  if ((long)M * N <= WS_FLOATS && n_tiles <= WS_TILES) {
    auto& W = workspace(dev);
    ws = W.ws.data_ptr<float>();
    cnt = W.cnt.data_ptr<int>();
  } else {
    per = ((per + kslabs - 1) / kslabs) * kslabs;  // whole tiles per CTA: no workspace needed
  }
  const int grid = (units + per - 1) / per;
  Params p{(const bf16*)x.data_ptr(), (const bf16*)w.data_ptr(), r, (bf16*)y.data_ptr(), ws, cnt, M, N, K, kslabs, units, per,
           (int)(weights_static() && pdl_enabled())};
  launch_pdl(kern, dim3(grid), dim3(THREADS), smem, stream(), p);
  AX_LAUNCH_OK();
  return y;
}
at::Tensor skinny_linear(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> residual) {
  return skinny_linear_out(x, w, residual, c10::nullopt);
}

}  // namespace ax
