// Trainer -> rollout weight sync: reshard + cast / 128x128 block-fp8 quantise + push.
//
// Reference counterpart: SGLangTensorWeightUpdater / SGLangDistributedWeightUpdater
// (axrl/utils/megatron/sglang_weight_updater.py:60-338) with per_block_cast_to_fp8
// (axrl/utils/megatron/fp8_quantizer.py:60-146): export HF tensors (gathering TP/EP shards),
// bucket them, optionally quantise, ship through CUDA IPC / NCCL broadcast, load in the engine.
//
// Here every trainer rank pushes its OWN shard.  The host precomputes a list of 128x128
// tiles, each fully inside one source shard and one destination shard:
//   (src_off, src_ld, dst_rank, dst_off, dst_ld, rows, cols, scale_off, scale_ld, scale_idx)
// One CTA per tile reads the tile from local HBM, optionally computes the block amax, and
// writes the bf16 / e4m3 values (and the fp32 inverse scale) straight into the destination
// rank's weight buffer with P2P stores over NVLink.  No gather, no staging, no rank-0 funnel.
#include <cuda_fp8.h>

#include "common.cuh"

namespace ax {

constexpr int SYNC_TILE = 128;

struct SyncTile {
  int64_t src_off, src_ld, dst_rank, dst_off, dst_ld, rows, cols, scale_off, scale_ld, scale_idx;
};
static_assert(sizeof(SyncTile) == 10 * 8, "tile record layout");

// mode 0: bf16 -> bf16 copy; mode 1: bf16 -> e4m3 with one fp32 inverse scale per 128x128 block.
__global__ void __launch_bounds__(256) sync_push_k(const SyncTile* __restrict__ tiles, const bf16* __restrict__ src,
                                                   const int64_t* __restrict__ dst_ptrs, int mode) {
  const SyncTile t = tiles[blockIdx.x];
  const bf16* s = src + t.src_off;
  char* dbase = reinterpret_cast<char*>(dst_ptrs[t.dst_rank]);
  int rows = (int)t.rows, cols = (int)t.cols;
  if (mode == 0) {
    bf16* d = reinterpret_cast<bf16*>(dbase) + t.dst_off;
    int c8 = cols / 8;
    for (int i = threadIdx.x; i < rows * c8; i += blockDim.x) {
      int r = i / c8, c = (i % c8) * 8;
      *reinterpret_cast<V8*>(d + (long)r * t.dst_ld + c) = *reinterpret_cast<const V8*>(s + (long)r * t.src_ld + c);
    }
    return;
  }
  __shared__ float sh[32];
  float amax = 0.f;
  int c8 = cols / 8;
  for (int i = threadIdx.x; i < rows * c8; i += blockDim.x) {
    int r = i / c8, c = (i % c8) * 8;
    float f[8];
    load8(s + (long)r * t.src_ld + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
  }
  // block max via warp shuffles + smem
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) sh[0] = v;
  }
  __syncthreads();
  amax = fmaxf(sh[0], 1e-12f);
  const float scale_inv = amax / 448.f;  // dequant: w = q * scale_inv
  const float qs = 448.f / amax;
  uint8_t* d = reinterpret_cast<uint8_t*>(dbase) + t.dst_off;
  for (int i = threadIdx.x; i < rows * c8; i += blockDim.x) {
    int r = i / c8, c = (i % c8) * 8;
    float f[8];
    load8(s + (long)r * t.src_ld + c, f);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_fp8_e4m3 a(f[j] * qs), b(f[j + 4] * qs);
      lo |= (uint32_t)a.__x << (8 * j);
      hi |= (uint32_t)b.__x << (8 * j);
    }
    *reinterpret_cast<uint2*>(d + (long)r * t.dst_ld + c) = make_uint2(lo, hi);
  }
  if (threadIdx.x == 0) reinterpret_cast<float*>(dbase + t.scale_off)[t.scale_idx] = scale_inv;
}

void sync_push(at::Tensor tiles, at::Tensor src, at::Tensor dst_ptrs, int64_t mode) {
  AX_CHECK(tiles.scalar_type() == at::kLong && tiles.is_cuda() && tiles.size(1) == 10, "tiles: int64 (n, 10) on device");
  AX_CHECK(src.scalar_type() == at::kBFloat16, "source must be bf16");
  int n = tiles.size(0);
  if (n == 0) return;
  sync_push_k<<<n, 256, 0, stream()>>>(reinterpret_cast<const SyncTile*>(tiles.data_ptr<int64_t>()), (const bf16*)src.data_ptr(),
                                      dst_ptrs.data_ptr<int64_t>(), (int)mode);
  AX_LAUNCH_OK();
}

}  // namespace ax
