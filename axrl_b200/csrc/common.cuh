// Torch-facing side of the sm_100a kernels: the pure-CUDA helpers plus the tensor types used by
// the wrappers that check, allocate and launch.  Only the light ATen headers are included
// (tensor class, the factory functions used here, the current CUDA stream); the Python module
// itself is built in bindings.cpp.
#pragma once
#include "cuda_common.cuh"

#include <ATen/core/Tensor.h>
#include <ATen/ops/empty.h>
#include <ATen/ops/empty_like.h>
#include <ATen/ops/full.h>
#include <ATen/ops/zeros.h>
#include <ATen/ops/zeros_like.h>
#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAStream.h>
#include <c10/util/Optional.h>

#define AX_CHECK(cond, ...) TORCH_CHECK(cond, __VA_ARGS__)

namespace ax {
inline cudaStream_t stream() { return c10::cuda::getCurrentCUDAStream().stream(); }
}  // namespace ax
