// Narrow-feature (d <= 16) squared-L2 cost and gradient kernels: host entry points used by the C ABI in
// sdtw_distance.cu.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

#include "sdtw_common.cuh"

namespace sdtw {

// Whether the narrow kernels take these sizes (d <= 16; B within one launch's grid).
bool narrow_supported(int64_t B, int64_t N, int64_t M, int64_t d);

// D = clamp((|x|^2 + |y|^2) - 2 X Y^T) with the clamp recorded as -0.0 and in clamp_flags (optional).
template <typename T>
cudaError_t narrow_pairwise_l2(const T* X, const T* Y, T* D, int* clamp_flags, int64_t B, int64_t N, int64_t M,
                               int64_t d, cudaStream_t s);

// grad_X = 2 g (rowsum(G) X - G Y), grad_Y = 2 g (colsum(G) Y - G^T X), G = E with the clamped cells of D
// (sign bit) zeroed in pairs whose flag is set (every pair when clamp_flags is null); gX / gY may be null.
template <typename T>
cudaError_t narrow_grad_l2(const T* X, const T* Y, const T* D, const T* E, const T* g, const int* clamp_flags, T* gX,
                           T* gY, int64_t B, int64_t N, int64_t M, int64_t d, cudaStream_t s);

}  // namespace sdtw
