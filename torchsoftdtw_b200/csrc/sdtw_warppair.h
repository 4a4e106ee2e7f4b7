// Warp-per-pair wavefront kernels (one warp per pair, strips swept one after the other, operands in
// global memory): host entry points used by the C ABI in sdtw_wavefront.cu.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#include "sdtw_common.cuh"

namespace sdtw {

constexpr int kWarpPairWarps = 4;    // warps (= pairs) per CTA
constexpr int kWarpPairMinCtas = 4;  // registers sized for at least 4 resident CTAs (16 warps) per SM

// Shared-memory bytes of one CTA (one row buffer per warp).
template <typename T>
size_t warp_fwd_smem_bytes(int64_t M);
template <typename T>
size_t warp_bwd_smem_bytes(int64_t M);

template <typename T>
cudaError_t warp_forward(const T* D, T* R, T* costs, const void* lx, const void* ly, int is32, int64_t B, int64_t N,
                         int64_t M, int64_t bw, double gamma, uint32_t* err, cudaStream_t stream);
template <typename T>
cudaError_t warp_backward(const T* R, T* E, const void* lx, const void* ly, int is32, int64_t B, int64_t N, int64_t M,
                          int64_t bw, double gamma, uint32_t* err, cudaStream_t stream);

}  // namespace sdtw
