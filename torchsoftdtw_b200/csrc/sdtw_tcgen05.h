// Tensor-core (tcgen05) kernels: host entry points used by the C ABI in sdtw_distance.cu.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace sdtw {

// The cells a pair's dynamic program reads: rows below lengths_x[b], columns below lengths_y[b] and inside
// the Sakoe-Chiba band of bandwidth bw (bw < 0: no band). Lengths are int32 (is32) or int64 device arrays;
// pairs whose lengths lie outside [0, N] x [0, M] read no cell (the wavefront kernels treat them as empty).
struct DpRegion {
    const void* px;
    const void* py;
    int is32;
    int64_t bw;
};

// Bytes of the tile list pairwise_tc_launch builds when given a region.
size_t pairwise_tc_region_ws_bytes(int64_t B, int64_t N, int64_t M);

// Whether the tcgen05 cost-matrix kernel handles these fp32 arguments (TMA needs 16-byte aligned bases
// and rows, hence d % 4 == 0 and M % 4 == 0).
bool pairwise_tc_supported(const void* X, const void* Y, const void* D, int64_t B, int64_t N, int64_t M, int64_t d);

// D = clamp(|x|^2 + |y|^2 - 2 X Y^T) for fp32 X (B,N,d), Y (B,M,d); clamp_flags (optional) as for
// sdtw_pairwise_l2. With cosine: D = 1 - X Y^T / (n(x) n(y)), n(v) = max(|v|, eps), no clamp. Every wait in
// the kernel is bounded by timeout_s. With a region (and ws, pairwise_tc_region_ws_bytes(B, N, M) bytes, 16-byte
// aligned): only the 128 x 128 tiles of D that hold a cell of the region are computed, listed first by a
// one-CTA kernel; the other cells of D are left as they were, and the clamp flags cover the computed tiles.
cudaError_t pairwise_tc_launch(const float* X, const float* Y, float* D, int* clamp_flags, int64_t B, int64_t N,
                               int64_t M, int64_t d, double timeout_s, cudaStream_t s, bool cosine = false,
                               float eps = 0.f, const DpRegion* region = nullptr, void* ws = nullptr);

// Whether the tcgen05 grad_X kernel handles these fp32 arguments (d <= 128, d % 4 == 0, M % 4 == 0,
// 16-byte aligned bases).
bool grad_tc_supported(const void* X, const void* Y, const void* D, const void* E, const void* gX, int64_t B,
                       int64_t N, int64_t M, int64_t d);

// grad_X = 2 g[b] (rowsum(G) X - G Y), G = E with the clamped cells of D (sign bit) zeroed in pairs whose
// clamp flag is set (every pair when clamp_flags is null). With ry (cosine; 1 / n(y_j) per row of Y, B x M,
// 16-byte aligned): P = E (Y / n(Y)) and grad_X = -g[b] / n(x_i) (P - [|x_i| >= eps] (x_i.P) x_i / n(x_i)^2);
// D and clamp_flags are not read. Every wait in the kernel is bounded by timeout_s. With a region, E must be
// zero outside it (as the backward wavefronts leave it): each row tile contracts only the 32-column chunks that
// hold a cell of the region, and reads D only there.
cudaError_t grad_x_tc_launch(const float* X, const float* Y, const float* D, const float* E, const float* g,
                             const int* clamp_flags, float* gX, int64_t B, int64_t N, int64_t M, int64_t d,
                             double timeout_s, cudaStream_t s, const float* ry = nullptr, float eps = 0.f,
                             const DpRegion* region = nullptr);

// grad_Y = 2 g[b] (colsum(G) Y - G^T X) on the same kernel, E read transposed; with rx (cosine; 1 / n(x_i) per
// row of X, B x N, 16-byte aligned): P = G^T (X / n(X)) and the cosine form of grad_X with the roles of X and
// Y swapped. Supported when grad_tc_supported(X, Y, D, E, gY, B, N, M, d) holds.
cudaError_t grad_y_tc_launch(const float* X, const float* Y, const float* D, const float* E, const float* g,
                             const int* clamp_flags, float* gY, int64_t B, int64_t N, int64_t M, int64_t d,
                             double timeout_s, cudaStream_t s, const float* rx = nullptr, float eps = 0.f,
                             const DpRegion* region = nullptr);

// The distance kernel family forced by sdtw_debug_force_distance_path (0: automatic, 1: no tcgen05,
// 2: CUDA cores only).
int distance_path();

// Reads and clears the tensor-core kernels' error bits (1: a wait ran out and a tile was written as NaN).
cudaError_t read_distance_errors(uint32_t& bits);

}  // namespace sdtw
