// Pair-resident wavefront kernels (one CTA per pair, strip boundaries in shared memory): host entry
// points used by the C ABI in sdtw_wavefront.cu.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#include "sdtw_common.cuh"

namespace sdtw {

// Launch bounds of the pair-resident kernels: at most SDTW_PAIR_THREADS threads per CTA, and registers
// sized for SDTW_PAIR_MIN_CTAS resident CTAs of that size per SM.
#ifndef SDTW_PAIR_THREADS
#define SDTW_PAIR_THREADS 512
#endif
#ifndef SDTW_PAIR_MIN_CTAS
#define SDTW_PAIR_MIN_CTAS 1
#endif
constexpr int kPairMaxWarps = SDTW_PAIR_THREADS / 32;  // warps per CTA at most
constexpr int kBufPad = 64;        // boundary rows are indexed by column + kBufPad
// Row length M for which the wavefront kernels are also compiled with M as a compile-time constant
// (immediate row offsets in the ring loads and stores); other lengths run the generic instantiation.
constexpr int kPairSpecialM = 512;

// Shared-memory bytes of one CTA with W warps.
template <typename T>
size_t pair_fwd_smem_bytes(int W, int64_t M);
template <typename T>
size_t pair_bwd_smem_bytes(int W, int64_t M);

// Sets the kernels' dynamic shared-memory limit (once per device).
template <typename T>
cudaError_t pair_init_attrs(int max_smem);

// Registers per thread of the forward / backward kernel.
template <typename T>
cudaError_t pair_regs(bool backward, int& regs);

// Largest W <= cap (and <= the strip count) whose CTA fits `budget` bytes; 0 if none.
template <typename T>
int pair_warps(bool backward, int64_t N, int64_t M, int cap, size_t budget);

// Progress keys stay below 2^30 for these sizes.
bool pair_keys_fit(int64_t N, int64_t M);

// R as strip tiles (the module path's layout between the pair-resident forward and backward): tile (b, s, k)
// is 32 x 32 elements, row l holding R[32 s + l][32 k + x - l - 1] log2(e) / gamma at x = 0..31 (R in units of
// gamma ln 2; +inf outside the band and the lengths); tiles of blocks a strip does not sweep are never
// written. Blocks per strip: pair_tile_blocks(M).
inline int pair_tile_blocks(int64_t M) { return static_cast<int>((M + 31) / 32) + 1; }

// Fused squared-L2 forward (fp32, R as strip tiles): the cost matrix D = (|x|^2 + |y|^2) - 2 x.y, clamped
// at 0, is computed tile by tile inside the forward from X (B, N, d) and Y (B, M, d) (d a multiple of 16,
// both 16-byte aligned) and never stored. Clamped cells inside the matrix set bit c % 32 of word
// cmask[(b N + i) ((M + 31) / 32) + c / 32] and cflags[b] (both zeroed by the caller).
size_t pair_fused_smem_bytes(int W, int64_t M);
cudaError_t pair_fused_regs(int& regs);
cudaError_t pair_forward_fused(const float* X, const float* Y, int64_t d, float* Rt, float* costs, uint32_t* cmask,
                               int* cflags, const void* lx, const void* ly, int is32, int64_t B, int64_t N, int64_t M,
                               int64_t bw, double gamma, int W, Sync sy, int64_t inject, cudaStream_t stream);

// Forward: writes the padded R (B, N+2, M+2) when Rt is null, else the tiles Rt (R unused).
template <typename T>
cudaError_t pair_forward(const T* D, T* R, T* Rt, T* costs, const void* lx, const void* ly, int is32, int64_t B,
                         int64_t N, int64_t M, int64_t bw, double gamma, int W, Sync sy, int64_t inject,
                         cudaStream_t stream);
// Backward: reads the padded R when Rt is null, else the tiles Rt written by pair_forward (R unused).
template <typename T>
cudaError_t pair_backward(const T* R, const T* Rt, T* E, const void* lx, const void* ly, int is32, int64_t B,
                          int64_t N, int64_t M, int64_t bw, double gamma, int W, Sync sy, int64_t inject,
                          cudaStream_t stream);

}  // namespace sdtw
