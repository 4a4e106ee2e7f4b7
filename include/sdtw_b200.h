/*
 * torchsoftdtw_b200 — C ABI of the sm_100a Soft-DTW kernel library (libsdtw_b200.so).
 *
 * Plain pointers and sizes only: no torch types. Every pointer argument named a "device pointer" is
 * CUDA global memory on the current device; `stream` is a cudaStream_t (0 = legacy default stream).
 * Calls only enqueue work on `stream`: none synchronises, none reads device data on the host, none
 * allocates device memory. Scratch memory is passed in by the caller as `workspace` (size from the
 * matching *_workspace_bytes function), so every call can be captured in a CUDA graph.
 *
 * Layouts (row-major, contiguous):
 *   D  (B, N, M)      pairwise cost matrix                        [reference: softdtw.cpp:342-345 schemas]
 *   R  (B, N+2, M+2)  forward DP table, +inf border, R[:,0,0] = 0  [reference: softdtw.cu:485-492]
 *   E  (B, N, M)      d costs / d D                                [reference: softdtw.cu:636-641]
 *   X  (B, N, d), Y (B, M, d) sequences for the fused distance path
 *   lengths_x, lengths_y: (B,) int64, or int32 when lengths_int32 != 0
 *
 * Errors: a negative status is an invalid argument (nothing was launched); a positive status is a
 * cudaError_t from a launch. Device-side failures (a strip wait that ran out, a length outside
 * [0, N]/[0, M]) are OR-ed into the caller's sticky `err_word` (device pointer to one uint32, see
 * SDTW_ERR_*); read it with sdtw_read_error_word (which synchronises the stream). Pairs with an
 * invalid length get a NaN cost.
 */
#ifndef SDTW_B200_H
#define SDTW_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int sdtw_status;

#define SDTW_OK 0
#define SDTW_EINVAL (-1)     /* a size, pointer or parameter is invalid */
#define SDTW_EDTYPE (-2)     /* unsupported dtype code */
#define SDTW_EWORKSPACE (-3) /* workspace missing or too small */
#define SDTW_EDEVICE (-4)    /* no usable sm_100 device / kernel image */
#define SDTW_ETOOLARGE (-5)  /* sdtw_forward_noalloc: the problem needs more than its static scratch */

#define SDTW_ERR_TIMEOUT 1u    /* a wait on a neighbouring strip's progress ran out (kernel returned early) */
#define SDTW_ERR_BAD_LENGTH 2u /* some lengths value was outside [0, N] or [0, M] */
#define SDTW_ERR_BOUNDS 4u     /* debug build (libsdtw_b200_debug.so) only: a kernel's global access fell outside
                                  its buffer and was skipped */

typedef enum { SDTW_F32 = 0, SDTW_F64 = 1 } sdtw_dtype;

/* Human-readable text of a status. */
const char* sdtw_status_string(sdtw_status status);

/* Columns [*lo, *hi] of row i that lie in the Sakoe-Chiba band of an (nx, ny) pair, intersected
 * with [0, ny). Host function. Restates the per-cell predicate in_band of the reference
 * (src/torchsoftdtw/csrc/band.h:23-38) as a per-row interval. */
void sdtw_band_row_range(int64_t i, int64_t nx, int64_t ny, int64_t bandwidth, int64_t* lo, int64_t* hi);

/* Number of DP cells evaluated for one pair: in-band cells (i, j) with i < nx, j < ny. Host function. */
int64_t sdtw_pair_cells(int64_t nx, int64_t ny, int64_t bandwidth);

/* Reads (synchronising `stream`) and clears the sticky device error word. Returns the SDTW_ERR_* bits,
 * or 0xffffffff if the copy failed. */
uint32_t sdtw_read_error_word(uint32_t* err_word, void* stream);

/* Upper bound (seconds) of every device-side wait on another strip; default 2.0. Process-wide. */
void sdtw_set_wait_timeout(double seconds);

/* ---------------------------------------------------------------------------------------------------
 * Forward: costs[b] = soft-DTW of D[b] restricted to [0, nx) x [0, ny), and the DP table R.
 * Replaces the reference CUDA launcher softdtw_cuda_forward (src/torchsoftdtw/csrc/cuda/softdtw.cu:464-540),
 * reached through the op torchsoftdtw::forward (src/torchsoftdtw/csrc/softdtw.cpp:343, :361-367).
 * D, R, costs are `dtype`; R must hold (B, N+2, M+2) elements; D may be any device pointer (no
 * alignment requirement). bandwidth < 0 disables the band.
 * ------------------------------------------------------------------------------------------------- */
size_t sdtw_forward_workspace_bytes(int64_t B, int64_t N, int64_t M, sdtw_dtype dtype);
sdtw_status sdtw_forward(sdtw_dtype dtype, const void* D, int64_t B, int64_t N, int64_t M,
                         const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                         int64_t bandwidth, void* R, void* costs, void* workspace, size_t workspace_bytes,
                         uint32_t* err_word, void* stream);

/* sdtw_forward for an R that only sdtw_backward (same lengths and bandwidth) reads, as the SoftDTW module
 * saves it: the same costs, and R identical in every cell that backward reads. Where the strip-ticket
 * kernels run both directions, R is prefilled with +inf only over the 32-column chunks around each strip's
 * band that the backward loads, instead of everywhere; cells outside them are left unwritten. */
sdtw_status sdtw_forward_band_r(sdtw_dtype dtype, const void* D, int64_t B, int64_t N, int64_t M,
                                const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                                int64_t bandwidth, void* R, void* costs, void* workspace, size_t workspace_bytes,
                                uint32_t* err_word, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Forward that allocates nothing (no counterpart in the reference, which always allocates its outputs
 * and temporaries through torch).
 * For callers that cannot allocate device memory on their hot path: a host that reaches this library
 * through its C ABI alone and owns no device allocator (a service in another language, with no torch
 * in the process), or one that must not call cudaMalloc there because it can synchronise the device.
 * Same arguments, work and results as sdtw_forward, minus the workspace: the call uses a file-scope
 * static device array of SDTW_NOALLOC_SCRATCH_BYTES (16 MiB) inside this library instead. The caller
 * still provides D, R, costs, lengths and err_word (err_word must start at zero, as for sdtw_forward);
 * nothing else needs to start at zero (the call resets its scratch on the stream before use).
 *   - Limit: the scratch must hold the workspace of the kernel this shape runs on. The pair-resident and
 *     warp-per-pair kernels need 256 bytes, so every shape they take fits; the strip-ticket kernels (few
 *     long pairs) need 256 bytes plus one row of M values per 32-row strip (sdtw_forward_workspace_bytes),
 *     and shapes beyond SDTW_NOALLOC_SCRATCH_BYTES are rejected with SDTW_ETOOLARGE before anything is
 *     enqueued (e.g. B=16, N=M=4096 fp32 needs 32 MiB).
 *   - Every call looks the scratch's address up on the current device (cudaGetSymbolAddress, which
 *     allocates nothing), so a cudaDeviceReset between calls does no harm. The first call on a device can
 *     load this library's kernels there: make it before any stream capture.
 *   - The scratch is shared by every call in the process on that device: calls that can overlap in time
 *     (different streams, or different host threads without ordering) race on it and give wrong results.
 *     Serialise them, e.g. on one stream.
 * ------------------------------------------------------------------------------------------------- */
#define SDTW_NOALLOC_SCRATCH_BYTES (16u << 20)
sdtw_status sdtw_forward_noalloc(sdtw_dtype dtype, const void* D, int64_t B, int64_t N, int64_t M,
                                 const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                                 int64_t bandwidth, void* R, void* costs, uint32_t* err_word, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Backward: E = d costs / d D (unscaled; the caller multiplies by the upstream gradient).
 * Replaces softdtw_cuda_backward (src/torchsoftdtw/csrc/cuda/softdtw.cu:543-642), reached through the op
 * torchsoftdtw::backward (src/torchsoftdtw/csrc/softdtw.cpp:344, :368-373). R must be the forward's
 * output for the same D, lengths, gamma and bandwidth: the successor weights are recomputed from R
 * alone (softmin weights of each cell's three predecessors), which equals the reference's
 * exp((R[s] - R[p] - D[s]) / gamma) whenever R[s] = D[s] + softmin(predecessors of s).
 * ------------------------------------------------------------------------------------------------- */
size_t sdtw_backward_workspace_bytes(int64_t B, int64_t N, int64_t M, sdtw_dtype dtype);
sdtw_status sdtw_backward(sdtw_dtype dtype, const void* D, const void* R, int64_t B, int64_t N, int64_t M,
                          const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                          int64_t bandwidth, void* E, void* workspace, size_t workspace_bytes,
                          uint32_t* err_word, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * R as strip tiles: the layout in which the module path hands R from the forward to the backward (no
 * counterpart in the reference, whose module keeps the padded R of the op; the padded R stays the layout of
 * sdtw_forward / sdtw_backward). Tile (b, s, k), s = 0 .. ceil(N/32)-1, k = 0 .. M/32 (integer division), is
 * 32 x 32 elements, contiguous: row l, element x is R[32 s + l][32 k + x - l - 1] * log2(e) / gamma (DP
 * indices; R in units of gamma ln 2, in which the dynamic program runs with two operations fewer per cell;
 * +inf outside the band and the lengths). The costs are returned in R's own units. Each tile row is written
 * and read as one bulk copy, against the per-element copies of the padded layout. Only available when both
 * directions run on the pair-resident kernels for the
 * shape: sdtw_r_tiled(...) != 0 (a property of the shape, the dtype and the current device).
 *   sdtw_r_tiles_elems: elements of the tile array (16-byte aligned device memory, any initial content).
 *   sdtw_forward_tiles / sdtw_backward_tiles: sdtw_forward / sdtw_backward with R_tiles in place of R;
 *     SDTW_EINVAL when sdtw_r_tiled is 0. Same workspace sizes. The backward takes the forward's tiles for the
 *     same D, lengths, gamma and bandwidth.
 * ------------------------------------------------------------------------------------------------- */
int sdtw_r_tiled(int64_t B, int64_t N, int64_t M, sdtw_dtype dtype);
int64_t sdtw_r_tiles_elems(int64_t B, int64_t N, int64_t M);
sdtw_status sdtw_forward_tiles(sdtw_dtype dtype, const void* D, int64_t B, int64_t N, int64_t M,
                               const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                               int64_t bandwidth, void* R_tiles, void* costs, void* workspace,
                               size_t workspace_bytes, uint32_t* err_word, void* stream);
sdtw_status sdtw_backward_tiles(sdtw_dtype dtype, const void* R_tiles, int64_t B, int64_t N, int64_t M,
                                const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                                int64_t bandwidth, void* E, void* workspace, size_t workspace_bytes,
                                uint32_t* err_word, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Fused squared-L2 forward (module path, fp32). Replaces the chain distances.py:14-18 (pairwise_l2_squared,
 * which stores D) -> sdtw_forward_tiles: the forward computes each 32 x 32 tile of
 * D = (|x|^2 + |y|^2) - 2 X Y^T, clamped at 0, from X (B, N, d) and Y (B, M, d) inside the wavefront, and D
 * never reaches memory. Outputs: costs, R as strip tiles (for sdtw_backward_tiles), and the clamp record the
 * gradient needs in place of D's sign: clamp_mask (sdtw_clamp_mask_words(B, N, M) uint32 words, bit c % 32
 * of word (b N + i) ceil(M / 32) + c / 32 set where cell (i, c) was clamped) and clamp_flags (B int32, nonzero
 * for pairs with a clamped cell). Both are overwritten (zeroed by the call first).
 *   sdtw_forward_l2_fused_ok: 1 when the fused forward runs this shape (the pair-resident kernels with
 *     tiles, d a positive multiple of 16); otherwise sdtw_forward_l2_tiles returns SDTW_EINVAL.
 *   X, Y and R_tiles 16-byte aligned; workspace as sdtw_forward_workspace_bytes(B, N, M, SDTW_F32).
 *   sdtw_apply_clamp_mask: E[b, i, c] = 0 at the recorded clamped cells of the flagged pairs (one launch; the
 *     other pairs cost one flag read). After it, the gradient kernels take E with all-zero clamp flags.
 * A memory-saving alternative, not the fast path: the products run on the warp-level tensor-core
 * instructions (3xTF32 mma.sync) between the wavefront's blocks, and on B200 the forward then takes
 * 0.67 ms at B=256, N=M=512, d=64 (0.42 ms at d=16), against 0.10 + 0.18 ms for sdtw_pairwise_l2 followed
 * by sdtw_forward_tiles. The module path uses it only with TORCHSOFTDTW_B200_FUSED_COST=1.
 * ------------------------------------------------------------------------------------------------- */
int sdtw_forward_l2_fused_ok(int64_t B, int64_t N, int64_t M, int64_t d);
int64_t sdtw_clamp_mask_words(int64_t B, int64_t N, int64_t M);
sdtw_status sdtw_forward_l2_tiles(const float* X, const float* Y, int64_t B, int64_t N, int64_t M, int64_t d,
                                  const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                                  int64_t bandwidth, void* R_tiles, float* costs, uint32_t* clamp_mask,
                                  int* clamp_flags, void* workspace, size_t workspace_bytes, uint32_t* err_word,
                                  void* stream);
sdtw_status sdtw_apply_clamp_mask(float* E, const uint32_t* clamp_mask, const int* clamp_flags, int64_t B, int64_t N,
                                  int64_t M, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Compensated fp32 forward / backward (no counterpart in the reference): the better-conditioned fp32 path.
 * The reference's fp32 backward takes its softmin weights from exp((R[s] - R[p] - D[s]) / gamma)
 * (src/torchsoftdtw/csrc/softdtw.cpp:248-256); an fp32 R carries an absolute error of about ulp(R), which a
 * small gamma turns into O(1) weight errors. These entry points keep R as an unevaluated sum of two floats
 * R_hi + R_lo (each cell accumulated exactly by TwoSum), so the weights come from R differences accurate to
 * far below ulp(R). Inputs and outputs are fp32; R_hi and R_lo have the padded layout of R (B, N+2, M+2).
 * costs = R_hi + R_lo of the terminal cell. Same lengths, band, error word and NaN conventions as
 * sdtw_forward / sdtw_backward; no workspace (one warp per pair, strips in sequence: slower than the default
 * kernels, for callers who need accurate fp32 gradients). M is limited by shared memory (about 6400).
 * ------------------------------------------------------------------------------------------------- */
sdtw_status sdtw_forward_x2(const float* D, int64_t B, int64_t N, int64_t M, const void* lengths_x,
                            const void* lengths_y, int lengths_int32, double gamma, int64_t bandwidth, float* R_hi,
                            float* R_lo, float* costs, uint32_t* err_word, void* stream);
sdtw_status sdtw_backward_x2(const float* R_hi, const float* R_lo, int64_t B, int64_t N, int64_t M,
                             const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                             int64_t bandwidth, float* E, uint32_t* err_word, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Pairwise squared Euclidean cost: D[b,i,j] = (|x_i|^2 + |y_j|^2) - 2 x_i.y_j, clamped at 0.
 * Replaces the reference's pairwise_l2_squared (src/torchsoftdtw/distances.py:4-18) on the module path.
 * Cells where the unclamped value is negative are stored as -0.0 (sign bit set), so that the
 * gradient kernel can reproduce the clamp's zero gradient there; -0.0 compares and adds as 0.
 * clamp_flags (optional, (B,) int32 device array): set non-zero for every pair that has such a cell.
 * fp32 with d % 4 == 0 and 16-byte aligned X, Y runs on the tensor cores (3xTF32, fp32 accuracy).
 * ------------------------------------------------------------------------------------------------- */
sdtw_status sdtw_pairwise_l2(sdtw_dtype dtype, const void* X, const void* Y, int64_t B, int64_t N, int64_t M,
                             int64_t d, void* D, int* clamp_flags, void* stream);

/* The same cost for a dynamic program that reads only part of D: the cells below the pair's lengths and
 * inside the Sakoe-Chiba band (bandwidth < 0: no band). On the tensor-core path only the 128 x 128 tiles of
 * D that hold such a cell are computed (a one-CTA kernel lists them first); the other cells of D are left
 * unwritten, and clamp_flags cover the computed tiles. Elsewhere all of D is computed. For D that feeds
 * this library's wavefronts with the same lengths and bandwidth (which read nothing else), as on the
 * SoftDTW module path with a band; the operator contract (R and E in full) is unchanged by it.
 * workspace: sdtw_pairwise_l2_band_workspace_bytes(B, N, M) bytes, 16-byte aligned. */
size_t sdtw_pairwise_l2_band_workspace_bytes(int64_t B, int64_t N, int64_t M);
sdtw_status sdtw_pairwise_l2_band(sdtw_dtype dtype, const void* X, const void* Y, int64_t B, int64_t N, int64_t M,
                                  int64_t d, const void* lengths_x, const void* lengths_y, int lengths_are_int32,
                                  int64_t bandwidth, void* D, int* clamp_flags, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * Gradient of sum_b g[b] * costs[b] through the squared-L2 cost (the autograd of distances.py:14-18):
 *   G = g[b] * E * [D >= 0 before the clamp]  (read from the sign bit written by sdtw_pairwise_l2)
 *   grad_X = 2 * (rowsum(G) * X - G @ Y),   grad_Y = 2 * (colsum(G) * Y - G^T @ X)
 * g is (B,) `dtype` on the device; grad_X / grad_Y may be NULL to skip them. clamp_flags (optional)
 * is sdtw_pairwise_l2's output: pairs whose flag is 0 skip reading D.
 * ------------------------------------------------------------------------------------------------- */
sdtw_status sdtw_grad_l2(sdtw_dtype dtype, const void* X, const void* Y, const void* D, const void* E,
                         const void* g, const int* clamp_flags, int64_t B, int64_t N, int64_t M, int64_t d,
                         void* grad_X, void* grad_Y, void* stream);

/* The same gradient for E that is zero outside the cells below the pair's lengths and inside the band (as
 * sdtw_backward leaves it): on the tensor-core path each 128-row tile contracts only the 32-wide chunks of
 * E that hold such a cell (zero chunks add nothing), and reads D only there, so D may come from
 * sdtw_pairwise_l2_band. Elsewhere it is sdtw_grad_l2. */
sdtw_status sdtw_grad_l2_band(sdtw_dtype dtype, const void* X, const void* Y, const void* D, const void* E,
                              const void* g, const int* clamp_flags, int64_t B, int64_t N, int64_t M, int64_t d,
                              const void* lengths_x, const void* lengths_y, int lengths_are_int32, int64_t bandwidth,
                              void* grad_X, void* grad_Y, void* stream);

/* ---------------------------------------------------------------------------------------------------
 * L1 and cosine cost matrices (the module's distance="l1" / "cosine" path) and their gradients.
 * Replace the reference's pairwise_l1 and pairwise_cosine (src/torchsoftdtw/distances.py:21-50) and their
 * autograd; the reference's L1 expression materialises a (B, N, M, d) difference tensor, these do not.
 *   kind SDTW_DIST_L1:      D[b,i,j] = sum_k |x_ik - y_jk|                     (eps unused, must be > 0)
 *   kind SDTW_DIST_COSINE:  D[b,i,j] = 1 - x_i.y_j / (max(|x_i|, eps) max(|y_j|, eps))
 * sdtw_grad_dist returns the gradient of sum_b g[b] * sum_ij E[b,i,j] D[b,i,j] (E from sdtw_backward,
 * g the (B,) upstream gradient of the costs): sgn(0) = 0 for L1, and no gradient through the eps floor of
 * a norm for cosine (torch's abs and clamp_min). D (the cost matrix) is read by the cosine gradient only.
 * grad_X / grad_Y may be NULL to skip them. fp32 or fp64. L1: CUDA-core kernels. Cosine in fp32 with
 * d % 4 == 0, M % 4 == 0 (and d <= 128 for grad_X) and 16-byte aligned arrays: the cost matrix and grad_X
 * run on the tcgen05 tensor cores (3xTF32), grad_X only when a workspace of
 * sdtw_grad_dist_workspace_bytes(B, M, dtype) bytes (device memory, any content, 16-byte aligned) is
 * given; with workspace NULL, or otherwise, CUDA-core kernels.
 * ------------------------------------------------------------------------------------------------- */
#define SDTW_DIST_L1 1
#define SDTW_DIST_COSINE 2
sdtw_status sdtw_pairwise_dist(sdtw_dtype dtype, int kind, const void* X, const void* Y, int64_t B, int64_t N,
                               int64_t M, int64_t d, double eps, void* D, void* stream);
size_t sdtw_grad_dist_workspace_bytes(int64_t B, int64_t M, sdtw_dtype dtype);
sdtw_status sdtw_grad_dist(sdtw_dtype dtype, int kind, const void* X, const void* Y, const void* D, const void* E,
                           const void* g, int64_t B, int64_t N, int64_t M, int64_t d, double eps, void* workspace,
                           void* grad_X, void* grad_Y, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SDTW_B200_H */
