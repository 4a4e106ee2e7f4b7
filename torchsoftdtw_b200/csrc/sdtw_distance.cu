// Squared-Euclidean cost matrix and its gradient for the module path (reference
// src/torchsoftdtw/distances.py:4-18 and its autograd), behind the C ABI of include/sdtw_b200.h.
//
// Both kernels are CUDA-core (FFMA) tiled contractions: 64x64 output tiles per 256-thread CTA,
// 4x4 outputs per thread, operands staged through shared memory in K-slices of 16.
#include <algorithm>

#include "sdtw_common.cuh"
#include "sdtw_b200.h"

namespace sdtw {

constexpr int kTile = 64;
constexpr int kKs = 16;

// D[b,i,j] = (|x_i|^2 + |y_j|^2) - 2 x_i.y_j; negative values (rounding, x_i ~ y_j) are stored as -0.0.
template <typename T>
__global__ void __launch_bounds__(256) pairwise_l2_kernel(const T* __restrict__ X, const T* __restrict__ Y,
                                                          T* __restrict__ D, int64_t N, int64_t M, int64_t d)
{
    __shared__ T Xs[kKs][kTile + 1];
    __shared__ T Ys[kKs][kTile + 1];
    const int64_t b = blockIdx.z;
    const int64_t i0 = static_cast<int64_t>(blockIdx.y) * kTile;
    const int64_t j0 = static_cast<int64_t>(blockIdx.x) * kTile;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const T* Xb = X + b * N * d;
    const T* Yb = Y + b * M * d;
    T acc[4][4];
    T xn[4], yn[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        xn[p] = yn[p] = T(0);
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[p][q] = T(0);
    }
    for (int64_t k0 = 0; k0 < d; k0 += kKs) {
        for (int e = threadIdx.x; e < kTile * kKs; e += 256) {
            const int r = e / kKs, kk = e % kKs;
            const int64_t gk = k0 + kk;
            const int64_t gi = i0 + r, gj = j0 + r;
            Xs[kk][r] = (gi < N && gk < d) ? Xb[gi * d + gk] : T(0);
            Ys[kk][r] = (gj < M && gk < d) ? Yb[gj * d + gk] : T(0);
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kKs; ++kk) {
            T xa[4], ya[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                xa[p] = Xs[kk][ty + 16 * p];
                ya[p] = Ys[kk][tx + 16 * p];
                xn[p] = fma(xa[p], xa[p], xn[p]);
                yn[p] = fma(ya[p], ya[p], yn[p]);
            }
#pragma unroll
            for (int p = 0; p < 4; ++p)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[p][q] = fma(xa[p], ya[q], acc[p][q]);
        }
        __syncthreads();
    }
    T* Db = D + b * N * M;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int64_t i = i0 + ty + 16 * p;
        if (i >= N) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t j = j0 + tx + 16 * q;
            if (j >= M) continue;
            const T v = (xn[p] + yn[q]) - T(2) * acc[p][q];
            Db[i * M + j] = v < T(0) ? -T(0) : v;
        }
    }
}

// out[b, r, c] = 2 * (sum_s G[r,s]) * A[b, r, c] - 2 * sum_s G[r,s] * Bm[b, s, c], where
// G[r,s] = g[b] * E[r,s] * [D[r,s] not negative-zero] and (r, s) index E/D as (i, j) when TRANS is
// false (grad_X: A = X, Bm = Y) or as (j, i) when TRANS is true (grad_Y: A = Y, Bm = X).
template <typename T, bool TRANS>
__global__ void __launch_bounds__(256) grad_l2_kernel(const T* __restrict__ A, const T* __restrict__ Bm,
                                                      const T* __restrict__ Dm, const T* __restrict__ E,
                                                      const T* __restrict__ g, T* __restrict__ out, int64_t R_,
                                                      int64_t S_, int64_t d, int64_t N, int64_t M)
{
    __shared__ T Gs[kKs][kTile + 1];  // [s][r]
    __shared__ T Bs[kKs][kTile + 1];  // [s][c]
    const int64_t b = blockIdx.z;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kTile;
    const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kTile;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const T gb = g[b];
    const T* Ab = A + b * R_ * d;
    const T* Bb = Bm + b * S_ * d;
    const T* Db = Dm + b * N * M;
    const T* Eb = E + b * N * M;
    T acc[4][4];
    T rs[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        rs[p] = T(0);
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[p][q] = T(0);
    }
    for (int64_t s0 = 0; s0 < S_; s0 += kKs) {
        for (int e = threadIdx.x; e < kTile * kKs; e += 256) {
            int r, ss;
            if (TRANS) {  // E/D rows are s (= i): read along r (= j) contiguously
                r = e % kTile;
                ss = e / kTile;
            } else {      // E/D rows are r (= i): read along s (= j) contiguously
                r = e / kKs;
                ss = e % kKs;
            }
            const int64_t gr = r0 + r, gs = s0 + ss;
            T gv = T(0);
            if (gr < R_ && gs < S_) {
                const int64_t off = TRANS ? gs * M + gr : gr * M + gs;
                const T dv = Db[off];
                gv = signbit(dv) ? T(0) : gb * Eb[off];
            }
            Gs[ss][r] = gv;
        }
        for (int e = threadIdx.x; e < kTile * kKs; e += 256) {
            const int c = e % kTile, ss = e / kTile;
            const int64_t gs = s0 + ss, gc = c0 + c;
            Bs[ss][c] = (gs < S_ && gc < d) ? Bb[gs * d + gc] : T(0);
        }
        __syncthreads();
#pragma unroll
        for (int ss = 0; ss < kKs; ++ss) {
            T ga[4], ba[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                ga[p] = Gs[ss][ty + 16 * p];
                ba[p] = Bs[ss][tx + 16 * p];
                rs[p] += ga[p];
            }
#pragma unroll
            for (int p = 0; p < 4; ++p)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[p][q] = fma(ga[p], ba[q], acc[p][q]);
        }
        __syncthreads();
    }
    T* ob = out + b * R_ * d;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int64_t r = r0 + ty + 16 * p;
        if (r >= R_) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t c = c0 + tx + 16 * q;
            if (c >= d) continue;
            ob[r * d + c] = T(2) * (rs[p] * Ab[r * d + c] - acc[p][q]);
        }
    }
}

namespace {
template <typename T>
sdtw_status launch_pairwise(const void* X, const void* Y, int64_t B, int64_t N, int64_t M, int64_t d, void* D,
                            cudaStream_t s)
{
    const dim3 grid(static_cast<unsigned>((M + kTile - 1) / kTile), static_cast<unsigned>((N + kTile - 1) / kTile),
                    static_cast<unsigned>(B));
    pairwise_l2_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(X), static_cast<const T*>(Y), static_cast<T*>(D),
                                               N, M, d);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
}

template <typename T>
sdtw_status launch_grad(const void* X, const void* Y, const void* D, const void* E, const void* g, int64_t B,
                        int64_t N, int64_t M, int64_t d, void* gX, void* gY, cudaStream_t s)
{
    const unsigned cblocks = static_cast<unsigned>((d + kTile - 1) / kTile);
    if (gX) {
        const dim3 grid(cblocks, static_cast<unsigned>((N + kTile - 1) / kTile), static_cast<unsigned>(B));
        grad_l2_kernel<T, false><<<grid, 256, 0, s>>>(static_cast<const T*>(X), static_cast<const T*>(Y),
                                                      static_cast<const T*>(D), static_cast<const T*>(E),
                                                      static_cast<const T*>(g), static_cast<T*>(gX), N, M, d, N, M);
    }
    if (gY) {
        const dim3 grid(cblocks, static_cast<unsigned>((M + kTile - 1) / kTile), static_cast<unsigned>(B));
        grad_l2_kernel<T, true><<<grid, 256, 0, s>>>(static_cast<const T*>(Y), static_cast<const T*>(X),
                                                     static_cast<const T*>(D), static_cast<const T*>(E),
                                                     static_cast<const T*>(g), static_cast<T*>(gY), M, N, d, N, M);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
}

bool sizes_ok(int64_t B, int64_t N, int64_t M, int64_t d)
{
    return B >= 0 && N >= 0 && M >= 0 && d >= 0 && B < 65536 * 1024 && N < (int64_t(1) << 31) / kTile * kTile &&
           M < (int64_t(1) << 31) / kTile * kTile && B <= 65535;
}
}  // namespace
}  // namespace sdtw

using namespace sdtw;

extern "C" {

sdtw_status sdtw_pairwise_l2(sdtw_dtype dtype, const void* X, const void* Y, int64_t B, int64_t N, int64_t M,
                             int64_t d, void* D, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!sizes_ok(B, N, M, d)) return SDTW_EINVAL;
    if (B == 0 || N == 0 || M == 0) return SDTW_OK;
    if (!D || (d > 0 && (!X || !Y))) return SDTW_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dtype == SDTW_F32 ? launch_pairwise<float>(X, Y, B, N, M, d, D, s)
                             : launch_pairwise<double>(X, Y, B, N, M, d, D, s);
}

sdtw_status sdtw_grad_l2(sdtw_dtype dtype, const void* X, const void* Y, const void* D, const void* E, const void* g,
                         int64_t B, int64_t N, int64_t M, int64_t d, void* grad_X, void* grad_Y, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!sizes_ok(B, N, M, d)) return SDTW_EINVAL;
    if (B == 0 || d == 0 || (!grad_X && !grad_Y)) return SDTW_OK;
    if (!X || !Y || !g || ((N * M > 0) && (!D || !E))) return SDTW_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dtype == SDTW_F32 ? launch_grad<float>(X, Y, D, E, g, B, N, M, d, grad_X, grad_Y, s)
                             : launch_grad<double>(X, Y, D, E, g, B, N, M, d, grad_X, grad_Y, s);
}

}  // extern "C"
