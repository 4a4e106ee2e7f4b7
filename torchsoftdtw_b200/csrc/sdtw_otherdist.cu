// L1 and cosine cost matrices and their gradients for the module path (reference
// src/torchsoftdtw/distances.py:21-50 and their autograd), behind the C ABI of include/sdtw_b200.h.
//
// The L1 kernels run on CUDA cores, because the L1 cost is not a contraction. The cost kernel tiles 128 x 64
// cells per CTA and 8 x 4 per thread; the gradient kernel tiles 64 x 64 outputs and 4 x 4 per thread.
// Both stage feature or sequence chunks of 16 in shared memory. The cosine cost and
// grad_X are contractions and run in fp32 on the tcgen05 kernels of sdtw_tcgen05.cu (cost: the epilogue
// forms 1 - acc / (n(x) n(y)); grad_X: B operand Y / n(Y), with the inverse norms of Y from
// row_inv_norm_kernel in the caller's workspace); fp64, unsupported shapes and grad_Y use the CUDA-core
// kernels here.
//
//   L1:      D[b,i,j] = sum_k |x_ik - y_jk|
//            dD/dx_ik = sgn(x_ik - y_jk), dD/dy_jk = -sgn(x_ik - y_jk), sgn(0) = 0 (torch's abs backward)
//   cosine:  D[b,i,j] = 1 - x_i.y_j / (n(x_i) n(y_j)),  n(v) = max(|v|, eps)
//            dD/dx_i  = -(y_j / n(y_j) - c(x_i) S_ij x_i / n(x_i)) / n(x_i),  S = 1 - D,
//            c(v) = [|v| >= eps] (the clamp passes no gradient below eps, like torch's clamp_min)
// The gradient kernels compute sum_b g[b] * sum_ij E[b,i,j] dD[b,i,j] without forming g * E.
#include "sdtw_b200.h"
#include "sdtw_common.cuh"
#include "sdtw_tcgen05.h"

namespace sdtw {

namespace {

constexpr int kDT = 64;  // tile rows = tile columns
constexpr int kDK = 16;  // chunk of the reduced dimension

template <typename T>
__device__ __forceinline__ T rsqrt_floor(T sumsq, T eps)  // 1 / max(sqrt(sumsq), eps)
{
    const T n = sqrt(sumsq);
    return T(1) / (n > eps ? n : eps);
}

// out[r] = 1 / max(|A_r|, eps) for `rows` rows of d features: one warp per row.
__global__ void __launch_bounds__(256) row_inv_norm_kernel(const float* __restrict__ A, int64_t rows, int64_t d,
                                                           float eps, float* __restrict__ out)
{
    const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const float* a = A + r * d;
    float ss = 0.f;
    for (int64_t k = lane; k < d; k += 32) ss = fmaf(a[k], a[k], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) out[r] = rsqrt_floor(ss, eps);
}

// n consecutive values from 16-byte aligned shared memory, in 16-byte loads.
template <int n>
__device__ __forceinline__ void lds_vec(const float* p, float* v)
{
#pragma unroll
    for (int u = 0; u < n; u += 4) {
        const float4 f = *reinterpret_cast<const float4*>(p + u);
        v[u] = f.x;
        v[u + 1] = f.y;
        v[u + 2] = f.z;
        v[u + 3] = f.w;
    }
}
template <int n>
__device__ __forceinline__ void lds_vec(const double* p, double* v)
{
#pragma unroll
    for (int u = 0; u < n; u += 2) {
        const double2 f = *reinterpret_cast<const double2*>(p + u);
        v[u] = f.x;
        v[u + 1] = f.y;
    }
}

// L1 cost matrix: 128 x 64 cells per CTA, 256 threads, 8 rows x 4 columns per thread; features in chunks
// of 16 staged transposed in shared memory (row strides 132 / 68: 16-byte aligned rows, at most 2-way
// bank conflicts on the transposing stores). Per feature a thread reads its 8 + 4 operands in 16-byte
// loads and does 32 x (subtract, add |.|): the FP32 pipe bounds it (2 instructions per cell-feature).
constexpr int kL1R = 128, kL1C = 64, kL1XS = kL1R + 4, kL1YS = kL1C + 4;

template <typename T>
__global__ void __launch_bounds__(256) pairwise_l1_kernel(const T* __restrict__ X, const T* __restrict__ Y,
                                                          T* __restrict__ D, int64_t N, int64_t M, int64_t d)
{
    __shared__ __align__(16) T Xs[kDK][kL1XS];
    __shared__ __align__(16) T Ys[kDK][kL1YS];
    const int64_t b = blockIdx.z;
    const int64_t i0 = static_cast<int64_t>(blockIdx.y) * kL1R, j0 = static_cast<int64_t>(blockIdx.x) * kL1C;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const T* Xb = X + b * N * d;
    const T* Yb = Y + b * M * d;
    T acc[8][4];
#pragma unroll
    for (int p = 0; p < 8; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[p][q] = T(0);
    for (int64_t k0 = 0; k0 < d; k0 += kDK) {
        // 16 consecutive threads read 16 consecutive features of one row
        for (int e = threadIdx.x; e < kL1R * kDK; e += 256) {
            const int kk = e & (kDK - 1), r = e >> 4;
            const int64_t gk = k0 + kk, gi = i0 + r;
            Xs[kk][r] = (gi < N && gk < d) ? Xb[gi * d + gk] : T(0);
        }
        for (int e = threadIdx.x; e < kL1C * kDK; e += 256) {
            const int kk = e & (kDK - 1), r = e >> 4;
            const int64_t gk = k0 + kk, gj = j0 + r;
            Ys[kk][r] = (gj < M && gk < d) ? Yb[gj * d + gk] : T(0);
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kDK; ++kk) {
            T xa[8], yb[4];
            lds_vec<8>(&Xs[kk][8 * ty], xa);
            lds_vec<4>(&Ys[kk][4 * tx], yb);
#pragma unroll
            for (int p = 0; p < 8; ++p)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[p][q] += fabs(xa[p] - yb[q]);
        }
        __syncthreads();
    }
    T* Db = D + b * N * M;
    const int64_t j = j0 + 4 * tx;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const int64_t i = i0 + 8 * ty + p;
        if (i >= N) continue;
        if constexpr (sizeof(T) == 4) {
            if (M % 4 == 0 && j + 3 < M) {  // 16-byte aligned: D's base is, and so is every row
                *reinterpret_cast<float4*>(Db + i * M + j) = make_float4(acc[p][0], acc[p][1], acc[p][2], acc[p][3]);
                continue;
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (j + q < M) Db[i * M + j + q] = acc[p][q];
    }
}

template <typename T, int KIND>
__global__ void __launch_bounds__(256) pairwise_dist_kernel(const T* __restrict__ X, const T* __restrict__ Y,
                                                            T* __restrict__ D, int64_t N, int64_t M, int64_t d,
                                                            T eps)
{
    __shared__ T Xs[kDK][kDT + 1];
    __shared__ T Ys[kDK][kDT + 1];
    const int64_t b = blockIdx.z;
    const int64_t i0 = static_cast<int64_t>(blockIdx.y) * kDT, j0 = static_cast<int64_t>(blockIdx.x) * kDT;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const T* Xb = X + b * N * d;
    const T* Yb = Y + b * M * d;
    T acc[4][4], xn[4], yn[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        xn[p] = yn[p] = T(0);
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[p][q] = T(0);
    }
    for (int64_t k0 = 0; k0 < d; k0 += kDK) {
        for (int e = threadIdx.x; e < kDT * kDK; e += 256) {
            const int r = e / kDK, kk = e % kDK;
            const int64_t gk = k0 + kk, gi = i0 + r, gj = j0 + r;
            Xs[kk][r] = (gi < N && gk < d) ? Xb[gi * d + gk] : T(0);
            Ys[kk][r] = (gj < M && gk < d) ? Yb[gj * d + gk] : T(0);
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kDK; ++kk) {
            T xa[4], ya[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                xa[p] = Xs[kk][ty + 16 * p];
                ya[p] = Ys[kk][tx + 16 * p];
            }
            if (KIND == SDTW_DIST_L1) {
#pragma unroll
                for (int p = 0; p < 4; ++p)
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[p][q] += fabs(xa[p] - ya[q]);
            } else {
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    xn[p] = fma(xa[p], xa[p], xn[p]);
                    yn[p] = fma(ya[p], ya[p], yn[p]);
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[p][q] = fma(xa[p], ya[q], acc[p][q]);
                }
            }
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
            Db[i * M + j] = KIND == SDTW_DIST_L1
                                ? acc[p][q]
                                : T(1) - acc[p][q] * (rsqrt_floor(xn[p], eps) * rsqrt_floor(yn[q], eps));
        }
    }
}

// out[b, r, c] for the rows r of A (X for grad_X, Y for grad_Y) and features c; the reduced index s runs
// over the rows of Bm (the other sequence). E and D are (B, N, M): indexed (r, s) when TRANS is false and
// (s, r) when it is true.
template <typename T, int KIND, bool TRANS>
__global__ void __launch_bounds__(256) grad_dist_kernel(const T* __restrict__ A, const T* __restrict__ Bm,
                                                        const T* __restrict__ Dm, const T* __restrict__ E,
                                                        const T* __restrict__ g, T* __restrict__ out, int64_t R_,
                                                        int64_t S_, int64_t d, int64_t N, int64_t M, T eps)
{
    __shared__ T Gs[kDK][kDT + 1];  // [s][r]: g * E
    __shared__ T Ss[kDK][kDT + 1];  // [s][r]: cosine similarity 1 - D
    __shared__ T Bs[kDK][kDT + 1];  // [s][c]
    __shared__ T inv_nb[kDK];       // 1 / n(Bm_s)
    __shared__ T inv_na[kDT];       // 1 / n(A_r)
    __shared__ T live_a[kDT];       // [|A_r| >= eps]
    const int64_t b = blockIdx.z;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kDT, c0 = static_cast<int64_t>(blockIdx.x) * kDT;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const T gb = g[b];
    const T* Ab = A + b * R_ * d;
    const T* Bb = Bm + b * S_ * d;
    const T* Db = Dm + b * N * M;
    const T* Eb = E + b * N * M;

    T av[4][4];  // A at this thread's outputs
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t r = r0 + ty + 16 * p, c = c0 + tx + 16 * q;
            av[p][q] = (r < R_ && c < d) ? Ab[r * d + c] : T(0);
        }
    if (KIND == SDTW_DIST_COSINE) {
        if (threadIdx.x < kDT) {
            const int64_t r = r0 + threadIdx.x;
            T ss = T(0);
            if (r < R_)
                for (int64_t k = 0; k < d; ++k) ss = fma(Ab[r * d + k], Ab[r * d + k], ss);
            inv_na[threadIdx.x] = rsqrt_floor(ss, eps);
            live_a[threadIdx.x] = sqrt(ss) >= eps ? T(1) : T(0);
        }
    }
    T acc[4][4], rs[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        rs[p] = T(0);
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[p][q] = T(0);
    }
    for (int64_t s0 = 0; s0 < S_; s0 += kDK) {
        for (int e = threadIdx.x; e < kDT * kDK; e += 256) {
            int r, ss;
            if (TRANS) {  // E/D rows are s: read along r contiguously
                r = e % kDT;
                ss = e / kDT;
            } else {      // E/D rows are r: read along s contiguously
                r = e / kDK;
                ss = e % kDK;
            }
            const int64_t gr = r0 + r, gs = s0 + ss;
            T gv = T(0), sv = T(0);
            if (gr < R_ && gs < S_) {
                const int64_t off = TRANS ? gs * M + gr : gr * M + gs;
                gv = gb * Eb[off];
                if (KIND == SDTW_DIST_COSINE) sv = T(1) - Db[off];
            }
            Gs[ss][r] = gv;
            if (KIND == SDTW_DIST_COSINE) Ss[ss][r] = sv;
        }
        for (int e = threadIdx.x; e < kDT * kDK; e += 256) {
            const int c = e % kDT, ss = e / kDT;
            const int64_t gs = s0 + ss, gc = c0 + c;
            Bs[ss][c] = (gs < S_ && gc < d) ? Bb[gs * d + gc] : T(0);
        }
        if (KIND == SDTW_DIST_COSINE) {
            // 16 rows of Bm, 16 threads per row (consecutive lanes), full norms over all d features.
            const int row = threadIdx.x >> 4, part = threadIdx.x & 15;
            const int64_t gs = s0 + row;
            T ss = T(0);
            if (gs < S_)
                for (int64_t k = part; k < d; k += 16) ss = fma(Bb[gs * d + k], Bb[gs * d + k], ss);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
            if (part == 0) inv_nb[row] = rsqrt_floor(ss, eps);
        }
        __syncthreads();
#pragma unroll
        for (int ss = 0; ss < kDK; ++ss) {
            T gp[4], bq[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                gp[p] = Gs[ss][ty + 16 * p];
                bq[p] = Bs[ss][tx + 16 * p];
            }
            if (KIND == SDTW_DIST_L1) {
#pragma unroll
                for (int p = 0; p < 4; ++p)
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        // gp * sgn(a - b) as two compare-to-float and two FMAs (a > b iff a - b > 0 without
                        // flush-to-zero; a tie adds nothing)
                        acc[p][q] = fma(gp[p], T(av[p][q] > bq[q]), acc[p][q]);
                        acc[p][q] = fma(-gp[p], T(av[p][q] < bq[q]), acc[p][q]);
                    }
            } else {
                const T w = inv_nb[ss];
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    rs[p] = fma(gp[p], Ss[ss][ty + 16 * p], rs[p]);
                    const T gw = gp[p] * w;
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[p][q] = fma(gw, bq[q], acc[p][q]);
                }
            }
        }
        __syncthreads();
    }
    T* ob = out + b * R_ * d;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int rl = ty + 16 * p;
        const int64_t r = r0 + rl;
        if (r >= R_) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t c = c0 + tx + 16 * q;
            if (c >= d) continue;
            T o;
            if (KIND == SDTW_DIST_L1) {
                o = acc[p][q];  // for grad_Y, av = y and bq = x: sgn(y - x) = d|x - y| / dy
            } else {
                const T ia = inv_na[rl];
                o = -(acc[p][q] - live_a[rl] * rs[p] * av[p][q] * ia) * ia;
            }
            ob[r * d + c] = o;
        }
    }
}

bool dist_sizes_ok(int64_t B, int64_t N, int64_t M, int64_t d)
{
    // grid.y = ceil(N / 64) (or M) is limited to 65535; batches run in chunks of kBatchChunk pairs
    return B >= 0 && N >= 0 && M >= 0 && d >= 0 && B < (int64_t(1) << 31) && N <= 65535 * kDT &&
           M <= 65535 * kDT && d < (int64_t(1) << 30);
}

template <typename T>
sdtw_status launch_pairwise_dist(int kind, const void* X, const void* Y, int64_t B, int64_t N, int64_t M, int64_t d,
                                 double eps, void* D, cudaStream_t s)
{
    if constexpr (sizeof(T) == 4) {
        if (kind == SDTW_DIST_COSINE && distance_path() == 0 && d > 0 && pairwise_tc_supported(X, Y, D, B, N, M, d)) {
            const cudaError_t e =
                pairwise_tc_launch(static_cast<const float*>(X), static_cast<const float*>(Y), static_cast<float*>(D),
                                   nullptr, B, N, M, d, wait_timeout_s(), s, true, static_cast<float>(eps));
            return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
        }
    }
    const dim3 grid(static_cast<unsigned>((M + kDT - 1) / kDT), static_cast<unsigned>((N + kDT - 1) / kDT),
                    static_cast<unsigned>(B));
    count_launch();
    if (kind == SDTW_DIST_L1)
        pairwise_l1_kernel<T><<<dim3(static_cast<unsigned>((M + kL1C - 1) / kL1C),
                                     static_cast<unsigned>((N + kL1R - 1) / kL1R), static_cast<unsigned>(B)),
                                256, 0, s>>>(static_cast<const T*>(X), static_cast<const T*>(Y), static_cast<T*>(D), N,
                                             M, d);
    else
        pairwise_dist_kernel<T, SDTW_DIST_COSINE><<<grid, 256, 0, s>>>(
            static_cast<const T*>(X), static_cast<const T*>(Y), static_cast<T*>(D), N, M, d, static_cast<T>(eps));
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
}

template <typename T, int KIND>
void launch_grad_dist_kind(const T* X, const T* Y, const T* D, const T* E, const T* g, int64_t B, int64_t N, int64_t M,
                           int64_t d, T eps, T* gX, T* gY, cudaStream_t s)
{
    const unsigned cblocks = static_cast<unsigned>((d + kDT - 1) / kDT);
    if (gX && N > 0) {
        const dim3 grid(cblocks, static_cast<unsigned>((N + kDT - 1) / kDT), static_cast<unsigned>(B));
        count_launch();
        grad_dist_kernel<T, KIND, false><<<grid, 256, 0, s>>>(X, Y, D, E, g, gX, N, M, d, N, M, eps);
    }
    if (gY && M > 0) {
        const dim3 grid(cblocks, static_cast<unsigned>((M + kDT - 1) / kDT), static_cast<unsigned>(B));
        count_launch();
        grad_dist_kernel<T, KIND, true><<<grid, 256, 0, s>>>(Y, X, D, E, g, gY, M, N, d, N, M, eps);
    }
}

template <typename T>
sdtw_status launch_grad_dist(int kind, const void* X, const void* Y, const void* D, const void* E, const void* g,
                             int64_t B, int64_t N, int64_t M, int64_t d, double eps, void* ws, void* gX, void* gY,
                             cudaStream_t s)
{
    if constexpr (sizeof(T) == 4) {
        if (kind == SDTW_DIST_COSINE && ws && gX && distance_path() == 0 && (reinterpret_cast<uintptr_t>(ws) & 15) == 0 &&
            grad_tc_supported(X, Y, D, E, gX, B, N, M, d)) {
            float* ry = static_cast<float*>(ws);
            count_launch();
            row_inv_norm_kernel<<<static_cast<unsigned>((B * M + 7) / 8), 256, 0, s>>>(
                static_cast<const float*>(Y), B * M, d, static_cast<float>(eps), ry);
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return static_cast<sdtw_status>(e);
            e = grad_x_tc_launch(static_cast<const float*>(X), static_cast<const float*>(Y),
                                 static_cast<const float*>(D), static_cast<const float*>(E),
                                 static_cast<const float*>(g), nullptr, static_cast<float*>(gX), B, N, M, d,
                                 wait_timeout_s(), s, ry, static_cast<float>(eps));
            if (e != cudaSuccess) return static_cast<sdtw_status>(e);
            gX = nullptr;  // done; grad_Y (if asked) below
            if (!gY) return SDTW_OK;
        }
    }
    if (kind == SDTW_DIST_L1)
        launch_grad_dist_kind<T, SDTW_DIST_L1>(static_cast<const T*>(X), static_cast<const T*>(Y),
                                               static_cast<const T*>(D), static_cast<const T*>(E),
                                               static_cast<const T*>(g), B, N, M, d, static_cast<T>(eps),
                                               static_cast<T*>(gX), static_cast<T*>(gY), s);
    else
        launch_grad_dist_kind<T, SDTW_DIST_COSINE>(static_cast<const T*>(X), static_cast<const T*>(Y),
                                                   static_cast<const T*>(D), static_cast<const T*>(E),
                                                   static_cast<const T*>(g), B, N, M, d, static_cast<T>(eps),
                                                   static_cast<T*>(gX), static_cast<T*>(gY), s);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
}

}  // namespace
}  // namespace sdtw

using namespace sdtw;

extern "C" {

sdtw_status sdtw_pairwise_dist(sdtw_dtype dtype, int kind, const void* X, const void* Y, int64_t B, int64_t N,
                               int64_t M, int64_t d, double eps, void* D, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if ((kind != SDTW_DIST_L1 && kind != SDTW_DIST_COSINE) || !dist_sizes_ok(B, N, M, d) || !(eps > 0))
        return SDTW_EINVAL;
    if (B == 0 || N == 0 || M == 0) return SDTW_OK;
    if (!D || (d > 0 && (!X || !Y))) return SDTW_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t es = dtype == SDTW_F32 ? 4 : 8;
    for (int64_t b0 = 0; b0 < B; b0 += kBatchChunk) {
        const int64_t nb = B - b0 < kBatchChunk ? B - b0 : kBatchChunk;
        const void* Xc = at_elem(X, b0 * N * d, es);
        const void* Yc = at_elem(Y, b0 * M * d, es);
        void* Dc = at_elem(D, b0 * N * M, es);
        const sdtw_status st = dtype == SDTW_F32 ? launch_pairwise_dist<float>(kind, Xc, Yc, nb, N, M, d, eps, Dc, s)
                                                 : launch_pairwise_dist<double>(kind, Xc, Yc, nb, N, M, d, eps, Dc, s);
        if (st != SDTW_OK) return st;
    }
    return SDTW_OK;
}

size_t sdtw_grad_dist_workspace_bytes(int64_t B, int64_t M, sdtw_dtype dtype)
{
    if (B < 0 || M < 0) return 0;
    return static_cast<size_t>(B * M) * (dtype == SDTW_F64 ? 8 : 4) + 16;
}

sdtw_status sdtw_grad_dist(sdtw_dtype dtype, int kind, const void* X, const void* Y, const void* D, const void* E,
                           const void* g, int64_t B, int64_t N, int64_t M, int64_t d, double eps, void* workspace,
                           void* grad_X, void* grad_Y, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if ((kind != SDTW_DIST_L1 && kind != SDTW_DIST_COSINE) || !dist_sizes_ok(B, N, M, d) || !(eps > 0))
        return SDTW_EINVAL;
    if (B == 0 || d == 0 || (!grad_X && !grad_Y)) return SDTW_OK;
    if (!X || !Y || !g || (N * M > 0 && (!E || (kind == SDTW_DIST_COSINE && !D)))) return SDTW_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t es = dtype == SDTW_F32 ? 4 : 8;
    // Chunks run in stream order, so each may reuse the start of the workspace.
    for (int64_t b0 = 0; b0 < B; b0 += kBatchChunk) {
        const int64_t nb = B - b0 < kBatchChunk ? B - b0 : kBatchChunk;
        const void* Xc = at_elem(X, b0 * N * d, es);
        const void* Yc = at_elem(Y, b0 * M * d, es);
        const void* Dc = at_elem(D, b0 * N * M, es);
        const void* Ec = at_elem(E, b0 * N * M, es);
        const void* gc = at_elem(g, b0, es);
        void* gXc = at_elem(grad_X, b0 * N * d, es);
        void* gYc = at_elem(grad_Y, b0 * M * d, es);
        const sdtw_status st =
            dtype == SDTW_F32
                ? launch_grad_dist<float>(kind, Xc, Yc, Dc, Ec, gc, nb, N, M, d, eps, workspace, gXc, gYc, s)
                : launch_grad_dist<double>(kind, Xc, Yc, Dc, Ec, gc, nb, N, M, d, eps, workspace, gXc, gYc, s);
        if (st != SDTW_OK) return st;
    }
    return SDTW_OK;
}

}  // extern "C"
