// Squared-L2 cost matrix and its gradient for narrow features (d <= 16), CUDA cores, fp32 and fp64.
//
// The tiled kernels of sdtw_distance.cu reduce over features in chunks of 16 and lay a 64 x 64 tile of
// features over the threads of the gradient; with d = 4 most of that work is padding. Here the feature
// loop is a compile-time width DW (4, 8 or 16, zero-padded) held in registers:
//   * cost: a CTA covers 64 rows x 64 columns of one pair; thread t owns column j = t % 64 (its y_j and
//     |y_j|^2 in registers) and rows t / 64 + 4p, p < 16, whose x_i it reads from shared memory (one
//     address per warp: a broadcast). A warp's stores cover 32 consecutive columns of one row.
//   * gradient: a warp owns 32 output rows (lane = row r of grad_X, or of grad_Y) of one pair and walks
//     the other sequence in chunks of 32 rows staged in shared memory; per cell it reads G, adds it to
//     the row sum and accumulates G * b_s over the DW features. E is read along the lane's row (grad_X:
//     each 32-byte sector serves the lane's next 8 / 4 cells from L1) or coalesced (grad_Y). D is read
//     only in pairs whose clamp flag is set (or every pair when no flags are given).
// Arithmetic and results follow the tiled kernels: D = (|x|^2 + |y|^2) - 2 x.y with the clamp recorded as
// -0.0 and in clamp_flags; grad = 2 g (rowsum(G) a - G b) with G = E masked by the clamp.
#include "sdtw_b200.h"
#include "sdtw_narrow.h"

namespace sdtw {

namespace {

constexpr int kNT = 64;  // cost tile: rows = columns

template <typename T, int DW>
__global__ void __launch_bounds__(256) pairwise_l2_narrow_kernel(const T* __restrict__ X, const T* __restrict__ Y,
                                                                 T* __restrict__ D, int* __restrict__ clamp_flags,
                                                                 int64_t N, int64_t M, int d)
{
    __shared__ T Xs[kNT][DW + 1];
    __shared__ T xn[kNT];
    const int64_t b = blockIdx.z;
    const int64_t i0 = static_cast<int64_t>(blockIdx.y) * kNT, j0 = static_cast<int64_t>(blockIdx.x) * kNT;
    const T* Xb = X + b * N * d;
    for (int e = threadIdx.x; e < kNT * DW; e += 256) {
        const int r = e / DW, k = e % DW;
        Xs[r][k] = (i0 + r < N && k < d) ? Xb[(i0 + r) * d + k] : T(0);
    }
    __syncthreads();
    if (threadIdx.x < kNT) {
        T s = T(0);
#pragma unroll
        for (int k = 0; k < DW; ++k) s = fma(Xs[threadIdx.x][k], Xs[threadIdx.x][k], s);
        xn[threadIdx.x] = s;
    }
    const int jl = threadIdx.x & (kNT - 1);
    const int64_t j = j0 + jl;
    T y[DW];
    T yn = T(0);
    const T* yr = Y + (b * M + (j < M ? j : 0)) * d;
#pragma unroll
    for (int k = 0; k < DW; ++k) {
        y[k] = (j < M && k < d) ? yr[k] : T(0);
        yn = fma(y[k], y[k], yn);
    }
    __syncthreads();
    T* Db = D + b * N * M;
    bool clamped = false;
#pragma unroll 4
    for (int p = 0; p < kNT / 4; ++p) {
        const int il = (threadIdx.x >> 6) + 4 * p;
        const int64_t i = i0 + il;
        T acc = T(0);
#pragma unroll
        for (int k = 0; k < DW; ++k) acc = fma(Xs[il][k], y[k], acc);
        const T v = (xn[il] + yn) - T(2) * acc;
        if (i < N && j < M) {
            clamped |= v < T(0);
            Db[i * M + j] = v < T(0) ? -T(0) : v;
        }
    }
    if (clamp_flags && __any_sync(0xffffffffu, clamped) && (threadIdx.x & 31) == 0) atomicOr(clamp_flags + b, 1);
}

constexpr int kNGWarps = 4;  // gradient: warps per CTA

// out[b, r, c] = 2 g[b] (sum_s G[r,s] A[b,r,c] - sum_s G[r,s] Bm[b,s,c]); (r, s) index E/D as (i, j) when
// TRANS is false (grad_X: A = X, Bm = Y) and as (j, i) when TRANS is true (grad_Y: A = Y, Bm = X).
template <typename T, int DW, bool TRANS>
__global__ void __launch_bounds__(kNGWarps * 32) grad_l2_narrow_kernel(const T* __restrict__ A,
                                                                       const T* __restrict__ Bm,
                                                                       const T* __restrict__ Dm,
                                                                       const T* __restrict__ E,
                                                                       const T* __restrict__ g,
                                                                       const int* __restrict__ clamp_flags,
                                                                       T* __restrict__ out, int64_t B, int64_t R_,
                                                                       int64_t S_, int d, int64_t N, int64_t M)
{
    __shared__ T bs_all[kNGWarps][32][DW];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t nrb = (R_ + 31) / 32;
    const int64_t w = static_cast<int64_t>(blockIdx.x) * kNGWarps + warp;
    if (w >= B * nrb) return;  // the whole warp; no CTA-wide barrier follows
    const int64_t b = w / nrb;
    const int64_t r = (w % nrb) * 32 + lane;
    const bool live = r < R_;
    const bool masked = clamp_flags == nullptr || clamp_flags[b] != 0;
    T (*bs)[DW] = bs_all[warp];
    const T* Bb = Bm + b * S_ * d;
    const T* Eb = E + b * N * M;
    const T* Db = Dm + b * N * M;
    // E / D offset of (r, s): row-major (i, j) with i = r (grad_X) or i = s (grad_Y)
    const int64_t base = TRANS ? r : r * M;
    const int64_t step = TRANS ? M : 1;
    T acc[DW];
#pragma unroll
    for (int k = 0; k < DW; ++k) acc[k] = T(0);
    T rs = T(0);
    for (int64_t s0 = 0; s0 < S_; s0 += 32) {
        const int64_t sl = s0 + lane;
#pragma unroll
        for (int k = 0; k < DW; ++k) bs[lane][k] = (sl < S_ && k < d) ? Bb[sl * d + k] : T(0);
        __syncwarp();
        const int ns = static_cast<int>(S_ - s0 < 32 ? S_ - s0 : 32);
        int64_t off = base + s0 * step;
#pragma unroll 4
        for (int ss = 0; ss < ns; ++ss, off += step) {
            T gv = live ? __ldg(Eb + off) : T(0);
            if (masked && live && signbit(__ldg(Db + off))) gv = T(0);
            rs += gv;
#pragma unroll
            for (int k = 0; k < DW; ++k) acc[k] = fma(gv, bs[ss][k], acc[k]);
        }
        __syncwarp();
    }
    if (!live) return;
    const T g2 = T(2) * g[b];
    const T* ar = A + (b * R_ + r) * d;
    T* o = out + (b * R_ + r) * d;
#pragma unroll
    for (int k = 0; k < DW; ++k)
        if (k < d) o[k] = g2 * (rs * ar[k] - acc[k]);
}

template <typename T, int DW>
void launch_pairwise_w(const T* X, const T* Y, T* D, int* flags, int64_t B, int64_t N, int64_t M, int64_t d,
                       cudaStream_t s)
{
    const dim3 grid(static_cast<unsigned>((M + kNT - 1) / kNT), static_cast<unsigned>((N + kNT - 1) / kNT),
                    static_cast<unsigned>(B));
    pairwise_l2_narrow_kernel<T, DW><<<grid, 256, 0, s>>>(X, Y, D, flags, N, M, static_cast<int>(d));
}

template <typename T, int DW, bool TRANS>
void launch_grad_w(const T* A, const T* Bm, const T* D, const T* E, const T* g, const int* flags, T* out, int64_t B,
                   int64_t R_, int64_t S_, int64_t d, int64_t N, int64_t M, cudaStream_t s)
{
    const int64_t warps = B * ((R_ + 31) / 32);
    const int64_t grid = (warps + kNGWarps - 1) / kNGWarps;
    grad_l2_narrow_kernel<T, DW, TRANS><<<static_cast<unsigned>(grid), kNGWarps * 32, 0, s>>>(
        A, Bm, D, E, g, flags, out, B, R_, S_, static_cast<int>(d), N, M);
}

}  // namespace

bool narrow_supported(int64_t B, int64_t N, int64_t M, int64_t d)
{
    return d >= 1 && d <= 16 && B <= 65535 && (N + kNT - 1) / kNT <= 65535 && B * ((N + 31) / 32 + (M + 31) / 32) <
           (int64_t(1) << 31) / 2;
}

template <typename T>
cudaError_t narrow_pairwise_l2(const T* X, const T* Y, T* D, int* clamp_flags, int64_t B, int64_t N, int64_t M,
                               int64_t d, cudaStream_t s)
{
    count_launch();
    if (d <= 4)
        launch_pairwise_w<T, 4>(X, Y, D, clamp_flags, B, N, M, d, s);
    else if (d <= 8)
        launch_pairwise_w<T, 8>(X, Y, D, clamp_flags, B, N, M, d, s);
    else
        launch_pairwise_w<T, 16>(X, Y, D, clamp_flags, B, N, M, d, s);
    return cudaGetLastError();
}
template cudaError_t narrow_pairwise_l2<float>(const float*, const float*, float*, int*, int64_t, int64_t, int64_t,
                                               int64_t, cudaStream_t);
template cudaError_t narrow_pairwise_l2<double>(const double*, const double*, double*, int*, int64_t, int64_t, int64_t,
                                                int64_t, cudaStream_t);

template <typename T>
cudaError_t narrow_grad_l2(const T* X, const T* Y, const T* D, const T* E, const T* g, const int* clamp_flags, T* gX,
                           T* gY, int64_t B, int64_t N, int64_t M, int64_t d, cudaStream_t s)
{
    if (gX) {
        count_launch();
        if (d <= 4)
            launch_grad_w<T, 4, false>(X, Y, D, E, g, clamp_flags, gX, B, N, M, d, N, M, s);
        else if (d <= 8)
            launch_grad_w<T, 8, false>(X, Y, D, E, g, clamp_flags, gX, B, N, M, d, N, M, s);
        else
            launch_grad_w<T, 16, false>(X, Y, D, E, g, clamp_flags, gX, B, N, M, d, N, M, s);
    }
    if (gY) {
        count_launch();
        if (d <= 4)
            launch_grad_w<T, 4, true>(Y, X, D, E, g, clamp_flags, gY, B, M, N, d, N, M, s);
        else if (d <= 8)
            launch_grad_w<T, 8, true>(Y, X, D, E, g, clamp_flags, gY, B, M, N, d, N, M, s);
        else
            launch_grad_w<T, 16, true>(Y, X, D, E, g, clamp_flags, gY, B, M, N, d, N, M, s);
    }
    return cudaGetLastError();
}
template cudaError_t narrow_grad_l2<float>(const float*, const float*, const float*, const float*, const float*,
                                           const int*, float*, float*, int64_t, int64_t, int64_t, int64_t,
                                           cudaStream_t);
template cudaError_t narrow_grad_l2<double>(const double*, const double*, const double*, const double*, const double*,
                                            const int*, double*, double*, int64_t, int64_t, int64_t, int64_t,
                                            cudaStream_t);

}  // namespace sdtw
