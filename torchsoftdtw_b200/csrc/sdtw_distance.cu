// Squared-Euclidean cost matrix and its gradient for the module path (reference
// src/torchsoftdtw/distances.py:4-18 and its autograd), behind the C ABI of include/sdtw_b200.h.
//
// fp32 (d a multiple of 4, 16-byte aligned rows): warp-level tensor-core kernels (mma.sync m16n8k8,
//   TF32 operands). Every fp32 operand x is split into a TF32 pair x = hi + lo (hi = round-to-nearest
//   TF32 of x, lo = TF32 of the remainder) and each product is formed as hi*hi + hi*lo + lo*hi with
//   fp32 accumulation ("3xTF32"), which keeps the contraction at fp32 accuracy (the dropped lo*lo term
//   and the TF32 rounding of lo are below 2^-21 relative). Operand tiles are staged through shared
//   memory with cp.async, double-buffered.
// fp64, and fp32 shapes the tensor-core kernels do not take: CUDA-core (FFMA / DFMA) tiled kernels.
#include <algorithm>

#include "sdtw_common.cuh"
#include "sdtw_b200.h"
#include "sdtw_narrow.h"
#include "sdtw_tcgen05.h"

namespace sdtw {

constexpr int kTile = 64;
constexpr int kKs = 16;

// D[b,i,j] = (|x_i|^2 + |y_j|^2) - 2 x_i.y_j; negative values (rounding, x_i ~ y_j) are stored as -0.0.
template <typename T>
__global__ void __launch_bounds__(256) pairwise_l2_kernel(const T* __restrict__ X, const T* __restrict__ Y,
                                                          T* __restrict__ D, int* __restrict__ clamp_flags, int64_t N,
                                                          int64_t M, int64_t d)
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
    bool clamped = false;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int64_t i = i0 + ty + 16 * p;
        if (i >= N) continue;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t j = j0 + tx + 16 * q;
            if (j >= M) continue;
            const T v = (xn[p] + yn[q]) - T(2) * acc[p][q];
            clamped |= v < T(0);
            Db[i * M + j] = v < T(0) ? -T(0) : v;
        }
    }
    if (clamp_flags && __any_sync(kFull, clamped) && (threadIdx.x & 31) == 0) atomicOr(clamp_flags + b, 1);
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

// ==================================================================================================
// Tensor-core (mma.sync TF32, 3-way split) kernels, fp32
// ==================================================================================================
__device__ __forceinline__ uint32_t to_tf32(float x)
{
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo)
{
    hi = to_tf32(x);
    lo = to_tf32(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2])
{
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// c += a * b at fp32 accuracy from split operands
__device__ __forceinline__ void mma_3x(float (&c)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                       const uint32_t (&bh)[2], const uint32_t (&bl)[2])
{
    mma_tf32(c, al, bh);
    mma_tf32(c, ah, bl);
    mma_tf32(c, ah, bh);
}

// ---- cost matrix: 128 x 128 tile of D per CTA, 8 warps as 2 (rows) x 4 (cols) of 64 x 32 -------------
constexpr int kPT = 128;         // tile rows = tile cols
constexpr int kPK = 32;          // K slice
constexpr int kPKS = kPK + 4;    // smem row stride (floats): conflict-free fragment reads
constexpr size_t kPairwiseSmem = (2 * 2 * kPT * kPKS + 2 * kPT) * sizeof(float);

// rows [r0, r0+128) x columns [k0, k0+32) of a (rows x d) matrix -> dst[128][kPKS]; zero outside
__device__ __forceinline__ void load_rows_slice(float* dst, const float* src, int64_t r0, int64_t rows, int64_t k0,
                                                int64_t d, int tid)
{
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int p = tid + 256 * q;  // 1024 16-byte pieces
        const int r = p >> 3, kq = (p & 7) * 4;
        const int64_t gr = r0 + r, gk = k0 + kq;
        const int64_t left = (d - gk) * 4;
        const int bytes = (gr < rows && left > 0) ? (left >= 16 ? 16 : static_cast<int>(left)) : 0;
        const float* s = src + (bytes ? gr * d + gk : 0);
        cp_async_16(dst + r * kPKS + kq, s, bytes);
    }
}

__global__ void __launch_bounds__(256, 2) pairwise_l2_mma_kernel(const float* __restrict__ X,
                                                              const float* __restrict__ Y, float* __restrict__ D,
                                                              int* __restrict__ clamp_flags, int64_t N, int64_t M,
                                                              int64_t d)
{
    extern __shared__ __align__(16) float psm[];
    float* Xs = psm;                       // [2][128][kPKS]
    float* Ys = psm + 2 * kPT * kPKS;      // [2][128][kPKS]
    float* xn = psm + 4 * kPT * kPKS;      // [128]
    float* yn = xn + kPT;                  // [128]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int64_t b = blockIdx.z;
    const int64_t i0 = static_cast<int64_t>(blockIdx.y) * kPT, j0 = static_cast<int64_t>(blockIdx.x) * kPT;
    const float* Xb = X + b * N * d;
    const float* Yb = Y + b * M * d;
    const int wi = warp >> 2, wj = warp & 3;

    float acc[4][4][4];
#pragma unroll
    for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mi][ni][e] = 0.f;
    float norm = 0.f;  // thread tid < 128: |x_{i0+tid}|^2, else |y_{j0+tid-128}|^2

    const int nk = static_cast<int>((d + kPK - 1) / kPK);
    load_rows_slice(Xs, Xb, i0, N, 0, d, tid);
    load_rows_slice(Ys, Yb, j0, M, 0, d, tid);
    cp_async_commit();
    for (int kc = 0; kc < nk; ++kc) {
        const int buf = kc & 1;
        if (kc + 1 < nk) {
            load_rows_slice(Xs + (buf ^ 1) * kPT * kPKS, Xb, i0, N, int64_t(kc + 1) * kPK, d, tid);
            load_rows_slice(Ys + (buf ^ 1) * kPT * kPKS, Yb, j0, M, int64_t(kc + 1) * kPK, d, tid);
        }
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const float* xs = Xs + buf * kPT * kPKS;
        const float* ys = Ys + buf * kPT * kPKS;
        {
            const float* row = (tid < kPT ? xs + tid * kPKS : ys + (tid - kPT) * kPKS);
#pragma unroll 8
            for (int k = 0; k < kPK; ++k) norm = fmaf(row[k], row[k], norm);
        }
#pragma unroll
        for (int ks = 0; ks < kPK; ks += 8) {
            uint32_t bh[4][2], bl[4][2];
#pragma unroll
            for (int ni = 0; ni < 4; ++ni) {
                const float* yr = ys + (32 * wj + 8 * ni + g) * kPKS + ks + t;
                split_tf32(yr[0], bh[ni][0], bl[ni][0]);
                split_tf32(yr[4], bh[ni][1], bl[ni][1]);
            }
#pragma unroll
            for (int mi = 0; mi < 4; ++mi) {
                uint32_t ah[4], al[4];
                const float* xr = xs + (64 * wi + 16 * mi + g) * kPKS + ks + t;
                split_tf32(xr[0], ah[0], al[0]);
                split_tf32(xr[8 * kPKS], ah[1], al[1]);
                split_tf32(xr[4], ah[2], al[2]);
                split_tf32(xr[8 * kPKS + 4], ah[3], al[3]);
#pragma unroll
                for (int ni = 0; ni < 4; ++ni) mma_3x(acc[mi][ni], ah, al, bh[ni], bl[ni]);
            }
        }
        __syncthreads();
    }
    if (tid < kPT)
        xn[tid] = norm;
    else
        yn[tid - kPT] = norm;
    __syncthreads();

    float* Db = D + b * N * M;
    bool clamped = false;
    const bool pair_store = (M % 2) == 0;
#pragma unroll
    for (int mi = 0; mi < 4; ++mi) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int rl = 64 * wi + 16 * mi + g + 8 * h;
            const int64_t i = i0 + rl;
            if (i >= N) continue;
#pragma unroll
            for (int ni = 0; ni < 4; ++ni) {
                const int cl = 32 * wj + 8 * ni + 2 * t;
                const int64_t j = j0 + cl;
                float v0 = (xn[rl] + yn[cl]) - 2.f * acc[mi][ni][2 * h];
                float v1 = (xn[rl] + yn[cl + 1]) - 2.f * acc[mi][ni][2 * h + 1];
                clamped |= (v0 < 0.f && j < M) || (v1 < 0.f && j + 1 < M);
                v0 = v0 < 0.f ? -0.f : v0;
                v1 = v1 < 0.f ? -0.f : v1;
                float* dst = Db + i * M + j;
                if (pair_store && j + 1 < M) {
                    *reinterpret_cast<float2*>(dst) = make_float2(v0, v1);
                } else {
                    if (j < M) dst[0] = v0;
                    if (j + 1 < M) dst[1] = v1;
                }
            }
        }
    }
    if (clamp_flags && __any_sync(kFull, clamped) && lane == 0) atomicOr(clamp_flags + b, 1);
}

// ---- grad_X: 128 rows x 64 feature columns per CTA, 8 warps as 4 (rows) x 2 (cols) of 32 x 32 ------
constexpr int kGR = 128;        // rows (i) per CTA
constexpr int kGC = 64;         // output feature columns per CTA
constexpr int kGK = 32;         // K slice (j)
constexpr int kGES = kGK + 4;   // E tile row stride
constexpr int kGYS = kGC + 8;   // Y tile row stride
constexpr size_t kGradSmem = (2 * kGR * kGES + 2 * kGK * kGYS + kGR) * sizeof(float);

__global__ void __launch_bounds__(256, 2) grad_x_mma_kernel(const float* __restrict__ X, const float* __restrict__ Y,
                                                         const float* __restrict__ Dm, const float* __restrict__ E,
                                                         const float* __restrict__ g, const int* __restrict__ clamp_flags,
                                                         float* __restrict__ out, int64_t N, int64_t M, int64_t d)
{
    extern __shared__ __align__(16) float gsm[];
    float* Es = gsm;                          // [2][128][kGES]
    float* Ys = gsm + 2 * kGR * kGES;         // [2][32][kGYS]
    float* rs_s = Ys + 2 * kGK * kGYS;        // [128]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, t = lane & 3;
    const int64_t b = blockIdx.z;
    const int64_t i0 = static_cast<int64_t>(blockIdx.y) * kGR, c0 = static_cast<int64_t>(blockIdx.x) * kGC;
    const float* Eb = E + b * N * M;
    const float* Db = Dm + b * N * M;
    const float* Yb = Y + b * M * d;
    const bool masked = clamp_flags == nullptr || clamp_flags[b] != 0;
    const int wi = warp >> 1, wc = warp & 1;

    auto load_tiles = [&](int buf, int64_t j0) {
        float* es = Es + buf * kGR * kGES;
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // E rows i0.., columns j0..j0+31: 1024 pieces
            const int p = tid + 256 * q;
            const int r = p >> 3, jq = (p & 7) * 4;
            const int64_t gi = i0 + r, gj = j0 + jq;
            const int64_t left = (M - gj) * 4;
            const int bytes = (gi < N && left > 0) ? (left >= 16 ? 16 : static_cast<int>(left)) : 0;
            cp_async_16(es + r * kGES + jq, Eb + (bytes ? gi * M + gj : 0), bytes);
        }
        float* ys = Ys + buf * kGK * kGYS;
#pragma unroll
        for (int q = 0; q < 2; ++q) {  // Y rows j0..j0+31, columns c0..c0+63: 512 pieces
            const int p = tid + 256 * q;
            const int r = p >> 4, cq = (p & 15) * 4;
            const int64_t gj = j0 + r, gc = c0 + cq;
            const int64_t left = (d - gc) * 4;
            const int bytes = (gj < M && left > 0) ? (left >= 16 ? 16 : static_cast<int>(left)) : 0;
            cp_async_16(ys + r * kGYS + cq, Yb + (bytes ? gj * d + gc : 0), bytes);
        }
    };

    float acc[2][4][4];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mi][ni][e] = 0.f;
    float rs = 0.f;  // thread tid < 128: row sum of G for row i0 + tid

    const int nk = static_cast<int>((M + kGK - 1) / kGK);
    load_tiles(0, 0);
    cp_async_commit();
    for (int kc = 0; kc < nk; ++kc) {
        const int buf = kc & 1;
        if (kc + 1 < nk) load_tiles(buf ^ 1, int64_t(kc + 1) * kGK);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        float* es = Es + buf * kGR * kGES;
        const float* ys = Ys + buf * kGK * kGYS;
        if (masked) {  // zero E where the clamp of the cost matrix was active (sign bit of D)
            const int64_t j0 = int64_t(kc) * kGK;
            for (int e = tid; e < kGR * kGK; e += 256) {
                const int r = e >> 5, jj = e & 31;
                const int64_t gi = i0 + r, gj = j0 + jj;
                if (gi < N && gj < M && signbit(Db[gi * M + gj])) es[r * kGES + jj] = 0.f;
            }
            __syncthreads();
        }
        if (tid < kGR) {
            const float* er = es + tid * kGES;
#pragma unroll 8
            for (int k = 0; k < kGK; ++k) rs += er[k];
        }
#pragma unroll
        for (int ks = 0; ks < kGK; ks += 8) {
            uint32_t bh[4][2], bl[4][2];
#pragma unroll
            for (int ni = 0; ni < 4; ++ni) {
                const float* yc = ys + (ks + t) * kGYS + 32 * wc + 8 * ni + gq;
                split_tf32(yc[0], bh[ni][0], bl[ni][0]);
                split_tf32(yc[4 * kGYS], bh[ni][1], bl[ni][1]);
            }
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) {
                uint32_t ah[4], al[4];
                const float* er = es + (32 * wi + 16 * mi + gq) * kGES + ks + t;
                split_tf32(er[0], ah[0], al[0]);
                split_tf32(er[8 * kGES], ah[1], al[1]);
                split_tf32(er[4], ah[2], al[2]);
                split_tf32(er[8 * kGES + 4], ah[3], al[3]);
#pragma unroll
                for (int ni = 0; ni < 4; ++ni) mma_3x(acc[mi][ni], ah, al, bh[ni], bl[ni]);
            }
        }
        __syncthreads();
    }
    if (tid < kGR) rs_s[tid] = rs;
    __syncthreads();

    const float gb2 = 2.f * g[b];
    const float* Xb = X + b * N * d;
    float* ob = out + b * N * d;
#pragma unroll
    for (int mi = 0; mi < 2; ++mi) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int rl = 32 * wi + 16 * mi + gq + 8 * h;
            const int64_t i = i0 + rl;
            if (i >= N) continue;
            const float r_s = rs_s[rl];
#pragma unroll
            for (int ni = 0; ni < 4; ++ni) {
                const int64_t c = c0 + 32 * wc + 8 * ni + 2 * t;
                if (c >= d) continue;  // d is a multiple of 4 on this path, so c + 1 < d as well
                const float2 xv = *reinterpret_cast<const float2*>(Xb + i * d + c);
                float2 o;
                o.x = gb2 * (r_s * xv.x - acc[mi][ni][2 * h]);
                o.y = gb2 * (r_s * xv.y - acc[mi][ni][2 * h + 1]);
                *reinterpret_cast<float2*>(ob + i * d + c) = o;
            }
        }
    }
}

namespace {
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// 0: automatic (tcgen05, then the narrow kernels for d <= 16, then mma.sync, then the tiled CUDA-core
// kernels), 1: mma.sync kernels (no tcgen05), 2: tiled CUDA-core kernels only, 3: narrow kernels where
// d <= 16, else the tiled CUDA-core kernels.
int g_distance_path = 0;
}  // namespace

int distance_path() { return g_distance_path; }

namespace {

template <typename T>
sdtw_status launch_pairwise(const void* X, const void* Y, int64_t B, int64_t N, int64_t M, int64_t d, void* D,
                            int* clamp_flags, cudaStream_t s, const DpRegion* region = nullptr, void* ws = nullptr)
{
    if constexpr (sizeof(T) == 4) {
        if (g_distance_path == 0 && pairwise_tc_supported(X, Y, D, B, N, M, d)) {
            const cudaError_t e = pairwise_tc_launch(static_cast<const float*>(X), static_cast<const float*>(Y),
                                                     static_cast<float*>(D), clamp_flags, B, N, M, d,
                                                     wait_timeout_s(), s, false, 0.f, region, ws);
            return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
        }
    }
    if ((g_distance_path == 0 || g_distance_path == 3) && narrow_supported(B, N, M, d)) {
        const cudaError_t e = narrow_pairwise_l2<T>(static_cast<const T*>(X), static_cast<const T*>(Y),
                                                    static_cast<T*>(D), clamp_flags, B, N, M, d, s);
        return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
    }
    if constexpr (sizeof(T) == 4) {
        if (g_distance_path < 2 && d % 4 == 0 && aligned16(X) && aligned16(Y)) {
            static bool attr_set = false;
            if (!attr_set) {
                const cudaError_t e = cudaFuncSetAttribute(pairwise_l2_mma_kernel,
                                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                           static_cast<int>(kPairwiseSmem));
                if (e != cudaSuccess) return static_cast<sdtw_status>(e);
                attr_set = true;
            }
            const dim3 grid(static_cast<unsigned>((M + kPT - 1) / kPT), static_cast<unsigned>((N + kPT - 1) / kPT),
                            static_cast<unsigned>(B));
            count_launch();
            pairwise_l2_mma_kernel<<<grid, 256, kPairwiseSmem, s>>>(static_cast<const float*>(X),
                                                                   static_cast<const float*>(Y),
                                                                   static_cast<float*>(D), clamp_flags, N, M, d);
            const cudaError_t e = cudaGetLastError();
            return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
        }
    }
    const dim3 grid(static_cast<unsigned>((M + kTile - 1) / kTile), static_cast<unsigned>((N + kTile - 1) / kTile),
                    static_cast<unsigned>(B));
    count_launch();
    pairwise_l2_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(X), static_cast<const T*>(Y), static_cast<T*>(D),
                                               clamp_flags, N, M, d);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
}

template <typename T>
sdtw_status launch_grad(const void* X, const void* Y, const void* D, const void* E, const void* g,
                        const int* clamp_flags, int64_t B, int64_t N, int64_t M, int64_t d, void* gX, void* gY,
                        cudaStream_t s, const DpRegion* region = nullptr)
{
    const unsigned cblocks = static_cast<unsigned>((d + kTile - 1) / kTile);
    bool gx_done = false, gy_done = false;
    if constexpr (sizeof(T) == 4) {
        if (g_distance_path == 0 && gX && grad_tc_supported(X, Y, D, E, gX, B, N, M, d)) {
            const cudaError_t e = grad_x_tc_launch(static_cast<const float*>(X), static_cast<const float*>(Y),
                                                   static_cast<const float*>(D), static_cast<const float*>(E),
                                                   static_cast<const float*>(g), clamp_flags, static_cast<float*>(gX),
                                                   B, N, M, d, wait_timeout_s(), s, nullptr, 0.f, region);
            if (e != cudaSuccess) return static_cast<sdtw_status>(e);
            gx_done = true;
        }
        // grad_Y: the same tensor-core kernel with E read transposed (autograd's G^T X bmm of the reference).
        if (g_distance_path == 0 && gY && grad_tc_supported(X, Y, D, E, gY, B, N, M, d)) {
            const cudaError_t e = grad_y_tc_launch(static_cast<const float*>(X), static_cast<const float*>(Y),
                                                   static_cast<const float*>(D), static_cast<const float*>(E),
                                                   static_cast<const float*>(g), clamp_flags, static_cast<float*>(gY),
                                                   B, N, M, d, wait_timeout_s(), s, nullptr, 0.f, region);
            if (e != cudaSuccess) return static_cast<sdtw_status>(e);
            gy_done = true;
        }
    }
    if (gx_done) gX = nullptr;
    if (gy_done) gY = nullptr;
    if (!gX && !gY) return SDTW_OK;
    if ((g_distance_path == 0 || g_distance_path == 3) && narrow_supported(B, N, M, d)) {
        // grad_X and grad_Y, each unless the tensor cores took it
        const cudaError_t e = narrow_grad_l2<T>(static_cast<const T*>(X), static_cast<const T*>(Y),
                                                static_cast<const T*>(D), static_cast<const T*>(E),
                                                static_cast<const T*>(g), clamp_flags, static_cast<T*>(gX),
                                                static_cast<T*>(gY), B, N, M, d, s);
        return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
    }
    if constexpr (sizeof(T) == 4) {
        if (!gx_done && g_distance_path < 2 && gX && d % 4 == 0 && M % 4 == 0 && aligned16(X) && aligned16(Y) && aligned16(E) &&
            aligned16(gX)) {
            static bool attr_set = false;
            if (!attr_set) {
                const cudaError_t e = cudaFuncSetAttribute(grad_x_mma_kernel,
                                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                           static_cast<int>(kGradSmem));
                if (e != cudaSuccess) return static_cast<sdtw_status>(e);
                attr_set = true;
            }
            const dim3 grid(static_cast<unsigned>((d + kGC - 1) / kGC), static_cast<unsigned>((N + kGR - 1) / kGR),
                            static_cast<unsigned>(B));
            count_launch();
            grad_x_mma_kernel<<<grid, 256, kGradSmem, s>>>(
                static_cast<const float*>(X), static_cast<const float*>(Y), static_cast<const float*>(D),
                static_cast<const float*>(E), static_cast<const float*>(g), clamp_flags, static_cast<float*>(gX), N,
                M, d);
            gx_done = true;
        }
    }
    if (gX && !gx_done) {
        const dim3 grid(cblocks, static_cast<unsigned>((N + kTile - 1) / kTile), static_cast<unsigned>(B));
        count_launch();
        grad_l2_kernel<T, false><<<grid, 256, 0, s>>>(static_cast<const T*>(X), static_cast<const T*>(Y),
                                                      static_cast<const T*>(D), static_cast<const T*>(E),
                                                      static_cast<const T*>(g), static_cast<T*>(gX), N, M, d, N, M);
    }
    if (gY) {
        const dim3 grid(cblocks, static_cast<unsigned>((M + kTile - 1) / kTile), static_cast<unsigned>(B));
        count_launch();
        grad_l2_kernel<T, true><<<grid, 256, 0, s>>>(static_cast<const T*>(Y), static_cast<const T*>(X),
                                                     static_cast<const T*>(D), static_cast<const T*>(E),
                                                     static_cast<const T*>(g), static_cast<T*>(gY), M, N, d, N, M);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e);
}

bool sizes_ok(int64_t B, int64_t N, int64_t M, int64_t d)
{
    return B >= 0 && N >= 0 && M >= 0 && d >= 0 && B < (int64_t(1) << 31) && N < (int64_t(1) << 31) / kTile * kTile &&
           M < (int64_t(1) << 31) / kTile * kTile;
}
}  // namespace
}  // namespace sdtw

using namespace sdtw;

extern "C" {

/* Test hook (not in the public header): 0 chooses the cost-matrix kernel by shape (tcgen05 where
 * supported), 1 forces the mma.sync kernels, 2 the CUDA-core kernels. */
void sdtw_debug_force_distance_path(int path) { g_distance_path = (path >= 0 && path <= 3) ? path : 0; }

size_t sdtw_pairwise_l2_band_workspace_bytes(int64_t B, int64_t N, int64_t M)
{
    if (!sizes_ok(B, N, M, 0)) return 0;
    const int64_t nb = B < kBatchChunk ? B : kBatchChunk;
    return pairwise_tc_region_ws_bytes(nb, N, M);
}

sdtw_status sdtw_pairwise_l2_band(sdtw_dtype dtype, const void* X, const void* Y, int64_t B, int64_t N, int64_t M,
                                  int64_t d, const void* lengths_x, const void* lengths_y, int lengths_are_int32,
                                  int64_t bandwidth, void* D, int* clamp_flags, void* workspace,
                                  size_t workspace_bytes, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!sizes_ok(B, N, M, d)) return SDTW_EINVAL;
    if (B == 0) return SDTW_OK;
    if (!lengths_x || !lengths_y) return SDTW_EINVAL;
    if (workspace_bytes < sdtw_pairwise_l2_band_workspace_bytes(B, N, M) || !workspace ||
        (reinterpret_cast<uintptr_t>(workspace) & 15))
        return SDTW_EWORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (clamp_flags) {
        const cudaError_t e = cudaMemsetAsync(clamp_flags, 0, static_cast<size_t>(B) * sizeof(int), s);
        if (e != cudaSuccess) return static_cast<sdtw_status>(e);
    }
    if (N == 0 || M == 0) return SDTW_OK;
    if (!D || (d > 0 && (!X || !Y))) return SDTW_EINVAL;
    const size_t es = dtype == SDTW_F32 ? 4 : 8;
    const size_t ls = lengths_are_int32 ? 4 : 8;
    for (int64_t b0 = 0; b0 < B; b0 += kBatchChunk) {
        const int64_t nb = B - b0 < kBatchChunk ? B - b0 : kBatchChunk;
        const void* Xc = at_elem(X, b0 * N * d, es);
        const void* Yc = at_elem(Y, b0 * M * d, es);
        void* Dc = at_elem(D, b0 * N * M, es);
        int* fc = clamp_flags ? clamp_flags + b0 : nullptr;
        const DpRegion region{at_elem(lengths_x, b0, ls), at_elem(lengths_y, b0, ls), lengths_are_int32 ? 1 : 0,
                              bandwidth};
        // The tile list needs the tensor-core kernel; every other path computes all of D (a superset).
        const sdtw_status st = dtype == SDTW_F32
                                   ? launch_pairwise<float>(Xc, Yc, nb, N, M, d, Dc, fc, s, &region, workspace)
                                   : launch_pairwise<double>(Xc, Yc, nb, N, M, d, Dc, fc, s);
        if (st != SDTW_OK) return st;
    }
    return SDTW_OK;
}

sdtw_status sdtw_pairwise_l2(sdtw_dtype dtype, const void* X, const void* Y, int64_t B, int64_t N, int64_t M,
                             int64_t d, void* D, int* clamp_flags, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!sizes_ok(B, N, M, d)) return SDTW_EINVAL;
    if (B == 0) return SDTW_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (clamp_flags) {
        const cudaError_t e = cudaMemsetAsync(clamp_flags, 0, static_cast<size_t>(B) * sizeof(int), s);
        if (e != cudaSuccess) return static_cast<sdtw_status>(e);
    }
    if (N == 0 || M == 0) return SDTW_OK;
    if (!D || (d > 0 && (!X || !Y))) return SDTW_EINVAL;
    const size_t es = dtype == SDTW_F32 ? 4 : 8;
    // Pairs in chunks of kBatchChunk: the kernels index pairs by grid.z (at most 65535).
    for (int64_t b0 = 0; b0 < B; b0 += kBatchChunk) {
        const int64_t nb = B - b0 < kBatchChunk ? B - b0 : kBatchChunk;
        const void* Xc = at_elem(X, b0 * N * d, es);
        const void* Yc = at_elem(Y, b0 * M * d, es);
        void* Dc = at_elem(D, b0 * N * M, es);
        int* fc = clamp_flags ? clamp_flags + b0 : nullptr;
        const sdtw_status st = dtype == SDTW_F32 ? launch_pairwise<float>(Xc, Yc, nb, N, M, d, Dc, fc, s)
                                                 : launch_pairwise<double>(Xc, Yc, nb, N, M, d, Dc, fc, s);
        if (st != SDTW_OK) return st;
    }
    return SDTW_OK;
}

}  // extern "C"

namespace sdtw {
namespace {
sdtw_status grad_l2_impl(sdtw_dtype dtype, const void* X, const void* Y, const void* D, const void* E, const void* g,
                         const int* clamp_flags, int64_t B, int64_t N, int64_t M, int64_t d, void* grad_X,
                         void* grad_Y, void* stream, const void* lengths_x, const void* lengths_y,
                         int lengths_are_int32, int64_t bandwidth)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!sizes_ok(B, N, M, d)) return SDTW_EINVAL;
    if (B == 0 || d == 0 || (!grad_X && !grad_Y)) return SDTW_OK;
    if (!X || !Y || !g || ((N * M > 0) && (!D || !E))) return SDTW_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // An empty side has an empty gradient; the other side's is zero (its contraction has no terms).
    if (N == 0) grad_X = nullptr;
    if (M == 0) grad_Y = nullptr;
    if (!grad_X && !grad_Y) return SDTW_OK;
    const size_t es = dtype == SDTW_F32 ? 4 : 8;
    for (int64_t b0 = 0; b0 < B; b0 += kBatchChunk) {
        const int64_t nb = B - b0 < kBatchChunk ? B - b0 : kBatchChunk;
        const void* Xc = at_elem(X, b0 * N * d, es);
        const void* Yc = at_elem(Y, b0 * M * d, es);
        const void* Dc = at_elem(D, b0 * N * M, es);
        const void* Ec = at_elem(E, b0 * N * M, es);
        const void* gc = at_elem(g, b0, es);
        const int* fc = clamp_flags ? clamp_flags + b0 : nullptr;
        void* gXc = grad_X ? at_elem(grad_X, b0 * N * d, es) : nullptr;
        void* gYc = grad_Y ? at_elem(grad_Y, b0 * M * d, es) : nullptr;
        const size_t ls = lengths_are_int32 ? 4 : 8;
        const DpRegion region{lengths_x ? at_elem(lengths_x, b0, ls) : nullptr,
                              lengths_y ? at_elem(lengths_y, b0, ls) : nullptr, lengths_are_int32 ? 1 : 0, bandwidth};
        const DpRegion* rp = lengths_x ? &region : nullptr;
        const sdtw_status st = dtype == SDTW_F32
                                   ? launch_grad<float>(Xc, Yc, Dc, Ec, gc, fc, nb, N, M, d, gXc, gYc, s, rp)
                                   : launch_grad<double>(Xc, Yc, Dc, Ec, gc, fc, nb, N, M, d, gXc, gYc, s);
        if (st != SDTW_OK) return st;
    }
    return SDTW_OK;
}
}  // namespace
}  // namespace sdtw

extern "C" {

sdtw_status sdtw_grad_l2(sdtw_dtype dtype, const void* X, const void* Y, const void* D, const void* E, const void* g,
                         const int* clamp_flags, int64_t B, int64_t N, int64_t M, int64_t d, void* grad_X,
                         void* grad_Y, void* stream)
{
    return grad_l2_impl(dtype, X, Y, D, E, g, clamp_flags, B, N, M, d, grad_X, grad_Y, stream, nullptr, nullptr, 0,
                        -1);
}

sdtw_status sdtw_grad_l2_band(sdtw_dtype dtype, const void* X, const void* Y, const void* D, const void* E,
                              const void* g, const int* clamp_flags, int64_t B, int64_t N, int64_t M, int64_t d,
                              const void* lengths_x, const void* lengths_y, int lengths_are_int32, int64_t bandwidth,
                              void* grad_X, void* grad_Y, void* stream)
{
    if (!lengths_x || !lengths_y) return SDTW_EINVAL;
    return grad_l2_impl(dtype, X, Y, D, E, g, clamp_flags, B, N, M, d, grad_X, grad_Y, stream, lengths_x, lengths_y,
                        lengths_are_int32, bandwidth);
}

}  // extern "C"
