// Compensated fp32 Soft-DTW wavefront (forward and backward) for sm_100a: R carried as an unevaluated sum
// R_hi + R_lo of two floats.
//
// Why: in plain fp32 every R value is rounded to ulp(R) (4e-3 at R = 5e4), and the backward's softmin weights
// exp(-(R_p - m) / gamma) turn that absolute error into a relative weight error of ulp(R) / gamma: O(1) for a
// small gamma. The reference's own fp32 backward (softdtw.cpp:248-256, weights exp((R[s] - R[p] - D[s]) /
// gamma)) is off by up to 0.67 on the 256 x 512 x 512 gamma = 0.1 workload and overflows on long sequences
// with gamma = 0.01. Here each cell's R = D + m - gamma ln(1 + e1 + e2) is accumulated exactly in the
// pair (TwoSum of m_hi + D, the small terms added to the low part), and every exponent uses the pair
// difference (m_hi - v_hi) + (m_lo - v_lo): the weights are then limited by the exp2 / log2 approximations
// (about 2^-22 relative per cell), not by the magnitude of R. fp32 arithmetic and fp32 storage throughout.
//
// Decomposition: one warp per pair, strips of 32 rows swept one after the other, operands in global memory
// (the warp-per-pair scheme of sdtw_warppair.cu): lane l holds row r0 + l and processes column tau - l at step
// tau; neighbouring rows exchange (hi, lo) pairs by warp shuffle, consecutive strips through two row buffers
// (hi and lo) per warp in shared memory. The pairs are independent and no warp waits for another.
//
// Every addition of the compensated steps is an explicit __fadd_rn / __fsub_rn (never contracted into an
// FMA), so the error-free transformations hold.
#include <climits>

#include "sdtw_b200.h"
#include "sdtw_strip.cuh"

namespace sdtw {

namespace {

constexpr int kX2Warps = 4;  // warps (= pairs) per CTA

struct X2FwdArgs {
    const float* D;
    float* Rh;
    float* Rl;
    float* costs;
    Lengths len;
    int64_t B, N, M, bw;
    float k, gl;
    uint32_t* err;
};

struct X2BwdArgs {
    const float* Rh;
    const float* Rl;
    float* E;
    Lengths len;
    int64_t B, N, M, bw;
    float k;
    uint32_t* err;
};

inline __host__ __device__ int64_t x2_strips(int64_t N) { return N > 0 ? (N + 31) / 32 : 1; }

// (hi, lo) of a value kept as an unevaluated sum.
struct F2 {
    float h, l;
};

__device__ __forceinline__ F2 sel(bool p, F2 a, F2 b) { return {p ? a.h : b.h, p ? a.l : b.l}; }

// a - b as one float, from the pair difference (exact in the high parts when a and b are close).
__device__ __forceinline__ float diff(F2 a, F2 b) { return __fadd_rn(__fsub_rn(a.h, b.h), __fsub_rn(a.l, b.l)); }

// Compensated forward cell: R = d + m - gamma ln(1 + e1 + e2), m <= x <= y the predecessors sorted by their
// high parts. Returns the pair (R_hi, R_lo).
__device__ __forceinline__ F2 fwd_cell_x2(float d, F2 diag, F2 up, F2 left, float k, float gl)
{
    const bool p1 = up.h <= left.h;
    const F2 a = sel(p1, up, left), y = sel(p1, left, up);
    const bool p2 = diag.h <= a.h;
    const F2 m = sel(p2, diag, a), x = sel(p2, a, diag);
    // m is +inf only when all three predecessors are (cells outside the band, masked by the caller).
    const F2 mc = {fminf(m.h, FLT_MAX), m.l};
    const float e1 = ex2f(diff(mc, x) * k);
    const float e2 = ex2f(diff(mc, y) * k);
    const float t = -gl * lg2f(__fadd_rn(__fadd_rn(1.f, e1), e2));
    // TwoSum(m_hi, d): s + e = m_hi + d exactly.
    const float s = __fadd_rn(m.h, d);
    const float bb = __fsub_rn(s, m.h);
    const float e = __fadd_rn(__fsub_rn(m.h, __fsub_rn(s, bb)), __fsub_rn(d, bb));
    const float lo = __fadd_rn(__fadd_rn(e, m.l), t);
    const float rh = __fadd_rn(s, lo);
    return {rh, __fsub_rn(lo, __fsub_rn(rh, s))};
}

// ---------------------------------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kX2Warps * 32) sdtw_fwd_x2_kernel(X2FwdArgs a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t b = static_cast<int64_t>(blockIdx.x) * kX2Warps + warp;
    if (b >= a.B) return;  // the whole warp; the kernel has no CTA-wide barrier
    const int64_t N = a.N, M = a.M, pitch = M + 2;
    const float INF = __int_as_float(0x7f800000);
    // buf_h[c + 1] + buf_l[c + 1] = R[r0 - 1][c]
    float* buf_h = reinterpret_cast<float*>(smem) + static_cast<int64_t>(warp) * 2 * (M + 1);
    float* buf_l = buf_h + (M + 1);
    float* Rbh = a.Rh + b * (N + 2) * pitch;
    float* Rbl = a.Rl + b * (N + 2) * pitch;
    // Padded rows 0 and N+1 (softdtw.cpp:114-121: +inf with R[b,0,0] = 0); the row above strip 0.
    for (int64_t c = lane; c < pitch; c += 32) {
        Rbh[c] = c == 0 ? 0.f : INF;
        Rbh[(N + 1) * pitch + c] = INF;
        Rbl[c] = 0.f;
        Rbl[(N + 1) * pitch + c] = 0.f;
    }
    for (int64_t c = lane; c <= M; c += 32) {
        buf_h[c] = c == 0 ? 0.f : INF;
        buf_l[c] = 0.f;
    }
    __syncwarp();
    const int S = static_cast<int>(x2_strips(N));
    const int src = (lane + 31) & 31;
    const bool lane0 = lane == 0, lane31 = lane == 31;
    for (int s = 0; s < S; ++s) {
        const int r0 = 32 * s;
        const int nmat = static_cast<int>(N - r0 < 32 ? N - r0 : 32);
        float* Rrh = Rbh + static_cast<int64_t>(r0 + 1) * pitch;  // padded row of DP row r0
        float* Rrl = Rbl + static_cast<int64_t>(r0 + 1) * pitch;
        Strip st;
        if (!make_strip(st, a.len, b, s, N, M, a.bw, lane)) {
            if (s == 0 && lane == 0) {
                if (st.bad) {
                    atomicOr(a.err, kErrBadLength);
                    a.costs[b] = __int_as_float(0x7fc00000);
                } else {
                    a.costs[b] = (st.nx == 0 && st.ny == 0) ? 0.f : INF;
                }
            }
            for (int r = 0; r < nmat; ++r)
                for (int64_t c = lane; c < pitch; c += 32) {
                    Rrh[r * pitch + c] = INF;
                    Rrl[r * pitch + c] = 0.f;
                }
            continue;  // every later strip of the pair is empty as well
        }
        // Cells outside each row's band interval [lo, hi] (and the border columns): +inf (low part 0).
        for (int r = 0; r < nmat; ++r) {
            const int lo = __shfl_sync(kFull, st.lo, r);
            const int hi = __shfl_sync(kFull, st.hi, r);
            for (int64_t c = lane; c < pitch; c += 32)
                if (c - 1 < lo || c - 1 > hi) {
                    Rrh[r * pitch + c] = INF;
                    Rrl[r * pitch + c] = 0.f;
                }
        }
        const int tb = st.c_begin;              // first step (lane 0's first column)
        const int te = st.c_end + st.rows - 1;  // last step
        const int i = r0 + lane;
        const float* Drow = a.D + (b * N + (i < N ? i : 0)) * M;
        float* Ch = Rrh + static_cast<int64_t>(lane) * pitch + 1;  // R[i][c] at Ch[c] + Cl[c]
        float* Cl = Rrl + static_cast<int64_t>(lane) * pitch + 1;
        const bool has_next = st.rows == 32 && r0 + 32 < st.nx;
        const int lstar = static_cast<int>(st.nx - 1 - r0);
        const int tstar = (lstar >= 0 && lstar < 32) ? static_cast<int>(st.ny - 1) + lstar : INT_MIN;
        F2 upp = lane0 ? F2{buf_h[tb], buf_l[tb]} : F2{INF, 0.f};  // lane 0's diagonal predecessor
        F2 outp = {INF, 0.f};
        float dn = (tb >= st.A && tb <= st.Z) ? __ldg(Drow + (tb - lane)) : 0.f;
#pragma unroll 1
        for (int tau = tb; tau <= te; ++tau) {
            const float d = dn;
            const int tn = tau + 1;
            dn = (tn >= st.A && tn <= st.Z) ? __ldg(Drow + (tn - lane)) : 0.f;  // next step's D, in flight
            const bool top_in = lane0 && tau < M;
            const F2 tv = {top_in ? buf_h[tau + 1] : INF, top_in ? buf_l[tau + 1] : 0.f};  // R[r0 - 1][tau]
            const F2 upw = {__shfl_sync(kFull, outp.h, src), __shfl_sync(kFull, outp.l, src)};
            const F2 up = sel(lane0, tv, upw);
            F2 r = fwd_cell_x2(d, upp, up, outp, a.k, a.gl);
            const bool valid = tau >= st.A && tau <= st.Z;
            r = valid ? r : F2{INF, 0.f};
            const int c = tau - lane;
            if (valid) {
                Ch[c] = r.h;
                Cl[c] = r.l;
            }
            if (tau == tstar && lane == lstar) a.costs[b] = __fadd_rn(r.h, r.l);
            if (lane31 && has_next && c >= -1 && c < M) {
                buf_h[c + 1] = r.h;
                buf_l[c + 1] = r.l;
            }
            upp = up;
            outp = r;
            if ((tau & 7) == 7) __syncwarp();  // orders lane 31's buffer writes before lane 0's reads
        }
        if (has_next) {
            // Columns of the last row this sweep did not reach are out of band: +inf.
            __syncwarp();
            for (int c = lane - 1; c < M; c += 32)
                if (c < tb - 31 || c > te - 31) {
                    buf_h[c + 1] = INF;
                    buf_l[c + 1] = 0.f;
                }
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------------------------------
// Backward (scatter form: each cell pushes E * softmin weight into its three predecessors)
// ---------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kX2Warps * 32) sdtw_bwd_x2_kernel(X2BwdArgs a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t b = static_cast<int64_t>(blockIdx.x) * kX2Warps + warp;
    if (b >= a.B) return;
    const int64_t N = a.N, M = a.M, pitch = M + 2;
    float* buf = reinterpret_cast<float*>(smem) + static_cast<int64_t>(warp) * (M > 0 ? M : 1);  // pushes into row r0+31
    for (int64_t c = lane; c < M; c += 32) buf[c] = 0.f;
    __syncwarp();
    float* Eb = a.E + b * N * M;
    const float* Rbh = a.Rh + b * (N + 2) * pitch;
    const float* Rbl = a.Rl + b * (N + 2) * pitch;
    const int S = static_cast<int>(x2_strips(N));
    const int src = (lane + 1) & 31;
    const bool lane0 = lane == 0, lane31 = lane == 31;
    for (int s = S - 1; s >= 0; --s) {
        const int r0 = 32 * s;
        const int nmat = static_cast<int>(N - r0 < 32 ? N - r0 : 32);
        float* Erow = Eb + static_cast<int64_t>(r0) * M;
        Strip st;
        if (!make_strip(st, a.len, b, s, N, M, a.bw, lane)) {
            if (st.bad && s == 0 && lane == 0) atomicOr(a.err, kErrBadLength);
            for (int r = 0; r < nmat; ++r)
                for (int64_t c = lane; c < M; c += 32) Erow[r * M + c] = 0.f;
            continue;  // the buffer stays zero: every strip below this one is empty too
        }
        for (int r = 0; r < nmat; ++r) {
            const int lo = __shfl_sync(kFull, st.lo, r);
            const int hi = __shfl_sync(kFull, st.hi, r);
            float* row = Erow + r * M;
            for (int64_t c = lane; c < M; c += 32)
                if (c < lo || c > hi) row[c] = 0.f;
        }
        const int tb = st.c_begin;
        const int te = st.c_end + st.rows - 1;
        const int i = r0 + lane;
        const int ip = i < N ? i : static_cast<int>(N);
        const float* Rdh = Rbh + static_cast<int64_t>(ip) * pitch;  // padded row i: R[i-1][c-1] at Rd[c]
        const float* Rdl = Rbl + static_cast<int64_t>(ip) * pitch;
        const float* Rlh = Rdh + pitch;  // padded row i+1: R[i][c-1] at Rl[c]
        const float* Rll = Rdl + pitch;
        float* Ecell = Erow + static_cast<int64_t>(lane) * M;
        const bool has_consumer = s > 0;
        const float seed = (i == st.nx - 1) ? 1.f : 0.f;
        F2 upc = {0.f, 0.f};
        float sendv = 0.f, pend = 0.f, acc = seed;
#pragma unroll 1
        for (int tau = te + 1; tau >= tb - 1; --tau) {
            const int c = tau - lane;
            const bool valid = tau >= st.A && tau <= st.Z;
            // R[i-1][c-1] is also loaded one step before the lane's first cell: it is that cell's R[i-1][c].
            const bool ld = tau >= st.A && tau <= st.Z + 1;
            const F2 rd = ld ? F2{Rdh[c], Rdl[c]} : F2{0.f, 0.f};
            const F2 rl = valid ? F2{Rlh[c], Rll[c]} : F2{0.f, 0.f};
            const F2 ru = upc;
            const float recvw = __shfl_sync(kFull, sendv, src);
            const int cb = tau - 31;
            const float bv = (lane31 && cb >= 0 && cb < M) ? buf[cb] : 0.f;
            const float recv = lane31 ? bv : recvw;
            const float Es = acc + recv;
            const F2 mm = sel(rd.h <= ru.h, rd, ru);
            const F2 m = sel(mm.h <= rl.h, mm, rl);
            const F2 mc = {fminf(m.h, FLT_MAX), m.l};
            const float ed = ex2f(diff(mc, rd) * a.k);
            const float eu = ex2f(diff(mc, ru) * a.k);
            const float el = ex2f(diff(mc, rl) * a.k);
            float q = Es * rcpf((ed + eu) + el);
            q = valid ? q : 0.f;
            acc = valid ? q * el : seed;
            sendv = fmaf(q, eu, pend);
            pend = q * ed;
            if (valid) Ecell[c] = Es;
            if (lane0 && has_consumer && c >= 0 && c < M) buf[c] = sendv;  // into R row r0 - 1, column c
            upc = rd;
            if ((tau & 7) == 0) __syncwarp();  // orders lane 0's buffer writes before lane 31's reads
        }
        if (has_consumer) {
            // Columns of the row above that received no push: zero.
            __syncwarp();
            for (int64_t c = lane; c < M; c += 32)
                if (c < tb - 1 || c > te) buf[c] = 0.f;
        }
        __syncwarp();
    }
}

inline sdtw_status from_cuda_x2(cudaError_t e) { return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e); }

inline int64_t clamp_bw_x2(int64_t bw, int64_t N, int64_t M) { return bw > N + M ? N + M : bw; }

bool x2_args_ok(int64_t B, int64_t N, int64_t M, double gamma)
{
    if (B < 0 || N < 0 || M < 0) return false;
    if (!(gamma > 0.0) || gamma > 3.0e38) return false;
    if (N > (1 << 29) || M > (1 << 29)) return false;
    // The row buffers of a CTA live in shared memory (2 x (M + 1) floats per warp in the forward).
    if (static_cast<int64_t>(kX2Warps) * 2 * (M + 1) * 4 > 200 * 1024) return false;
    return true;
}

}  // namespace

}  // namespace sdtw

using namespace sdtw;

extern "C" {

sdtw_status sdtw_forward_x2(const float* D, int64_t B, int64_t N, int64_t M, const void* lengths_x,
                            const void* lengths_y, int lengths_int32, double gamma, int64_t bandwidth, float* R_hi,
                            float* R_lo, float* costs, uint32_t* err_word, void* stream)
{
    if (!x2_args_ok(B, N, M, gamma)) return SDTW_EINVAL;
    if (B == 0) return SDTW_OK;
    if (!lengths_x || !lengths_y || !R_hi || !R_lo || !costs || !err_word || (N * M > 0 && !D)) return SDTW_EINVAL;
    const size_t smem = static_cast<size_t>(kX2Warps) * 2 * static_cast<size_t>(M + 1) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(sdtw_fwd_x2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return from_cuda_x2(e);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Every cost starts as NaN, like sdtw_forward's.
    e = cudaMemsetAsync(costs, 0xff, static_cast<size_t>(B) * sizeof(float), s);
    if (e != cudaSuccess) return from_cuda_x2(e);
    X2FwdArgs a;
    a.D = D;
    a.Rh = R_hi;
    a.Rl = R_lo;
    a.costs = costs;
    a.len = Lengths{lengths_x, lengths_y, lengths_int32};
    a.B = B;
    a.N = N;
    a.M = M;
    a.bw = clamp_bw_x2(bandwidth, N, M);
    a.k = static_cast<float>(1.4426950408889634 / gamma);
    a.gl = static_cast<float>(gamma * 0.6931471805599453);
    a.err = err_word;
    const int64_t grid = (B + kX2Warps - 1) / kX2Warps;
    count_launch();
    sdtw_fwd_x2_kernel<<<static_cast<unsigned>(grid), kX2Warps * 32, smem, s>>>(a);
    return from_cuda_x2(cudaGetLastError());
}

sdtw_status sdtw_backward_x2(const float* R_hi, const float* R_lo, int64_t B, int64_t N, int64_t M,
                             const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                             int64_t bandwidth, float* E, uint32_t* err_word, void* stream)
{
    if (!x2_args_ok(B, N, M, gamma)) return SDTW_EINVAL;
    if (B == 0 || N == 0 || M == 0) return SDTW_OK;
    if (!lengths_x || !lengths_y || !R_hi || !R_lo || !E || !err_word) return SDTW_EINVAL;
    const size_t smem = static_cast<size_t>(kX2Warps) * static_cast<size_t>(M) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(sdtw_bwd_x2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return from_cuda_x2(e);
    X2BwdArgs a;
    a.Rh = R_hi;
    a.Rl = R_lo;
    a.E = E;
    a.len = Lengths{lengths_x, lengths_y, lengths_int32};
    a.B = B;
    a.N = N;
    a.M = M;
    a.bw = clamp_bw_x2(bandwidth, N, M);
    a.k = static_cast<float>(1.4426950408889634 / gamma);
    a.err = err_word;
    const int64_t grid = (B + kX2Warps - 1) / kX2Warps;
    count_launch();
    sdtw_bwd_x2_kernel<<<static_cast<unsigned>(grid), kX2Warps * 32, smem, static_cast<cudaStream_t>(stream)>>>(a);
    return from_cuda_x2(cudaGetLastError());
}

}  // extern "C"
