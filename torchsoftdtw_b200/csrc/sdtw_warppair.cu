// Warp-per-pair Soft-DTW wavefront kernels for sm_100a: large batches of short pairs.
//
// One warp owns one pair and sweeps its 32-row strips one after the other (the forward top-down, the
// backward bottom-up). Lane l holds row r0 + l and processes column tau - l at step tau, exactly as in
// the strip kernels of sdtw_wavefront.cu / sdtw_pairwave.cu, with the row above (forward) or the pushes
// from the row below (backward) arriving by warp shuffle. What differs is where the operands live:
//   * consecutive strips of a pair hand over their boundary row through ONE row buffer per warp in shared
//     memory, updated in place: at step tau the strip reads column tau (forward, lane 0) or tau - 31
//     (backward, lane 31) of it and overwrites column tau - 31 (forward, lane 31) or tau (backward,
//     lane 0), a column it read 31 steps earlier. No warp ever waits for another warp.
//   * D, R and E are read and written in place in global memory, one element per lane and step. A lane
//     walks along its own row, so each 32-byte sector it touches serves 4 (fp64) or 8 (fp32) consecutive
//     steps from L1 or L2, and the row buffer is the only shared memory a warp needs.
// The pair-resident and strip-ticket kernels stage operands in skewed shared-memory rings of 32 rows; for
// short pairs those rings, not the arithmetic, limit how many warps an SM holds (about 10 for fp64
// 64 x 64 pairs). Here an SM holds as many warps as its registers allow, which hides the latency of the
// dependent exp2 / log2 chain of each step (software sequences in fp64).
//
// The kernels write every element of their outputs (R with its +inf border and the cells outside the band
// or the lengths; E with its zeros).
#include <climits>

#include "sdtw_b200.h"
#include "sdtw_strip.cuh"
#include "sdtw_warppair.h"

namespace sdtw {

namespace {

template <typename T>
struct WarpFwdArgs {
    const T* D;
    T* R;
    T* costs;
    Lengths len;
    int64_t B, N, M, bw;
    T k, gl;
    uint32_t* err;
};

template <typename T>
struct WarpBwdArgs {
    const T* R;
    T* E;
    Lengths len;
    int64_t B, N, M, bw;
    T k;
    uint32_t* err;
};

inline __host__ __device__ int64_t n_strips(int64_t N) { return N > 0 ? (N + 31) / 32 : 1; }

// ---------------------------------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kWarpPairWarps * 32, kWarpPairMinCtas) sdtw_fwd_warp_kernel(WarpFwdArgs<T> a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t b = static_cast<int64_t>(blockIdx.x) * kWarpPairWarps + warp;
    if (b >= a.B) return;  // the whole warp; the kernel has no CTA-wide barrier
    const int64_t N = a.N, M = a.M, pitch = M + 2;
    const T INF = Num<T>::inf();
    T* buf = reinterpret_cast<T*>(smem) + static_cast<int64_t>(warp) * (M + 1);  // buf[c + 1] = R[r0 - 1][c]
    T* Rb = a.R + b * (N + 2) * pitch;
    // Padded rows 0 and N+1 (softdtw.cpp:114-121: +inf with R[b,0,0] = 0); the row above strip 0.
    for (int64_t c = lane; c < pitch; c += 32) {
        Rb[c] = c == 0 ? T(0) : INF;
        Rb[(N + 1) * pitch + c] = INF;
    }
    for (int64_t c = lane; c <= M; c += 32) buf[c] = c == 0 ? T(0) : INF;
    __syncwarp();
    const int S = static_cast<int>(n_strips(N));
    const int src = (lane + 31) & 31;
    const bool lane0 = lane == 0, lane31 = lane == 31;
    for (int s = 0; s < S; ++s) {
        const int r0 = 32 * s;
        const int nmat = static_cast<int>(N - r0 < 32 ? N - r0 : 32);
        T* Rrow = Rb + static_cast<int64_t>(r0 + 1) * pitch;  // padded row of DP row r0
        Strip st;
        if (!make_strip(st, a.len, b, s, N, M, a.bw, lane)) {
            if (s == 0 && lane == 0) {
                if (st.bad) {
                    atomicOr(a.err, kErrBadLength);
                    a.costs[b] = Num<T>::nan();
                } else {
                    a.costs[b] = (st.nx == 0 && st.ny == 0) ? T(0) : INF;
                }
            }
            for (int r = 0; r < nmat; ++r)
                for (int64_t c = lane; c < pitch; c += 32) Rrow[r * pitch + c] = INF;
            continue;  // every later strip of the pair is empty as well
        }
        // Cells outside each row's band interval [lo, hi] (and the border columns): +inf.
        for (int r = 0; r < nmat; ++r) {
            const int lo = __shfl_sync(kFull, st.lo, r);
            const int hi = __shfl_sync(kFull, st.hi, r);
            T* row = Rrow + r * pitch;
            for (int64_t c = lane; c < pitch; c += 32)
                if (c - 1 < lo || c - 1 > hi) row[c] = INF;
        }
        const int tb = st.c_begin;               // first step (lane 0's first column)
        const int te = st.c_end + st.rows - 1;   // last step
        const int i = r0 + lane;
        const T* Drow = a.D + (b * N + (i < N ? i : 0)) * M;
        T* Rcell = Rrow + static_cast<int64_t>(lane) * pitch + 1;  // R[i][c] at Rcell[c]
        const bool has_next = st.rows == 32 && r0 + 32 < st.nx;  // the next strip reads this one's last row
        const int lstar = static_cast<int>(st.nx - 1 - r0);
        const int tstar = (lstar >= 0 && lstar < 32) ? static_cast<int>(st.ny - 1) + lstar : INT_MIN;
        T upp = lane0 ? buf[tb] : INF;  // lane 0's diagonal predecessor R[r0 - 1][tb - 1]
        T outp = INF;
        T dn = (tb >= st.A && tb <= st.Z) ? __ldg(Drow + (tb - lane)) : T(0);
#pragma unroll 1
        for (int tau = tb; tau <= te; ++tau) {
            const T d = dn;
            const int tn = tau + 1;
            dn = (tn >= st.A && tn <= st.Z) ? __ldg(Drow + (tn - lane)) : T(0);  // next step's D, in flight
            const T tv = (lane0 && tau < M) ? buf[tau + 1] : INF;              // R[r0 - 1][tau]
            const T upw = __shfl_sync(kFull, outp, src);
            const T up = lane0 ? tv : upw;
            T r = fwd_cell<T>(d, upp, up, outp, a.k, a.gl);
            const bool valid = tau >= st.A && tau <= st.Z;
            r = valid ? r : INF;
            const int c = tau - lane;
            if (valid) Rcell[c] = r;
            if (tau == tstar && lane == lstar) a.costs[b] = r;
            if (lane31 && has_next && c >= -1 && c < M) buf[c + 1] = r;
            upp = up;
            outp = r;
            if ((tau & 7) == 7) __syncwarp();  // orders lane 31's buffer writes before lane 0's reads
        }
        if (has_next) {
            // Columns of the last row this sweep did not reach are out of band: +inf.
            __syncwarp();
            for (int c = lane - 1; c < M; c += 32)
                if (c < tb - 31 || c > te - 31) buf[c + 1] = INF;
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------------------------------
// Backward (scatter form: each cell pushes E * softmin weight into its three predecessors)
// ---------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kWarpPairWarps * 32, kWarpPairMinCtas) sdtw_bwd_warp_kernel(WarpBwdArgs<T> a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t b = static_cast<int64_t>(blockIdx.x) * kWarpPairWarps + warp;
    if (b >= a.B) return;
    const int64_t N = a.N, M = a.M, pitch = M + 2;
    const T big = Num<T>::big();
    T* buf = reinterpret_cast<T*>(smem) + static_cast<int64_t>(warp) * (M > 0 ? M : 1);  // pushes into row r0+31
    for (int64_t c = lane; c < M; c += 32) buf[c] = T(0);
    __syncwarp();
    T* Eb = a.E + b * N * M;
    const T* Rb = a.R + b * (N + 2) * pitch;
    const int S = static_cast<int>(n_strips(N));
    const int src = (lane + 1) & 31;
    const bool lane0 = lane == 0, lane31 = lane == 31;
    for (int s = S - 1; s >= 0; --s) {
        const int r0 = 32 * s;
        const int nmat = static_cast<int>(N - r0 < 32 ? N - r0 : 32);
        T* Erow = Eb + static_cast<int64_t>(r0) * M;
        Strip st;
        if (!make_strip(st, a.len, b, s, N, M, a.bw, lane)) {
            if (st.bad && s == 0 && lane == 0) atomicOr(a.err, kErrBadLength);
            for (int r = 0; r < nmat; ++r)
                for (int64_t c = lane; c < M; c += 32) Erow[r * M + c] = T(0);
            continue;  // the buffer stays zero: every strip below this one is empty too
        }
        for (int r = 0; r < nmat; ++r) {
            const int lo = __shfl_sync(kFull, st.lo, r);
            const int hi = __shfl_sync(kFull, st.hi, r);
            T* row = Erow + r * M;
            for (int64_t c = lane; c < M; c += 32)
                if (c < lo || c > hi) row[c] = T(0);
        }
        const int tb = st.c_begin;
        const int te = st.c_end + st.rows - 1;
        const int i = r0 + lane;
        const int ip = i < N ? i : static_cast<int>(N);
        const T* Rd = Rb + static_cast<int64_t>(ip) * pitch;  // padded row i: R[i-1][c-1] at Rd[c]
        const T* Rl = Rd + pitch;                             // padded row i+1: R[i][c-1] at Rl[c]
        T* Ecell = Erow + static_cast<int64_t>(lane) * M;
        const bool has_consumer = s > 0;
        const T seed = (i == st.nx - 1) ? T(1) : T(0);
        T upc = T(0), sendv = T(0), pend = T(0), acc = seed;
        // From te + 1 (a step without cells, which loads R[i-1][hi] for the lanes whose first cell comes
        // at te) down to tb - 1 (a step without cells, in which lane 0 pushes its last diagonal term).
#pragma unroll 1
        for (int tau = te + 1; tau >= tb - 1; --tau) {
            const int c = tau - lane;
            const bool valid = tau >= st.A && tau <= st.Z;
            // R[i-1][c-1] is also loaded one step before the lane's first cell: it is that cell's R[i-1][c].
            const bool ld = tau >= st.A && tau <= st.Z + 1;
            const T rd = ld ? Rd[c] : T(0);
            const T rl = valid ? Rl[c] : T(0);
            const T ru = upc;
            const T recvw = __shfl_sync(kFull, sendv, src);
            const int cb = tau - 31;
            const T bv = (lane31 && cb >= 0 && cb < M) ? buf[cb] : T(0);
            const T recv = lane31 ? bv : recvw;
            const T Es = acc + recv;
            const T m = Num<T>::mn(Num<T>::mn(rd, ru), rl);
            const T mc = Num<T>::mn(m, big);
            const T ed = Num<T>::exp2_((mc - rd) * a.k);
            const T eu = Num<T>::exp2_((mc - ru) * a.k);
            const T el = Num<T>::exp2_((mc - rl) * a.k);
            T q = Es * Num<T>::rcp_((ed + eu) + el);
            q = valid ? q : T(0);
            acc = valid ? q * el : seed;
            sendv = fma(q, eu, pend);
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
                if (c < tb - 1 || c > te) buf[c] = T(0);
        }
        __syncwarp();
    }
}

}  // namespace

template <typename T>
size_t warp_fwd_smem_bytes(int64_t M)
{
    return static_cast<size_t>(kWarpPairWarps) * static_cast<size_t>(M + 1) * sizeof(T);
}
template <typename T>
size_t warp_bwd_smem_bytes(int64_t M)
{
    return static_cast<size_t>(kWarpPairWarps) * static_cast<size_t>(M > 0 ? M : 1) * sizeof(T);
}
template size_t warp_fwd_smem_bytes<float>(int64_t);
template size_t warp_fwd_smem_bytes<double>(int64_t);
template size_t warp_bwd_smem_bytes<float>(int64_t);
template size_t warp_bwd_smem_bytes<double>(int64_t);

template <typename T>
cudaError_t warp_forward(const T* D, T* R, T* costs, const void* lx, const void* ly, int is32, int64_t B, int64_t N,
                         int64_t M, int64_t bw, double gamma, uint32_t* err, cudaStream_t stream)
{
    WarpFwdArgs<T> a;
    a.D = D;
    a.R = R;
    a.costs = costs;
    a.len = Lengths{lx, ly, is32};
    a.B = B;
    a.N = N;
    a.M = M;
    a.bw = bw;
    a.k = static_cast<T>(1.4426950408889634 / gamma);
    a.gl = static_cast<T>(gamma * 0.6931471805599453);
    a.err = err;
    const int64_t grid = (B + kWarpPairWarps - 1) / kWarpPairWarps;
    count_launch();
    sdtw_fwd_warp_kernel<T><<<static_cast<unsigned>(grid), kWarpPairWarps * 32, warp_fwd_smem_bytes<T>(M), stream>>>(a);
    return cudaGetLastError();
}
template cudaError_t warp_forward<float>(const float*, float*, float*, const void*, const void*, int, int64_t, int64_t,
                                         int64_t, int64_t, double, uint32_t*, cudaStream_t);
template cudaError_t warp_forward<double>(const double*, double*, double*, const void*, const void*, int, int64_t,
                                          int64_t, int64_t, int64_t, double, uint32_t*, cudaStream_t);

template <typename T>
cudaError_t warp_backward(const T* R, T* E, const void* lx, const void* ly, int is32, int64_t B, int64_t N, int64_t M,
                          int64_t bw, double gamma, uint32_t* err, cudaStream_t stream)
{
    WarpBwdArgs<T> a;
    a.R = R;
    a.E = E;
    a.len = Lengths{lx, ly, is32};
    a.B = B;
    a.N = N;
    a.M = M;
    a.bw = bw;
    a.k = static_cast<T>(1.4426950408889634 / gamma);
    a.err = err;
    const int64_t grid = (B + kWarpPairWarps - 1) / kWarpPairWarps;
    count_launch();
    sdtw_bwd_warp_kernel<T><<<static_cast<unsigned>(grid), kWarpPairWarps * 32, warp_bwd_smem_bytes<T>(M), stream>>>(a);
    return cudaGetLastError();
}
template cudaError_t warp_backward<float>(const float*, float*, const void*, const void*, int, int64_t, int64_t, int64_t,
                                          int64_t, double, uint32_t*, cudaStream_t);
template cudaError_t warp_backward<double>(const double*, double*, const void*, const void*, int, int64_t, int64_t,
                                           int64_t, int64_t, double, uint32_t*, cudaStream_t);

}  // namespace sdtw
