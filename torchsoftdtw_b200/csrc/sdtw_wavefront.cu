// Soft-DTW forward / backward wavefront kernels for sm_100a, behind the C ABI of include/sdtw_b200.h.
//
// Work decomposition (both directions)
//   * A pair's (nx, ny) DP grid is cut into strips of 32 rows. One warp owns one strip: lane l owns row
//     r0 + l and processes column (tau - l) at step tau, so every warp step is one anti-diagonal and
//     neighbouring rows exchange values with one warp shuffle per step; no block-wide barrier exists.
//   * Strips are claimed from a global ticket counter in dependency order (forward: strip 0 of every
//     pair, then strip 1, ...; backward: the last strip first). A strip only ever waits on the strip
//     claimed just before it in the same pair, which was claimed earlier by a running warp, so the
//     persistent grid cannot deadlock, whatever its size.
//   * The boundary row between strips goes through a workspace buffer in global memory (L2): the
//     forward passes each strip's last row of R down, the backward passes the contributions pushed
//     from a strip's first row up. The buffer starts as an all-ones NaN pattern and every value is
//     written once with st.relaxed, so a consumer knows a value has arrived when it is no longer the
//     pattern: no flags, no fences. Values are handed over per group of steps (8 steps in the backward
//     and the fp64 forward, a 32-step block in the fp32 forward): after each group the producer publishes
//     the boundary values it finished, and before each group the consumer waits for the ones that group
//     reads, having read them from L2 ahead of time; every wait is bounded in time (the launch aborts with
//     SDTW_ERR_TIMEOUT, never hangs).
//   * Per warp, a shared-memory ring of 4 chunks x 32 columns holds the operands of the swept rows
//     (forward: D, overwritten in place by R; backward: R, overwritten in place by E); chunks are
//     prefetched two blocks ahead with cp.async and written back with coalesced row stores.
//   * Only in-band columns of each strip are swept (the Sakoe-Chiba band and the lengths clip every
//     row to an interval), so out-of-band cells cost nothing beyond the 32-step skew of a strip.
//
// Arithmetic
//   Forward:  R[i,j] = D[i,j] + m - gamma*ln(1 + e^{-(x-m)/gamma} + e^{-(y-m)/gamma}),
//             m <= x <= y the three predecessors sorted: two exp2 + one log2 per cell.
//   Backward: scatter form. When E[s] is final, cell s pushes E[s] * w_p to each predecessor p, where
//             w_p = e^{-(R_p - m_s)/gamma} / sum_q e^{-(R_q - m_s)/gamma} is the softmin weight of p in
//             the forward of s. These are the reference's exp((R[s]-R[p]-D[s])/gamma) weights
//             (softdtw.cpp:248-256) written without the cancellation R[s]-D[s]: three exp2 and one
//             reciprocal per cell, and no read of D.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <mutex>

#include "sdtw_b200.h"
#include "sdtw_pairwave.h"
#include "sdtw_warppair.h"
#include "sdtw_tcgen05.h"
#include "sdtw_strip.cuh"

namespace sdtw {

// ==================================================================================================
// Forward
// ==================================================================================================
template <typename T>
struct FwdArgs {
    const T* D;
    T* R;
    T* costs;
    Lengths len;
    T* bnd;       // (B, S, M): last row of R of each strip, read by the strip below
    int* ticket;  // strip ticket counter
    int64_t B, N, M, bw;
    int S;
    T k;   // log2(e) / gamma
    T gl;  // gamma * ln(2)
    Sync sy;
    int inject_skip;  // ticket whose strip never writes its boundary row (failure-detection test); -1 = none
    int vec;          // D rows are 16-byte aligned: 16-byte cp.async
};

// The G forward steps tau = tau0 + GQ .. tau0 + GQ + G - 1 of one warp (group Q of the block at tau0).
template <typename T, bool MASKED, int G, int Q>
__device__ __forceinline__ void fwd_group(T* myrow, const T* top, int tau0, int lane, int A, int Z, T k, T gl,
                                          T& outp, T& upp)
{
    const T INF = Num<T>::inf();
    const int src = (lane + 31) & 31;
    const bool lane0 = lane == 0;
    const int base = tau0 - lane;
    const T* topb = top + (tau0 & kSideMask);
#pragma unroll
    for (int u = G * Q; u < G * Q + G; ++u) {
        T* cell = myrow + ((base + u) & kRingMask);
        const T d = *cell;
        const T upw = __shfl_sync(kFull, outp, src);
        const T tv = topb[u];
        const T up = lane0 ? tv : upw;
        T r = fwd_cell<T>(d, upp, up, outp, k, gl);
        if (MASKED) {
            const int tau = tau0 + u;
            r = (tau >= A && tau <= Z) ? r : INF;
        }
        *cell = r;
        upp = up;
        outp = r;
    }
}

// D chunk kk (columns [32kk, 32kk+32) of the strip's rows) -> ring, asynchronously.
template <typename T>
__device__ __forceinline__ void fwd_load_chunk(const FwdArgs<T>& a, const T* Db, T* ring, int kk, int rows, int lane)
{
    const int64_t M = a.M;
    const int col0 = 32 * kk;
    if (a.vec && rows == 32) {
        // Full strip: lane l copies piece l % PPR of rows l / PPR, l / PPR + RPI, ...; one column and byte count
        // per lane, so the loop is PPR copies with pointer increments (the general loop below recomputes the
        // row, column and byte count of every piece, on each warp's path between blocks).
        constexpr int EPP = 16 / sizeof(T);  // elements per 16-byte piece
        constexpr int PPR = 32 / EPP;        // pieces per row of a chunk
        constexpr int RPI = 32 / PPR;        // rows per warp-wide copy
        const int col = col0 + (lane % PPR) * EPP;
        const int64_t left = (M - col) * static_cast<int64_t>(sizeof(T));
        const int bytes = left >= 16 ? 16 : (left > 0 ? static_cast<int>(left) : 0);
        const int r = lane / PPR;
        const T* src = Db + static_cast<int64_t>(r) * M + (bytes > 0 ? col : 0);
        T* dst = ring + r * kRing + (col & kRingMask);
#pragma unroll
        for (int i = 0; i < PPR; ++i) cp_async_16(dst + i * RPI * kRing, src + i * RPI * M, bytes);
    } else if (a.vec) {
        constexpr int EPP = 16 / sizeof(T);  // elements per 16-byte piece
        constexpr int PPR = 32 / EPP;        // pieces per row of a chunk
#pragma unroll 4
        for (int p = lane; p < 32 * PPR; p += 32) {
            const int r = p / PPR;
            if (r >= rows) break;
            const int col = col0 + (p % PPR) * EPP;
            const int64_t left = (M - col) * static_cast<int64_t>(sizeof(T));
            const int bytes = left >= 16 ? 16 : (left > 0 ? static_cast<int>(left) : 0);
            const T* src = Db + static_cast<int64_t>(r) * M + (bytes > 0 ? col : 0);
            cp_async_16(ring + r * kRing + (col & kRingMask), src, bytes);
        }
    } else {
        const int col = col0 + lane;
        const bool in = col < M;
        for (int r = 0; r < rows; ++r) {
            const T* src = Db + static_cast<int64_t>(r) * M + (in ? col : 0);
            cp_async_scalar<sizeof(T)>(ring + r * kRing + (col & kRingMask), src, in ? static_cast<int>(sizeof(T)) : 0);
        }
    }
}

// Completed R chunk kk -> global R (padded layout), columns clipped to the swept range.
template <typename T>
__device__ __forceinline__ void fwd_store_chunk(const FwdArgs<T>& a, T* Rb, const T* ring, int kk, const Strip& st,
                                                int lane)
{
    const int col = 32 * kk + lane;
    if (col < st.c_begin || col > st.c_end) return;
    const int64_t pitch = a.M + 2;
    T* dst = Rb + static_cast<int64_t>(st.r0 + 1) * pitch + col + 1;
    const T* srcp = ring + (col & kRingMask);
    if (st.rows == 32) {
        // Unrolled, so the 32 shared-memory loads issue back to back instead of each store waiting for its
        // own load (16 pairs of 4096 x 4096, band 256: the forward took 6% longer with the rolled loop).
#pragma unroll
        for (int r = 0; r < 32; ++r) dst[r * pitch] = srcp[r * kRing];
    } else {
        for (int r = 0; r < st.rows; ++r) dst[r * pitch] = srcp[r * kRing];
    }
}

// Steps per boundary hand-over in the strip-ticket forward. Groups of 8 steps cut the lag between strips
// from 64 steps to 40 but cost each group a wait and a publish, which the short fp32 steps do not earn back.
// Measured on one B200: fp32, 16 pairs of 4096 x 4096, band 256: 1.60 ms with whole blocks, 1.61 with groups
// of 16, 1.68 with groups of 8; fp64, 4 pairs of 2048 x 2048: 3.99 ms with groups of 8, 4.46 with blocks.
template <typename T>
struct FwdGroup {
    static constexpr int value = sizeof(T) == 8 ? 8 : 32;
};

// One block of 32 steps as 32 / G groups of G. Lane l holds in `nv` the value of the row above at column
// tau0 + l (read from L2 ahead of time, possibly before the strip above wrote it). Group q reads columns
// tau0 + Gq .. tau0 + Gq + G - 1 of the row above (through lane 0), complete once the strip above finished the
// same group of the next block. Before group q the G lanes that hold them wait for their values, hand them to
// the side ring and read the next block's value of their column ahead, and the lanes of group q + 1 re-read
// theirs; after the group, G lanes publish the G values of the last row it finished. Returns false if the
// launch aborted.
template <typename T, bool MASKED, int G, int Q>
__device__ __forceinline__ bool fwd_group_step(const FwdArgs<T>& a, T* ring, T* top, const T* bnd_in, T* bnd_out, int tau0,
                                               const Strip& st, int plo, int phi, bool has_above, bool has_consumer,
                                               int lane, T& nv, T& outp, T& upp)
{
    constexpr int NG = 32 / G;
    const T INF = Num<T>::inf();
    const int grp = lane / G;
    if (has_above) {
        const int c = tau0 + lane;
        const bool need = c >= plo && c <= phi;
        if (!await_boundary(nv, bnd_in + c, need && grp == Q, a.sy, lane)) return false;
        if (grp == Q) {
            top[c & kSideMask] = need ? nv : INF;
            const int cn = c + 32;
            nv = (cn >= plo && cn <= phi) ? ld_relaxed(bnd_in + cn) : INF;
        } else if (NG > 1 && grp == (Q + 1) % NG) {
            const int cr = Q == NG - 1 ? c + 32 : c;  // after the last group: the next block's first group
            if (cr >= plo && cr <= phi) nv = ld_relaxed(bnd_in + cr);
        }
    } else if (grp == Q) {
        top[(tau0 + lane) & kSideMask] = INF;
    }
    __syncwarp();
    fwd_group<T, MASKED, G, Q>(ring + lane * kRing, top, tau0, lane, st.A, st.Z, a.k, a.gl, outp, upp);
    __syncwarp();
    if (has_consumer && lane < G) {
        // Last row (lane 31) finished columns [tau0 + GQ - 31, tau0 + GQ + G - 32] in this group.
        const int c = tau0 + G * Q - 31 + lane;
        if (c >= st.c_begin && c <= st.c_end) st_relaxed(bnd_out + c, ring[31 * kRing + (c & kRingMask)]);
    }
    return true;
}
template <typename T, bool MASKED, int G, int Q = 0>
__device__ __forceinline__ bool fwd_block_groups(const FwdArgs<T>& a, T* ring, T* top, const T* bnd_in, T* bnd_out,
                                                 int tau0, const Strip& st, int plo, int phi, bool has_above,
                                                 bool has_consumer, int lane, T& nv, T& outp, T& upp)
{
    if (!fwd_group_step<T, MASKED, G, Q>(a, ring, top, bnd_in, bnd_out, tau0, st, plo, phi, has_above, has_consumer,
                                         lane, nv, outp, upp))
        return false;
    if constexpr (Q + 1 < 32 / G)
        return fwd_block_groups<T, MASKED, G, Q + 1>(a, ring, top, bnd_in, bnd_out, tau0, st, plo, phi, has_above,
                                                     has_consumer, lane, nv, outp, upp);
    else
        return true;
}

template <typename T>
__device__ void fwd_strip(const FwdArgs<T>& a, T* ring, T* top, int64_t b, int s, int lane, bool skip_publish)
{
    const T INF = Num<T>::inf();
    Strip st;
    if (!make_strip(st, a.len, b, s, a.N, a.M, a.bw, lane)) {
        if (s == 0 && lane == 0) {
            if (st.bad) {
                atomicOr(a.sy.err, kErrBadLength);
                a.costs[b] = Num<T>::nan();
            } else {
                a.costs[b] = (st.nx == 0 && st.ny == 0) ? T(0) : INF;
            }
        }
        return;
    }
    const int64_t pitch = a.M + 2;
    const T* Db = a.D + (b * a.N + st.r0) * a.M;
    T* Rb = a.R + b * (a.N + 2) * pitch;
    const int k0 = st.c_begin >> 5;
    const int k1 = (st.c_end + 31) >> 5;
    const int kc = st.c_end >> 5;
    const bool has_consumer = st.rows == 32 && st.r0 + 32 < st.nx && !skip_publish;
    T* bnd_out = a.bnd + (b * a.S + s) * a.M;
    const T* bnd_in = a.bnd + (b * a.S + s - 1) * a.M;
    int plo = 0, phi = -1;  // in-band columns of the row above (row r0-1), the ones the strip above wrote
    if (s > 0) {
        int64_t l64, h64;
        band_row_range(st.r0 - 1, st.nx, st.ny, a.bw, l64, h64);
        plo = static_cast<int>(l64);
        phi = static_cast<int>(h64);
    }

#pragma unroll 1
    for (int q = 0; q < 3; ++q) {
        if (k0 + q <= kc) fwd_load_chunk<T>(a, Db, ring, k0 + q, st.rows, lane);
        cp_async_commit();
    }

    T outp = INF;
    T upp = (s == 0 && lane == 0) ? T(0) : INF;
    T* myrow = ring + lane * kRing;

    // Row above, lane `lane`'s column of the next block (prefetched one block ahead).
    T nv = INF;
    if (s > 0) {
        // lane 0's diagonal predecessor of column 32*k0 (column 32*k0 - 1 of the row above)
        const int cd = 32 * k0 - 1;
        const bool need_d = lane == 0 && cd >= plo && cd <= phi;
        T vd = need_d ? ld_relaxed(bnd_in + cd) : INF;
        if (!await_boundary(vd, bnd_in + cd, need_d, a.sy, lane)) return;
        if (lane == 0) upp = vd;
        const int c = 32 * k0 + lane;
        if (c >= plo && c <= phi) nv = ld_relaxed(bnd_in + c);
    }

#pragma unroll 1
    for (int blk = k0; blk <= k1; ++blk) {
        const int tau0 = 32 * blk;
        cp_async_wait<2>();
        __syncwarp();
        const bool full = tau0 >= st.Amax && tau0 + 31 <= st.Zmin;
        constexpr int G = FwdGroup<T>::value;
        if (!(full ? fwd_block_groups<T, false, G>(a, ring, top, bnd_in, bnd_out, tau0, st, plo, phi, s > 0,
                                                    has_consumer, lane, nv, outp, upp)
                   : fwd_block_groups<T, true, G>(a, ring, top, bnd_in, bnd_out, tau0, st, plo, phi, s > 0,
                                                   has_consumer, lane, nv, outp, upp)))
            return;
        if (blk - 1 >= k0) fwd_store_chunk<T>(a, Rb, ring, blk - 1, st, lane);
        __syncwarp();
        if (blk + 3 <= kc) fwd_load_chunk<T>(a, Db, ring, blk + 3, st.rows, lane);
        cp_async_commit();
    }
    cp_async_wait<0>();
    __syncwarp();
    if (kc == k1) fwd_store_chunk<T>(a, Rb, ring, kc, st, lane);
    if (st.nx - 1 - st.r0 == lane) a.costs[b] = ring[lane * kRing + ((st.ny - 1) & kRingMask)];
    __syncwarp();
}

// Warps per CTA of the strip-ticket forward (independent warps, as in the backward): fp64 6, the most
// whose rings fit one SM (4-warp CTAs fit once: 4 warps per SM); fp32 4, two CTAs per SM.
template <typename T>
struct FwdWarps {
    static constexpr int value = sizeof(T) == 8 ? 6 : kWarpsPerCta;
};

template <typename T>
__global__ void __launch_bounds__(FwdWarps<T>::value * 32) sdtw_fwd_kernel(FwdArgs<T> a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    T* ring = reinterpret_cast<T*>(smem) + static_cast<size_t>(warp) * (32 * kRing + kSide);
    T* top = ring + 32 * kRing;
    for (int e = lane; e < 32 * kRing + kSide; e += 32) ring[e] = T(0);
    __syncwarp();
    const int64_t total = a.B * a.S;
    while (true) {
        int tk = 0;
        if (lane == 0) tk = aborted(a.sy) ? static_cast<int>(total) : atomicAdd(a.ticket, 1);
        tk = __shfl_sync(kFull, tk, 0);
        if (tk >= total) break;
        const int s = static_cast<int>(tk / a.B);
        const int64_t b = tk % a.B;
        fwd_strip<T>(a, ring, top, b, s, lane, tk == a.inject_skip);
    }
}

// R <- +inf everywhere, R[:, 0, 0] <- 0 (softdtw.cpp:114-121).
template <typename T>
__global__ void sdtw_fill_r_kernel(T* R, int64_t total, int64_t slab)
{
    const T INF = Num<T>::inf();
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x)
        R[e] = (e % slab == 0) ? T(0) : INF;
}

// The part of R the strip-ticket backward reads, set to +inf (R[b, 0, 0] to 0), for an R that only that
// backward reads: for strip s of pair b, the padded rows r0 .. r0 + rows (D rows r0 - 1 .. r0 + rows - 1) over
// the 32-column chunks bwd_load_chunk loads, D columns [32 kmin, 32 k1 + 31] with kmin = (c_begin - 1) >> 5,
// k1 = (c_end + 31) >> 5, clipped to the padding. The forward then writes its swept cells over it. One CTA
// per strip; strips without cells (past the length, empty or invalid pairs) are not read and not filled.
template <typename T>
__global__ void sdtw_fill_r_band_kernel(T* R, Lengths len, int64_t N, int64_t M, int64_t bw, int S)
{
    const T INF = Num<T>::inf();
    const int64_t b = blockIdx.x / S;
    const int s = static_cast<int>(blockIdx.x % S);
    const int64_t nx = len.x(b), ny = len.y(b);
    if (nx <= 0 || nx > N || ny <= 0 || ny > M) return;
    const int64_t r0 = 32 * static_cast<int64_t>(s);
    if (r0 >= nx) return;
    const int64_t rows = nx - r0 < 32 ? nx - r0 : 32;
    int64_t lo, hi, lo1, hi1;
    band_row_range(r0, nx, ny, bw, lo, hi);
    band_row_range(r0 + rows - 1, nx, ny, bw, lo1, hi1);
    const int64_t kmin = floor_div(lo - 1, 32), k1 = (hi1 + 31) >> 5;
    const int64_t p0 = 32 * kmin + 1 > 0 ? 32 * kmin + 1 : 0;       // padded columns [p0, p1]
    const int64_t p1 = 32 * k1 + 32 < M + 1 ? 32 * k1 + 32 : M + 1;
    const int64_t pitch = M + 2;
    T* Rb = R + b * (N + 2) * pitch;
    for (int64_t r = r0; r <= r0 + rows; ++r)
        for (int64_t c = p0 + threadIdx.x; c <= p1; c += blockDim.x) Rb[r * pitch + c] = (r == 0 && c == 0) ? T(0) : INF;
}

// ==================================================================================================
// Backward
// ==================================================================================================
template <typename T>
struct BwdArgs {
    const T* R;
    T* E;
    T* bnd;  // (B, S, M): contributions pushed from the first row of strip s+1 into the last row of strip s
    Lengths len;
    int* ticket;
    int64_t B, N, M, bw;
    int S;
    T k;
    Sync sy;
    int inject_skip;
};

// The 8 backward steps tau = tau0 + 8Q + 7 down to tau0 + 8Q of one warp (group Q of the block at tau0). The
// group's R values and lane 31's contributions are read from shared memory first and its E values and lane 0's
// pushes written after (every position it reads is read before the group would overwrite it: step u reads
// column c - 1 = base + u - 1, which step u - 1 overwrites later), so a step's dependency chain holds the
// shuffle from the row below and no other shared-memory operation (fp32, 16 pairs of 4096 x 4096, band 256:
// 1.25 ms against 1.35 with the accesses step by step).
template <typename T, bool MASKED, int Q>
__device__ __forceinline__ void bwd_group(T* rowA, T* rowB, const T* bndring, T* sendring, int tau0, int lane, int A,
                                          int Z, T k, T seed, T& upc, T& sendv, T& pend, T& acc)
{
    const T big = Num<T>::big();
    const int src = (lane + 1) & 31;
    const bool lane31 = lane == 31;
    const bool lane0 = lane == 0;
    const int base = tau0 - lane + 8 * Q;
    // Boundary values of lane 31's column c live at (c + 31) & 63, so a block reads them without wrapping.
    const T* bndb = bndring + (tau0 & kSideMask) + 8 * Q;
    T ra[8], rb[8], bv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        ra[j] = rowA[(base + j - 1) & kRingMask];  // R[i-1][c-1]
        rb[j] = rowB[(base + j - 1) & kRingMask];  // R[i][c-1]
        bv[j] = bndb[j];                           // column tau0 + 8Q + j - 31
    }
#pragma unroll
    for (int j = 7; j >= 0; --j) {
        const T rd = ra[j];
        const T rl = rb[j];
        const T ru = upc;  // R[i-1][c]
        const T recvw = __shfl_sync(kFull, sendv, src);
        const T recv = lane31 ? bv[j] : recvw;
        const T Es = acc + recv;
        const T m = Num<T>::mn(Num<T>::mn(rd, ru), rl);
        const T mc = Num<T>::mn(m, big);
        const T ed = Num<T>::exp2_((mc - rd) * k);
        const T eu = Num<T>::exp2_((mc - ru) * k);
        const T el = Num<T>::exp2_((mc - rl) * k);
        T q = Es * Num<T>::rcp_((ed + eu) + el);
        T Eo = Es;
        if (MASKED) {
            const int tau = tau0 + 8 * Q + j;
            const bool valid = tau >= A && tau <= Z;
            q = valid ? q : T(0);
            acc = valid ? q * el : seed;
            Eo = valid ? Es : T(0);
        } else {
            acc = q * el;
        }
        sendv = fma(q, eu, pend);
        pend = q * ed;
        rb[j] = Eo;     // E[i][c], written back below
        bv[j] = sendv;  // lane 0's push into column c of the row above
        upc = rd;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) rowB[(base + j) & kRingMask] = rb[j];
    if (lane0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) sendring[(base + j) & kSideMask] = bv[j];
    }
}

// R chunk kk (padded rows r0 .. r0+rows, D-columns [32kk, 32kk+32)) -> ring rows 0..rows. M is a
// compile-time constant in the kernels specialized on it (immediate row offsets in the full-strip case).
template <typename T>
__device__ __forceinline__ void bwd_load_chunk(int64_t M, const T* Rb, T* ring, int kk, int r0, int rows, int lane)
{
    const int64_t pitch = M + 2;
    const int c = 32 * kk + lane;  // D-column; padded column c+1 exists for -1 <= c <= M
    const bool in = c >= -1 && c <= M;
    const T* src = Rb + static_cast<int64_t>(r0) * pitch + (in ? c + 1 : 0);
    T* dst = ring + (c & kRingMask);
    const int bytes = in ? static_cast<int>(sizeof(T)) : 0;
    if (rows == 32) {
#pragma unroll
        for (int q = 0; q <= 32; ++q) cp_async_scalar<sizeof(T)>(dst + q * kRing, src + q * pitch, bytes);
    } else {
        for (int q = 0; q <= rows; ++q) cp_async_scalar<sizeof(T)>(dst + q * kRing, src + q * pitch, bytes);
    }
}

template <typename T>
__device__ __forceinline__ void bwd_store_chunk(int64_t M, T* Eb, const T* ring, int kk, const Strip& st, int lane)
{
    const int col = 32 * kk + lane;
    if (col < st.c_begin || col > st.c_end) return;
    T* dst = Eb + static_cast<int64_t>(st.r0) * M + col;
    const T* srcp = ring + kRing + (col & kRingMask);
    if (st.rows == 32) {
#pragma unroll
        for (int r = 0; r < 32; ++r) dst[r * M] = srcp[r * kRing];
    } else {
        for (int r = 0; r < st.rows; ++r) dst[r * M] = srcp[r * kRing];
    }
}

// Column c of the row below's boundary (the contributions its first row pushes into this strip's last row)
// is written by the strip below.
__device__ __forceinline__ bool bwd_needed(int c, bool has_producer, int plo, int phi)
{
    return has_producer && c >= 0 && c >= plo - 1 && c <= phi;
}

// One block of 32 backward steps as four groups of 8, taken from the last (Q = 3) to the first. Lane l holds
// in `nv` the contribution into lane 31's column tau0 - 31 + l, read from L2 ahead of time. Before group q the
// lanes of that group wait for their values, hand them to the side ring and read their column of the next
// block ahead, and the lanes of the group after it re-read theirs; after the group, 8 lanes publish lane 0's
// pushes into the row above for the 8 columns the group finished (the lag between strips is 40 steps instead
// of 64 with whole blocks: fp32, 16 pairs of 4096 x 4096, band 256, measured on one B200 at 1.35 ms against
// 1.60). Returns false if the launch aborted.
template <typename T, bool MASKED, int Q>
__device__ __forceinline__ bool bwd_group_step(const BwdArgs<T>& a, T* rowA, T* rowB, T* bndring, T* sendring,
                                               const T* bnd_in, T* bnd_out, int tau0, const Strip& st, int hi0,
                                               bool has_producer, bool has_consumer, int plo, int phi, int lane,
                                               T seed, T& nv, T& upc, T& sendv, T& pend, T& acc)
{
    const int grp = lane >> 3;
    const int c = tau0 - 31 + lane;
    const bool need = bwd_needed(c, has_producer, plo, phi);
    if (!await_boundary(nv, bnd_in + c, need && grp == Q, a.sy, lane)) return false;
    if (grp == Q) {
        bndring[(c + 31) & kSideMask] = need ? nv : T(0);
        const int cn = c - 32;
        nv = bwd_needed(cn, has_producer, plo, phi) ? ld_relaxed(bnd_in + cn) : T(0);
    } else if (grp == ((Q + 3) & 3)) {
        const int cr = Q == 0 ? c - 32 : c;  // after the last group: the next block's first group
        if (bwd_needed(cr, has_producer, plo, phi)) nv = ld_relaxed(bnd_in + cr);
    }
    __syncwarp();
    bwd_group<T, MASKED, Q>(rowA, rowB, bndring, sendring, tau0, lane, st.A, st.Z, a.k, seed, upc, sendv, pend, acc);
    __syncwarp();
    if (has_consumer && lane < 8) {
        // Lane 0 finished its pushes into row r0-1 for columns [tau0 + 8Q, tau0 + 8Q + 7].
        const int cp = tau0 + 8 * Q + lane;
        if (cp >= 0 && cp >= st.c_begin - 1 && cp <= hi0) st_relaxed(bnd_out + cp, sendring[cp & kSideMask]);
    }
    return true;
}
template <typename T, bool MASKED>
__device__ __forceinline__ bool bwd_block_groups(const BwdArgs<T>& a, T* rowA, T* rowB, T* bndring, T* sendring,
                                                 const T* bnd_in, T* bnd_out, int tau0, const Strip& st, int hi0,
                                                 bool has_producer, bool has_consumer, int plo, int phi, int lane,
                                                 T seed, T& nv, T& upc, T& sendv, T& pend, T& acc)
{
    return bwd_group_step<T, MASKED, 3>(a, rowA, rowB, bndring, sendring, bnd_in, bnd_out, tau0, st, hi0,
                                        has_producer, has_consumer, plo, phi, lane, seed, nv, upc, sendv, pend, acc) &&
           bwd_group_step<T, MASKED, 2>(a, rowA, rowB, bndring, sendring, bnd_in, bnd_out, tau0, st, hi0,
                                        has_producer, has_consumer, plo, phi, lane, seed, nv, upc, sendv, pend, acc) &&
           bwd_group_step<T, MASKED, 1>(a, rowA, rowB, bndring, sendring, bnd_in, bnd_out, tau0, st, hi0,
                                        has_producer, has_consumer, plo, phi, lane, seed, nv, upc, sendv, pend, acc) &&
           bwd_group_step<T, MASKED, 0>(a, rowA, rowB, bndring, sendring, bnd_in, bnd_out, tau0, st, hi0,
                                        has_producer, has_consumer, plo, phi, lane, seed, nv, upc, sendv, pend, acc);
}

template <typename T, int MC>
__device__ void bwd_strip(const BwdArgs<T>& a, T* ring, T* bndring, T* sendring, int64_t b, int s, int lane,
                          bool skip_publish)
{
    const int64_t M = MC > 0 ? MC : a.M;
    Strip st;
    T* Eb = a.E + b * a.N * M;
    const int nmat = static_cast<int>(a.N - 32 * s < 32 ? a.N - 32 * s : 32);  // rows of E this strip owns
    if (!make_strip(st, a.len, b, s, a.N, M, a.bw, lane)) {
        if (st.bad && s == 0 && lane == 0) atomicOr(a.sy.err, kErrBadLength);
        T* row0 = Eb + static_cast<int64_t>(32 * s) * M;
        for (int r = 0; r < nmat; ++r)
            for (int c = lane; c < M; c += 32) row0[r * M + c] = T(0);
        return;
    }
    // E is written in full: zeros outside the swept columns [c_begin, c_end] and in rows past the length.
    for (int r = 0; r < nmat; ++r) {
        T* row = Eb + static_cast<int64_t>(st.r0 + r) * M;
        const int lo = r < st.rows ? st.c_begin : static_cast<int>(M);
        const int hi = r < st.rows ? st.c_end : static_cast<int>(M);
        for (int c = lane; c < lo; c += 32) row[c] = T(0);
        for (int c = hi + 1 + lane; c < M; c += 32) row[c] = T(0);
    }
    const int64_t pitch = M + 2;
    const T* Rb = a.R + b * (a.N + 2) * pitch;
    const int k0 = st.c_begin >> 5;
    const int k1 = (st.c_end + 31) >> 5;
    const int kmin = (st.c_begin - 1) >> 5;  // arithmetic shift: -1 when c_begin == 0
    const bool has_producer = st.r0 + 32 < st.nx;
    const bool has_consumer = s > 0 && !skip_publish;
    int plo = 0, phi = -1;  // the producer's first row (row r0+32) pushes into columns [plo-1, phi]
    if (has_producer) {
        int64_t l64, h64;
        band_row_range(st.r0 + 32, st.nx, st.ny, a.bw, l64, h64);
        plo = static_cast<int>(l64);
        phi = static_cast<int>(h64);
    }
    const T* bnd_in = a.bnd + (b * a.S + s) * M;
    T* bnd_out = a.bnd + (b * a.S + (s - 1)) * M;
    // Terminal cell (nx-1, ny-1): E = 1 (the reference's sentinel, softdtw.cpp:225-227). Masked steps of
    // the terminal row leave `acc` = seed, so its first valid cell (column ny-1) starts from 1.
    const T seed = (st.r0 + lane == st.nx - 1) ? T(1) : T(0);
    const int hi0 = __shfl_sync(kFull, st.hi, 0);

#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
        if (k1 - q >= kmin) bwd_load_chunk<T>(M, Rb, ring, k1 - q, st.r0, st.rows, lane);
        cp_async_commit();
    }

    T* rowA = ring + lane * kRing;
    T* rowB = rowA + kRing;
    T upc = T(0), sendv = T(0), pend = T(0), acc = seed;

    // Contributions from the row below into lane 31's columns of the next block, prefetched.
    T nv = T(0);
    {
        const int c = 32 * k1 - 31 + lane;
        if (bwd_needed(c, has_producer, plo, phi)) nv = ld_relaxed(bnd_in + c);
    }

#pragma unroll 1
    for (int blk = k1; blk >= k0; --blk) {
        const int tau0 = 32 * blk;
        cp_async_wait<2>();
        __syncwarp();
        if (blk == k1) upc = rowA[(tau0 + 31 - lane) & kRingMask];
        const bool full = tau0 >= st.Amax && tau0 + 31 <= st.Zmin;
        if (!(full ? bwd_block_groups<T, false>(a, rowA, rowB, bndring, sendring, bnd_in, bnd_out, tau0, st, hi0,
                                                 has_producer, has_consumer, plo, phi, lane, seed, nv, upc, sendv,
                                                 pend, acc)
                   : bwd_block_groups<T, true>(a, rowA, rowB, bndring, sendring, bnd_in, bnd_out, tau0, st, hi0,
                                                has_producer, has_consumer, plo, phi, lane, seed, nv, upc, sendv,
                                                pend, acc)))
            return;
        bwd_store_chunk<T>(M, Eb, ring, blk, st, lane);
        __syncwarp();
        if (blk - 4 >= kmin) bwd_load_chunk<T>(M, Rb, ring, blk - 4, st.r0, st.rows, lane);
        cp_async_commit();
    }
    cp_async_wait<0>();
    // When the sweep starts exactly at a chunk boundary, lane 0's last diagonal push (into column
    // c_begin-1 of the row above) was never followed by another step: write it out now.
    if (has_consumer && lane == 0 && st.c_begin == 32 * k0 && st.c_begin >= 1) st_relaxed(bnd_out + st.c_begin - 1, pend);
    __syncwarp();
}

// Warps per CTA of the strip-ticket backward (its warps share nothing but the ticket counter). fp64: 6,
// the most whose rings fit one SM's 227 KB (4-warp CTAs fit once: 4 warps per SM); the fp64 backward of
// 65536 x 64 x 64 pairs takes 10.3 ms instead of 14.8. fp32: 4, three CTAs per SM (12 warps); one
// 13-warp CTA per SM measured slower on the headline workload (288 us against 279).
template <typename T>
struct BwdWarps {
    static constexpr int value = sizeof(T) == 8 ? 6 : kWarpsPerCta;
};
template <typename T>
constexpr int bwd_warps()
{
    return BwdWarps<T>::value;
}

template <typename T, int MC>
__global__ void __launch_bounds__(BwdWarps<T>::value * 32) sdtw_bwd_kernel(BwdArgs<T> a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    constexpr int per_warp = 33 * kRing + 2 * kSide;
    T* ring = reinterpret_cast<T*>(smem) + static_cast<size_t>(warp) * per_warp;
    T* bndring = ring + 33 * kRing;
    T* sendring = bndring + kSide;
    for (int e = lane; e < per_warp; e += 32) ring[e] = T(0);
    __syncwarp();
    const int64_t total = a.B * a.S;
    while (true) {
        int tk = 0;
        if (lane == 0) tk = aborted(a.sy) ? static_cast<int>(total) : atomicAdd(a.ticket, 1);
        tk = __shfl_sync(kFull, tk, 0);
        if (tk >= total) break;
        const int s = a.S - 1 - static_cast<int>(tk / a.B);
        const int64_t b = tk % a.B;
        bwd_strip<T, MC>(a, ring, bndring, sendring, b, s, lane, tk == a.inject_skip);
    }
}

// ==================================================================================================
// Host side
// ==================================================================================================
std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// Scratch of sdtw_forward_noalloc: one forward's workspace (launch header + strip boundary rows) as a
// file-scope device array, so that the call allocates nothing. Its device address is looked up once per
// device (cudaGetSymbolAddress) on the first call.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SDTW_NOALLOC_SCRATCH_BYTES];

namespace {
double g_timeout_s = 2.0;
}  // namespace
double wait_timeout_s() { return g_timeout_s; }

namespace {

int g_inject_skip = -1;  // set only through sdtw_debug_inject_stall (tests of the failure path)
int g_force_path = 0;    // 0: automatic, 1: strip-ticket kernels, 2: pair-resident kernels, 3: warp-per-pair
int g_pair_warps = kPairMaxWarps;  // warps per CTA of the pair-resident kernels (upper bound)

// E[b, i, c] = 0 where bit c % 32 of clamp_mask[(b N + i) MW + c / 32] is set, in pairs whose clamp flag is
// set (one CTA per pair; the others return at once). The fused forward's clamp record applied to the
// backward's E, so that the gradient kernels see the clamp of the cost matrix already folded in.
__global__ void sdtw_clamp_mask_kernel(float* E, const uint32_t* clamp_mask, const int* clamp_flags, int64_t N,
                                       int64_t M)
{
    const int64_t b = blockIdx.x;
    if (clamp_flags[b] == 0) return;
    const int64_t MW = (M + 31) / 32;
    const uint32_t* mb = clamp_mask + b * N * MW;
    for (int64_t w = threadIdx.x; w < N * MW; w += blockDim.x) {
        uint32_t bits = mb[w];
        const int64_t i = w / MW, c0 = (w % MW) * 32;
        while (bits != 0) {
            const int k = __ffs(static_cast<int>(bits)) - 1;
            bits &= bits - 1;
            if (c0 + k < M) E[(b * N + i) * M + c0 + k] = 0.f;
        }
    }
}

struct DeviceInfo {
    bool ready = false;
    int sms = 0;
    int max_smem = 0;  // opt-in dynamic shared memory per CTA
    int sm_smem = 0;   // shared memory per SM
    int sm_regs = 0;   // 32-bit registers per SM
    int pair_regs[2][2] = {{0, 0}, {0, 0}};  // [fp64][backward]: registers per thread of the pair kernels
    int occ_fwd[2] = {0, 0};
    int occ_bwd[2] = {0, 0};
};
std::mutex g_mu;
DeviceInfo g_dev[128];

template <typename T>
constexpr size_t fwd_smem_bytes()
{
    return static_cast<size_t>(FwdWarps<T>::value) * (32 * kRing + kSide) * sizeof(T);
}
template <typename T>
constexpr size_t bwd_smem_bytes()
{
    return static_cast<size_t>(bwd_warps<T>()) * (33 * kRing + 2 * kSide) * sizeof(T);
}

template <typename T>
cudaError_t init_kernel_attrs(int& occ_f, int& occ_b)
{
    cudaError_t e = cudaFuncSetAttribute(sdtw_fwd_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(fwd_smem_bytes<T>()));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(sdtw_bwd_kernel<T, kPairSpecialM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(bwd_smem_bytes<T>()));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(sdtw_bwd_kernel<T, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(bwd_smem_bytes<T>()));
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_f, sdtw_fwd_kernel<T>, FwdWarps<T>::value * 32,
                                                      fwd_smem_bytes<T>());
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_b, sdtw_bwd_kernel<T, 0>, bwd_warps<T>() * 32,
                                                         bwd_smem_bytes<T>());
}

cudaError_t device_info(const DeviceInfo*& out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceInfo& di = g_dev[dev];
    if (!di.ready) {
        e = cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&di.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&di.sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&di.sm_regs, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
        if (e != cudaSuccess) return e;
        e = pair_init_attrs<float>(di.max_smem);
        if (e != cudaSuccess) return e;
        e = pair_init_attrs<double>(di.max_smem);
        if (e != cudaSuccess) return e;
        for (int bwd = 0; bwd < 2; ++bwd) {
            e = pair_regs<float>(bwd != 0, di.pair_regs[0][bwd]);
            if (e != cudaSuccess) return e;
            e = pair_regs<double>(bwd != 0, di.pair_regs[1][bwd]);
            if (e != cudaSuccess) return e;
        }
        e = init_kernel_attrs<float>(di.occ_fwd[0], di.occ_bwd[0]);
        if (e != cudaSuccess) return e;
        e = init_kernel_attrs<double>(di.occ_fwd[1], di.occ_bwd[1]);
        if (e != cudaSuccess) return e;
        di.ready = true;
    }
    out = &di;
    return cudaSuccess;
}

constexpr size_t kHeader = 256;  // ticket, abort word
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline int64_t strips_of(int64_t N) { return N > 0 ? (N + 31) / 32 : 1; }
// Boundary buffer: one row of M values per strip.
inline size_t bnd_bytes(int64_t B, int64_t N, int64_t M, size_t es)
{
    return align_up(static_cast<size_t>(B * strips_of(N) * M) * es, 256);
}
inline size_t elem_size(sdtw_dtype t) { return t == SDTW_F64 ? 8 : 4; }

inline sdtw_status from_cuda(cudaError_t e) { return e == cudaSuccess ? SDTW_OK : static_cast<sdtw_status>(e); }

// A bandwidth beyond N+M admits every cell, exactly like an unconstrained band; clamping keeps the
// integer band arithmetic far from overflow.
inline int64_t clamp_bw(int64_t bw, int64_t N, int64_t M) { return bw > N + M ? N + M : bw; }

bool common_args_ok(int64_t B, int64_t N, int64_t M, double gamma)
{
    if (B < 0 || N < 0 || M < 0) return false;
    if (!(gamma > 0.0) || !std::isfinite(gamma)) return false;
    if (N > (1 << 29) || M > (1 << 29)) return false;
    if (B * strips_of(N) >= (int64_t(1) << 31)) return false;
    return true;
}

Sync make_sync(void* workspace, uint32_t* err_word)
{
    Sync sy;
    sy.err = err_word;
    sy.abort = reinterpret_cast<int*>(static_cast<char*>(workspace) + 4);
    sy.timeout_ns = static_cast<uint64_t>(g_timeout_s * 1e9);
    return sy;
}

// Pair-resident kernels (one CTA per pair) when the batch fills the GPU and a CTA fits in shared
// memory; otherwise the strip-ticket kernels, which spread a few long pairs over every SM. Returns the
// pair kernels' warps per CTA, or 0 for the strip-ticket kernels.
template <typename T>
int choose_pair_warps(const DeviceInfo& di, bool backward, int64_t B, int64_t N, int64_t M)
{
    if (g_force_path == 1) return 0;
    // Measured on B200, fp32, forward op (pair-resident / strip-ticket): 256 x 512 x 512 0.230 / 0.313 ms,
    // 512 x 256 x 256 0.148 / 0.172, 512 x 192 x 192 0.109 / 0.118, 1024 x 160 x 160 0.150 / 0.137,
    // 65536 x 64 x 64 2.08 / 1.30; backward op at 256 x 512 x 512: 0.243 / 0.272 ms. Both directions switch
    // together (the module path then hands R over as tiles), for pairs of at least 6 strips. Batches smaller
    // than the SM count stay on the pair-resident kernels while one warp per strip fits a CTA (at most 16
    // strips): every strip of a pair then runs at once and a pair takes its dependency chain's time, where the
    // strip-ticket kernels' coarser hand-over through L2 makes the chain longer (128 x 512 x 512 forward:
    // strip-ticket 0.233 ms).
    // Pairs of more than 16 strips in batches smaller than the SM count: the pair-resident kernels sweep the
    // strips in rounds on one SM per pair and still win while the boundary rows leave room for enough warps
    // (fp32, forward / backward, pair-resident against strip-ticket: 64 x 768 x 768 0.258 / 0.231 against
    // 0.326 / 0.326 ms; 16 x 2048 x 2048 band 128 0.613 / 0.590 against 0.736 / 0.743; 32 x 1024 x 1024
    // 0.412 / 0.378 against 0.389 / 0.395); with 128 strips of 4096 columns the strip-ticket kernels spread
    // the work over every SM and are faster (16 x 4096 x 4096 band 256: 2.20 / 2.64 against 1.63 / 1.59 ms).
    // (fp64 rings and rows are twice the size: those batches stay on the strip-ticket kernels.)
    const bool many_strips =
        B < di.sms && strips_of(N) > kPairMaxWarps && (strips_of(N) > 64 || M > 2048 || sizeof(T) == 8);
    if (g_force_path != 2 && (many_strips || strips_of(N) < 6)) return 0;
    if (B > 0x7fffffff || !pair_keys_fit(N, M)) return 0;
    // Enough CTAs per SM for the whole batch to be resident at once (up to 8), each as wide as its
    // share of the SM's shared memory and registers allows.
    const int64_t want = std::min<int64_t>(8, std::max<int64_t>(1, (B + di.sms - 1) / di.sms));
    const size_t share = static_cast<size_t>(di.sm_smem) / static_cast<size_t>(want);
    const size_t budget = std::min<size_t>(static_cast<size_t>(di.max_smem), share > 1024 ? share - 1024 : 0);
    const int regs = std::max(1, di.pair_regs[sizeof(T) == 8 ? 1 : 0][backward ? 1 : 0]);
    const int reg_warps = static_cast<int>(di.sm_regs / (want * 32 * regs));
    const int W = pair_warps<T>(backward, N, M, std::min(g_pair_warps, std::max(1, reg_warps)), budget);
    return W > 0 ? W : pair_warps<T>(backward, N, M, g_pair_warps, static_cast<size_t>(di.max_smem));
}

// Warp-per-pair kernels for large fp64 batches of short pairs (at most 4 strips): one warp per pair and no
// shared-memory rings, so an SM holds as many warps as its registers allow. Measured on B200, forward /
// backward op in ms:
//   fp64 65536 x 64 x 64: warp-per-pair 4.62 / 4.55, strip-ticket 11.1 / 10.2, pair-resident 7.61 / 15.0
//   fp64 2048 x 128 x 128: 0.60 / 0.68, 1.29 / 1.08, 0.92 / 2.06
//   fp32 65536 x 64 x 64: 2.43 / 2.31, strip-ticket 1.30 / 1.44 (fp32 stays on the strip-ticket kernels)
// Forced with path 3 whenever the row buffers fit.
template <typename T>
bool use_warp_kernels(const DeviceInfo& di, int64_t B, int64_t N, int64_t M)
{
    const bool fits = warp_fwd_smem_bytes<T>(M) <= 48 * 1024 && warp_bwd_smem_bytes<T>(M) <= 48 * 1024;
    if (!fits || g_force_path == 1 || g_force_path == 2) return false;
    if (g_force_path == 3) return true;
    return sizeof(T) == 8 && strips_of(N) <= 4 && B >= 8 * static_cast<int64_t>(di.sms);
}

// Workspace bytes the forward kernel chosen for this shape needs: the header alone for the warp-per-pair
// and pair-resident kernels, the header and the strip boundary rows for the strip-ticket kernels.
template <typename T>
size_t forward_ws_needed(const DeviceInfo& di, int64_t B, int64_t N, int64_t M)
{
    if (use_warp_kernels<T>(di, B, N, M) || choose_pair_warps<T>(di, false, B, N, M) > 0) return kHeader;
    return kHeader + bnd_bytes(B, N, M, sizeof(T));
}

// True when both directions run on the pair-resident kernels for this shape (the module path then keeps R
// as the forward's strip tiles).
template <typename T>
bool uses_tiles(const DeviceInfo& di, int64_t B, int64_t N, int64_t M)
{
    if (use_warp_kernels<T>(di, B, N, M)) return false;
    return choose_pair_warps<T>(di, false, B, N, M) > 0 && choose_pair_warps<T>(di, true, B, N, M) > 0;
}

// Rt non-null: the forward writes R as strip tiles (only when uses_tiles; R unused), else the padded R.
template <typename T>
sdtw_status launch_forward(const void* D, int64_t B, int64_t N, int64_t M, const void* lx, const void* ly, int is32,
                           double gamma, int64_t bw, void* R, void* costs, void* ws, uint32_t* err,
                           cudaStream_t stream, void* Rt = nullptr, bool band_r = false)
{
    const DeviceInfo* di = nullptr;
    cudaError_t e = device_info(di);
    if (e != cudaSuccess) return from_cuda(e);
    // Every cost starts as NaN (all-ones bits): a pair whose strips never finish (a launch that aborted on
    // a wait timeout) then reads as NaN even when nobody checks the error word.
    e = cudaMemsetAsync(costs, 0xff, static_cast<size_t>(B) * sizeof(T), stream);
    if (e != cudaSuccess) return from_cuda(e);
    if (Rt != nullptr && !uses_tiles<T>(*di, B, N, M)) return SDTW_EINVAL;
    if (use_warp_kernels<T>(*di, B, N, M))
        return from_cuda(warp_forward<T>(static_cast<const T*>(D), static_cast<T*>(R), static_cast<T*>(costs), lx, ly,
                                         is32, B, N, M, clamp_bw(bw, N, M), gamma, err, stream));
    const int64_t S = strips_of(N);
    e = cudaMemsetAsync(ws, 0, kHeader, stream);
    if (e != cudaSuccess) return from_cuda(e);
    const int W = choose_pair_warps<T>(*di, false, B, N, M);
    if (Rt != nullptr && W == 0) return SDTW_EINVAL;  // tiles exist only between the pair-resident kernels
    if (W > 0)
        return from_cuda(pair_forward<T>(static_cast<const T*>(D), static_cast<T*>(R), static_cast<T*>(Rt),
                                         static_cast<T*>(costs), lx, ly, is32, B, N, M, clamp_bw(bw, N, M), gamma, W,
                                         make_sync(ws, err), g_inject_skip, stream));
    e = cudaMemsetAsync(static_cast<char*>(ws) + kHeader, 0xff, bnd_bytes(B, N, M, sizeof(T)), stream);
    if (e != cudaSuccess) return from_cuda(e);
    const int64_t slab = (N + 2) * (M + 2);
    if (band_r && !use_warp_kernels<T>(*di, B, N, M) && choose_pair_warps<T>(*di, true, B, N, M) == 0) {
        // R for the strip-ticket backward alone: only the chunks it loads.
        count_launch();
        sdtw_fill_r_band_kernel<T><<<static_cast<unsigned>(B * S), 256, 0, stream>>>(
            static_cast<T*>(R), Lengths{lx, ly, is32}, N, M, clamp_bw(bw, N, M), static_cast<int>(S));
    } else {
        const int64_t total = B * slab;
        const int threads = 256;
        const int64_t want = (total + threads - 1) / threads;
        const int blocks = static_cast<int>(std::min<int64_t>(want, int64_t(di->sms) * 16));
        count_launch();
        sdtw_fill_r_kernel<T><<<std::max(blocks, 1), threads, 0, stream>>>(static_cast<T*>(R), total, slab);
    }
    FwdArgs<T> a;
    a.D = static_cast<const T*>(D);
    a.R = static_cast<T*>(R);
    a.costs = static_cast<T*>(costs);
    a.len = Lengths{lx, ly, is32};
    a.ticket = reinterpret_cast<int*>(ws);
    a.bnd = reinterpret_cast<T*>(static_cast<char*>(ws) + kHeader);
    a.B = B;
    a.N = N;
    a.M = M;
    a.bw = clamp_bw(bw, N, M);
    a.S = static_cast<int>(S);
    a.k = static_cast<T>(1.4426950408889634 / gamma);
    a.gl = static_cast<T>(gamma * 0.6931471805599453);
    a.sy = make_sync(ws, err);
    a.inject_skip = g_inject_skip;
    a.vec = (M % (16 / sizeof(T)) == 0) && (reinterpret_cast<uintptr_t>(D) % 16 == 0);
    const int occ = di->occ_fwd[sizeof(T) == 8 ? 1 : 0];
    constexpr int FW = FwdWarps<T>::value;
    const int64_t ctas_needed = (B * S + FW - 1) / FW;
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ctas_needed, int64_t(di->sms) * std::max(occ, 1))));
    count_launch();
    sdtw_fwd_kernel<T><<<grid, FW * 32, fwd_smem_bytes<T>(), stream>>>(a);
    return from_cuda(cudaGetLastError());
}

template <typename T>
sdtw_status launch_backward(const void* R, int64_t B, int64_t N, int64_t M, const void* lx, const void* ly, int is32,
                            double gamma, int64_t bw, void* E, void* ws, uint32_t* err, cudaStream_t stream,
                            const void* Rt = nullptr)
{
    const DeviceInfo* di = nullptr;
    cudaError_t e = device_info(di);
    if (e != cudaSuccess) return from_cuda(e);
    if (Rt != nullptr && !uses_tiles<T>(*di, B, N, M)) return SDTW_EINVAL;
    if (use_warp_kernels<T>(*di, B, N, M))
        return from_cuda(warp_backward<T>(static_cast<const T*>(R), static_cast<T*>(E), lx, ly, is32, B, N, M,
                                          clamp_bw(bw, N, M), gamma, err, stream));
    const int64_t S = strips_of(N);
    e = cudaMemsetAsync(ws, 0, kHeader, stream);
    if (e != cudaSuccess) return from_cuda(e);
    const int W = choose_pair_warps<T>(*di, true, B, N, M);
    if (Rt != nullptr && W == 0) return SDTW_EINVAL;
    if (W > 0)
        return from_cuda(pair_backward<T>(static_cast<const T*>(R), static_cast<const T*>(Rt), static_cast<T*>(E), lx,
                                          ly, is32, B, N, M,
                                          clamp_bw(bw, N, M), gamma, W, make_sync(ws, err), g_inject_skip, stream));
    e = cudaMemsetAsync(static_cast<char*>(ws) + kHeader, 0xff, bnd_bytes(B, N, M, sizeof(T)), stream);
    if (e != cudaSuccess) return from_cuda(e);
    BwdArgs<T> a;
    a.R = static_cast<const T*>(R);
    a.E = static_cast<T*>(E);
    a.bnd = reinterpret_cast<T*>(static_cast<char*>(ws) + kHeader);
    a.len = Lengths{lx, ly, is32};
    a.ticket = reinterpret_cast<int*>(ws);
    a.B = B;
    a.N = N;
    a.M = M;
    a.bw = clamp_bw(bw, N, M);
    a.S = static_cast<int>(S);
    a.k = static_cast<T>(1.4426950408889634 / gamma);
    a.sy = make_sync(ws, err);
    a.inject_skip = g_inject_skip;
    const int occ = di->occ_bwd[sizeof(T) == 8 ? 1 : 0];
    constexpr int BW = bwd_warps<T>();
    const int64_t ctas_needed = (B * S + BW - 1) / BW;
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ctas_needed, int64_t(di->sms) * std::max(occ, 1))));
    count_launch();
    if (M == kPairSpecialM)
        sdtw_bwd_kernel<T, kPairSpecialM><<<grid, BW * 32, bwd_smem_bytes<T>(), stream>>>(a);
    else
        sdtw_bwd_kernel<T, 0><<<grid, BW * 32, bwd_smem_bytes<T>(), stream>>>(a);
    return from_cuda(cudaGetLastError());
}

}  // namespace
}  // namespace sdtw

using namespace sdtw;

extern "C" {

const char* sdtw_status_string(sdtw_status status)
{
    switch (status) {
        case SDTW_OK: return "ok";
        case SDTW_EINVAL: return "invalid argument (size, pointer, gamma or bandwidth)";
        case SDTW_EDTYPE: return "unsupported dtype (expected SDTW_F32 or SDTW_F64)";
        case SDTW_EWORKSPACE: return "workspace missing or smaller than the *_workspace_bytes size";
        case SDTW_EDEVICE: return "no usable sm_100 device";
        case SDTW_ETOOLARGE:
            return "problem needs more scratch than sdtw_forward_noalloc's static scratch "
                   "(SDTW_NOALLOC_SCRATCH_BYTES); use sdtw_forward with a workspace";
        default: break;
    }
    if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
    return "unknown status";
}

void sdtw_band_row_range(int64_t i, int64_t nx, int64_t ny, int64_t bandwidth, int64_t* lo, int64_t* hi)
{
    int64_t l, h;
    band_row_range(i, nx, ny, clamp_bw(bandwidth, nx, ny), l, h);
    *lo = l;
    *hi = h;
}

int64_t sdtw_pair_cells(int64_t nx, int64_t ny, int64_t bandwidth)
{
    if (nx <= 0 || ny <= 0) return 0;
    int64_t total = 0;
    for (int64_t i = 0; i < nx; ++i) {
        int64_t l, h;
        band_row_range(i, nx, ny, clamp_bw(bandwidth, nx, ny), l, h);
        if (h >= l) total += h - l + 1;
    }
    return total;
}

uint32_t sdtw_read_error_word(uint32_t* err_word, void* stream)
{
    uint32_t v = 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&v, err_word, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess) return 0xffffffffu;
    if (cudaStreamSynchronize(s) != cudaSuccess) return 0xffffffffu;
    if (v != 0 && cudaMemsetAsync(err_word, 0, 4, s) != cudaSuccess) return 0xffffffffu;
    if (cudaStreamSynchronize(s) != cudaSuccess) return 0xffffffffu;
    // The tensor-core cost kernel has no caller error word: its timeouts live in the library's own device
    // word and are reported here as SDTW_ERR_TIMEOUT.
    uint32_t tc = 0;
    if (read_distance_errors(tc) != cudaSuccess) return 0xffffffffu;
    return v | (tc ? SDTW_ERR_TIMEOUT : 0u);
}

void sdtw_set_wait_timeout(double seconds)
{
    if (seconds > 0 && std::isfinite(seconds)) g_timeout_s = seconds;
}

/* Failure-path test hook (not in the public header's main API): the strip holding ticket `ticket` of
 * every following launch completes its cells but never writes its boundary row, so the strip after it
 * runs into the bounded wait. -1 switches it off. */
void sdtw_debug_inject_stall(int ticket) { g_inject_skip = ticket; }

/* Test and tuning hooks (not in the public header): `path` 0 chooses the kernels by shape, 1 forces the
 * strip-ticket kernels, 2 the pair-resident kernels (when a CTA fits), 3 the warp-per-pair kernels (when
 * their row buffers fit); `warps` caps the pair-resident
 * kernels' warps per CTA (1..16). With the pair-resident kernels, sdtw_debug_inject_stall's argument
 * names strip s of pair b as b * ceil(N/32) + s. */
/* Number of kernels this library has launched in this process (all entry points). */
uint64_t sdtw_debug_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

void sdtw_debug_force_path(int path) { g_force_path = (path >= 0 && path <= 3) ? path : 0; }
void sdtw_debug_set_pair_warps(int warps) { g_pair_warps = (warps >= 1 && warps <= kPairMaxWarps) ? warps : kPairMaxWarps; }

size_t sdtw_forward_workspace_bytes(int64_t B, int64_t N, int64_t M, sdtw_dtype dtype)
{
    if (B < 0 || N < 0 || M < 0) return 0;
    return kHeader + bnd_bytes(B, N, M, elem_size(dtype));
}

size_t sdtw_backward_workspace_bytes(int64_t B, int64_t N, int64_t M, sdtw_dtype dtype)
{
    if (B < 0 || N < 0 || M < 0) return 0;
    return kHeader + bnd_bytes(B, N, M, elem_size(dtype));
}

/* Forward for callers that cannot allocate device memory (see the header): the workspace is the static
 * device array g_noalloc_scratch. Every call looks the array's address up on the current device
 * (cudaGetSymbolAddress allocates nothing; the first lookup on a device may load this library's module
 * there), so the address is never stale, also after a cudaDeviceReset. The launch resets the scratch itself
 * (cudaMemsetAsync of the header to 0 and of the boundary rows to 0xFF), so its content between calls does
 * not matter. The size limit applies to the workspace of the kernel this shape runs on. */
sdtw_status sdtw_forward_noalloc(sdtw_dtype dtype, const void* D, int64_t B, int64_t N, int64_t M,
                                 const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                                 int64_t bandwidth, void* R, void* costs, uint32_t* err_word, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!common_args_ok(B, N, M, gamma)) return SDTW_EINVAL;
    if (B == 0) return SDTW_OK;
    if (!lengths_x || !lengths_y || !R || !costs || !err_word || (N * M > 0 && !D)) return SDTW_EINVAL;
    const DeviceInfo* di = nullptr;
    cudaError_t e = device_info(di);
    if (e != cudaSuccess) return from_cuda(e);
    const size_t need = dtype == SDTW_F32 ? forward_ws_needed<float>(*di, B, N, M)
                                          : forward_ws_needed<double>(*di, B, N, M);
    if (need > SDTW_NOALLOC_SCRATCH_BYTES) return SDTW_ETOOLARGE;
    void* ws = nullptr;
    e = cudaGetSymbolAddress(&ws, g_noalloc_scratch);
    if (e != cudaSuccess) return from_cuda(e);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == SDTW_F32)
        return launch_forward<float>(D, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, R, costs, ws,
                                     err_word, s);
    return launch_forward<double>(D, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, R, costs, ws,
                                  err_word, s);
}

sdtw_status sdtw_forward_band_r(sdtw_dtype dtype, const void* D, int64_t B, int64_t N, int64_t M,
                                const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                                int64_t bandwidth, void* R, void* costs, void* workspace, size_t workspace_bytes,
                                uint32_t* err_word, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!common_args_ok(B, N, M, gamma)) return SDTW_EINVAL;
    if (B == 0) return SDTW_OK;
    if (!lengths_x || !lengths_y || !R || !costs || !err_word || (N * M > 0 && !D)) return SDTW_EINVAL;
    if (!workspace || workspace_bytes < sdtw_forward_workspace_bytes(B, N, M, dtype)) return SDTW_EWORKSPACE;
    if (B * strips_of(N) >= (int64_t(1) << 31)) return SDTW_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == SDTW_F32)
        return launch_forward<float>(D, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, R, costs,
                                     workspace, err_word, s, nullptr, true);
    return launch_forward<double>(D, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, R, costs,
                                  workspace, err_word, s, nullptr, true);
}

sdtw_status sdtw_forward(sdtw_dtype dtype, const void* D, int64_t B, int64_t N, int64_t M, const void* lengths_x,
                         const void* lengths_y, int lengths_int32, double gamma, int64_t bandwidth, void* R,
                         void* costs, void* workspace, size_t workspace_bytes, uint32_t* err_word, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!common_args_ok(B, N, M, gamma)) return SDTW_EINVAL;
    if (B == 0) return SDTW_OK;
    if (!lengths_x || !lengths_y || !R || !costs || !err_word || (N * M > 0 && !D)) return SDTW_EINVAL;
    if (!workspace || workspace_bytes < sdtw_forward_workspace_bytes(B, N, M, dtype)) return SDTW_EWORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == SDTW_F32)
        return launch_forward<float>(D, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, R, costs,
                                     workspace, err_word, s);
    return launch_forward<double>(D, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, R, costs,
                                  workspace, err_word, s);
}

int sdtw_r_tiled(int64_t B, int64_t N, int64_t M, sdtw_dtype dtype)
{
    if (B <= 0 || N <= 0 || M <= 0 || (dtype != SDTW_F32 && dtype != SDTW_F64)) return 0;
    const DeviceInfo* di = nullptr;
    if (device_info(di) != cudaSuccess) return 0;
    return dtype == SDTW_F32 ? uses_tiles<float>(*di, B, N, M) : uses_tiles<double>(*di, B, N, M);
}

int64_t sdtw_r_tiles_elems(int64_t B, int64_t N, int64_t M)
{
    if (B < 0 || N < 0 || M < 0) return 0;
    return B * strips_of(N) * static_cast<int64_t>(pair_tile_blocks(M)) * 1024;
}

sdtw_status sdtw_forward_tiles(sdtw_dtype dtype, const void* D, int64_t B, int64_t N, int64_t M, const void* lengths_x,
                               const void* lengths_y, int lengths_int32, double gamma, int64_t bandwidth,
                               void* R_tiles, void* costs, void* workspace, size_t workspace_bytes,
                               uint32_t* err_word, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!common_args_ok(B, N, M, gamma)) return SDTW_EINVAL;
    if (B == 0) return SDTW_OK;
    if (!sdtw_r_tiled(B, N, M, dtype)) return SDTW_EINVAL;
    if (!lengths_x || !lengths_y || !R_tiles || !costs || !err_word || !D) return SDTW_EINVAL;
    if (reinterpret_cast<uintptr_t>(R_tiles) % 16 != 0) return SDTW_EINVAL;
    if (!workspace || workspace_bytes < sdtw_forward_workspace_bytes(B, N, M, dtype)) return SDTW_EWORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == SDTW_F32)
        return launch_forward<float>(D, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, nullptr,
                                     costs, workspace, err_word, s, R_tiles);
    return launch_forward<double>(D, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, nullptr, costs,
                                  workspace, err_word, s, R_tiles);
}

int sdtw_forward_l2_fused_ok(int64_t B, int64_t N, int64_t M, int64_t d)
{
    if (B <= 0 || N <= 0 || M <= 0 || d <= 0 || d % 16 != 0 || d > (int64_t(1) << 20)) return 0;
    const DeviceInfo* di = nullptr;
    if (device_info(di) != cudaSuccess || !uses_tiles<float>(*di, B, N, M)) return 0;
    const int W = choose_pair_warps<float>(*di, false, B, N, M);
    return W > 0 && pair_fused_smem_bytes(W, M) <= static_cast<size_t>(di->max_smem);
}

int64_t sdtw_clamp_mask_words(int64_t B, int64_t N, int64_t M)
{
    if (B < 0 || N < 0 || M < 0) return 0;
    return B * N * ((M + 31) / 32);
}

sdtw_status sdtw_forward_l2_tiles(const float* X, const float* Y, int64_t B, int64_t N, int64_t M, int64_t d,
                                  const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                                  int64_t bandwidth, void* R_tiles, float* costs, uint32_t* clamp_mask,
                                  int* clamp_flags, void* workspace, size_t workspace_bytes, uint32_t* err_word,
                                  void* stream)
{
    if (!common_args_ok(B, N, M, gamma) || d < 0) return SDTW_EINVAL;
    if (B == 0) return SDTW_OK;
    if (!sdtw_forward_l2_fused_ok(B, N, M, d)) return SDTW_EINVAL;
    if (!X || !Y || !lengths_x || !lengths_y || !R_tiles || !costs || !clamp_mask || !clamp_flags || !err_word)
        return SDTW_EINVAL;
    if (reinterpret_cast<uintptr_t>(R_tiles) % 16 != 0 || reinterpret_cast<uintptr_t>(X) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(Y) % 16 != 0)
        return SDTW_EINVAL;
    if (!workspace || workspace_bytes < sdtw_forward_workspace_bytes(B, N, M, SDTW_F32)) return SDTW_EWORKSPACE;
    const DeviceInfo* di = nullptr;
    cudaError_t e = device_info(di);
    if (e != cudaSuccess) return from_cuda(e);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    e = cudaMemsetAsync(costs, 0xff, static_cast<size_t>(B) * sizeof(float), s);  // NaN until the pair finishes
    if (e == cudaSuccess) e = cudaMemsetAsync(workspace, 0, kHeader, s);
    if (e == cudaSuccess)
        e = cudaMemsetAsync(clamp_mask, 0, static_cast<size_t>(sdtw_clamp_mask_words(B, N, M)) * sizeof(uint32_t), s);
    if (e == cudaSuccess) e = cudaMemsetAsync(clamp_flags, 0, static_cast<size_t>(B) * sizeof(int), s);
    if (e != cudaSuccess) return from_cuda(e);
    const int W = choose_pair_warps<float>(*di, false, B, N, M);
    return from_cuda(pair_forward_fused(X, Y, d, static_cast<float*>(R_tiles), costs, clamp_mask, clamp_flags,
                                        lengths_x, lengths_y, lengths_int32, B, N, M, clamp_bw(bandwidth, N, M), gamma,
                                        W, make_sync(workspace, err_word), g_inject_skip, s));
}

sdtw_status sdtw_apply_clamp_mask(float* E, const uint32_t* clamp_mask, const int* clamp_flags, int64_t B, int64_t N,
                                  int64_t M, void* stream)
{
    if (B < 0 || N < 0 || M < 0 || B > 0x7fffffff) return SDTW_EINVAL;
    if (B == 0 || N == 0 || M == 0) return SDTW_OK;
    if (!E || !clamp_mask || !clamp_flags) return SDTW_EINVAL;
    count_launch();
    sdtw_clamp_mask_kernel<<<static_cast<unsigned>(B), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        E, clamp_mask, clamp_flags, N, M);
    return from_cuda(cudaGetLastError());
}

sdtw_status sdtw_backward_tiles(sdtw_dtype dtype, const void* R_tiles, int64_t B, int64_t N, int64_t M,
                                const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                                int64_t bandwidth, void* E, void* workspace, size_t workspace_bytes,
                                uint32_t* err_word, void* stream)
{
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!common_args_ok(B, N, M, gamma)) return SDTW_EINVAL;
    if (B == 0) return SDTW_OK;
    if (!sdtw_r_tiled(B, N, M, dtype)) return SDTW_EINVAL;
    if (!lengths_x || !lengths_y || !R_tiles || !E || !err_word) return SDTW_EINVAL;
    if (reinterpret_cast<uintptr_t>(R_tiles) % 16 != 0) return SDTW_EINVAL;
    if (!workspace || workspace_bytes < sdtw_backward_workspace_bytes(B, N, M, dtype)) return SDTW_EWORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == SDTW_F32)
        return launch_backward<float>(nullptr, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, E,
                                      workspace, err_word, s, R_tiles);
    return launch_backward<double>(nullptr, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, E,
                                   workspace, err_word, s, R_tiles);
}

sdtw_status sdtw_backward(sdtw_dtype dtype, const void* D, const void* R, int64_t B, int64_t N, int64_t M,
                          const void* lengths_x, const void* lengths_y, int lengths_int32, double gamma,
                          int64_t bandwidth, void* E, void* workspace, size_t workspace_bytes, uint32_t* err_word,
                          void* stream)
{
    (void)D;
    if (dtype != SDTW_F32 && dtype != SDTW_F64) return SDTW_EDTYPE;
    if (!common_args_ok(B, N, M, gamma)) return SDTW_EINVAL;
    if (B == 0 || N == 0 || M == 0) return SDTW_OK;
    if (!lengths_x || !lengths_y || !R || !E || !err_word) return SDTW_EINVAL;
    if (!workspace || workspace_bytes < sdtw_backward_workspace_bytes(B, N, M, dtype)) return SDTW_EWORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == SDTW_F32)
        return launch_backward<float>(R, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, E, workspace,
                                      err_word, s);
    return launch_backward<double>(R, B, N, M, lengths_x, lengths_y, lengths_int32, gamma, bandwidth, E, workspace,
                                   err_word, s);
}

}  // extern "C"
