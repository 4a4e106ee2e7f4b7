// Pair-resident Soft-DTW wavefront kernels for sm_100a (forward and backward).
//
// One CTA owns one pair. Its W warps sweep the pair's 32-row strips round-robin (warp w takes strips
// w, w+W, ...; the backward walks the strips bottom-up), and consecutive strips hand their boundary
// row to each other through shared memory:
//   * every warp owns a full-width boundary row in shared memory (forward: the last row of R of its
//     current strip; backward: the contributions its first row pushes into the row above) and a
//     progress counter. The producing lane writes a value per step; after every 8 steps the counter is
//     raised with st.release.cta, and the consuming warp reads it with ld.acquire.cta before it reads
//     the 8 values it needs. A strip therefore starts 40 steps after the strip it depends on.
//   * A warp only ever waits on a strip with a smaller index in sweep order, which is always held by a
//     running warp of the same CTA, so the CTA cannot deadlock. A boundary row is rewritten (by the
//     strip W positions later) only after a chain of acquires through every warp in between, so each
//     value has been read before it is replaced. Every wait is bounded in time.
//   * Operands live in a per-warp ring in shared memory whose rows are skewed: the element of row l,
//     column c sits at position c + l, so at step tau every lane reads and writes position tau of its
//     own row (immediate offsets, no index arithmetic, conflict-free with an odd row stride). Slots of
//     32 positions are filled with cp.async one block ahead and written back row by row.
//   * The kernels write every element of their outputs (R including its +inf border and the cells
//     outside the band or the lengths; E including its zeros), so no fill or memset pass precedes them.
#include <climits>

#include "sdtw_b200.h"
#include "sdtw_pairwave.h"
#include "sdtw_strip.cuh"

namespace sdtw {

namespace {

// ---- shared-memory acquire / release on a CTA-scope progress counter ------------------------------
__device__ __forceinline__ int ld_acquire_cta(const int* p)
{
    int v;
    asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_cta_if(int* p, int v, bool pred)
{
    asm volatile(
        "{ .reg .pred q; setp.ne.u32 q, %2, 0; @q st.release.cta.shared::cta.b32 [%0], %1; }" ::"r"(smem_addr(p)),
        "r"(v), "r"(static_cast<unsigned>(pred))
        : "memory");
}

// ---- forward progress barriers -------------------------------------------------------------------
// The forward publishes its strip's last row in groups of 8 steps. Group g (= step / 8) of the strip held
// by warp w completes mbarrier g of warp w's array (count 1, arrived by lane 0 after the group's values
// are in shared memory). Each barrier completes exactly once per non-empty strip that warp sweeps (the
// groups the sweep does not reach are completed when the strip ends), so the consumer of the strip in
// round r of that warp waits for parity r & 1. A round can only complete a barrier after the consumer of
// the previous round has passed it: the strip W positions later depends, through the W-1 strips between,
// on that consumer being 4 groups further on. An empty strip (rows past the pair's length) completes
// nothing, and nothing waits after it. A waiting warp is suspended by mbarrier.try_wait instead of polling.
__device__ __forceinline__ void fbar_init(uint32_t bar) { asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory"); }
__device__ __forceinline__ void fbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool fbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.b32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}
// Warp-collective bounded wait for the phase of `bar` with the given parity. Returns false if the launch
// aborted or the wait ran out (which raises kErrTimeout and aborts the launch).
__device__ __forceinline__ bool fbar_wait(uint32_t bar, uint32_t parity, const Sync& sy, int lane)
{
    if (fbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        if (fbar_try_wait(bar, parity)) return true;
        int stop = 0;
        if (lane == 0) {
            if (aborted(sy)) {
                stop = 1;
            } else if (global_ns() - t0 > sy.timeout_ns) {
                raise_error(sy, kErrTimeout);
                stop = 1;
            }
        }
        if (__shfl_sync(kFull, stop, 0)) return false;
    }
}
// Progress barriers per warp for rows of M columns: groups 0 .. 4 * (blocks + 1) - 1.
inline __host__ __device__ int fwd_groups(int64_t M) { return 4 * (static_cast<int>((M + 30) / 32) + 2); }

// Warp-collective bounded wait until *prog >= need. `seen` caches the last value read (all lanes read
// the same word, so it is warp-uniform). Keys count columns, so need - seen is the number of steps the
// producer still has to take: the warp sleeps for about that many steps (~100 ns each, at most 2 us)
// between polls instead of spinning, which leaves the issue slots to the warps that compute. Returns
// false if the launch aborted or the wait ran out.
__device__ __forceinline__ bool wait_key(const int* prog, int need, int& seen, const Sync& sy, int lane)
{
    if (seen >= need) return true;
    seen = ld_acquire_cta(prog);
    if (seen >= need) return true;
    const uint64_t t0 = global_ns();
    unsigned spins = 0;
    while (true) {
        const int deficit = need - seen;
        __nanosleep(deficit >= 20 ? 2000u : 64u + 96u * static_cast<unsigned>(deficit));
        seen = ld_acquire_cta(prog);
        if (seen >= need) return true;
        if ((++spins & 15u) == 0) {
            int stop = 0;
            if (lane == 0) {
                if (aborted(sy)) {
                    stop = 1;
                } else if (global_ns() - t0 > sy.timeout_ns) {
                    raise_error(sy, kErrTimeout);
                    stop = 1;
                }
            }
            if (__shfl_sync(kFull, stop, 0)) return false;
        }
    }
}

inline __host__ __device__ int buf_len(int64_t M) { return static_cast<int>((M + 128 + 3) / 4 * 4); }

// Ring slot of block `blk` (blk >= -1) in the backward's three-slot ring.
__device__ __forceinline__ int slot3(int blk) { return (blk + 3) % 3; }

}  // namespace

// ==================================================================================================
// Forward
// ==================================================================================================
template <typename T>
struct PairFwdArgs {
    const T* D;
    T* R;
    T* costs;
    Lengths len;
    int64_t B, N, M, bw;
    int S, W, BL, G;  // strips, warps, boundary row length, progress barriers per warp
    T k, gl;
    Sync sy;
    int64_t inject;  // b * S + s: that strip never publishes its boundary row (failure-path test); -1 = none
};

// D rows r0..r0+31, skewed slot of block `blk` (positions 32*blk + lane) <- global, asynchronously.
// Rows at or beyond `nrows` and columns outside [0, M) are zero-filled.
template <typename T>
__device__ __forceinline__ void fwd_pair_load(const T* Db, int64_t M, T* ring, int blk, int nrows, int lane)
{
    T* dst = ring + (blk & 1) * 32 + lane;
    const int c0 = 32 * blk + lane;  // column read by row 0; row r reads column c0 - r
    if (32 * blk - 31 >= 0 && 32 * blk + 31 < M && nrows == 32) {
        const T* src = Db + c0;
        const int64_t step = M - 1;  // a compile-time constant in the kernels specialized on M
#pragma unroll
        for (int r = 0; r < 32; ++r)
            cp_async_scalar<sizeof(T)>(dst + r * kFwdStride, src + r * step, static_cast<int>(sizeof(T)));
    } else {
        for (int r = 0; r < 32; ++r) {
            const int c = c0 - r;
            const bool in = r < nrows && c >= 0 && c < M;
            cp_async_scalar<sizeof(T)>(dst + r * kFwdStride, in ? Db + static_cast<int64_t>(r) * M + c : Db,
                                       in ? static_cast<int>(sizeof(T)) : 0);
        }
    }
}

// Finished slot of block `blk` -> R (padded layout; Rrow = padded row of DP row r0), rows < nmat.
template <typename T>
__device__ __forceinline__ void fwd_pair_store(T* Rrow, int64_t pitch, int64_t M, const T* ring, int blk, int nmat,
                                               int lane)
{
    const T* src = ring + (blk & 1) * 32 + lane;
    const int c0 = 32 * blk + lane;
    if (32 * blk - 31 >= 0 && 32 * blk + 31 < M && nmat == 32) {
        T* dst = Rrow + c0 + 1;
        const int64_t step = pitch - 1;
#pragma unroll
        for (int r = 0; r < 32; ++r) dst[r * step] = src[r * kFwdStride];
    } else {
        for (int r = 0; r < nmat; ++r) {
            const int c = c0 - r;
            if (c >= 0 && c < M) Rrow[r * pitch + c + 1] = src[r * kFwdStride];
        }
    }
}

// 8 forward steps tau0 .. tau0+7 of one warp. `cell` is this lane's ring row at position tau0, `top`
// the row above (boundary row) at column tau0.
template <typename T, bool MASKED>
__device__ __forceinline__ void fwd_pair_steps8(T* cell, const T* top, int tau0, int A, int Z, T k, T gl,
                                                int src_lane, bool lane0, T& outp, T& upp)
{
    const T INF = Num<T>::inf();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const T d = cell[j];
        const T tv = top[j];
        const T upw = __shfl_sync(kFull, outp, src_lane);
        const T up = lane0 ? tv : upw;
        T r = fwd_cell<T>(d, upp, up, outp, k, gl);
        if (MASKED) {
            const int tau = tau0 + j;
            r = (tau >= A && tau <= Z) ? r : INF;
        }
        cell[j] = r;
        upp = up;
        outp = r;
    }
}

// One strip of the forward. Returns false if the launch aborted. MC > 0: the kernel is specialized on
// M == MC, so every row offset in the ring's loads and stores is a compile-time constant.
template <typename T, int MC>
__device__ bool fwd_pair_strip(const PairFwdArgs<T>& a, T* ring, const T* bin, uint32_t bars_in, uint32_t par_in,
                               T* bout, uint32_t bars_out, int64_t b, int s, int lane)
{
    const T INF = Num<T>::inf();
    const int64_t N = a.N, M = MC > 0 ? MC : a.M, pitch = M + 2;
    const int r0 = 32 * s;
    const int nmat = static_cast<int>(N - r0 < 32 ? N - r0 : 32);
    T* Rrow = a.R + b * (N + 2) * pitch + static_cast<int64_t>(r0 + 1) * pitch;
    Strip st;
    if (!make_strip(st, a.len, b, s, N, M, a.bw, lane)) {
        if (s == 0 && lane == 0) {
            if (st.bad) {
                atomicOr(a.sy.err, kErrBadLength);
                a.costs[b] = Num<T>::nan();
            } else {
                a.costs[b] = (st.nx == 0 && st.ny == 0) ? T(0) : INF;
            }
        }
        for (int r = 0; r < nmat; ++r)
            for (int c = lane; c < M + 2; c += 32) Rrow[r * pitch + c] = INF;
        // No barrier arrivals: every later strip of this pair is empty too, so nothing waits on this
        // warp's barriers again (arriving here could lap the phase the strip below the previous round
        // is still waiting for).
        return true;
    }
    const int k0 = st.c_begin >> 5;
    const int k1 = (st.c_end + 31) >> 5;
    const bool skip = b * a.S + s == a.inject;
    const bool has_consumer = st.rows == 32 && r0 + 32 < st.nx && !skip;
    const T* Db = a.D + (b * N + r0) * M;

    cp_async_wait<0>();
    __syncwarp();
    fwd_pair_load<T>(Db, M, ring, k0, st.rows, lane);
    cp_async_commit();
    if (k0 + 1 <= k1) fwd_pair_load<T>(Db, M, ring, k0 + 1, st.rows, lane);
    cp_async_commit();

    // Columns of each row outside the swept range [32*k0 - r, 32*k1 + 31 - r], and the border: +inf.
    for (int r = 0; r < nmat; ++r) {
        T* row = Rrow + r * pitch;
        int pe = 32 * k0 - r;
        pe = pe < 0 ? 0 : pe;
        int ss = 32 * k1 + 32 - r;
        ss = ss > M ? static_cast<int>(M) : ss;
        for (int c = lane; c <= pe; c += 32) row[c] = INF;
        for (int c = ss + 1 + lane; c < M + 2; c += 32) row[c] = INF;
    }

    // Terminal cell (nx-1, ny-1): lane lstar at step tstar.
    const int lstar = static_cast<int>(st.nx - 1 - r0);
    const int tstar = static_cast<int>(st.ny - 1) + lstar;
    const int bstar = (lstar >= 0 && lstar < 32) ? (tstar >> 5) : INT_MIN;

    // Group g of the strip above publishes its last row through column 8g - 24, so the columns up to
    // 8g + 7 that group g of this strip reads are complete with its group g + 4 (or, past its sweep, with
    // the barriers completed when it ends).
    const int glast = a.G - 1;
    if (s > 0 && !fbar_wait(bars_in + 8 * min(4 * k0 + 4, glast), par_in, a.sy, lane)) return false;
    T upp = lane == 0 ? bin[32 * k0 - 1 + kBufPad] : INF;  // lane 0's diagonal predecessor
    T outp = INF;
    const int src_lane = (lane + 31) & 31;
    const bool lane0 = lane == 0;

#pragma unroll 1
    for (int blk = k0; blk <= k1; ++blk) {
        cp_async_wait<1>();
        __syncwarp();
        const int tau0 = 32 * blk;
        T* cell = ring + lane * kFwdStride + (blk & 1) * 32;
        const T* top = bin + tau0 + kBufPad;
        const T* last = ring + 31 * kFwdStride + (blk & 1) * 32;  // the strip's last row, positions tau0 ..
        const bool full = tau0 >= st.Amax && tau0 + 31 <= st.Zmin;
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
            const int t8 = tau0 + 8 * q;
            if (s > 0 && !fbar_wait(bars_in + 8 * min(t8 / 8 + 4, glast), par_in, a.sy, lane)) return false;
            if (full)
                fwd_pair_steps8<T, false>(cell + 8 * q, top + 8 * q, t8, st.A, st.Z, a.k, a.gl, src_lane, lane0,
                                          outp, upp);
            else
                fwd_pair_steps8<T, true>(cell + 8 * q, top + 8 * q, t8, st.A, st.Z, a.k, a.gl, src_lane, lane0,
                                         outp, upp);
            if (!skip) {
                // Publish the last row's 8 new values (columns t8 - 31 .. t8 - 24) from the ring.
                __syncwarp();
                if (has_consumer && lane < 8) bout[t8 + lane - 31 + kBufPad] = last[8 * q + lane];
                __syncwarp();
                if (lane == 0) fbar_arrive(bars_out + 8 * (t8 / 8));
            }
        }
        __syncwarp();
        fwd_pair_store<T>(Rrow, pitch, M, ring, blk, nmat, lane);
        if (blk == bstar && lane == lstar) a.costs[b] = cell[tstar - tau0];
        __syncwarp();
        if (blk + 2 <= k1) fwd_pair_load<T>(Db, M, ring, blk + 2, st.rows, lane);
        cp_async_commit();
    }
    if (!skip) {
        // The strip below may read columns past this sweep as its row above: they are out of band (+inf).
        if (has_consumer)
            for (int c = 32 * k1 + 1 + lane; c + kBufPad < a.BL; c += 32) bout[c + kBufPad] = INF;
        __syncwarp();
        // Complete the barriers of the groups this sweep did not reach (every barrier once per strip).
        for (int g = lane; g < a.G; g += 32)
            if (g < 4 * k0 || g > 4 * k1 + 3) fbar_arrive(bars_out + 8 * g);
    }
    return true;
}

template <typename T, int MC>
__global__ void __launch_bounds__(SDTW_PAIR_THREADS, SDTW_PAIR_MIN_CTAS) sdtw_fwd_pair_kernel(PairFwdArgs<T> a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int W = a.W;
    T* rings = reinterpret_cast<T*>(smem);
    T* bufs = rings + static_cast<size_t>(W) * 32 * kFwdStride;
    T* crow = bufs + static_cast<size_t>(W) * a.BL;
    T* scratch = crow + a.BL;  // 32 elements per warp
    const uint32_t bars = (smem_addr(scratch + static_cast<size_t>(W) * 32) + 7u) & ~7u;  // [W][G] mbarriers
    const int64_t b = blockIdx.x;
    const T INF = Num<T>::inf();
    // Zero the rings and boundary rows (stale shared memory must not feed NaN patterns to masked
    // cells); the row above strip 0 is +inf with R[-1][-1] = 0.
    for (int e = threadIdx.x; e < W * (32 * kFwdStride + a.BL); e += blockDim.x) rings[e] = T(0);
    for (int e = threadIdx.x; e < a.BL; e += blockDim.x) crow[e] = e == kBufPad - 1 ? T(0) : INF;
    for (int e = threadIdx.x; e < W * a.G; e += blockDim.x) fbar_init(bars + 8 * e);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // Padded rows 0 and N+1 of R (softdtw.cpp:114-121: +inf with R[b,0,0] = 0).
    T* Rb = a.R + b * (a.N + 2) * (a.M + 2);
    for (int64_t e = threadIdx.x; e < a.M + 2; e += blockDim.x) {
        Rb[e] = e == 0 ? T(0) : INF;
        Rb[(a.N + 1) * (a.M + 2) + e] = INF;
    }
    __syncthreads();
    T* ring = rings + static_cast<size_t>(warp) * 32 * kFwdStride;
    for (int s = warp; s < a.S; s += W) {
        const int wp = (s + W - 1) % W;
        const T* bin = s > 0 ? bufs + static_cast<size_t>(wp) * a.BL : crow;
        const uint32_t par_in = static_cast<uint32_t>(((s - 1) / W) & 1);  // round of the strip above in its warp
        if (!fwd_pair_strip<T, MC>(a, ring, bin, bars + 8 * wp * a.G, par_in, bufs + static_cast<size_t>(warp) * a.BL,
                                   bars + 8 * warp * a.G, b, s, lane))
            break;
    }
    cp_async_wait<0>();
}

// ==================================================================================================
// Backward (scatter form, see sdtw_wavefront.cu)
// ==================================================================================================
template <typename T>
struct PairBwdArgs {
    const T* R;
    T* E;
    Lengths len;
    int64_t B, N, M, bw;
    int S, W, BL, P;
    T k;
    Sync sy;
    int64_t inject;
};

// Padded R rows r0 .. r0+32 (DP rows r0-1 .. r0+31), skewed slot of block `blk` <- global.
template <typename T>
__device__ __forceinline__ void bwd_pair_load(const T* Rb, int64_t N, int64_t M, T* ring, int blk, int r0, int lane)
{
    const int64_t pitch = M + 2;
    T* dst = ring + slot3(blk) * 32 + lane;
    const int c0 = 32 * blk + lane;  // column read by ring row 0; ring row p reads column c0 - p
    if (32 * blk - 31 >= 0 && 32 * blk + 32 <= M + 1 && r0 + 32 <= N + 1) {
        const T* src = Rb + static_cast<int64_t>(r0) * pitch + c0 + 1;
        const int64_t step = pitch - 1;
#pragma unroll 11
        for (int p = 0; p < 33; ++p) {
            cp_async_scalar<sizeof(T)>(dst + p * kBwdStride, src, static_cast<int>(sizeof(T)));
            src += step;
        }
    } else {
        for (int p = 0; p < 33; ++p) {
            const int pc = c0 - p + 1;  // padded column
            const bool in = r0 + p <= N + 1 && pc >= 0 && pc <= M + 1;
            cp_async_scalar<sizeof(T)>(dst + p * kBwdStride,
                                       in ? Rb + static_cast<int64_t>(r0 + p) * pitch + pc : Rb,
                                       in ? static_cast<int>(sizeof(T)) : 0);
        }
    }
}

// E of slot `blk` -> global (Erow = E row of DP row r0). Positions outside [lo_pos, hi_pos] were never
// written by the sweep: their cells lie outside the band and get 0.
template <typename T>
__device__ __forceinline__ void bwd_pair_store(T* Erow, int64_t M, const T* ring, int blk, int lo_pos, int hi_pos,
                                               int nmat, int lane)
{
    const T* src = ring + kBwdStride + slot3(blk) * 32 + lane;  // ring row p = r + 1 holds DP row r0 + r
    const int pos = 32 * blk + lane;
    const int c0 = pos - 1;  // column of row 0; row r: c0 - r
    if (32 * blk - 32 >= 0 && 32 * blk + 30 < M && nmat == 32 && 32 * blk >= lo_pos && 32 * blk + 31 <= hi_pos) {
        T* dst = Erow + c0;
        const int64_t step = M - 1;
#pragma unroll 8
        for (int r = 0; r < 32; ++r) {
            *dst = src[r * kBwdStride];
            dst += step;
        }
    } else {
        const bool written = pos >= lo_pos && pos <= hi_pos;
        for (int r = 0; r < nmat; ++r) {
            const int c = c0 - r;
            if (c >= 0 && c < M) Erow[r * M + c] = written ? src[r * kBwdStride] : T(0);
        }
    }
}

// Backward steps tau = tau0 + u for u = UHI down to ULO. `A` is this lane's ring row (the row above its
// own) at the block's slot; position tau-1 of it is R[i-1][c-1], position tau of the next ring row is
// R[i][c-1], and E[i][c] is written at position tau+1 of the next ring row. The first position of the
// block (u = 0 reads tau-1 = 32*blk - 1) and the last (u = 31 writes 32*blk + 32) lie in neighbouring
// slots: `edge_rd` / `edge_e` point there.
template <typename T, bool MASKED, int UHI, int ULO>
__device__ __forceinline__ void bwd_pair_steps(T* A, const T* edge_rd, T* edge_e, const T* bin, T* bout, int tau0,
                                               int Av, int Zv, T k, T seed, int src_lane, bool lane31, T& upc,
                                               T& sendv, T& pend, T& acc)
{
    const T big = Num<T>::big();
    T* A1 = A + kBwdStride;
#pragma unroll
    for (int u = UHI; u >= ULO; --u) {
        const T rd = (u == 0) ? *edge_rd : A[u - 1];
        const T rl = A1[u];
        const T ru = upc;
        const T recvw = __shfl_sync(kFull, sendv, src_lane);
        const T bv = bin[u];
        const T recv = lane31 ? bv : recvw;
        const T Es = acc + recv;
        const T m = Num<T>::mn(Num<T>::mn(rd, ru), rl);
        const T mc = Num<T>::mn(m, big);
        const T ed = Num<T>::exp2_((mc - rd) * k);
        const T eu = Num<T>::exp2_((mc - ru) * k);
        const T el = Num<T>::exp2_((mc - rl) * k);
        T q = Es * Num<T>::rcp_((ed + eu) + el);
        T Eo = Es;
        if (MASKED) {
            const int tau = tau0 + u;
            const bool valid = tau >= Av && tau <= Zv;
            q = valid ? q : T(0);
            acc = valid ? q * el : seed;
            Eo = valid ? Es : T(0);
        } else {
            acc = q * el;
        }
        sendv = fma(q, eu, pend);
        pend = q * ed;
        if (u == 31)
            *edge_e = Eo;
        else
            A1[u + 1] = Eo;
        bout[u] = sendv;  // lane 0: the boundary row; other lanes: a scratch area
        upc = rd;
    }
}

template <typename T, bool MASKED>
__device__ __forceinline__ void bwd_pair_block(T* A, const T* edge_rd, T* edge_e, const T* bin, T* bout, int tau0,
                                               const Strip& st, T k, T seed, int src_lane, bool lane31, T& upc,
                                               T& sendv, T& pend, T& acc, int q)
{
    // q selects the 8-step group; the block's first and last steps are run by the caller.
    switch (q) {
        case 3:
            bwd_pair_steps<T, MASKED, 30, 24>(A, edge_rd, edge_e, bin, bout, tau0, st.A, st.Z, k, seed,
                                              src_lane, lane31, upc, sendv, pend, acc);
            break;
        case 2:
            bwd_pair_steps<T, MASKED, 23, 16>(A, edge_rd, edge_e, bin, bout, tau0, st.A, st.Z, k, seed,
                                              src_lane, lane31, upc, sendv, pend, acc);
            break;
        case 1:
            bwd_pair_steps<T, MASKED, 15, 8>(A, edge_rd, edge_e, bin, bout, tau0, st.A, st.Z, k, seed,
                                             src_lane, lane31, upc, sendv, pend, acc);
            break;
        default:
            bwd_pair_steps<T, MASKED, 7, 1>(A, edge_rd, edge_e, bin, bout, tau0, st.A, st.Z, k, seed,
                                            src_lane, lane31, upc, sendv, pend, acc);
            break;
    }
}

// One strip of the backward; `t` is its position in sweep order (strip S-1-t). Returns false if the
// launch aborted.
template <typename T>
__device__ bool bwd_pair_strip(const PairBwdArgs<T>& a, T* ring, const T* bin, const int* pin, const T* zrow,
                               T* bout, int* pout, T* scratch, int64_t b, int s, int t, int lane)
{
    const int64_t N = a.N, M = a.M;
    const int r0 = 32 * s;
    const int nmat = static_cast<int>(N - r0 < 32 ? N - r0 : 32);
    T* Erow = a.E + (b * N + r0) * M;
    Strip st;
    if (!make_strip(st, a.len, b, s, N, M, a.bw, lane)) {
        if (st.bad && s == 0 && lane == 0) atomicOr(a.sy.err, kErrBadLength);
        for (int r = 0; r < nmat; ++r)
            for (int c = lane; c < M; c += 32) Erow[r * M + c] = T(0);
        return true;
    }
    const int k0 = st.c_begin >> 5;
    const int k1 = (st.c_end + 31) >> 5;
    const int kmin = (32 * k0 - 1) >> 5;  // arithmetic shift: -1 when k0 == 0
    const bool has_producer = r0 + 32 < st.nx;
    const bool skip = b * a.S + s == a.inject;
    const bool has_consumer = s > 0 && !skip;
    if (!has_producer) bin = zrow;
    const T seed = (r0 + lane == st.nx - 1) ? T(1) : T(0);
    const T* Rb = a.R + b * (N + 2) * (M + 2);

    cp_async_wait<0>();
    __syncwarp();
    bwd_pair_load<T>(Rb, N, M, ring, k1, r0, lane);
    cp_async_commit();
    if (k1 - 1 >= kmin) bwd_pair_load<T>(Rb, N, M, ring, k1 - 1, r0, lane);
    cp_async_commit();

    // Columns of each row outside the stored range [32*k0 - r - 1, 32*k1 + 62 - r]: zero.
    for (int r = 0; r < nmat; ++r) {
        T* row = Erow + r * M;
        int pe = 32 * k0 - r - 1;
        pe = pe < 0 ? 0 : (pe > M ? static_cast<int>(M) : pe);
        int ss = 32 * k1 + 63 - r;
        ss = ss > M ? static_cast<int>(M) : ss;
        for (int c = lane; c < pe; c += 32) row[c] = T(0);
        for (int c = ss + lane; c < M; c += 32) row[c] = T(0);
    }

    const int P = a.P;
    const int H = static_cast<int>(M) + 63;
    const int key_in = (t - 1) * P + H;  // the strip below has pushed into every column >= c: key_in - c
    const int key_out = t * P + H;
    const int lo_pos = 32 * k0 + 1;
    const int hi_pos = 32 * k1 + 32;
    int seen = INT_MIN;
    T upc = T(0), sendv = T(0), pend = T(0), acc = seed;
    const int src_lane = (lane + 1) & 31;
    const bool lane31 = lane == 31;
    const bool put_out = has_consumer && lane == 0;

#pragma unroll 1
    for (int blk = k1; blk >= k0; --blk) {
        cp_async_wait<1>();
        __syncwarp();
        const int tau0 = 32 * blk;
        T* A = ring + lane * kBwdStride + slot3(blk) * 32;
        if (blk == k1) upc = A[31];  // R[i-1][c] of the first step
        const T* edge_rd = ring + lane * kBwdStride + slot3(blk - 1) * 32 + 31;
        T* edge_e = ring + (lane + 1) * kBwdStride + slot3(blk + 1) * 32;
        const T* bi = bin + tau0 - 31 + kBufPad;
        T* bo = put_out ? bout + tau0 + kBufPad : scratch;
        const bool full = tau0 >= st.Amax && tau0 + 31 <= st.Zmin;
#pragma unroll 1
        for (int q = 3; q >= 0; --q) {
            const int t8 = tau0 + 8 * q;
            if (has_producer && !wait_key(pin, key_in - (t8 - 31), seen, a.sy, lane)) return false;
            if (q == 3) {
                if (full)
                    bwd_pair_steps<T, false, 31, 31>(A, edge_rd, edge_e, bi, bo, tau0, st.A, st.Z, a.k, seed,
                                                     src_lane, lane31, upc, sendv, pend, acc);
                else
                    bwd_pair_steps<T, true, 31, 31>(A, edge_rd, edge_e, bi, bo, tau0, st.A, st.Z, a.k, seed,
                                                    src_lane, lane31, upc, sendv, pend, acc);
                // Slot blk+1 is now final: write its E back and refill it with slot blk-2.
                __syncwarp();
                bwd_pair_store<T>(Erow, M, ring, blk + 1, lo_pos, hi_pos, nmat, lane);
                __syncwarp();
                if (blk - 2 >= kmin) bwd_pair_load<T>(Rb, N, M, ring, blk - 2, r0, lane);
                cp_async_commit();
            }
            if (full)
                bwd_pair_block<T, false>(A, edge_rd, edge_e, bi, bo, tau0, st, a.k, seed, src_lane,
                                         lane31, upc, sendv, pend, acc, q);
            else
                bwd_pair_block<T, true>(A, edge_rd, edge_e, bi, bo, tau0, st, a.k, seed, src_lane,
                                        lane31, upc, sendv, pend, acc, q);
            if (q == 0) {
                cp_async_wait<1>();  // slot blk-1 (read by the last step)
                __syncwarp();
                if (full)
                    bwd_pair_steps<T, false, 0, 0>(A, edge_rd, edge_e, bi, bo, tau0, st.A, st.Z, a.k, seed,
                                                   src_lane, lane31, upc, sendv, pend, acc);
                else
                    bwd_pair_steps<T, true, 0, 0>(A, edge_rd, edge_e, bi, bo, tau0, st.A, st.Z, a.k, seed,
                                                  src_lane, lane31, upc, sendv, pend, acc);
            }
            st_release_cta_if(pout, key_out - t8, put_out);
        }
    }
    cp_async_wait<0>();
    __syncwarp();
    bwd_pair_store<T>(Erow, M, ring, k0, lo_pos, hi_pos, nmat, lane);
    if (has_consumer) {
        // Lane 0's last diagonal push (into column 32*k0 - 1) and zeros below the sweep.
        if (lane == 0) bout[32 * k0 - 1 + kBufPad] = pend;
        for (int c = -kBufPad + lane; c <= 32 * k0 - 2; c += 32) bout[c + kBufPad] = T(0);
        __threadfence_block();
        __syncwarp();
        st_release_cta_if(pout, t * P + P - 1, lane == 0);
    }
    __syncwarp();
    return true;
}

template <typename T>
__global__ void __launch_bounds__(SDTW_PAIR_THREADS, SDTW_PAIR_MIN_CTAS) sdtw_bwd_pair_kernel(PairBwdArgs<T> a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int W = a.W;
    T* rings = reinterpret_cast<T*>(smem);
    T* bufs = rings + static_cast<size_t>(W) * 33 * kBwdStride;
    T* zrow = bufs + static_cast<size_t>(W) * a.BL;
    T* scratch = zrow + a.BL;  // 32 elements per warp
    int* prog = reinterpret_cast<int*>(scratch + static_cast<size_t>(W) * 32);
    const int64_t b = blockIdx.x;
    for (int e = threadIdx.x; e < W * (33 * kBwdStride + a.BL) + a.BL; e += blockDim.x) rings[e] = T(0);
    if (threadIdx.x < W) prog[threadIdx.x] = -1;
    __syncthreads();
    T* ring = rings + static_cast<size_t>(warp) * 33 * kBwdStride;
    for (int t = warp; t < a.S; t += W) {
        const int wp = (t + W - 1) % W;
        if (!bwd_pair_strip<T>(a, ring, bufs + static_cast<size_t>(wp) * a.BL, prog + wp, zrow,
                               bufs + static_cast<size_t>(warp) * a.BL, prog + warp,
                               scratch + static_cast<size_t>(warp) * 32, b, a.S - 1 - t, t, lane))
            break;
    }
    cp_async_wait<0>();
}

// ==================================================================================================
// Host side
// ==================================================================================================
template <typename T>
size_t pair_fwd_smem_bytes(int W, int64_t M)
{
    return (static_cast<size_t>(W) * (32 * kFwdStride + 32) + static_cast<size_t>(W + 1) * buf_len(M)) * sizeof(T) +
           8 + static_cast<size_t>(W) * fwd_groups(M) * 8;
}
template <typename T>
size_t pair_bwd_smem_bytes(int W, int64_t M)
{
    return (static_cast<size_t>(W) * (33 * kBwdStride + 32) + static_cast<size_t>(W + 1) * buf_len(M)) * sizeof(T) +
           static_cast<size_t>(W) * sizeof(int);
}

template <typename T>
cudaError_t pair_init_attrs(int max_smem)
{
    cudaError_t e = cudaFuncSetAttribute(sdtw_fwd_pair_kernel<T, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(sdtw_fwd_pair_kernel<T, kPairSpecialM>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(sdtw_bwd_pair_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}
template cudaError_t pair_init_attrs<float>(int);
template cudaError_t pair_init_attrs<double>(int);

template <typename T>
cudaError_t pair_regs(bool backward, int& regs)
{
    cudaFuncAttributes fa;
    const cudaError_t e = backward ? cudaFuncGetAttributes(&fa, sdtw_bwd_pair_kernel<T>)
                                   : cudaFuncGetAttributes(&fa, sdtw_fwd_pair_kernel<T, 0>);
    regs = e == cudaSuccess ? fa.numRegs : 0;
    return e;
}
template cudaError_t pair_regs<float>(bool, int&);
template cudaError_t pair_regs<double>(bool, int&);

// Warps per CTA: at most `cap` and the pair's strip count, and few enough for the CTA to fit `budget`.
template <typename T>
int pair_warps(bool backward, int64_t N, int64_t M, int cap, size_t budget)
{
    const int64_t S = N > 0 ? (N + 31) / 32 : 1;
    int W = static_cast<int>(S < cap ? S : cap);
    if (W > kPairMaxWarps) W = kPairMaxWarps;
    while (W >= 1) {
        const size_t bytes = backward ? pair_bwd_smem_bytes<T>(W, M) : pair_fwd_smem_bytes<T>(W, M);
        if (bytes <= budget) return W;
        --W;
    }
    return 0;
}
template int pair_warps<float>(bool, int64_t, int64_t, int, size_t);
template int pair_warps<double>(bool, int64_t, int64_t, int, size_t);

bool pair_keys_fit(int64_t N, int64_t M)
{
    const int64_t S = N > 0 ? (N + 31) / 32 : 1;
    return (S + 1) * (M + 128) < (int64_t(1) << 30);
}

template <typename T>
cudaError_t pair_forward(const T* D, T* R, T* costs, const void* lx, const void* ly, int is32, int64_t B, int64_t N,
                         int64_t M, int64_t bw, double gamma, int W, Sync sy, int64_t inject, cudaStream_t stream)
{
    PairFwdArgs<T> a;
    a.D = D;
    a.R = R;
    a.costs = costs;
    a.len = Lengths{lx, ly, is32};
    a.B = B;
    a.N = N;
    a.M = M;
    a.bw = bw;
    a.S = static_cast<int>(N > 0 ? (N + 31) / 32 : 1);
    a.W = W;
    a.BL = buf_len(M);
    a.G = fwd_groups(M);
    a.k = static_cast<T>(1.4426950408889634 / gamma);
    a.gl = static_cast<T>(gamma * 0.6931471805599453);
    a.sy = sy;
    a.inject = inject;
    count_launch();
    if (M == kPairSpecialM)
        sdtw_fwd_pair_kernel<T, kPairSpecialM><<<static_cast<unsigned>(B), W * 32, pair_fwd_smem_bytes<T>(W, M), stream>>>(a);
    else
        sdtw_fwd_pair_kernel<T, 0><<<static_cast<unsigned>(B), W * 32, pair_fwd_smem_bytes<T>(W, M), stream>>>(a);
    return cudaGetLastError();
}
template cudaError_t pair_forward<float>(const float*, float*, float*, const void*, const void*, int, int64_t, int64_t,
                                         int64_t, int64_t, double, int, Sync, int64_t, cudaStream_t);
template cudaError_t pair_forward<double>(const double*, double*, double*, const void*, const void*, int, int64_t,
                                          int64_t, int64_t, int64_t, double, int, Sync, int64_t, cudaStream_t);

template <typename T>
cudaError_t pair_backward(const T* R, T* E, const void* lx, const void* ly, int is32, int64_t B, int64_t N, int64_t M,
                          int64_t bw, double gamma, int W, Sync sy, int64_t inject, cudaStream_t stream)
{
    PairBwdArgs<T> a;
    a.R = R;
    a.E = E;
    a.len = Lengths{lx, ly, is32};
    a.B = B;
    a.N = N;
    a.M = M;
    a.bw = bw;
    a.S = static_cast<int>(N > 0 ? (N + 31) / 32 : 1);
    a.W = W;
    a.BL = buf_len(M);
    a.P = static_cast<int>(M + 128);
    a.k = static_cast<T>(1.4426950408889634 / gamma);
    a.sy = sy;
    a.inject = inject;
    count_launch();
    sdtw_bwd_pair_kernel<T><<<static_cast<unsigned>(B), W * 32, pair_bwd_smem_bytes<T>(W, M), stream>>>(a);
    return cudaGetLastError();
}
template cudaError_t pair_backward<float>(const float*, float*, const void*, const void*, int, int64_t, int64_t,
                                          int64_t, int64_t, double, int, Sync, int64_t, cudaStream_t);
template cudaError_t pair_backward<double>(const double*, double*, const void*, const void*, int, int64_t, int64_t,
                                           int64_t, int64_t, double, int, Sync, int64_t, cudaStream_t);

}  // namespace sdtw
