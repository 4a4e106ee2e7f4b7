// Pair-resident Soft-DTW wavefront kernels for sm_100a (forward and backward).
//
// One CTA owns one pair. Its W warps sweep the pair's 32-row strips round-robin (warp w takes strips
// w, w+W, ...; the backward walks the strips bottom-up), and consecutive strips hand their boundary
// row to each other through shared memory:
//   * every warp owns a full-width boundary row in shared memory (forward: the last row of R of its
//     current strip; backward: the contributions its first row pushes into the row above) and one
//     mbarrier per group of 8 steps. After every second group the 16 new values are copied into the row
//     and the group's barrier completes; the consuming warp waits on it (mbarrier.try_wait, bounded)
//     once per pair of its own groups. A strip therefore starts about 48 steps after the strip it
//     depends on.
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

// ---- progress barriers between strips -----------------------------------------------------------
// A strip publishes its boundary row (forward: its last row of R; backward: the contributions its first row
// pushes into the row above) two groups of 8 steps at a time: after the pair of groups (g, g + 1) of the
// strip held by warp w (forward; g + 1 and g going downwards in the backward), the 16 values are in shared
// memory and mbarrier g + 1 (forward) / g (backward) of warp w's array completes. Only those barriers, odd
// (forward) or even (backward), are used; a consumer waits once per pair of its own groups, on the later
// producer group the pair needs, which costs a few steps of lag and halves the waits and the publishing.
// Each used barrier completes exactly once per non-empty strip that warp sweeps (the groups the sweep does
// not reach are completed when the strip ends), so the consumer of the strip in round r of that warp waits
// for parity r & 1. A round can only complete a barrier after the consumer of the previous round has passed
// it: the strip W positions later depends, through the W-1 strips between, on that consumer being 5 groups
// further on. An empty forward strip (rows past the pair's length) completes nothing, and nothing waits
// after it. A waiting warp is suspended by mbarrier.try_wait instead of polling.
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
// Progress barriers per warp for rows of M columns: groups 0 .. 4 * (blocks + 1) - 1 (both directions).
inline __host__ __device__ int fwd_groups(int64_t M) { return 4 * (static_cast<int>((M + 30) / 32) + 2); }

inline __host__ __device__ int buf_len(int64_t M) { return static_cast<int>((M + 128 + 3) / 4 * 4); }


}  // namespace

// ==================================================================================================
// Forward
// ==================================================================================================
// Forward ring row stride in elements: 2 slots of 32 positions + pad. 68 floats / 66 doubles are 272 / 528
// bytes, 16-byte multiples whose word stride is 4 (mod 32), so the per-lane 16-byte accesses of a quarter
// warp (8 lanes, 8 rows) fall into 8 distinct 16-byte bank groups, and a whole row read or written one lane
// per position is conflict-free.
template <typename T>
struct FwdRing {
    static constexpr int S = sizeof(T) == 4 ? 68 : 66;
};

// Fused forward: byte offset of the |y|^2 array in shared memory (after the rings, boundary rows, scratch and
// barriers of pair_fwd_smem_bytes<float>), and the CTA's total.
inline __host__ __device__ size_t fused_y2_offset(int W, int64_t M)
{
    const size_t end = (static_cast<size_t>(W) * (32 * FwdRing<float>::S + 32) + static_cast<size_t>(W + 1) * buf_len(M)) *
                           sizeof(float) +
                       8 + static_cast<size_t>(W) * fwd_groups(M) * 8;
    return (end + 15) / 16 * 16;
}
inline size_t fused_smem_bytes(int W, int64_t M) { return fused_y2_offset(W, M) + static_cast<size_t>(M + 96) * 4; }

// Inputs of the fused squared-L2 forward (the cost matrix computed inside the wavefront, never stored).
struct FusedL2 {
    const float* X;   // (B, N, d)
    const float* Y;   // (B, M, d)
    int d;            // a multiple of 16
    uint32_t* cmask;  // (B, N, MW): bit c % 32 of word c / 32 set where the clamp at 0 was active
    int* cflags;      // (B,): set for pairs with a clamped cell
    int MW;
    Extent xX, xY, xMask, xFlags;
};

template <typename T>
struct PairFwdArgs {
    const T* D;
    T* R;   // padded R (B, N+2, M+2), or null when Rt is given
    T* Rt;  // R as strip tiles (B, S, NBt, 32, 32), or null (see pair_forward)
    int NBt;
    T* costs;
    Lengths len;
    int64_t B, N, M, bw;
    int S, W, BL, G;  // strips, warps, boundary row length, progress barriers per warp
    T k, gl;
    Extent xD, xR, xRt, xC;  // buffers, for the debug build's bounds checks
    Sync sy;
    int64_t inject;  // b * S + s: that strip never publishes its boundary row (failure-path test); -1 = none
    FusedL2 f;       // the fused kernel's inputs (D unused)
};

// ---- cost rectangles of the fused squared-L2 forward ------------------------------------------------------
// D = (|x|^2 + |y|^2) - 2 x.y clamped at 0, the form of distances.py:14-18, with x.y from 3xTF32 warp MMAs:
// each operand splits into a head (the nearest TF32 value) and a tail (the nearest TF32 value of the
// remainder), the split of the tcgen05 cost kernel, and x.y = head.head + head.tail + tail.head; the
// tail.tail term left out is below 2^-22 of |x||y| and has no fixed sign after round-to-nearest, so the
// products of identical rows land on either side of |x|^2 like an fp32 dot product does.
__device__ __forceinline__ void mma_tf32(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void tf32_split(float v, uint32_t& hi, uint32_t& lo)
{
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(v));
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(v - __uint_as_float(hi)));
}
__device__ __forceinline__ float f4c(const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// D of the 32 x 32 rectangle rows r0 .. r0+31, columns 32K .. 32K+31 of one pair -> the forward ring: element
// (r, c) at position (c + r + 1) mod 64 of ring row r, the position the forward sweep reads it at. Xs: row r0 of
// X; Yb: row 0 of Y; x2[i]: |x|^2 of row r0 + lane/4 + 8i; y2: |y|^2 by column (zero outside [0, M), 32 before
// column 0 and 64 after M-1 readable). Rows past N and columns outside [0, M) read zero operands; the sweep
// masks those cells. A clamp of a cell inside the matrix sets its bit in the pair's clamp mask and its flag.
//
// Fragment layout (mma.m16n8k8 .tf32): lane = 4 g + t holds A rows g, g+8 at k = t, t+4, B column g at
// k = t, t+4, and C rows g, g+8 at columns 2t, 2t+1. The 8 k of MMA step 2p+ks are the feature dimensions
// 16p + 4t + 2ks + {0, 1} (k = t -> +0, k = t+4 -> +1): a permutation of the 16 dimensions of chunk p that is
// the same for both operands, so each lane loads its operands as whole 16-byte vectors.
__device__ __forceinline__ void fused_rect(const FusedL2& f, float* ring, const float* Xs, const float* Yb,
                                           const float (&x2)[4], const float* y2, int64_t b, int r0, int64_t N,
                                           int64_t M, int K, int lane, uint32_t* err)
{
    constexpr int RS = FwdRing<float>::S;
    const int g = lane >> 2, t = lane & 3, d = f.d;
    const int cb = 32 * K;
    // Operand rows: rows past N and columns outside [0, M) read a row of the matrix instead (any finite
    // value will do, the sweep masks those cells), so the loads need no predicate.
    int xo[4], yo[4];  // element offsets from Xs and Yb
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t row = min(static_cast<int64_t>(r0 + g + 8 * i), N - 1) - r0;
        xo[i] = static_cast<int>(row * d) + 4 * t;
        const int64_t col = min(static_cast<int64_t>(max(cb + 8 * i + g, 0)), M - 1);
        yo[i] = static_cast<int>(col * d) + 4 * t;
    }
    float acc[2][4][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[mt][nt][c] = 0.f;
#pragma unroll 1
    for (int p = 0; p < d / 16; ++p) {
        float4 xa[4], yb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4* xq = reinterpret_cast<const float4*>(Xs + xo[i] + 16 * p);
            const float4* yq = reinterpret_cast<const float4*>(Yb + yo[i] + 16 * p);
            xa[i] = SDTW_IN_BOUNDS(f.xX, xq, 16, err) ? __ldg(xq) : make_float4(0.f, 0.f, 0.f, 0.f);
            yb[i] = SDTW_IN_BOUNDS(f.xY, yq, 16, err) ? __ldg(yq) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            uint32_t ah[4][2], al[4][2];  // [row set][k = t, t + 4]
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int h = 0; h < 2; ++h) tf32_split(f4c(xa[i], 2 * ks + h), ah[i][h], al[i][h]);
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                uint32_t bh[2], bl[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) tf32_split(f4c(yb[nt], 2 * ks + h), bh[h], bl[h]);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    mma_tf32(acc[mt][nt], al[2 * mt][0], al[2 * mt + 1][0], al[2 * mt][1], al[2 * mt + 1][1], bh[0],
                             bh[1]);
                    mma_tf32(acc[mt][nt], ah[2 * mt][0], ah[2 * mt + 1][0], ah[2 * mt][1], ah[2 * mt + 1][1], bl[0],
                             bl[1]);
                    mma_tf32(acc[mt][nt], ah[2 * mt][0], ah[2 * mt + 1][0], ah[2 * mt][1], ah[2 * mt + 1][1], bh[0],
                             bh[1]);
                }
            }
        }
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int r = 16 * mt + g + 8 * (c >> 1);
                const int cc = 8 * nt + 2 * t + (c & 1);
                float v = (x2[2 * mt + (c >> 1)] + y2[cb + cc]) - 2.f * acc[mt][nt][c];
                if (v < 0.f) {
                    const int64_t row = r0 + r;
                    const int col = cb + cc;
                    if (row < N && col >= 0 && col < M) {
                        uint32_t* w = f.cmask + (b * N + row) * f.MW + (col >> 5);
                        if (SDTW_IN_BOUNDS(f.xMask, w, 4, err)) atomicOr(w, 1u << (col & 31));
                        if (SDTW_IN_BOUNDS(f.xFlags, f.cflags + b, 4, err)) f.cflags[b] = 1;
                    }
                    v = 0.f;
                }
                ring[r * RS + ((cb + cc + r + 1) & 63)] = v;
            }
}

// D rows r0..r0+31, skewed slot of block `blk` (positions 32*blk + lane) <- global, asynchronously. Ring row
// r holds column c at position c + r + 1. Rows at or beyond `nrows` and columns outside [0, M) are zero-filled.
template <typename T>
__device__ __forceinline__ void fwd_pair_load(const T* Db, int64_t M, T* ring, int blk, int nrows, int lane,
                                              const Extent& xD, uint32_t* err)
{
    constexpr int S = FwdRing<T>::S;
    T* dst = ring + (blk & 1) * 32 + lane;
    const int c0 = 32 * blk + lane - 1;  // column read by row 0; row r reads column c0 - r
    if (32 * blk - 32 >= 0 && 32 * blk + 30 < M && nrows == 32) {
        const T* src = Db + c0;
        const int64_t step = M - 1;  // a compile-time constant in the kernels specialized on M
#pragma unroll
        for (int r = 0; r < 32; ++r) {
            const bool ok = SDTW_IN_BOUNDS(xD, src + r * step, sizeof(T), err);
            cp_async_scalar<sizeof(T)>(dst + r * S, ok ? src + r * step : Db, ok ? static_cast<int>(sizeof(T)) : 0);
        }
    } else {
        for (int r = 0; r < 32; ++r) {
            const int c = c0 - r;
            bool in = r < nrows && c >= 0 && c < M;
            if (in) in = SDTW_IN_BOUNDS(xD, Db + static_cast<int64_t>(r) * M + c, sizeof(T), err);
            cp_async_scalar<sizeof(T)>(dst + r * S, in ? Db + static_cast<int64_t>(r) * M + c : Db,
                                       in ? static_cast<int>(sizeof(T)) : 0);
        }
    }
}

// Finished slot of block `blk` -> R (padded layout; Rrow = padded row of DP row r0), rows < nmat.
template <typename T>
__device__ __forceinline__ void fwd_pair_store(T* Rrow, int64_t pitch, int64_t M, const T* ring, int blk, int nmat,
                                               int lane, const Extent& xR, uint32_t* err)
{
    constexpr int S = FwdRing<T>::S;
    const T* src = ring + (blk & 1) * 32 + lane;
    const int c0 = 32 * blk + lane - 1;  // column of row 0; row r: c0 - r
    if (32 * blk - 32 >= 0 && 32 * blk + 30 < M && nmat == 32) {
        T* dst = Rrow + c0 + 1;
        const int64_t step = pitch - 1;
#pragma unroll
        for (int r = 0; r < 32; ++r)
            if (SDTW_IN_BOUNDS(xR, dst + r * step, sizeof(T), err)) dst[r * step] = src[r * S];
    } else {
        for (int r = 0; r < nmat; ++r) {
            const int c = c0 - r;
            if (c >= 0 && c < M && SDTW_IN_BOUNDS(xR, Rrow + r * pitch + c + 1, sizeof(T), err))
                Rrow[r * pitch + c + 1] = src[r * S];
        }
    }
}

// 8 consecutive elements <-> shared memory, 16-byte accesses (p 16-byte aligned).
__device__ __forceinline__ void lds8(float (&v)[8], const float* p)
{
    const float4 x = reinterpret_cast<const float4*>(p)[0], y = reinterpret_cast<const float4*>(p)[1];
    v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w, v[4] = y.x, v[5] = y.y, v[6] = y.z, v[7] = y.w;
}
__device__ __forceinline__ void lds8(double (&v)[8], const double* p)
{
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const double2 x = reinterpret_cast<const double2*>(p)[i];
        v[2 * i] = x.x, v[2 * i + 1] = x.y;
    }
}
__device__ __forceinline__ void sts8(float* p, const float (&v)[8])
{
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void sts8(double* p, const double (&v)[8])
{
#pragma unroll
    for (int i = 0; i < 4; ++i) reinterpret_cast<double2*>(p)[i] = make_double2(v[2 * i], v[2 * i + 1]);
}

// Arrive (count `n`) on a forward progress barrier when `pred`.
__device__ __forceinline__ void fbar_arrive_n_if(uint32_t bar, uint32_t n, bool pred)
{
    asm volatile("{ .reg .pred q; setp.ne.u32 q, %2, 0; @q mbarrier.arrive.shared::cta.b64 _, [%0], %1; }" ::"r"(bar),
                 "r"(n), "r"(static_cast<unsigned>(pred))
                 : "memory");
}
// Lanes that publish a group of the boundary row: each arrives once, so a barrier phase completes after all
// of them stored their value (each arrive releases its own store; no second warp barrier is needed).
constexpr int kPubLanes = 8;

// Out-of-line part of the bounded wait (the common case, a phase already complete, is one try_wait).
__device__ __noinline__ bool fbar_wait_slow(uint32_t bar, uint32_t parity, Sync sy, int lane)
{
    return fbar_wait(bar, parity, sy, lane);
}
__device__ __forceinline__ bool fbar_wait_fast(uint32_t bar, uint32_t parity, const Sync& sy, int lane)
{
    if (__all_sync(kFull, fbar_try_wait(bar, parity))) return true;
    return fbar_wait_slow(bar, parity, sy, lane);
}

// 8 forward steps tau0 .. tau0+7 of one warp. `cell` is this lane's ring row at position tau0 (read and
// written with 16-byte accesses), `top` the row above (boundary row) at column tau0.
// Finished slot of block `blk` -> its 32 x 32 tile (module path): 16-byte pieces, each store instruction writing
// whole 128-byte tile rows (4 rows of floats, 2 of doubles), read from the ring row by row.
template <typename T>
__device__ __forceinline__ void fwd_tile_store(T* tile, const T* ring, int blk, int lane, const Extent& xRt,
                                               uint32_t* err)
{
    constexpr int RS = FwdRing<T>::S;
    constexpr int EPP = 16 / sizeof(T);  // elements per piece
    constexpr int CPR = 32 / EPP;        // pieces per row
    constexpr int RPI = 32 / CPR;        // rows per store instruction
    const int r = lane / CPR, c = (lane % CPR) * EPP;
    const T* src = ring + r * RS + (blk & 1) * 32 + c;
    T* dst = tile + r * 32 + c;
#pragma unroll
    for (int i = 0; i < 32; i += RPI) {
        const uint4 v = *reinterpret_cast<const uint4*>(src + i * RS);
        if (SDTW_IN_BOUNDS(xRt, dst + i * 32, 16, err)) *reinterpret_cast<uint4*>(dst + i * 32) = v;
    }
}

// SCALED: the values are R in units of gamma ln 2 (fwd_cell_scaled); D arrives in its own units and is
// scaled here.
template <typename T, bool MASKED, bool SCALED>
__device__ __forceinline__ void fwd_pair_steps8(T* cell, const T* top, int tau0, int A, int Z, T k, T gl,
                                                int src_lane, bool lane0, T& outp, T& upp)
{
    const T INF = Num<T>::inf();
    T dv[8], tv[8];
    lds8(dv, cell);
    lds8(tv, top);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const T upw = __shfl_sync(kFull, outp, src_lane);
        const T up = lane0 ? tv[j] : upw;
        T r = SCALED ? fwd_cell_scaled<T>(dv[j] * k, upp, up, outp) : fwd_cell<T>(dv[j], upp, up, outp, k, gl);
        if (MASKED) {
            const int tau = tau0 + j;
            r = (tau >= A && tau <= Z) ? r : INF;
        }
        dv[j] = r;
        upp = up;
        outp = r;
    }
    sts8(cell, dv);
}

// Groups Q0 .. Q1 (Q0 even, Q1 odd) of the 32 steps of block `tau0 / 32` (four groups of 8), in pairs: before
// an even group q, wait for the strip above to have published its group g + 5 (group g of this strip reads
// columns up to 8g + 7 of the row above, complete with the group g + 4 of the strip above; g + 5 covers
// groups q and q + 1 with one wait); sweep the two groups; publish the 16 values of the last row that they
// finished, completing the barrier of the odd group. Only odd barriers are used. Returns false if the
// launch aborted.
template <typename T, bool MASKED, int Q0, int Q1, bool SCALED>
__device__ __forceinline__ bool fwd_pair_block(T* cell, const T* top, const T* last, T* bout, int tau0, int A, int Z,
                                               T k, T gl, bool wait_in, uint32_t bars_in, uint32_t par_in, int glast,
                                               bool publish, bool has_consumer, uint32_t bars_out, const Sync& sy,
                                               int src_lane, int lane, T& outp, T& upp)
{
    static_assert(Q0 % 2 == 0 && Q1 % 2 == 1, "groups come in pairs");
    const bool lane0 = lane == 0;
    const bool pub_lane = lane < kPubLanes;
    const int g0 = tau0 / 8;
#pragma unroll
    for (int q = Q0; q <= Q1; ++q) {
        if ((q & 1) == 0 && wait_in && !fbar_wait_fast(bars_in + 8 * min(g0 + q + 5, glast), par_in, sy, lane))
            return false;
        fwd_pair_steps8<T, MASKED, SCALED>(cell + 8 * q, top + 8 * q, tau0 + 8 * q, A, Z, k, gl, src_lane, lane0, outp,
                                           upp);
        if (publish && (q & 1) == 1) {
            // Columns tau0 + 8(q-1) - 31 .. tau0 + 8q - 24 of the last row (groups q - 1 and q), written by lane
            // 31 above: 8 lanes, 2 values each, then each arrives once.
            __syncwarp();
            const T v0 = last[8 * (q - 1) + (lane & (kPubLanes - 1))];
            const T v1 = last[8 * q + (lane & (kPubLanes - 1))];
            if (pub_lane && has_consumer) {
                bout[tau0 + 8 * (q - 1) + lane - 31 + kBufPad] = v0;
                bout[tau0 + 8 * q + lane - 31 + kBufPad] = v1;
            }
            fbar_arrive_n_if(bars_out + 8 * (g0 + q), 1, pub_lane);
        }
    }
    return true;
}

// One strip of the forward. Returns false if the launch aborted. MC > 0: the kernel is specialized on
// M == MC, so every row offset in the ring's loads and stores is a compile-time constant.
//
// Lane l processes column c at step tau = c + l + 1 (ring position tau), one step later than the skew of the
// strip-ticket kernels: a block's slot then holds, for row l, exactly the columns 32*blk + x - l - 1 that the
// backward's ring row l + 1 needs at its positions 32*blk + x, so that R can travel between the two as whole
// 32 x 32 tiles (PairFwdArgs::Rt). The boundary rows are indexed by column + kBufPad + 1.
//
// FUSED (float only, tiles only): D comes from fused_rect instead of a.D. Rectangle K lands in the slots of
// blocks K and K + 1, so it is computed after block K - 1 has written back its slot and before block K starts
// (rectangles k0 - 1 and k0 before the first block).
//
// SCALED (tiles only): R is kept, and written to the tiles, in units of gamma ln 2 (k R, k = log2(e) / gamma);
// the cost is converted back (times gamma ln 2) when the terminal cell writes it.
template <typename T, int MC, bool FUSED, bool SCALED>
__device__ bool fwd_pair_strip(const PairFwdArgs<T>& a, T* ring, const T* bin, uint32_t bars_in, uint32_t par_in,
                               T* bout, uint32_t bars_out, const float* y2, int64_t b, int s, int lane)
{
    constexpr int RS = FwdRing<T>::S;
    const T INF = Num<T>::inf();
    const int64_t N = a.N, M = MC > 0 ? MC : a.M, pitch = M + 2;
    const bool tiles = a.Rt != nullptr;
    const int r0 = 32 * s;
    const int nmat = static_cast<int>(N - r0 < 32 ? N - r0 : 32);
    T* Rrow = tiles ? nullptr : a.R + b * (N + 2) * pitch + static_cast<int64_t>(r0 + 1) * pitch;
    Strip st;
    if (!make_strip(st, a.len, b, s, N, M, a.bw, lane)) {
        if (s == 0 && lane == 0 && SDTW_IN_BOUNDS(a.xC, a.costs + b, sizeof(T), a.sy.err)) {
            if (st.bad) {
                atomicOr(a.sy.err, kErrBadLength);
                a.costs[b] = Num<T>::nan();
            } else {
                a.costs[b] = (st.nx == 0 && st.ny == 0) ? T(0) : INF;
            }
        }
        if (!tiles)
            for (int r = 0; r < nmat; ++r)
                for (int c = lane; c < M + 2; c += 32)
                    if (SDTW_IN_BOUNDS(a.xR, Rrow + r * pitch + c, sizeof(T), a.sy.err)) Rrow[r * pitch + c] = INF;
        // No barrier arrivals: every later strip of this pair is empty too, so nothing waits on this
        // warp's barriers again (arriving here could lap the phase the strip below the previous round
        // is still waiting for).
        return true;
    }
    // Valid steps of this lane and of the whole warp, in this kernel's step numbering.
    const int A = st.A + 1, Z = st.Z + 1, Amax = st.Amax + 1, Zmin = st.Zmin + 1;
    const int k0 = (st.c_begin + 1) >> 5;
    const int k1 = (st.c_end + 32) >> 5;
    const bool skip = b * a.S + s == a.inject;
    const bool has_consumer = st.rows == 32 && r0 + 32 < st.nx && !skip;
    const T* Db = a.D + (b * N + r0) * M;
    T* tile0 = tiles ? a.Rt + (b * a.S + s) * static_cast<int64_t>(a.NBt) * 1024 : nullptr;

    float x2[4];  // FUSED: |x|^2 of rows r0 + lane/4 + 8i
    const float* Xs = nullptr;
    const float* Yb = nullptr;
    if constexpr (FUSED) {
        Xs = a.f.X + (b * N + r0) * a.f.d;
        Yb = a.f.Y + b * M * a.f.d;
        float xn = 0.f;
        if (r0 + lane < N) {
            const float4* xr = reinterpret_cast<const float4*>(Xs + static_cast<int64_t>(lane) * a.f.d);
            for (int q = 0; q < a.f.d / 4; ++q) {
                const float4 v = SDTW_IN_BOUNDS(a.f.xX, xr + q, 16, a.sy.err) ? __ldg(xr + q)
                                                                               : make_float4(0.f, 0.f, 0.f, 0.f);
                xn = fmaf(v.x, v.x, xn);
                xn = fmaf(v.y, v.y, xn);
                xn = fmaf(v.z, v.z, xn);
                xn = fmaf(v.w, v.w, xn);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) x2[i] = __shfl_sync(kFull, xn, (lane >> 2) + 8 * i);
        __syncwarp();
        if (k0 > 0) fused_rect(a.f, ring, Xs, Yb, x2, y2, b, r0, N, M, k0 - 1, lane, a.sy.err);
        fused_rect(a.f, ring, Xs, Yb, x2, y2, b, r0, N, M, k0, lane, a.sy.err);
        __syncwarp();
    } else {
        cp_async_wait<0>();
        __syncwarp();
        fwd_pair_load<T>(Db, M, ring, k0, st.rows, lane, a.xD, a.sy.err);
        cp_async_commit();
    }

    if (!tiles) {
        // Padded columns of each row outside the swept range (columns 32*k0 - r - 1 .. 32*k1 + 30 - r, padded
        // index + 1), and the border: +inf.
        for (int r = 0; r < nmat; ++r) {
            T* row = Rrow + r * pitch;
            int pe = 32 * k0 - r - 1;
            pe = pe < 0 ? 0 : pe;
            int ss = 32 * k1 + 32 - r;
            ss = ss > M + 1 ? static_cast<int>(M + 1) : ss;
            for (int c = lane; c <= pe; c += 32)
                if (SDTW_IN_BOUNDS(a.xR, row + c, sizeof(T), a.sy.err)) row[c] = INF;
            for (int c = ss + lane; c < M + 2; c += 32)
                if (SDTW_IN_BOUNDS(a.xR, row + c, sizeof(T), a.sy.err)) row[c] = INF;
        }
    }

    // Terminal cell (nx-1, ny-1): lane lstar at step tstar.
    const int lstar = static_cast<int>(st.nx - 1 - r0);
    const int tstar = static_cast<int>(st.ny - 1) + lstar + 1;
    const int bstar = (lstar >= 0 && lstar < 32) ? (tstar >> 5) : INT_MIN;

    const int glast = a.G - 1;
    const bool wait_in = s > 0;
    // (Group 4 k0 + 4 of the strip above holds the values the first group reads; its barriers complete in
    // pairs, on the odd group.)
    if (wait_in && !fbar_wait(bars_in + 8 * min(4 * k0 + 5, glast), par_in, a.sy, lane)) return false;
    T upp = lane == 0 ? bin[32 * k0 - 1 + kBufPad] : INF;  // lane 0's diagonal predecessor (column 32*k0 - 2)
    T outp = INF;
    const int src_lane = (lane + 31) & 31;

    // D of the first block is in flight; each block prefetches D of the next one into the other slot as it
    // starts (that slot's R was written back, synchronously, at the end of the block before).
#pragma unroll 1
    for (int blk = k0; blk <= k1; ++blk) {
        if constexpr (!FUSED) {
            cp_async_wait<0>();
            __syncwarp();
            if (blk + 1 <= k1) fwd_pair_load<T>(Db, M, ring, blk + 1, st.rows, lane, a.xD, a.sy.err);
            cp_async_commit();
        }
        const int tau0 = 32 * blk;
        T* cell = ring + lane * RS + (blk & 1) * 32;
        const T* top = bin + tau0 + kBufPad;
        const T* last = ring + 31 * RS + (blk & 1) * 32;  // the strip's last row, positions tau0 ..
        const bool ok = (tau0 >= Amax && tau0 + 31 <= Zmin)
                            ? fwd_pair_block<T, false, 0, 3, SCALED>(cell, top, last, bout, tau0, A, Z, a.k, a.gl, wait_in,
                                                             bars_in, par_in, glast, !skip, has_consumer, bars_out,
                                                             a.sy, src_lane, lane, outp, upp)
                            : fwd_pair_block<T, true, 0, 3, SCALED>(cell, top, last, bout, tau0, A, Z, a.k, a.gl, wait_in,
                                                            bars_in, par_in, glast, !skip, has_consumer, bars_out,
                                                            a.sy, src_lane, lane, outp, upp);
        if (!ok) return false;
        __syncwarp();
        if (tiles)
            fwd_tile_store<T>(tile0 + static_cast<int64_t>(blk) * 1024, ring, blk, lane, a.xRt, a.sy.err);
        else
            fwd_pair_store<T>(Rrow, pitch, M, ring, blk, nmat, lane, a.xR, a.sy.err);
        if (blk == bstar && lane == lstar && SDTW_IN_BOUNDS(a.xC, a.costs + b, sizeof(T), a.sy.err))
            a.costs[b] = SCALED ? cell[tstar - tau0] * a.gl : cell[tstar - tau0];
        __syncwarp();
        if constexpr (FUSED) {
            if (blk + 1 <= k1) {
                fused_rect(a.f, ring, Xs, Yb, x2, y2, b, r0, N, M, blk + 1, lane, a.sy.err);
                __syncwarp();
            }
        }
    }
    if (!skip) {
        // The strip below may read columns past this sweep as its row above: they are out of band (+inf).
        if (has_consumer)
            for (int c = 32 * k1 + 1 + lane; c + kBufPad < a.BL; c += 32) bout[c + kBufPad] = INF;
        __syncwarp();
        // Complete the barriers of the groups this sweep did not reach (every odd barrier once per strip; each
        // phase expects kPubLanes arrivals).
        for (int g = lane; g < a.G; g += 32)
            if ((g & 1) == 1 && (g < 4 * k0 || g > 4 * k1 + 3)) fbar_arrive_n_if(bars_out + 8 * g, kPubLanes, true);
    }
    return true;
}

template <typename T, int MC, bool FUSED, bool SCALED>
__global__ void __launch_bounds__(SDTW_PAIR_THREADS, SDTW_PAIR_MIN_CTAS) sdtw_fwd_pair_kernel(PairFwdArgs<T> a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int RS = FwdRing<T>::S;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int W = a.W;
    T* rings = reinterpret_cast<T*>(smem);
    T* bufs = rings + static_cast<size_t>(W) * 32 * RS;
    T* crow = bufs + static_cast<size_t>(W) * a.BL;
    T* scratch = crow + a.BL;  // 32 elements per warp
    const uint32_t bars = (smem_addr(scratch + static_cast<size_t>(W) * 32) + 7u) & ~7u;  // [W][G] mbarriers
    const int64_t b = blockIdx.x;
    const T INF = Num<T>::inf();
    // Zero the rings and boundary rows (stale shared memory must not feed NaN patterns to masked
    // cells); the row above strip 0 is +inf with R[-1][-1] = 0.
    for (int e = threadIdx.x; e < W * (32 * RS + a.BL); e += blockDim.x) rings[e] = T(0);
    for (int e = threadIdx.x; e < a.BL; e += blockDim.x) crow[e] = e == kBufPad ? T(0) : INF;  // column -1: 0
    for (int e = threadIdx.x; e < W * a.G; e += blockDim.x)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bars + 8 * e), "r"(kPubLanes) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // FUSED: |y|^2 of the pair's columns, zero-padded by 32 before column 0 and 64 after M - 1.
    float* y2 = nullptr;
    if constexpr (FUSED) {
        float* y2s = reinterpret_cast<float*>(smem + fused_y2_offset(W, a.M));
        const float* Yb = a.f.Y + b * a.M * a.f.d;
        for (int e = threadIdx.x; e < a.M + 96; e += blockDim.x) {
            const int64_t c = e - 32;
            float sq = 0.f;
            if (c >= 0 && c < a.M) {
                const float4* yr = reinterpret_cast<const float4*>(Yb + c * a.f.d);
                for (int q = 0; q < a.f.d / 4; ++q) {
                    const float4 v = SDTW_IN_BOUNDS(a.f.xY, yr + q, 16, a.sy.err) ? __ldg(yr + q)
                                                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
                    sq = fmaf(v.x, v.x, sq);
                    sq = fmaf(v.y, v.y, sq);
                    sq = fmaf(v.z, v.z, sq);
                    sq = fmaf(v.w, v.w, sq);
                }
            }
            y2s[e] = sq;
        }
        y2 = y2s + 32;
    }
    // Padded rows 0 and N+1 of R (softdtw.cpp:114-121: +inf with R[b,0,0] = 0).
    if (a.Rt == nullptr) {
        T* Rb = a.R + b * (a.N + 2) * (a.M + 2);
        for (int64_t e = threadIdx.x; e < a.M + 2; e += blockDim.x) {
            if (SDTW_IN_BOUNDS(a.xR, Rb + e, sizeof(T), a.sy.err)) Rb[e] = e == 0 ? T(0) : INF;
            T* last_row = Rb + (a.N + 1) * (a.M + 2) + e;
            if (SDTW_IN_BOUNDS(a.xR, last_row, sizeof(T), a.sy.err)) *last_row = INF;
        }
    }
    __syncthreads();
    T* ring = rings + static_cast<size_t>(warp) * 32 * RS;
    for (int s = warp; s < a.S; s += W) {
        const int wp = (s + W - 1) % W;
        const T* bin = s > 0 ? bufs + static_cast<size_t>(wp) * a.BL : crow;
        const uint32_t par_in = static_cast<uint32_t>(((s - 1) / W) & 1);  // round of the strip above in its warp
        if (!fwd_pair_strip<T, MC, FUSED, SCALED>(a, ring, bin, bars + 8 * wp * a.G, par_in,
                                          bufs + static_cast<size_t>(warp) * a.BL, bars + 8 * warp * a.G, y2, b, s,
                                          lane))
            break;
    }
    cp_async_wait<0>();
}

// ==================================================================================================
// Backward (scatter form, see sdtw_wavefront.cu)
// ==================================================================================================
// Backward ring of a warp: 33 rows (ring row p = padded R row r0 + p = DP row r0 - 1 + p) x 2 slots of 32
// positions, row p holding DP column c at position c + p (the forward's skew). At step tau, lane l (DP row
// i = r0 + l, column c = tau - l) reads R[i-1][c-1] and R[i-1][c] at positions tau - 1 and tau of ring row l,
// and R[i][c-1] at position tau of ring row l + 1, and writes E[i][c] in place of the last (R[i][c-1] is not
// read again: the cells that need it, (i, c) itself and the row below, have already run). A group of 8 steps
// therefore reads and writes aligned 16-byte vectors. Strides as in FwdRing (2 slots + pad).
template <typename T>
struct BwdRing {
    static constexpr int S = sizeof(T) == 4 ? 68 : 66;
};

template <typename T>
struct PairBwdArgs {
    const T* R;   // padded R (B, N+2, M+2), or null when Rt is given
    const T* Rt;  // R as the forward's strip tiles (B, S, NBt, 32, 32), or null
    int NBt;
    T* E;
    Lengths len;
    int64_t B, N, M, bw;
    int S, W, BL, G;  // strips, warps, boundary row length, progress barriers per warp
    T k;
    Extent xR, xRt, xE;  // buffers, for the debug build's bounds checks
    Sync sy;
    int64_t inject;
};

// Padded R rows r0 .. r0+32 (DP rows r0-1 .. r0+31), skewed slot of block `blk` <- global.
template <typename T>
__device__ __forceinline__ void bwd_pair_load(const T* Rb, int64_t N, int64_t M, T* ring, int blk, int r0, int lane,
                                              const Extent& xR, uint32_t* err)
{
    constexpr int S = BwdRing<T>::S;
    const int64_t pitch = M + 2;
    T* dst = ring + (blk & 1) * 32 + lane;
    const int c0 = 32 * blk + lane;  // column read by ring row 0; ring row p reads column c0 - p
    if (32 * blk - 31 >= 0 && 32 * blk + 32 <= M + 1 && r0 + 32 <= N + 1) {
        const T* src = Rb + static_cast<int64_t>(r0) * pitch + c0 + 1;
        const int64_t step = pitch - 1;
#pragma unroll 11
        for (int p = 0; p < 33; ++p) {
            const bool ok = SDTW_IN_BOUNDS(xR, src, sizeof(T), err);
            cp_async_scalar<sizeof(T)>(dst + p * S, ok ? src : Rb, ok ? static_cast<int>(sizeof(T)) : 0);
            src += step;
        }
    } else {
        for (int p = 0; p < 33; ++p) {
            const int pc = c0 - p + 1;  // padded column
            bool in = r0 + p <= N + 1 && pc >= 0 && pc <= M + 1;
            if (in) in = SDTW_IN_BOUNDS(xR, Rb + static_cast<int64_t>(r0 + p) * pitch + pc, sizeof(T), err);
            cp_async_scalar<sizeof(T)>(dst + p * S, in ? Rb + static_cast<int64_t>(r0 + p) * pitch + pc : Rb,
                                       in ? static_cast<int>(sizeof(T)) : 0);
        }
    }
}

// Slot of block `blk` <- R tiles written by the forward, asynchronously (cp.async, 16-byte pieces): ring rows
// 1..32 from tile (s, blk), each lane copying its own row, and ring row 0 from row 31 of tile (s-1, blk+1)
// (the forward's skew puts both at the positions this ring expects). Tiles outside the forward's swept blocks
// ([kf0, kf1] for strip s, [kp0, kp1] for strip s-1) were never written: their cells are outside the band or
// the lengths, +inf, and are filled here instead (the row above strip 0 is R's border row, +inf with
// R[-1][-1] = 0).
template <typename T>
__device__ __forceinline__ void bwd_tile_load(const PairBwdArgs<T>& a, T* ring, int blk, int64_t b, int s, int kf0,
                                              int kf1, int kp0, int kp1, int lane)
{
    constexpr int RS = BwdRing<T>::S;
    constexpr int EPP = 16 / sizeof(T);  // elements per 16-byte piece
    const T INF = Num<T>::inf();
    T* slot = ring + (blk & 1) * 32;
    T* row = slot + (lane + 1) * RS;
    if (blk >= kf0 && blk <= kf1) {
        const T* src = a.Rt + (((b * a.S + s) * static_cast<int64_t>(a.NBt) + blk) * 32 + lane) * 32;
#pragma unroll
        for (int i = 0; i < 32; i += EPP) {
            const bool ok = SDTW_IN_BOUNDS(a.xRt, src + i, 16, a.sy.err);
            cp_async_16(row + i, ok ? src + i : a.Rt, ok ? 16 : 0);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) row[i] = INF;
    }
    if (s > 0 && blk + 1 >= kp0 && blk + 1 <= kp1) {
        const T* src = a.Rt + (((b * a.S + s - 1) * static_cast<int64_t>(a.NBt) + blk + 1) * 32 + 31) * 32;
        if (lane < 32 / EPP) {
            const bool ok = SDTW_IN_BOUNDS(a.xRt, src + lane * EPP, 16, a.sy.err);
            cp_async_16(slot + lane * EPP, ok ? src + lane * EPP : a.Rt, ok ? 16 : 0);
        }
    } else {
        slot[lane] = (s == 0 && blk == -1 && lane == 31) ? T(0) : INF;
    }
}

// E of slot `blk` -> global (Erow = E row of DP row r0): ring row r + 1 holds E[r0 + r][c] at position c + r.
// Every position of the slot was written by the block's sweep (zeros where a step was outside the band).
template <typename T>
__device__ __forceinline__ void bwd_pair_store(T* Erow, int64_t M, const T* ring, int blk, int nmat, int lane,
                                               const Extent& xE, uint32_t* err)
{
    constexpr int S = BwdRing<T>::S;
    const T* src = ring + S + (blk & 1) * 32 + lane;
    const int c0 = 32 * blk + lane;  // column of row 0; row r: c0 - r
    if (32 * blk - 31 >= 0 && 32 * blk + 31 < M && nmat == 32) {
        T* dst = Erow + c0;
        const int64_t step = M - 1;
#pragma unroll 8
        for (int r = 0; r < 32; ++r) {
            if (SDTW_IN_BOUNDS(xE, dst, sizeof(T), err)) *dst = src[r * S];
            dst += step;
        }
    } else {
        for (int r = 0; r < nmat; ++r) {
            const int c = c0 - r;
            if (c >= 0 && c < M && SDTW_IN_BOUNDS(xE, Erow + r * M + c, sizeof(T), err)) Erow[r * M + c] = src[r * S];
        }
    }
}

// 8 backward steps tau = t8+7 .. t8 of one warp. A: ring row l at positions t8 .. t8+7, am1: position t8-1;
// Bv: ring row l+1 at positions t8 .. t8+7 (R in, E out); bvv: lane 31's contributions from the strip below
// (columns t8-31 .. t8-24); sv: the values lane 0 pushes into the row above (columns t8 .. t8+7).
// SCALED: R arrives in units of gamma ln 2 (the forward's tiles), so the weights need no product with k.
template <typename T, bool MASKED, bool SCALED>
__device__ __forceinline__ void bwd_pair_steps8(const T (&A)[8], T am1, T (&Bv)[8], const T (&bvv)[8], T (&sv)[8],
                                                int t8, int Av, int Zv, T k, T seed, int src_lane, bool lane31,
                                                T& sendv, T& pend, T& acc)
{
    const T big = Num<T>::big();
#pragma unroll
    for (int j = 7; j >= 0; --j) {
        const T rd = j > 0 ? A[j > 0 ? j - 1 : 0] : am1;  // R[i-1][c-1]
        const T ru = A[j];                                // R[i-1][c]
        const T rl = Bv[j];                               // R[i][c-1]
        const T recvw = __shfl_sync(kFull, sendv, src_lane);
        const T recv = lane31 ? bvv[j] : recvw;
        const T Es = acc + recv;
        const T m = Num<T>::mn(Num<T>::mn(rd, ru), rl);
        const T mc = Num<T>::mn(m, big);
        const T ed = Num<T>::exp2_(SCALED ? mc - rd : (mc - rd) * k);
        const T eu = Num<T>::exp2_(SCALED ? mc - ru : (mc - ru) * k);
        const T el = Num<T>::exp2_(SCALED ? mc - rl : (mc - rl) * k);
        T q = Es * Num<T>::rcp_((ed + eu) + el);
        T Eo = Es;
        if (MASKED) {
            const int tau = t8 + j;
            const bool valid = tau >= Av && tau <= Zv;
            q = valid ? q : T(0);
            acc = valid ? q * el : seed;
            Eo = valid ? Es : T(0);
        } else {
            acc = q * el;
        }
        sendv = fma(q, eu, pend);
        pend = q * ed;
        Bv[j] = Eo;
        sv[j] = sendv;
    }
}

// The 32 steps of block tau0 / 32 as four groups of 8, top group first. Before group g (steps 8g .. 8g+7)
// the strip below must have completed its group g - 4: lane 31 reads the contributions into columns
// 8g - 31 .. 8g - 24, pushed by the strip below at its steps 8g - 31 .. 8g - 24 (groups g - 4 and g - 3; the
// strip below sweeps downwards, so g - 3 completes first). The groups go in pairs: before an odd group g, one
// wait on group g - 5 of the strip below covers g and g - 1; after the even group, the 16 pushes of the pair
// are published and the even group's barrier completes (only even barriers are used). `bcar` carries the
// contribution at column 8g - 24, loaded with the group above. Returns false if the launch aborted.
template <typename T, bool MASKED, bool SCALED>
__device__ __forceinline__ bool bwd_pair_block(T* ring, const T* bin, T* bout, int tau0, const Strip& st, T k, T seed,
                                               bool wait_in, uint32_t bars_in, uint32_t par_in, bool publish,
                                               uint32_t bars_out, bool slot_below_pending, const Sync& sy,
                                               int src_lane, int lane, T& sendv, T& pend, T& acc, T& bcar)
{
    constexpr int RS = BwdRing<T>::S;
    const bool lane31 = lane == 31;
    T* rowA = ring + lane * RS + (tau0 & 32);  // ring row l, positions tau0 .. (slot of this block)
    T* rowB = rowA + RS;                       // ring row l + 1
    const int g0 = tau0 / 8;
    T svp[8];  // the pushes of the odd group, published with the even group below it
#pragma unroll
    for (int q = 3; q >= 0; --q) {
        const int t8 = tau0 + 8 * q;
        if ((q & 1) == 1 && wait_in && !fbar_wait_fast(bars_in + 8 * max(g0 + q - 5, 0), par_in, sy, lane))
            return false;
        if (q == 0 && slot_below_pending) {  // position tau0 - 1 lies in the slot of the block below
            cp_async_wait<0>();
            __syncwarp();
        }
        T A[8], Bv[8], bvv[8], sv[8];
        lds8(A, rowA + 8 * q);
        // Position t8 - 1 of ring row l: the slot of the block below for the group q = 0.
        const T am1 = q > 0 ? rowA[8 * q - 1] : ring[lane * RS + ((tau0 - 1) & 63)];
        lds8(Bv, rowB + 8 * q);
        {
            T v[8];
            lds8(v, bin + t8 - 32 + kBufPad);
#pragma unroll
            for (int j = 0; j < 7; ++j) bvv[j] = v[j + 1];
            bvv[7] = bcar;
            bcar = v[0];
        }
        bwd_pair_steps8<T, MASKED, SCALED>(A, am1, Bv, bvv, sv, t8, st.A, st.Z, k, seed, src_lane, lane31, sendv, pend,
                                           acc);
        __syncwarp();  // every lane has read ring row l+1 [t8, t8+8) (its A) before lane l overwrites it
        sts8(rowB + 8 * q, Bv);
        if (publish) {
            if (q & 1) {
#pragma unroll
                for (int j = 0; j < 8; ++j) svp[j] = sv[j];
            } else {
                if (lane == 0) {
                    sts8(bout + t8 + 8 + kBufPad, svp);
                    sts8(bout + t8 + kBufPad, sv);
                }
                fbar_arrive_n_if(bars_out + 8 * (g0 + q), 1, lane == 0);
            }
        }
    }
    return true;
}

// One strip of the backward; `t` is its position in sweep order (strip S-1-t). Returns false if the
// launch aborted.
template <typename T, int MC, bool SCALED>
__device__ bool bwd_pair_strip(const PairBwdArgs<T>& a, T* ring, const T* bin, uint32_t bars_in, uint32_t par_in,
                               const T* zrow, T* bout, uint32_t bars_out, int64_t b, int s, int lane)
{
    const int64_t N = a.N, M = MC > 0 ? MC : a.M;
    const int r0 = 32 * s;
    const int nmat = static_cast<int>(N - r0 < 32 ? N - r0 : 32);
    T* Erow = a.E + (b * N + r0) * M;
    Strip st;
    if (!make_strip(st, a.len, b, s, N, M, a.bw, lane)) {
        if (st.bad && s == 0 && lane == 0) atomicOr(a.sy.err, kErrBadLength);
        for (int r = 0; r < nmat; ++r)
            for (int c = lane; c < M; c += 32)
                if (SDTW_IN_BOUNDS(a.xE, Erow + r * M + c, sizeof(T), a.sy.err)) Erow[r * M + c] = T(0);
        // Empty strips (rows past the pair's length) come first in the bottom-up order, and their warps sweep
        // non-empty strips in later rounds: complete every barrier once here too, so that a warp's barrier
        // phases keep counting its rounds (nothing waits on these arrivals: the strip above an empty strip
        // has no producer).
        for (int g = lane; g < a.G; g += 32)
            if ((g & 1) == 0) fbar_arrive_n_if(bars_out + 8 * g, 1, true);
        return true;
    }
    const int k0 = st.c_begin >> 5;
    const int k1 = (st.c_end + 31) >> 5;
    const int kmin = (32 * k0 - 1) >> 5;  // arithmetic shift: -1 when k0 == 0
    const bool has_producer = r0 + 32 < st.nx;
    const bool skip = b * a.S + s == a.inject;
    const bool publish = s > 0 && !skip;
    if (!has_producer) bin = zrow;
    const T seed = (r0 + lane == st.nx - 1) ? T(1) : T(0);
    const bool tiles = a.Rt != nullptr;
    const T* Rb = tiles ? nullptr : a.R + b * (N + 2) * (M + 2);
    // Blocks of the forward's tiles of this strip and of the strip above (the forward's skew is one step later).
    const int kf0 = (st.c_begin + 1) >> 5, kf1 = (st.c_end + 32) >> 5;
    int kp0 = 0, kp1 = -1;
    if (tiles && s > 0) {
        int64_t lo, hi, lo2, hi2;
        band_row_range(r0 - 32, st.nx, st.ny, a.bw, lo, hi);
        band_row_range(r0 - 1, st.nx, st.ny, a.bw, lo2, hi2);
        kp0 = static_cast<int>((lo + 1) >> 5);
        kp1 = static_cast<int>((hi2 + 32) >> 5);
    }

    cp_async_wait<0>();
    __syncwarp();
    if (tiles)
        bwd_tile_load<T>(a, ring, k1, b, s, kf0, kf1, kp0, kp1, lane);
    else
        bwd_pair_load<T>(Rb, N, M, ring, k1, r0, lane, a.xR, a.sy.err);
    cp_async_commit();
    if (k1 - 1 >= kmin) {
        if (tiles)
            bwd_tile_load<T>(a, ring, k1 - 1, b, s, kf0, kf1, kp0, kp1, lane);
        else
            bwd_pair_load<T>(Rb, N, M, ring, k1 - 1, r0, lane, a.xR, a.sy.err);
    }
    cp_async_commit();

    // Columns of each row outside the stored range [32*k0 - r, 32*k1 + 31 - r]: zero.
    for (int r = 0; r < nmat; ++r) {
        T* row = Erow + r * M;
        int pe = 32 * k0 - r;
        pe = pe < 0 ? 0 : (pe > M ? static_cast<int>(M) : pe);
        int ss = 32 * k1 + 32 - r;
        ss = ss > M ? static_cast<int>(M) : ss;
        for (int c = lane; c < pe; c += 32)
            if (SDTW_IN_BOUNDS(a.xE, row + c, sizeof(T), a.sy.err)) row[c] = T(0);
        for (int c = ss + lane; c < M; c += 32)
            if (SDTW_IN_BOUNDS(a.xE, row + c, sizeof(T), a.sy.err)) row[c] = T(0);
    }

    T sendv = T(0), pend = T(0), acc = seed;
    // The carry of the top group g = 4*k1 + 3 (lane 31's contribution at column 8g - 24 = 32*k1) comes from the
    // strip below's group 4*k1, complete once the group's own wait (on group g - 4) returns.
    T bcar = T(0);
    bool first = true;
    const int src_lane = (lane + 1) & 31;

#pragma unroll 1
    for (int blk = k1; blk >= k0; --blk) {
        cp_async_wait<1>();
        __syncwarp();
        const int tau0 = 32 * blk;
        if (first) {
            // Group 4 k1 - 1 of the strip below holds the carry; its barrier completes with the pair's even
            // group 4 k1 - 2.
            if (has_producer && !fbar_wait_fast(bars_in + 8 * max(4 * k1 - 2, 0), par_in, a.sy, lane))
                return false;
            bcar = bin[32 * k1 + kBufPad];
            first = false;
        }
        const bool below = blk - 1 >= kmin;
        const bool ok = (tau0 >= st.Amax && tau0 + 31 <= st.Zmin)
                            ? bwd_pair_block<T, false, SCALED>(ring, bin, bout, tau0, st, a.k, seed, has_producer, bars_in,
                                                       par_in, publish, bars_out, below, a.sy, src_lane, lane, sendv,
                                                       pend, acc, bcar)
                            : bwd_pair_block<T, true, SCALED>(ring, bin, bout, tau0, st, a.k, seed, has_producer, bars_in,
                                                      par_in, publish, bars_out, below, a.sy, src_lane, lane, sendv,
                                                      pend, acc, bcar);
        if (!ok) return false;
        __syncwarp();
        bwd_pair_store<T>(Erow, M, ring, blk, nmat, lane, a.xE, a.sy.err);
        __syncwarp();
        if (blk - 2 >= kmin) {
            if (tiles)
                bwd_tile_load<T>(a, ring, blk - 2, b, s, kf0, kf1, kp0, kp1, lane);
            else
                bwd_pair_load<T>(Rb, N, M, ring, blk - 2, r0, lane, a.xR, a.sy.err);
        }
        cp_async_commit();
    }
    cp_async_wait<0>();
    __syncwarp();
    if (publish) {
        // Lane 0's last diagonal push (into column 32*k0 - 1) and zeros below the sweep; then complete the
        // barriers of the groups below the sweep (every barrier once per strip).
        if (lane == 0) bout[32 * k0 - 1 + kBufPad] = pend;
        for (int c = -kBufPad + lane; c <= 32 * k0 - 2; c += 32) bout[c + kBufPad] = T(0);
        __syncwarp();
        for (int g = lane; g < 4 * k0; g += 32)
            if ((g & 1) == 0) fbar_arrive_n_if(bars_out + 8 * g, 1, true);
    }
    __syncwarp();
    return true;
}

template <typename T, int MC, bool SCALED>
__global__ void __launch_bounds__(SDTW_PAIR_THREADS, SDTW_PAIR_MIN_CTAS) sdtw_bwd_pair_kernel(PairBwdArgs<T> a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int RS = BwdRing<T>::S;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int W = a.W;
    T* rings = reinterpret_cast<T*>(smem);
    T* bufs = rings + static_cast<size_t>(W) * 33 * RS;
    T* zrow = bufs + static_cast<size_t>(W) * a.BL;
    const uint32_t bars = (smem_addr(zrow + a.BL) + 7u) & ~7u;  // [W][G] progress mbarriers
    const int64_t b = blockIdx.x;
    for (int e = threadIdx.x; e < W * (33 * RS + a.BL) + a.BL; e += blockDim.x) rings[e] = T(0);
    for (int e = threadIdx.x; e < W * a.G; e += blockDim.x)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bars + 8 * e), "r"(1) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    T* ring = rings + static_cast<size_t>(warp) * 33 * RS;
    for (int t = warp; t < a.S; t += W) {
        const int wp = (t + W - 1) % W;
        const uint32_t par_in = static_cast<uint32_t>(((t - 1) / W) & 1);  // round of the strip below in its warp
        if (!bwd_pair_strip<T, MC, SCALED>(a, ring, bufs + static_cast<size_t>(wp) * a.BL, bars + 8 * wp * a.G, par_in, zrow,
                                   bufs + static_cast<size_t>(warp) * a.BL, bars + 8 * warp * a.G, b, a.S - 1 - t,
                                   lane))
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
    return (static_cast<size_t>(W) * (32 * FwdRing<T>::S + 32) + static_cast<size_t>(W + 1) * buf_len(M)) * sizeof(T) +
           8 + static_cast<size_t>(W) * fwd_groups(M) * 8;
}
template <typename T>
size_t pair_bwd_smem_bytes(int W, int64_t M)
{
    return (static_cast<size_t>(W) * 33 * BwdRing<T>::S + static_cast<size_t>(W + 1) * buf_len(M)) * sizeof(T) + 8 +
           static_cast<size_t>(W) * fwd_groups(M) * 8;
}

// The kernel instantiations: M specialized (MC = kPairSpecialM) or not; R in its own units (padded R) or in
// units of gamma ln 2 (R tiles, SCALED); the fused cost forward (float, tiles).
template <typename T>
cudaError_t pair_init_attrs(int max_smem)
{
    const auto set = [max_smem](const void* f) {
        return cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    };
    const void* kernels[] = {
        reinterpret_cast<const void*>(sdtw_fwd_pair_kernel<T, 0, false, false>),
        reinterpret_cast<const void*>(sdtw_fwd_pair_kernel<T, kPairSpecialM, false, false>),
        reinterpret_cast<const void*>(sdtw_fwd_pair_kernel<T, 0, false, true>),
        reinterpret_cast<const void*>(sdtw_fwd_pair_kernel<T, kPairSpecialM, false, true>),
        reinterpret_cast<const void*>(sdtw_bwd_pair_kernel<T, 0, false>),
        reinterpret_cast<const void*>(sdtw_bwd_pair_kernel<T, kPairSpecialM, false>),
        reinterpret_cast<const void*>(sdtw_bwd_pair_kernel<T, 0, true>),
        reinterpret_cast<const void*>(sdtw_bwd_pair_kernel<T, kPairSpecialM, true>),
    };
    for (const void* f : kernels) {
        const cudaError_t e = set(f);
        if (e != cudaSuccess) return e;
    }
    if constexpr (sizeof(T) == 4) {
        cudaError_t e = set(reinterpret_cast<const void*>(sdtw_fwd_pair_kernel<float, 0, true, true>));
        if (e == cudaSuccess) e = set(reinterpret_cast<const void*>(sdtw_fwd_pair_kernel<float, kPairSpecialM, true, true>));
        return e;
    }
    return cudaSuccess;
}
template cudaError_t pair_init_attrs<float>(int);
template cudaError_t pair_init_attrs<double>(int);

template <typename T>
cudaError_t pair_regs(bool backward, int& regs)
{
    // The largest count over the direction's instantiations (the ones specialized on M can need more).
    const void* fwd[] = {reinterpret_cast<const void*>(sdtw_fwd_pair_kernel<T, 0, false, false>),
                         reinterpret_cast<const void*>(sdtw_fwd_pair_kernel<T, kPairSpecialM, false, false>),
                         reinterpret_cast<const void*>(sdtw_fwd_pair_kernel<T, 0, false, true>),
                         reinterpret_cast<const void*>(sdtw_fwd_pair_kernel<T, kPairSpecialM, false, true>)};
    const void* bwd[] = {reinterpret_cast<const void*>(sdtw_bwd_pair_kernel<T, 0, false>),
                         reinterpret_cast<const void*>(sdtw_bwd_pair_kernel<T, kPairSpecialM, false>),
                         reinterpret_cast<const void*>(sdtw_bwd_pair_kernel<T, 0, true>),
                         reinterpret_cast<const void*>(sdtw_bwd_pair_kernel<T, kPairSpecialM, true>)};
    regs = 0;
    for (const void* f : backward ? bwd : fwd) {
        cudaFuncAttributes fa;
        const cudaError_t e = cudaFuncGetAttributes(&fa, f);
        if (e != cudaSuccess) {
            regs = 0;
            return e;
        }
        regs = fa.numRegs > regs ? fa.numRegs : regs;
    }
    return cudaSuccess;
}
template cudaError_t pair_regs<float>(bool, int&);
template cudaError_t pair_regs<double>(bool, int&);

size_t pair_fused_smem_bytes(int W, int64_t M) { return fused_smem_bytes(W, M); }

cudaError_t pair_fused_regs(int& regs)
{
    cudaFuncAttributes fa, fb;
    cudaError_t e = cudaFuncGetAttributes(&fa, sdtw_fwd_pair_kernel<float, 0, true, true>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fb, sdtw_fwd_pair_kernel<float, kPairSpecialM, true, true>);
    regs = e == cudaSuccess ? (fa.numRegs > fb.numRegs ? fa.numRegs : fb.numRegs) : 0;
    return e;
}

// Warps per CTA: at most `cap` and the pair's strip count, and few enough for the CTA to fit `budget`.
template <typename T>
int pair_warps(bool backward, int64_t N, int64_t M, int cap, size_t budget)
{
    const int64_t S = N > 0 ? (N + 31) / 32 : 1;
    int W = static_cast<int>(S < cap ? S : cap);
    if (W > kPairMaxWarps) W = kPairMaxWarps;
    while (W >= 1) {
        const size_t bytes = backward ? pair_bwd_smem_bytes<T>(W, M) : pair_fwd_smem_bytes<T>(W, M);
        if (bytes <= budget) {
            // As few warps as give the same number of rounds over the strips (16 strips on 9 warps take 2 rounds
            // like 8 warps, with an idle warp in the second): fewer registers and less shared memory per CTA.
            const int64_t rounds = (S + W - 1) / W;
            return static_cast<int>((S + rounds - 1) / rounds);
        }
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
cudaError_t pair_forward(const T* D, T* R, T* Rt, T* costs, const void* lx, const void* ly, int is32, int64_t B,
                         int64_t N, int64_t M, int64_t bw, double gamma, int W, Sync sy, int64_t inject,
                         cudaStream_t stream)
{
    PairFwdArgs<T> a;
    a.D = D;
    a.R = R;
    a.Rt = Rt;
    a.NBt = pair_tile_blocks(M);
    const size_t es = sizeof(T);
    const int64_t S = N > 0 ? (N + 31) / 32 : 1;
    a.xD = Extent{D, static_cast<size_t>(B * N * M) * es};
    a.xR = Extent{R, R ? static_cast<size_t>(B * (N + 2) * (M + 2)) * es : 0};
    a.xRt = Extent{Rt, Rt ? static_cast<size_t>(B * S * a.NBt) * 1024 * es : 0};
    a.xC = Extent{costs, static_cast<size_t>(B) * es};
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
    const dim3 grid(static_cast<unsigned>(B)), block(static_cast<unsigned>(W * 32));
    const size_t smem = pair_fwd_smem_bytes<T>(W, M);
    if (Rt != nullptr) {  // R stays in the library: units of gamma ln 2
        if (M == kPairSpecialM)
            sdtw_fwd_pair_kernel<T, kPairSpecialM, false, true><<<grid, block, smem, stream>>>(a);
        else
            sdtw_fwd_pair_kernel<T, 0, false, true><<<grid, block, smem, stream>>>(a);
    } else {
        if (M == kPairSpecialM)
            sdtw_fwd_pair_kernel<T, kPairSpecialM, false, false><<<grid, block, smem, stream>>>(a);
        else
            sdtw_fwd_pair_kernel<T, 0, false, false><<<grid, block, smem, stream>>>(a);
    }
    return cudaGetLastError();
}
cudaError_t pair_forward_fused(const float* X, const float* Y, int64_t d, float* Rt, float* costs, uint32_t* cmask,
                               int* cflags, const void* lx, const void* ly, int is32, int64_t B, int64_t N, int64_t M,
                               int64_t bw, double gamma, int W, Sync sy, int64_t inject, cudaStream_t stream)
{
    PairFwdArgs<float> a;
    a.D = nullptr;
    a.R = nullptr;
    a.Rt = Rt;
    a.NBt = pair_tile_blocks(M);
    const int64_t S = N > 0 ? (N + 31) / 32 : 1;
    a.xD = Extent{nullptr, 0};
    a.xR = Extent{nullptr, 0};
    a.xRt = Extent{Rt, static_cast<size_t>(B * S * a.NBt) * 1024 * sizeof(float)};
    a.xC = Extent{costs, static_cast<size_t>(B) * sizeof(float)};
    a.costs = costs;
    a.len = Lengths{lx, ly, is32};
    a.B = B;
    a.N = N;
    a.M = M;
    a.bw = bw;
    a.S = static_cast<int>(S);
    a.W = W;
    a.BL = buf_len(M);
    a.G = fwd_groups(M);
    a.k = static_cast<float>(1.4426950408889634 / gamma);
    a.gl = static_cast<float>(gamma * 0.6931471805599453);
    a.sy = sy;
    a.inject = inject;
    a.f.X = X;
    a.f.Y = Y;
    a.f.d = static_cast<int>(d);
    a.f.cmask = cmask;
    a.f.cflags = cflags;
    a.f.MW = static_cast<int>((M + 31) / 32);
    a.f.xX = Extent{X, static_cast<size_t>(B * N * d) * sizeof(float)};
    a.f.xY = Extent{Y, static_cast<size_t>(B * M * d) * sizeof(float)};
    a.f.xMask = Extent{cmask, static_cast<size_t>(B * N * a.f.MW) * sizeof(uint32_t)};
    a.f.xFlags = Extent{cflags, static_cast<size_t>(B) * sizeof(int)};
    count_launch();
    if (M == kPairSpecialM)
        sdtw_fwd_pair_kernel<float, kPairSpecialM, true, true><<<static_cast<unsigned>(B), W * 32, fused_smem_bytes(W, M), stream>>>(a);
    else
        sdtw_fwd_pair_kernel<float, 0, true, true><<<static_cast<unsigned>(B), W * 32, fused_smem_bytes(W, M), stream>>>(a);
    return cudaGetLastError();
}

template cudaError_t pair_forward<float>(const float*, float*, float*, float*, const void*, const void*, int, int64_t,
                                         int64_t, int64_t, int64_t, double, int, Sync, int64_t, cudaStream_t);
template cudaError_t pair_forward<double>(const double*, double*, double*, double*, const void*, const void*, int,
                                          int64_t, int64_t, int64_t, int64_t, double, int, Sync, int64_t,
                                          cudaStream_t);

template <typename T>
cudaError_t pair_backward(const T* R, const T* Rt, T* E, const void* lx, const void* ly, int is32, int64_t B,
                          int64_t N, int64_t M, int64_t bw, double gamma, int W, Sync sy, int64_t inject,
                          cudaStream_t stream)
{
    PairBwdArgs<T> a;
    a.R = R;
    a.Rt = Rt;
    a.NBt = pair_tile_blocks(M);
    const size_t es = sizeof(T);
    const int64_t S = N > 0 ? (N + 31) / 32 : 1;
    a.xR = Extent{R, R ? static_cast<size_t>(B * (N + 2) * (M + 2)) * es : 0};
    a.xRt = Extent{Rt, Rt ? static_cast<size_t>(B * S * a.NBt) * 1024 * es : 0};
    a.xE = Extent{E, static_cast<size_t>(B * N * M) * es};
    a.E = E;
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
    a.sy = sy;
    a.inject = inject;
    count_launch();
    const dim3 grid(static_cast<unsigned>(B)), block(static_cast<unsigned>(W * 32));
    const size_t smem = pair_bwd_smem_bytes<T>(W, M);
    if (Rt != nullptr) {  // the forward's tiles, in units of gamma ln 2
        if (M == kPairSpecialM)
            sdtw_bwd_pair_kernel<T, kPairSpecialM, true><<<grid, block, smem, stream>>>(a);
        else
            sdtw_bwd_pair_kernel<T, 0, true><<<grid, block, smem, stream>>>(a);
    } else {
        if (M == kPairSpecialM)
            sdtw_bwd_pair_kernel<T, kPairSpecialM, false><<<grid, block, smem, stream>>>(a);
        else
            sdtw_bwd_pair_kernel<T, 0, false><<<grid, block, smem, stream>>>(a);
    }
    return cudaGetLastError();
}
template cudaError_t pair_backward<float>(const float*, const float*, float*, const void*, const void*, int, int64_t,
                                          int64_t, int64_t, int64_t, double, int, Sync, int64_t, cudaStream_t);
template cudaError_t pair_backward<double>(const double*, const double*, double*, const void*, const void*, int,
                                           int64_t, int64_t, int64_t, int64_t, double, int, Sync, int64_t,
                                           cudaStream_t);

}  // namespace sdtw
