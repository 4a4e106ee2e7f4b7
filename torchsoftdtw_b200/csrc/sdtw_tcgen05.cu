// Tensor-core (tcgen05, sm_100a) kernels of the squared-L2 module path, both fp32 with 3xTF32 products:
// the cost matrix D = |x|^2 + |y|^2 - 2 X Y^T (clamped at 0, the clamp recorded as -0.0) and the gradient
// grad_X = 2 g (rowsum(G) X - G Y). Both are persistent and warp-specialized: a TMA warp streams operand
// chunks into this CTA's own shared memory, split warps turn each fp32 operand into a TF32 head and tail
// (x = head + tail to about 2^-22) so that head.head + head.tail + tail.head keeps fp32 accuracy, one thread
// issues tcgen05.mma into fp32 accumulators in tensor memory, and epilogue warps read the accumulators back
// with tcgen05.ld while the next tile's products run. Every mbarrier wait is bounded in time.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "sdtw_b200.h"
#include "sdtw_common.cuh"
#include "sdtw_strip.cuh"
#include "sdtw_tcgen05.h"

namespace sdtw {

namespace {

constexpr int kT = 128;                // tile rows (X) = tile columns (Y) = UMMA M = N
constexpr int kKC = 32;                // features per K step: one 128-byte swizzle atom of fp32
constexpr int kChunk = kT * kKC * 4;   // 16 KB: one operand's K step
// UMMA instruction descriptor: D fp32, A and B TF32, both K-major, M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t(kT) >> 3) << 17) |
                            ((uint32_t(kT) >> 4) << 24);

__device__ uint32_t g_distance_err;  // bit 1: a wait of the tensor-core cost kernel ran out

// Shared-memory matrix descriptor of a K-major operand in the 128-byte swizzled layout written by TMA:
// rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), leading byte offset unused (1).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version of sm_100
    d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.b32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity; false if it did not complete within timeout_ns.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t timeout_ns)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > timeout_ns) return false;
    }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2)
{
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate)
{
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p; }" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32])
{
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Nearest TF32 value (round to nearest, ties away; low 13 mantissa bits zero).
__device__ __forceinline__ float to_tf32(float x)
{
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Split the 32 features of one swizzled 128-byte row (row index `row`) in place into head | tail, both
// exact TF32 values (head = tf32(x), tail = tf32(x - head)), and return the row's sum of squares. The
// split is elementwise, so each thread visits its row's 16-byte units in the row's swizzle order
// (u ^ row % 8): the 32 rows of a warp then touch 8 different unit positions at every step, which spreads
// the accesses over all banks.
__device__ __forceinline__ float split_row(unsigned char* head, unsigned char* tail, int row)
{
    float s = 0.f;
#pragma unroll
    for (int u0 = 0; u0 < 8; ++u0) {
        const int u = u0 ^ (row & 7);
        float4 v = *reinterpret_cast<float4*>(head + 16 * u);
        s = fmaf(v.x, v.x, s);
        s = fmaf(v.y, v.y, s);
        s = fmaf(v.z, v.z, s);
        s = fmaf(v.w, v.w, s);
        float4 h, t;
        h.x = to_tf32(v.x);
        h.y = to_tf32(v.y);
        h.z = to_tf32(v.z);
        h.w = to_tf32(v.w);
        t.x = to_tf32(v.x - h.x);
        t.y = to_tf32(v.y - h.y);
        t.z = to_tf32(v.z - h.z);
        t.w = to_tf32(v.w - h.w);
        *reinterpret_cast<float4*>(head + 16 * u) = h;
        *reinterpret_cast<float4*>(tail + 16 * u) = t;
    }
    return s;
}

// ==================================================================================================
// grad_X = 2 g[b] (rowsum(G) X - G Y), G = E masked by the clamp of the cost matrix, on tcgen05.
//
// A tile is 128 rows of grad_X (UMMA M) x all features; its K loop runs over the columns j of E in chunks
// of 32. The B operand is [Y | 1]: DPAD features (d <= 128 padded to 16/32/64/96/128) and 16 more rows,
// the first all ones, so the accumulator's column DPAD is rowsum(G). The kernel is persistent (tiles
// blockIdx.x, blockIdx.x + gridDim.x, ...; chunks numbered q = 0, 1, ... across them) and its warps
// specialise, communicating only through mbarriers:
//   * warp 0 (TMA): E[128 rows x 32 columns] (128-byte swizzled) and Y[32 rows x DPAD] (plain boxes) of
//     chunk q into raw stage q % S;
//   * warps 2..17 (split, 512 threads): zero the clamped cells of E in flagged pairs (sign bit of D), split
//     E into TF32 head | tail (3xTF32) in place of the 128-byte swizzled rows of split buffer q % P, and
//     transpose + split Y into its K-major rows; release the raw stage and mark the split buffer full;
//   * warp 1 (MMA): 3 x 4 tcgen05.mma kind::tf32 per chunk into accumulator (tile & 1) in tensor memory,
//     commit to the split buffer's "empty" barrier, and after a tile's last chunk to the accumulator's
//     "full" barrier;
//   * the last 8 warps (epilogue, two groups of four, one per feature half): read their 32 accumulator
//     lanes (rows) with tcgen05.ld and write grad_X rows; the accumulator is double-buffered, so this
//     overlaps the next tile's MMAs.
// Every wait is bounded in time. A wait that runs out raises an abort word in shared memory that every
// role polls, sets bit 1 of the library's distance error word, and the epilogue writes NaN into the rows
// it has not finished; the TMA and MMA warps wait (bounded) for their own operations before the CTA
// releases its tensor memory.
//
// TRANS: the same kernel computes grad_Y = 2 g[b] (colsum(G) Y - G^T X), the contraction of E over its
// rows. The roles swap (output rows are the columns of E; B operand [X | 1]; the epilogue reads Y), and E
// is read transposed: the TMA warp loads E[32 rows x 128 columns] (unswizzled) and the split threads
// gather each output row's 32 K values from that box's column, so the A operand is Gᵀ in the same
// 128-byte swizzled K-major layout. GradTcArgs then describes the transposed problem: N = output rows
// (the columns of E), M = the K extent (the rows of E); E and D are (B, M, N) in memory.
// ==================================================================================================
constexpr int kGT = 128;                    // grad_X rows per tile (UMMA M)
constexpr int kGKC = 32;                    // columns of E per chunk (one 128-byte swizzle atom of fp32)
constexpr int kEChunk = kGT * kGKC * 4;     // 16 KB
constexpr int kGradSplitWarps = 16;
constexpr int kGradSplitThreads = 32 * kGradSplitWarps;
constexpr int kGradEpiWarps = 8;  // two groups of four (one per column half), each covering the 128 lanes
constexpr int kGradThreads = 32 * (2 + kGradSplitWarps + kGradEpiWarps);  // TMA, MMA, split, epilogue
constexpr int kGradEpiWarp0 = 2 + kGradSplitWarps;
constexpr int kGradSmemBudget = 218 * 1024;

template <int DPAD>
struct GradGeom {
    static constexpr int NB = DPAD + 16;                                    // UMMA N: features + ones block
    static constexpr int YB = DPAD < 32 ? DPAD : 32;                        // features per Y box
    static constexpr int NBOX = DPAD / YB;
    static constexpr int YRAW = DPAD * 128;                                 // raw Y: 32 K rows x DPAD fp32
    static constexpr int YT = NB * 128;                                     // Y^T (one of head / tail)
    static constexpr int RAW = kEChunk + YRAW;                              // one raw stage
    static constexpr int SPL = 2 * kEChunk + 2 * YT;                        // E head, E tail, Y^T head, Y^T tail
    static constexpr int P = 2;                                             // split buffers
    static constexpr int S0 = (kGradSmemBudget - P * SPL) / RAW;
    static constexpr int S = S0 > 4 ? 4 : S0;                               // raw stages
    static constexpr int OFF_SPL = S * RAW;
    static constexpr int OFF_BAR = OFF_SPL + P * SPL;
    // barriers: raw_full[S], raw_empty[S], spl_full[P], spl_empty[P], acc_full[2], acc_empty[2]
    static constexpr int NBAR = 2 * S + 2 * P + 4;
    static constexpr int OFF_TMEM = OFF_BAR + 8 * NBAR;
    static constexpr int OFF_ABORT = OFF_TMEM + 8;
    static constexpr int BYTES = OFF_ABORT + 8 + 1024;                      // + slack to align the base
    static constexpr uint32_t ACC_COLS = NB <= 32 ? 32u : (NB <= 64 ? 64u : (NB <= 128 ? 128u : 256u));
    static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
    // Y split: TPN threads per feature, KPER consecutive K rows each (whole 16-byte units).
    static constexpr int TPN = DPAD * 8 <= kGradSplitThreads ? 8 : (DPAD * 4 <= kGradSplitThreads ? 4 : 2);
    static constexpr int KPER = kGKC / TPN;
    static constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t(NB) >> 3) << 17) |
                                      ((uint32_t(kGT) >> 4) << 24);
    static_assert(S >= 2, "grad_X tensor-core kernel: fewer than two raw stages fit");
    static_assert(DPAD % 16 == 0 && NB <= 256, "UMMA N");
    static_assert(BYTES <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void umma_tf32_id(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                             uint32_t accumulate)
{
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p; }" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// 16 consecutive fp32 accumulator columns of this thread's lane (no wait).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, float* v)
{
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float4 split_hi(float4 v)
{
    return make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
}
__device__ __forceinline__ float4 split_lo(float4 v, float4 h)
{
    return make_float4(to_tf32(v.x - h.x), to_tf32(v.y - h.y), to_tf32(v.z - h.z), to_tf32(v.w - h.w));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Bounded wait that also gives up when another role of the CTA raised the abort word. On its own
// timeout it raises the abort word and the library's distance error bit.
__device__ __forceinline__ bool wait_role(uint32_t bar, uint32_t parity, uint64_t timeout_ns, volatile int* abort)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    unsigned ns = 32;
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 4; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        __nanosleep(ns);  // back off: waiting warps leave the issue slots to the working ones
        ns = ns < 512 ? 2 * ns : 512;
        if (*abort) return false;
        if (global_ns() - t0 > timeout_ns) {
            *abort = 1;
            atomicOr(&g_distance_err, 1u);
            return false;
        }
    }
}

// ---- the cells a pair's dynamic program reads --------------------------------------------------------
// Columns [c0, c1] that hold the in-band cells of rows i0 .. i1 of pair b lying below its lengths (rows
// i < nx, columns j < ny), for E (or D) of nrows x ncols. With trans the rows are E's columns (the band is
// symmetric in its two axes: band_row_range(j, ny, nx, bw) is the row interval of column j). Band intervals
// are non-decreasing in the row, so the first and last rows bound them. False when no such cell exists: rows
// past the length, an empty side, or lengths outside [0, nrows] x [0, ncols] (an empty pair for the
// wavefront kernels).
__device__ __forceinline__ bool dp_cols_of_rows(const Lengths& len, int64_t b, int64_t nrows, int64_t ncols,
                                                int64_t bw, int64_t i0, int64_t i1, bool trans, int64_t& c0,
                                                int64_t& c1)
{
    const int64_t nx = len.x(b), ny = len.y(b);
    if (nx <= 0 || nx > nrows || ny <= 0 || ny > ncols) return false;
    const int64_t nr = trans ? ny : nx, nc = trans ? nx : ny;
    if (i0 >= nr) return false;
    if (i1 > nr - 1) i1 = nr - 1;
    int64_t lo, hi, lo1, hi1;
    band_row_range(i0, nr, nc, bw, lo, hi);
    band_row_range(i1, nr, nc, bw, lo1, hi1);
    c0 = lo;
    c1 = hi1;
    return c0 <= c1;
}

// The tiles of D (B pairs of nit x njt tiles of 128 x 128) that hold a cell of the region, as tile ids
// (b * nit + row tile) * njt + column tile in increasing order, and their count. One CTA of 1024 threads,
// one (pair, row tile) per thread per round, an exclusive scan of the per-row counts placing the ids.
__global__ void __launch_bounds__(1024) band_tile_list_kernel(Lengths len, int B, int N, int M, int64_t bw,
                                                              int nit, int njt, int* count, int* list)
{
    __shared__ int wsum[32];
    __shared__ int base;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) base = 0;
    __syncthreads();
    const int rows = B * nit;
    for (int e0 = 0; e0 < rows; e0 += 1024) {
        const int e = e0 + tid;
        int ct0 = 0, n = 0;
        if (e < rows) {
            const int b = e / nit, rt = e % nit;
            int64_t c0, c1;
            if (dp_cols_of_rows(len, b, N, M, bw, static_cast<int64_t>(rt) * kT, static_cast<int64_t>(rt) * kT + kT - 1,
                                false, c0, c1)) {
                ct0 = static_cast<int>(c0 / kT);
                n = static_cast<int>(c1 / kT) - ct0 + 1;
            }
        }
        int v = n;  // inclusive scan within the warp
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(kFull, v, o);
            if (lane >= o) v += t;
        }
        if (lane == 31) wsum[warp] = v;
        __syncthreads();
        if (warp == 0) {
            int w = wsum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(kFull, w, o);
                if (lane >= o) w += t;
            }
            wsum[lane] = w;
        }
        __syncthreads();
        const int at = base + (warp > 0 ? wsum[warp - 1] : 0) + v - n;
        for (int k = 0; k < n; ++k) list[at + k] = e * njt + ct0 + k;
        __syncthreads();
        if (tid == 0) base += wsum[31];
        __syncthreads();
    }
    if (tid == 0) *count = base;
}

struct GradTcArgs {
    const float* X;
    const float* D;
    const float* g;
    const int* clamp_flags;  // may be null: every pair is masked
    const float* ry;         // cosine: 1 / max(|y_j|, eps) per row of Y (B x M); null: squared L2
    float eps;               // cosine: the floor of the norms
    float* out;
    int B, N, M, d;
    int nrt;                 // row tiles per pair
    int nk;                  // chunks per tile
    unsigned long long timeout_ns;
    Lengths len;             // BANDED kernels: E is zero outside the region of len and bw
    int64_t bw;
};

// The K chunks (32 columns of E; rows of E with TRANS) a row tile contracts: with BANDED, those that hold a
// cell of the region (one chunk of zeros where the tile holds none, so that its accumulator is written), else
// all. BANDED is a template parameter so that the kernel without a region keeps its registers (the split
// warps run at the 72-register cap of 832 threads).
template <bool TRANS, bool BANDED>
__device__ __forceinline__ void grad_chunk_range(const GradTcArgs& a, int b, int rt, int& kc0, int& nkc)
{
    kc0 = 0;
    nkc = a.nk;
    if constexpr (!BANDED) return;
    const int64_t ne = TRANS ? a.M : a.N, me = TRANS ? a.N : a.M;  // E is (B, ne, me)
    int64_t c0, c1;
    if (!dp_cols_of_rows(a.len, b, ne, me, a.bw, static_cast<int64_t>(rt) * kGT,
                         static_cast<int64_t>(rt) * kGT + kGT - 1, TRANS, c0, c1)) {
        nkc = 1;
        return;
    }
    kc0 = static_cast<int>(c0 / kGKC);
    nkc = static_cast<int>(c1 / kGKC) - kc0 + 1;
}

template <int DPAD, bool TRANS, bool BANDED>
__global__ void __launch_bounds__(kGradThreads, 1) grad_x_tc_kernel(const __grid_constant__ CUtensorMap me,
                                                                    const __grid_constant__ CUtensorMap my,
                                                                    GradTcArgs a)
{
    using G = GradGeom<DPAD>;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw0 = smem_addr(smem_raw);
    unsigned char* sm = smem_raw + ((1024u - (raw0 & 1023u)) & 1023u);
    const uint32_t base = smem_addr(sm);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t raw_full = base + G::OFF_BAR;
    const uint32_t raw_empty = raw_full + 8 * G::S;
    const uint32_t spl_full = raw_empty + 8 * G::S;
    const uint32_t spl_empty = spl_full + 8 * G::P;
    const uint32_t acc_full = spl_empty + 8 * G::P;
    const uint32_t acc_empty = acc_full + 16;
    volatile int* abort = reinterpret_cast<volatile int*>(sm + G::OFF_ABORT);

    const int ntiles = a.B * a.nrt;
    const int my_tiles = blockIdx.x < static_cast<unsigned>(ntiles)
                             ? (ntiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                             : 0;
    if (tid == 0) {
        for (int s = 0; s < G::S; ++s) {
            mbar_init(raw_full + 8 * s, 1);
            mbar_init(raw_empty + 8 * s, kGradSplitWarps);
        }
        for (int p = 0; p < G::P; ++p) {
            mbar_init(spl_full + 8 * p, kGradSplitWarps);
            mbar_init(spl_empty + 8 * p, 1);
        }
        for (int c = 0; c < 2; ++c) {
            mbar_init(acc_full + 8 * c, 1);
            mbar_init(acc_empty + 8 * c, kGradEpiWarps);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // The ones block of [Y | 1]^T in every split buffer: row DPAD of the head all ones, rows DPAD+1..NB-1
    // of the head and all 16 rows of the tail zero (written once; the split only writes rows < DPAD).
    for (int e = tid; e < G::P * 16 * 32; e += kGradThreads) {
        const int p = e / (16 * 32), r = (e / 32) % 16, k = e % 32;
        float* yh = reinterpret_cast<float*>(sm + G::OFF_SPL + p * G::SPL + 2 * kEChunk + 128 * (DPAD + r));
        yh[k] = r == 0 ? 1.f : 0.f;
        yh[G::YT / 4 + k] = 0.f;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(base + G::OFF_TMEM),
                     "r"(G::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + G::OFF_TMEM);

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int issued = 0, q = 0;
            bool ok = true;
            for (int tl = 0; tl < my_tiles && ok; ++tl) {
                const int t = static_cast<int>(blockIdx.x) + tl * static_cast<int>(gridDim.x);
                const int b = t / a.nrt, rt = t % a.nrt;
                int kc0, nkc;
                grad_chunk_range<TRANS, BANDED>(a, b, rt, kc0, nkc);
                for (int kc = kc0; kc < kc0 + nkc; ++kc, ++q) {
                    const int s = q % G::S;
                    if (q >= G::S && !wait_role(raw_empty + 8 * s, ((q / G::S) - 1) & 1, a.timeout_ns, abort)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = base + s * G::RAW;
                    mbar_expect_tx(raw_full + 8 * s, G::RAW);
                    if constexpr (TRANS)  // E rows kc*32.., columns rt*128..
                        tma_load_3d(dst, &me, raw_full + 8 * s, rt * kGT, kc * kGKC, b);
                    else
                        tma_load_3d(dst, &me, raw_full + 8 * s, kc * kGKC, rt * kGT, b);
#pragma unroll
                    for (int bx = 0; bx < G::NBOX; ++bx)
                        tma_load_3d(dst + kEChunk + bx * (kGKC * G::YB * 4), &my, raw_full + 8 * s, bx * G::YB,
                                    kc * kGKC, b);
                    issued = q + 1;
                }
            }
            // Before the CTA ends: every load issued into each stage has landed (the last one per stage
            // completes after all earlier ones, which the split released).
            for (int q = issued - G::S < 0 ? 0 : issued - G::S; q < issued; ++q)
                (void)mbar_wait(raw_full + 8 * (q % G::S), (q / G::S) & 1, a.timeout_ns);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int q = 0;
            int last_commit_bar = -1;
            uint32_t last_commit_parity = 0;
            bool ok = true;
            for (int tl = 0; tl < my_tiles && ok; ++tl) {
                const int ab = tl & 1;
                if (tl >= 2 && !wait_role(acc_empty + 8 * ab, ((tl >> 1) - 1) & 1, a.timeout_ns, abort)) break;
                const uint32_t acc = tmem + static_cast<uint32_t>(ab) * G::ACC_COLS;
                int kc0, nkc;
                {
                    const int t = static_cast<int>(blockIdx.x) + tl * static_cast<int>(gridDim.x);
                    grad_chunk_range<TRANS, BANDED>(a, t / a.nrt, t % a.nrt, kc0, nkc);
                }
                for (int kc = 0; kc < nkc; ++kc, ++q) {
                    const int p = q % G::P;
                    if (!wait_role(spl_full + 8 * p, (q / G::P) & 1, a.timeout_ns, abort)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t sb = base + G::OFF_SPL + p * G::SPL;
                    const uint64_t ah = sw128_desc(sb), al = sw128_desc(sb + kEChunk);
                    const uint64_t bh = sw128_desc(sb + 2 * kEChunk), bl = sw128_desc(sb + 2 * kEChunk + G::YT);
#pragma unroll
                    for (int kk = 0; kk < kGKC / 8; ++kk) {
                        const uint64_t st = static_cast<uint64_t>((kk * 32) >> 4);  // 8 TF32 = 32 bytes along K
                        umma_tf32_id(acc, ah + st, bh + st, G::IDESC, (kc > 0 || kk > 0) ? 1u : 0u);
                        umma_tf32_id(acc, ah + st, bl + st, G::IDESC, 1u);
                        umma_tf32_id(acc, al + st, bh + st, G::IDESC, 1u);
                    }
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     spl_empty + 8 * p)
                                 : "memory");
                    last_commit_bar = 0;
                    last_commit_parity = static_cast<uint32_t>((q / G::P) & 1);
                    if (kc == nkc - 1) {
                        asm volatile(
                            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                acc_full + 8 * ab)
                            : "memory");
                    }
                }
                if (ok && q > 0) last_commit_bar = 1 + (q - 1) % G::P;
            }
            // Before the CTA ends: the last MMAs have completed (their commit arrived).
            if (q > 0) {
                const int ql = q - 1;
                (void)mbar_wait(spl_empty + 8 * (ql % G::P), (ql / G::P) & 1, a.timeout_ns);
            }
            (void)last_commit_bar;
            (void)last_commit_parity;
        }
    } else if (warp < kGradEpiWarp0) {
        // ---------------- split ----------------
        constexpr int EU = 8 * kGT / kGradSplitThreads;  // E units (16 bytes) per split thread
        const int st = tid - 64;                          // 0 .. kGradSplitThreads - 1
        const int er = st & (kGT - 1), eu0 = (st >> 7) * EU;  // E: row er, logical units eu0 .. eu0+EU-1
        const bool y_active = st < DPAD * G::TPN;
        const int yn = st % DPAD, yh = st / DPAD;         // Y: feature yn, K units [yh*KPER/4, ...)
        int q = 0;
        for (int tl = 0; tl < my_tiles; ++tl) {
            const int t = static_cast<int>(blockIdx.x) + tl * static_cast<int>(gridDim.x);
            const int b = t / a.nrt, rt = t % a.nrt;
            const int i_e = rt * kGT + er;
            const bool masked = !a.ry && (a.clamp_flags == nullptr || a.clamp_flags[b] != 0) && i_e < a.N;
            const float* Drow = a.D + (static_cast<int64_t>(b) * a.N + (i_e < a.N ? i_e : 0)) * a.M;
            int kc0, nkc;
            grad_chunk_range<TRANS, BANDED>(a, b, rt, kc0, nkc);
            bool ok = true;
            for (int kc = kc0; kc < kc0 + nkc; ++kc, ++q) {
                const int s = q % G::S, p = q % G::P;
                if (!wait_role(raw_full + 8 * s, (q / G::S) & 1, a.timeout_ns, abort) ||
                    (q >= G::P && !wait_role(spl_empty + 8 * p, ((q / G::P) - 1) & 1, a.timeout_ns, abort))) {
                    ok = false;
                    break;
                }
                const unsigned char* raw = sm + s * G::RAW;
                unsigned char* spl = sm + G::OFF_SPL + p * G::SPL;
                const int j0 = kc * kGKC;
#pragma unroll
                for (int w = 0; w < EU; ++w) {
                    const int lu = eu0 + w;
                    const int off = 128 * er + 16 * (lu ^ (er & 7));
                    if constexpr (TRANS) {
                        // Output row er's K values 4 lu .. 4 lu + 3: column er of E's rows j0 + 4 lu + t (the
                        // raw box is [32 rows][128 columns]; a warp reads 32 consecutive columns per row).
                        const float* rc = reinterpret_cast<const float*>(raw) + er;
                        float4 v = make_float4(rc[128 * (4 * lu)], rc[128 * (4 * lu + 1)], rc[128 * (4 * lu + 2)],
                                               rc[128 * (4 * lu + 3)]);
                        if (masked) {
                            // D is (B, M, N) here: D[b][j][i_e]; rows j past the K extent read zero E anyway.
                            const float* Dc = a.D + static_cast<int64_t>(b) * a.M * a.N + i_e;
                            const int j = j0 + 4 * lu;
                            if (j < a.M && signbit(__ldg(Dc + static_cast<int64_t>(j) * a.N))) v.x = 0.f;
                            if (j + 1 < a.M && signbit(__ldg(Dc + static_cast<int64_t>(j + 1) * a.N))) v.y = 0.f;
                            if (j + 2 < a.M && signbit(__ldg(Dc + static_cast<int64_t>(j + 2) * a.N))) v.z = 0.f;
                            if (j + 3 < a.M && signbit(__ldg(Dc + static_cast<int64_t>(j + 3) * a.N))) v.w = 0.f;
                        }
                        const float4 h = split_hi(v);
                        *reinterpret_cast<float4*>(spl + off) = h;
                        *reinterpret_cast<float4*>(spl + kEChunk + off) = split_lo(v, h);
                        continue;
                    }
                    float4 v = *reinterpret_cast<const float4*>(raw + off);
                    if (masked) {
                        const int j = j0 + 4 * lu;  // M % 4 == 0: the four columns are all in or all out
                        if (j < a.M) {
                            const float4 dv = __ldg(reinterpret_cast<const float4*>(Drow + j));
                            if (signbit(dv.x)) v.x = 0.f;
                            if (signbit(dv.y)) v.y = 0.f;
                            if (signbit(dv.z)) v.z = 0.f;
                            if (signbit(dv.w)) v.w = 0.f;
                        }
                    }
                    const float4 h = split_hi(v);
                    *reinterpret_cast<float4*>(spl + off) = h;
                    *reinterpret_cast<float4*>(spl + kEChunk + off) = split_lo(v, h);
                }
                if (y_active) {
                    const float* yr =
                        reinterpret_cast<const float*>(raw + kEChunk + (yn / G::YB) * (kGKC * G::YB * 4)) + (yn % G::YB);
                    unsigned char* yhb = spl + 2 * kEChunk + 128 * yn;
#pragma unroll
                    for (int u = 0; u < G::KPER / 4; ++u) {
                        const int lu = yh * (G::KPER / 4) + u;
                        float4 v;
                        v.x = yr[(4 * lu + 0) * G::YB];
                        v.y = yr[(4 * lu + 1) * G::YB];
                        v.z = yr[(4 * lu + 2) * G::YB];
                        v.w = yr[(4 * lu + 3) * G::YB];
                        if (a.ry) {  // cosine: rows of Y / n(Y); M % 4 == 0, the four rows all in or all out
                            const int j = j0 + 4 * lu;
                            if (j < a.M) {
                                const float4 r4 =
                                    __ldg(reinterpret_cast<const float4*>(a.ry + static_cast<int64_t>(b) * a.M + j));
                                v.x *= r4.x;
                                v.y *= r4.y;
                                v.z *= r4.z;
                                v.w *= r4.w;
                            }
                        }
                        const float4 h = split_hi(v);
                        const int off = 16 * (lu ^ (yn & 7));
                        *reinterpret_cast<float4*>(yhb + off) = h;
                        *reinterpret_cast<float4*>(yhb + G::YT + off) = split_lo(v, h);
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(raw_empty + 8 * s);
                    mbar_arrive(spl_full + 8 * p);
                }
            }
            if (!ok) break;
        }
    } else {
        // ---------------- epilogue ----------------
        // Group eg (0, 1) writes features [eg * NC, eg * NC + NC) of its rows. The row of X it needs is
        // loaded before the accumulator wait, so its latency overlaps the tile's products.
        constexpr int NC = DPAD / 2;
        constexpr bool kHoist = NC <= 32;  // X half row held in registers (NC / 4 float4)
        const int row = 32 * (warp & 3) + lane;  // accumulator lane of this thread
        const int eg = (warp - kGradEpiWarp0) >> 2;
        const int c0 = eg * NC;
        int tl = 0;
        for (; tl < my_tiles; ++tl) {
            const int ab = tl & 1;
            const int t = static_cast<int>(blockIdx.x) + tl * static_cast<int>(gridDim.x);
            const int b = t / a.nrt, i = (t % a.nrt) * kGT + row;
            const float* xr = a.X + (static_cast<int64_t>(b) * a.N + (i < a.N ? i : 0)) * a.d;
            float4 xv[kHoist ? NC / 4 : 1];
            if constexpr (kHoist) {
#pragma unroll
                for (int e = 0; e < NC / 4; ++e)
                    xv[e] = (i < a.N && c0 + 4 * e < a.d) ? __ldg(reinterpret_cast<const float4*>(xr + c0 + 4 * e))
                                                         : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (!wait_role(acc_full + 8 * ab, (tl >> 1) & 1, a.timeout_ns, abort)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t acc = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) +
                                 static_cast<uint32_t>(ab) * G::ACC_COLS;
            float* orow = a.out + (static_cast<int64_t>(b) * a.N + i) * a.d;
            if (a.ry) {
                // Cosine: P = G (Y / n(Y)) in the accumulator. Pass 1 over the whole row: |x_i|^2 and x_i.P;
                // pass 2 over this group's features: -g / n(x_i) (P - c(x_i) (x_i.P) x_i / n(x_i)^2).
                float ss = 0.f, dot = 0.f;
#pragma unroll
                for (int cc = 0; cc < DPAD; cc += 8) {
                    uint32_t r[8];
                    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                                   "=r"(r[6]), "=r"(r[7])
                                 : "r"(acc + static_cast<uint32_t>(cc)));
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int e = 0; e < 8; e += 4) {
                        if (i < a.N && cc + e < a.d) {
                            const float4 x4 = __ldg(reinterpret_cast<const float4*>(xr + cc + e));
                            ss = fmaf(x4.x, x4.x, ss);
                            ss = fmaf(x4.y, x4.y, ss);
                            ss = fmaf(x4.z, x4.z, ss);
                            ss = fmaf(x4.w, x4.w, ss);
                            dot = fmaf(x4.x, __uint_as_float(r[e]), dot);
                            dot = fmaf(x4.y, __uint_as_float(r[e + 1]), dot);
                            dot = fmaf(x4.z, __uint_as_float(r[e + 2]), dot);
                            dot = fmaf(x4.w, __uint_as_float(r[e + 3]), dot);
                        }
                    }
                }
                const float nrm = sqrtf(ss);
                const float inv = 1.f / fmaxf(nrm, a.eps);
                const float coef = nrm >= a.eps ? dot * inv * inv : 0.f;
                const float ginv = a.g[b] * inv;
#pragma unroll
                for (int cc = 0; cc < NC; cc += 8) {
                    uint32_t r[8];
                    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                                   "=r"(r[6]), "=r"(r[7])
                                 : "r"(acc + static_cast<uint32_t>(c0 + cc)));
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    if (i < a.N) {
#pragma unroll
                        for (int e = 0; e < 8; e += 4) {
                            const int n = c0 + cc + e;
                            if (n < a.d) {
                                const float4 x4 = __ldg(reinterpret_cast<const float4*>(xr + n));
                                float4 o;
                                o.x = -ginv * (__uint_as_float(r[e]) - coef * x4.x);
                                o.y = -ginv * (__uint_as_float(r[e + 1]) - coef * x4.y);
                                o.z = -ginv * (__uint_as_float(r[e + 2]) - coef * x4.z);
                                o.w = -ginv * (__uint_as_float(r[e + 3]) - coef * x4.w);
                                *reinterpret_cast<float4*>(orow + n) = o;
                            }
                        }
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(acc_empty + 8 * ab);
                continue;
            }
            float v[16];
            tmem_ld16_nowait(acc + DPAD, v);  // column DPAD: rowsum(G)
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            const float rsum = v[0];
            const float g2 = 2.f * a.g[b];
#pragma unroll
            for (int cc = 0; cc < NC; cc += 8) {
                uint32_t r[8];
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                             : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                               "=r"(r[7])
                             : "r"(acc + static_cast<uint32_t>(c0 + cc)));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (i < a.N) {
#pragma unroll
                    for (int e = 0; e < 8; e += 4) {
                        const int n = c0 + cc + e;
                        if (n < a.d) {
                            float4 x4;
                            if constexpr (kHoist)
                                x4 = xv[(cc + e) / 4];
                            else
                                x4 = __ldg(reinterpret_cast<const float4*>(xr + n));
                            float4 o;
                            o.x = g2 * (rsum * x4.x - __uint_as_float(r[e]));
                            o.y = g2 * (rsum * x4.y - __uint_as_float(r[e + 1]));
                            o.z = g2 * (rsum * x4.z - __uint_as_float(r[e + 2]));
                            o.w = g2 * (rsum * x4.w - __uint_as_float(r[e + 3]));
                            *reinterpret_cast<float4*>(orow + n) = o;
                        }
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + 8 * ab);
        }
        // Rows of tiles not finished (a wait ran out): NaN.
        for (; tl < my_tiles; ++tl) {
            const int t = static_cast<int>(blockIdx.x) + tl * static_cast<int>(gridDim.x);
            const int b = t / a.nrt, i = (t % a.nrt) * kGT + row;
            if (i < a.N)
                for (int n = c0; n < c0 + NC && n < a.d; ++n)
                    a.out[(static_cast<int64_t>(b) * a.N + i) * a.d + n] = __int_as_float(0x7fc00000);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G::TMEM_COLS)
                     : "memory");
}

// ==================================================================================================
// Cost matrix, persistent and warp-specialized: D[b,i,j] = (|x_i|^2 + |y_j|^2) - 2 x_i.y_j, clamped at 0
// with the clamp recorded as -0.0 and in clamp_flags[b].
//
// A tile is 128 x 128 cells of one pair (UMMA M = N = 128); its K loop runs over the features in chunks of
// 32 (one 128-byte swizzle atom of fp32). Tiles blockIdx.x, blockIdx.x + gridDim.x, ... (the tiles of a pair
// are consecutive, so X and Y rows are reused from L2); chunks are numbered q across the CTA's tiles.
//   * warp 0 (TMA): X[128 rows x 32 features] and Y[128 x 32] of chunk q into stage q % S (128-byte
//     swizzled); three stages, so the load of a chunk has two chunks' products to arrive in;
//   * warps 2..9 (split): thread r (< 128) takes X row r, thread 128 + r takes Y row r: split in place into a
//     TF32 head and, in tail buffer q % 2, a TF32 tail (3xTF32), and accumulate the row's squared norm over
//     the tile's chunks (written to norm buffer tile % 4 at the tile's last chunk);
//   * warp 1 (MMA): 3 x 4 tcgen05.mma kind::tf32 per chunk into accumulator (tile & 1), commit to the
//     stage's and the tail buffer's "empty" barriers, and after the tile's last chunk to "acc full";
//   * warps 10..17 (epilogue, two groups of four, one per column half): per 32-column slice, read the
//     accumulator row (tcgen05.ld), form D, write it 128-byte swizzled into the group's staging buffer and
//     store it with TMA; release the accumulator after the last slice.
// Every wait is bounded; a wait that runs out raises the CTA's abort word and bit 1 of the distance error
// word, and the epilogue writes NaN into the tiles it has not finished.
// ==================================================================================================
constexpr int kDThreads = 32 * (2 + 8 + 8);
constexpr int kDSplit0 = 64;                        // first split thread
constexpr int kDEpiWarp0 = 10;                      // epilogue warps 10..17: lane quarter w % 4, column half
constexpr int kDStage = 2 * kChunk;                 // X head, Y head (TMA destination, split in place): 32 KB
constexpr int kDS = 3;                              // stages
constexpr int kDP = 2;                              // tail buffers (X tail, Y tail: 32 KB each)
constexpr int kDOffStage = 0;
constexpr int kDOffTail = kDS * kDStage;
constexpr int kDOffOut = kDOffTail + kDP * 2 * kChunk;  // 2 column halves x 16 KB output staging
constexpr int kDOffNorm = kDOffOut + 2 * kChunk;    // x2[4][128], y2[4][128]
constexpr int kDOffBar = kDOffNorm + 2 * 4 * kT * 4;
// full[S], ready[S], empty[S], tail_empty[P], acc_full[2], acc_empty[2], norm[4]
constexpr int kDNBar = 3 * kDS + kDP + 8;
constexpr int kDOffTmem = kDOffBar + 8 * kDNBar;
constexpr int kDOffAbort = kDOffTmem + 8;
constexpr int kDSmemBytes = kDOffAbort + 8 + 1024;
constexpr uint32_t kDTmemCols = 2 * kT;             // two 128-column fp32 accumulators
static_assert(kDSmemBytes <= 227 * 1024, "shared memory");

struct PairwiseTcArgs {
    float* D;
    int* clamp_flags;
    int cosine;  // 0: squared L2; 1: D = 1 - x.y / (n(x) n(y)), n(v) = max(|v|, eps), no clamp
    float eps;
    int B, N, M, d;
    int nit, njt, nk;  // row tiles, column tiles, feature chunks
    unsigned long long timeout_ns;
    const int* tiles;    // non-null: compute only these tile ids (band_tile_list_kernel), tile_count of them
    const int* tile_count;
};

__global__ void __launch_bounds__(kDThreads, 1) pairwise_l2_tc_kernel(const __grid_constant__ CUtensorMap mx,
                                                                       const __grid_constant__ CUtensorMap my,
                                                                       const __grid_constant__ CUtensorMap md,
                                                                       PairwiseTcArgs a)
{
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw0 = smem_addr(smem_raw);
    unsigned char* sm = smem_raw + ((1024u - (raw0 & 1023u)) & 1023u);
    const uint32_t base = smem_addr(sm);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t full = base + kDOffBar;
    const uint32_t split = full + 8 * kDS;       // "ready": heads (stage) and tails (buffer) of chunk q written
    const uint32_t empty = split + 8 * kDS;
    const uint32_t tail_empty = empty + 8 * kDS;
    const uint32_t acc_full = tail_empty + 8 * kDP;
    const uint32_t acc_empty = acc_full + 16;
    const uint32_t norm_full = acc_empty + 16;  // [4]: the split wrote the norms of tile t (t % 4)
    volatile int* abort = reinterpret_cast<volatile int*>(sm + kDOffAbort);
    float* x2s = reinterpret_cast<float*>(sm + kDOffNorm);  // [4][128]
    float* y2s = x2s + 4 * kT;                              // [4][128]

    const int per_pair = a.nit * a.njt;
    const int ntiles = a.tiles ? *a.tile_count : a.B * per_pair;
    const int my_tiles = blockIdx.x < static_cast<unsigned>(ntiles)
                             ? (ntiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                             : 0;
    auto tile_of = [&](int tl, int& b, int& i0, int& j0) {
        int t = static_cast<int>(blockIdx.x) + tl * static_cast<int>(gridDim.x);
        if (a.tiles) t = a.tiles[t];
        b = t / per_pair;
        const int r = t % per_pair;
        i0 = (r / a.njt) * kT;
        j0 = (r % a.njt) * kT;
    };

    if (tid == 0) {
        for (int s = 0; s < kDS; ++s) {
            mbar_init(full + 8 * s, 1);
            mbar_init(split + 8 * s, 8);
            mbar_init(empty + 8 * s, 1);
        }
        for (int p = 0; p < kDP; ++p) mbar_init(tail_empty + 8 * p, 1);
        for (int c = 0; c < 2; ++c) {
            mbar_init(acc_full + 8 * c, 1);
            mbar_init(acc_empty + 8 * c, 8);
        }
        for (int c = 0; c < 4; ++c) mbar_init(norm_full + 8 * c, 8);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(base + kDOffTmem),
                     "r"(kDTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + kDOffTmem);

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const int Q = my_tiles * a.nk;
            int issued = 0;
            for (int q = 0; q < Q; ++q) {
                const int s = q % kDS;
                if (q >= kDS && !wait_role(empty + 8 * s, ((q / kDS) - 1) & 1, a.timeout_ns, abort)) break;
                int b, i0, j0;
                tile_of(q / a.nk, b, i0, j0);
                const int kc = q % a.nk;
                const uint32_t st = base + kDOffStage + s * kDStage;
                mbar_expect_tx(full + 8 * s, kDStage);
                tma_load_3d(st, &mx, full + 8 * s, kc * kKC, i0, b);
                tma_load_3d(st + kChunk, &my, full + 8 * s, kc * kKC, j0, b);
                issued = q + 1;
            }
            for (int q = issued - kDS < 0 ? 0 : issued - kDS; q < issued; ++q)
                (void)mbar_wait(full + 8 * (q % kDS), (q / kDS) & 1, a.timeout_ns);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int q = 0;
            bool ok = true;
            for (int tl = 0; tl < my_tiles && ok; ++tl) {
                const int ab = tl & 1;
                if (tl >= 2 && !wait_role(acc_empty + 8 * ab, ((tl >> 1) - 1) & 1, a.timeout_ns, abort)) break;
                const uint32_t acc = tmem + static_cast<uint32_t>(ab * kT);
                for (int kc = 0; kc < a.nk; ++kc, ++q) {
                    const int s = q % kDS;
                    if (!wait_role(split + 8 * s, (q / kDS) & 1, a.timeout_ns, abort)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t st = base + kDOffStage + s * kDStage;
                    const uint32_t tb = base + kDOffTail + (q % kDP) * 2 * kChunk;
                    const uint64_t xh = sw128_desc(st), yh = sw128_desc(st + kChunk);
                    const uint64_t xl = sw128_desc(tb), yl = sw128_desc(tb + kChunk);
#pragma unroll
                    for (int kk = 0; kk < kKC / 8; ++kk) {
                        const uint64_t o = static_cast<uint64_t>((kk * 32) >> 4);  // 8 TF32 = 32 bytes along K
                        umma_tf32(acc, xh + o, yh + o, (kc > 0 || kk > 0) ? 1u : 0u);
                        umma_tf32(acc, xh + o, yl + o, 1u);
                        umma_tf32(acc, xl + o, yh + o, 1u);
                    }
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     empty + 8 * s)
                                 : "memory");
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     tail_empty + 8 * (q % kDP))
                                 : "memory");
                    if (kc == a.nk - 1)
                        asm volatile(
                            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                acc_full + 8 * ab)
                            : "memory");
                }
            }
            if (q > 0) (void)mbar_wait(empty + 8 * ((q - 1) % kDS), ((q - 1) / kDS) & 1, a.timeout_ns);
        }
    } else if (warp < kDEpiWarp0) {
        // ---------------- split ----------------
        const int st_id = tid - kDSplit0;          // 0..255
        const bool is_y = st_id >= kT;
        const int row = st_id & (kT - 1);
        int q = 0;
        for (int tl = 0; tl < my_tiles; ++tl) {
            float nrm = 0.f;
            bool ok = true;
            for (int kc = 0; kc < a.nk; ++kc, ++q) {
                const int s = q % kDS, p = q % kDP;
                if (!wait_role(full + 8 * s, (q / kDS) & 1, a.timeout_ns, abort) ||
                    (q >= kDP && !wait_role(tail_empty + 8 * p, ((q / kDP) - 1) & 1, a.timeout_ns, abort))) {
                    ok = false;
                    break;
                }
                unsigned char* st = sm + kDOffStage + s * kDStage + (is_y ? kChunk : 0);
                unsigned char* tb = sm + kDOffTail + p * 2 * kChunk + (is_y ? kChunk : 0);
                nrm += split_row(st + 128 * row, tb + 128 * row, row);
                if (kc == a.nk - 1)
                    (is_y ? y2s : x2s)[(tl & 3) * kT + row] = a.cosine ? 1.f / fmaxf(sqrtf(nrm), a.eps) : nrm;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(split + 8 * s);
                    if (kc == a.nk - 1) mbar_arrive(norm_full + 8 * (tl & 3));
                }
            }
            if (!ok) break;
        }
    } else {
        // ---------------- epilogue ----------------
        // Two groups of four warps; group h writes column slices 2h and 2h+1 of every tile through its own
        // two staging buffers, synchronised by named barrier 1 + h.
        const int row = 32 * (warp & 3) + lane;     // accumulator lane = tile row
        const int eg = (warp - kDEpiWarp0) >> 2;    // column half
        const int et = tid - 32 * kDEpiWarp0 - 128 * eg;  // 0..127 within the group
        const bool leader = et == 0;
        const uint32_t gbar = 1 + eg;
        unsigned char* const gout = sm + kDOffOut + eg * kChunk;
        int tl = 0;
        for (; tl < my_tiles; ++tl) {
            const int ab = tl & 1;
            if (!wait_role(acc_full + 8 * ab, (tl >> 1) & 1, a.timeout_ns, abort) ||
                !wait_role(norm_full + 8 * (tl & 3), (tl >> 2) & 1, a.timeout_ns, abort))
                break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            int b, i0, j0;
            tile_of(tl, b, i0, j0);
            const float x2 = x2s[(tl & 3) * kT + row];
            const float* y2 = y2s + (tl & 3) * kT;
            const int i = i0 + row;
            bool clamped = false;
#pragma unroll 1
            for (int qs = 2 * eg; qs < 2 * eg + 2; ++qs) {
                float acc[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + static_cast<uint32_t>(ab * kT + 32 * qs),
                          acc);
                // The group's staging buffer was last read by its previous store.
                if (leader) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                asm volatile("bar.sync %0, 128;" ::"r"(gbar) : "memory");
                unsigned char* ob = gout + 128 * row;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    float o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int jl = 32 * qs + 4 * u + e;
                        if (a.cosine) {  // x2, y2 hold the inverse norms
                            o[e] = 1.f - acc[4 * u + e] * (x2 * y2[jl]);
                        } else {
                            const float v = (x2 + y2[jl]) - 2.f * acc[4 * u + e];
                            clamped |= v < 0.f && i < a.N && j0 + jl < a.M;
                            o[e] = v < 0.f ? -0.f : v;
                        }
                    }
                    *reinterpret_cast<float4*>(ob + 16 * (u ^ (row & 7))) = make_float4(o[0], o[1], o[2], o[3]);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                asm volatile("bar.sync %0, 128;" ::"r"(gbar) : "memory");
                if (leader) {
                    tma_store_3d(&md, smem_addr(gout), j0 + 32 * qs, i0, b);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + 8 * ab);
            if (a.clamp_flags && __any_sync(kFull, clamped) && lane == 0) atomicOr(a.clamp_flags + b, 1);
        }
        if (leader) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        if (tl < my_tiles) {
            // A wait ran out: NaN into this thread's row of every tile not finished.
            for (; tl < my_tiles; ++tl) {
                int b, i0, j0;
                tile_of(tl, b, i0, j0);
                const int i = i0 + row;
                if (i < a.N)
                    for (int jl = 64 * eg; jl < 64 * eg + 64 && j0 + jl < a.M; ++jl)
                        a.D[(static_cast<int64_t>(b) * a.N + i) * a.M + j0 + jl] = __int_as_float(0x7fc00000);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kDTmemCols) : "memory");
}

// ---- host -------------------------------------------------------------------------------------------
std::mutex g_tc_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
bool g_attr_set[128] = {};

cudaError_t get_encode(PFN_cuTensorMapEncodeTiled_v12000& fn)
{
    std::lock_guard<std::mutex> lock(g_tc_mu);
    if (!g_encode) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (e != cudaSuccess) return e;
        if (q != cudaDriverEntryPointSuccess || !p) return cudaErrorNotSupported;
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    fn = g_encode;
    return cudaSuccess;
}

// 3-D tensor map of a (batch, rows, cols) fp32 array with a box of box_cols x box_rows x 1. Elements
// outside the array read as zero.
bool make_map_box(PFN_cuTensorMapEncodeTiled_v12000 encode, CUtensorMap* map, const void* ptr, int64_t B,
                  int64_t rows, int64_t cols, int box_cols, int box_rows, CUtensorMapSwizzle swizzle)
{
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(B)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 4, static_cast<cuuint64_t>(rows * cols) * 4};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Box of 32 columns x 128 rows, 128-byte swizzle (the operand tiles of both tensor-core kernels).
bool make_map(PFN_cuTensorMapEncodeTiled_v12000 encode, CUtensorMap* map, const void* ptr, int64_t B,
              int64_t rows, int64_t cols)
{
    return make_map_box(encode, map, ptr, B, rows, cols, kKC, kT, CU_TENSOR_MAP_SWIZZLE_128B);
}

int g_sm_count[128] = {};
bool g_grad_attr_set[128][20] = {};

// TRANS == false: grad_X of E (B, N, M) against Y (B, M, d), rows of X. TRANS == true: the caller passes the
// transposed problem (X := Y, Y := X, N := M, M := N, out := grad_Y, ry := the inverse norms of X's rows),
// and E, D stay the (B, M, N) arrays they are in memory.
template <int DPAD, bool TRANS, bool BANDED>
cudaError_t grad_tc_launch_t(const float* X, const float* Y, const float* D, const float* E, const float* g,
                             const int* clamp_flags, float* gX, int64_t B, int64_t N, int64_t M, int64_t d,
                             double timeout_s, cudaStream_t s, int dev, int slot,
                             PFN_cuTensorMapEncodeTiled_v12000 encode, const float* ry, float eps,
                             const DpRegion* region)
{
    using G = GradGeom<DPAD>;
    {
        std::lock_guard<std::mutex> lock(g_tc_mu);
        const int sl = slot + (TRANS ? 5 : 0) + (BANDED ? 10 : 0);
        if (!g_grad_attr_set[dev][sl]) {
            const cudaError_t e = cudaFuncSetAttribute(grad_x_tc_kernel<DPAD, TRANS, BANDED>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, G::BYTES);
            if (e != cudaSuccess) return e;
            g_grad_attr_set[dev][sl] = true;
        }
    }
    CUtensorMap me, my;
    // E's box: 32 columns x 128 rows, 128-byte swizzled (grad_X), or 128 columns x 32 rows, unswizzled
    // (grad_Y, from the (B, M, N) array: rows are the K extent).
    const bool me_ok = TRANS ? make_map_box(encode, &me, E, B, M, N, kGT, kGKC, CU_TENSOR_MAP_SWIZZLE_NONE)
                             : make_map(encode, &me, E, B, N, M);
    if (!me_ok || !make_map_box(encode, &my, Y, B, M, d, G::YB, kGKC, CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    GradTcArgs a;
    a.X = X;
    a.D = D;
    a.g = g;
    a.clamp_flags = clamp_flags;
    a.ry = ry;
    a.eps = eps;
    a.out = gX;
    a.B = static_cast<int>(B);
    a.N = static_cast<int>(N);
    a.M = static_cast<int>(M);
    a.d = static_cast<int>(d);
    a.nrt = static_cast<int>((N + kGT - 1) / kGT);
    a.nk = static_cast<int>((M + kGKC - 1) / kGKC);
    a.timeout_ns = static_cast<unsigned long long>(timeout_s * 1e9);
    a.len = Lengths{BANDED ? region->px : nullptr, BANDED ? region->py : nullptr, BANDED ? region->is32 : 0};
    a.bw = BANDED ? (region->bw > N + M ? N + M : region->bw) : -1;
    const int64_t tiles = B * a.nrt;
    const int grid = static_cast<int>(tiles < g_sm_count[dev] ? tiles : g_sm_count[dev]);
    count_launch();
    grad_x_tc_kernel<DPAD, TRANS, BANDED><<<grid, kGradThreads, G::BYTES, s>>>(me, my, a);
    return cudaGetLastError();
}

}  // namespace

bool grad_tc_supported(const void* X, const void* Y, const void* D, const void* E, const void* gX, int64_t B,
                       int64_t N, int64_t M, int64_t d)
{
    const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    // (The row-tile count bounds both contractions: grad_X tiles over N, grad_Y over M.)
    return d >= 1 && d <= 128 && d % 4 == 0 && M % 4 == 0 && N >= 1 && M >= 1 && al(X) && al(Y) && al(D) &&
           al(E) && al(gX) && N < (1 << 30) && M < (1 << 30) && B >= 1 && B * ((N + kGT - 1) / kGT) < (1ll << 31) &&
           B * ((M + kGT - 1) / kGT) < (1ll << 31);
}

namespace {
// The SM count and the tensor-map encoder, for the calling thread's current device.
cudaError_t tc_prepare(PFN_cuTensorMapEncodeTiled_v12000& encode, int& dev)
{
    cudaError_t e = get_encode(encode);
    if (e != cudaSuccess) return e;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_tc_mu);
    if (g_sm_count[dev] == 0) {
        int n = 0;
        e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        g_sm_count[dev] = n > 0 ? n : 1;
    }
    return cudaSuccess;
}

// grad_tc_launch_t for d's padded width, with or without a region.
template <bool TRANS>
cudaError_t grad_tc_dispatch(const float* X, const float* Y, const float* D, const float* E, const float* g,
                             const int* clamp_flags, float* out, int64_t B, int64_t N, int64_t M, int64_t d,
                             double timeout_s, cudaStream_t s, int dev, PFN_cuTensorMapEncodeTiled_v12000 encode,
                             const float* r, float eps, const DpRegion* region)
{
    if (region && region->px) {
        if (d <= 16) return grad_tc_launch_t<16, TRANS, true>(X, Y, D, E, g, clamp_flags, out, B, N, M, d, timeout_s, s, dev, 0, encode, r, eps, region);
        if (d <= 32) return grad_tc_launch_t<32, TRANS, true>(X, Y, D, E, g, clamp_flags, out, B, N, M, d, timeout_s, s, dev, 1, encode, r, eps, region);
        if (d <= 64) return grad_tc_launch_t<64, TRANS, true>(X, Y, D, E, g, clamp_flags, out, B, N, M, d, timeout_s, s, dev, 2, encode, r, eps, region);
        if (d <= 96) return grad_tc_launch_t<96, TRANS, true>(X, Y, D, E, g, clamp_flags, out, B, N, M, d, timeout_s, s, dev, 3, encode, r, eps, region);
        return grad_tc_launch_t<128, TRANS, true>(X, Y, D, E, g, clamp_flags, out, B, N, M, d, timeout_s, s, dev, 4, encode, r, eps, region);
    }
    if (d <= 16) return grad_tc_launch_t<16, TRANS, false>(X, Y, D, E, g, clamp_flags, out, B, N, M, d, timeout_s, s, dev, 0, encode, r, eps, nullptr);
    if (d <= 32) return grad_tc_launch_t<32, TRANS, false>(X, Y, D, E, g, clamp_flags, out, B, N, M, d, timeout_s, s, dev, 1, encode, r, eps, nullptr);
    if (d <= 64) return grad_tc_launch_t<64, TRANS, false>(X, Y, D, E, g, clamp_flags, out, B, N, M, d, timeout_s, s, dev, 2, encode, r, eps, nullptr);
    if (d <= 96) return grad_tc_launch_t<96, TRANS, false>(X, Y, D, E, g, clamp_flags, out, B, N, M, d, timeout_s, s, dev, 3, encode, r, eps, nullptr);
    return grad_tc_launch_t<128, TRANS, false>(X, Y, D, E, g, clamp_flags, out, B, N, M, d, timeout_s, s, dev, 4, encode, r, eps, nullptr);
}
}  // namespace

cudaError_t grad_y_tc_launch(const float* X, const float* Y, const float* D, const float* E, const float* g,
                             const int* clamp_flags, float* gY, int64_t B, int64_t N, int64_t M, int64_t d,
                             double timeout_s, cudaStream_t s, const float* rx, float eps, const DpRegion* region)
{
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    int dev = 0;
    const cudaError_t e = tc_prepare(encode, dev);
    if (e != cudaSuccess) return e;
    // The transposed problem: output rows are Y's (M of them), the K extent is N, B operand X.
    return grad_tc_dispatch<true>(Y, X, D, E, g, clamp_flags, gY, B, M, N, d, timeout_s, s, dev, encode, rx, eps,
                                  region);
}

cudaError_t grad_x_tc_launch(const float* X, const float* Y, const float* D, const float* E, const float* g,
                             const int* clamp_flags, float* gX, int64_t B, int64_t N, int64_t M, int64_t d,
                             double timeout_s, cudaStream_t s, const float* ry, float eps, const DpRegion* region)
{
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    int dev = 0;
    const cudaError_t e = tc_prepare(encode, dev);
    if (e != cudaSuccess) return e;
    return grad_tc_dispatch<false>(X, Y, D, E, g, clamp_flags, gX, B, N, M, d, timeout_s, s, dev, encode, ry, eps,
                                   region);
}

size_t pairwise_tc_region_ws_bytes(int64_t B, int64_t N, int64_t M)
{
    return 16 + 4 * static_cast<size_t>(B) * static_cast<size_t>((N + kT - 1) / kT) *
                    static_cast<size_t>((M + kT - 1) / kT);
}

bool pairwise_tc_supported(const void* X, const void* Y, const void* D, int64_t B, int64_t N, int64_t M, int64_t d)
{
    const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return d >= 1 && d % 4 == 0 && M % 4 == 0 && al(X) && al(Y) && al(D) && N <= (1 << 30) && M <= (1 << 30) &&
           d <= (1 << 20) && B <= 65535 && (N + kT - 1) / kT <= 65535;
}

cudaError_t pairwise_tc_launch(const float* X, const float* Y, float* D, int* clamp_flags, int64_t B, int64_t N,
                               int64_t M, int64_t d, double timeout_s, cudaStream_t s, bool cosine, float eps,
                               const DpRegion* region, void* ws)
{
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    cudaError_t e = get_encode(encode);
    if (e != cudaSuccess) return e;
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    {
        std::lock_guard<std::mutex> lock(g_tc_mu);
        if (!g_attr_set[dev]) {
            e = cudaFuncSetAttribute(pairwise_l2_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDSmemBytes);
            if (e != cudaSuccess) return e;
            g_attr_set[dev] = true;
        }
        if (g_sm_count[dev] == 0) {
            int n = 0;
            e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess) return e;
            g_sm_count[dev] = n > 0 ? n : 1;
        }
    }
    CUtensorMap mx, my, md;
    if (!make_map(encode, &mx, X, B, N, d) || !make_map(encode, &my, Y, B, M, d) || !make_map(encode, &md, D, B, N, M))
        return cudaErrorInvalidValue;
    PairwiseTcArgs a;
    a.D = D;
    a.clamp_flags = clamp_flags;
    a.cosine = cosine ? 1 : 0;
    a.eps = eps;
    a.B = static_cast<int>(B);
    a.N = static_cast<int>(N);
    a.M = static_cast<int>(M);
    a.d = static_cast<int>(d);
    a.nit = static_cast<int>((N + kT - 1) / kT);
    a.njt = static_cast<int>((M + kT - 1) / kT);
    a.nk = static_cast<int>((d + kKC - 1) / kKC);
    a.timeout_ns = static_cast<unsigned long long>(timeout_s * 1e9);
    a.tiles = nullptr;
    a.tile_count = nullptr;
    const int64_t tiles = B * a.nit * a.njt;
    if (region && region->px && ws && tiles < (int64_t(1) << 31)) {
        int* count = static_cast<int*>(ws);
        int* list = count + 4;
        const Lengths len{region->px, region->py, region->is32};
        const int64_t bw = region->bw > N + M ? N + M : region->bw;
        count_launch();
        band_tile_list_kernel<<<1, 1024, 0, s>>>(len, a.B, a.N, a.M, bw, a.nit, a.njt, count, list);
        a.tiles = list;
        a.tile_count = count;
    }
    const int grid = static_cast<int>(tiles < g_sm_count[dev] ? tiles : g_sm_count[dev]);
    count_launch();
    pairwise_l2_tc_kernel<<<grid, kDThreads, kDSmemBytes, s>>>(mx, my, md, a);
    return cudaGetLastError();
}

cudaError_t read_distance_errors(uint32_t& bits)
{
    uint32_t zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&bits, g_distance_err, sizeof(bits));
    if (e != cudaSuccess) return e;
    return bits ? cudaMemcpyToSymbol(g_distance_err, &zero, sizeof(zero)) : cudaSuccess;
}

}  // namespace sdtw
