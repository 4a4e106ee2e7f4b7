// Squared-L2 cost matrix on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// D[b,i,j] = (|x_i|^2 + |y_j|^2) - 2 x_i.y_j, clamped at 0 with the clamp recorded as -0.0, for fp32 X, Y.
// One CTA (128 threads) computes a 128 x 128 tile of D:
//   * TMA (cp.async.bulk.tensor, no multicast) brings 128 rows x 32 features of X and of Y into shared
//     memory per K step, 128-byte swizzled, completing on an mbarrier;
//   * each thread splits one row of each in place into a TF32 head and a TF32 tail (both rounded to
//     nearest: x = head + tail to about 2^-22) and accumulates the row's squared norm in fp32;
//   * one thread issues tcgen05.mma kind::tf32 (M = N = 128, K = 8) for head.head + head.tail + tail.head
//     (3xTF32: the x.y products keep fp32 accuracy) into a 128-column fp32 accumulator in tensor memory,
//     and tcgen05.commit signals an mbarrier when they are done;
//   * the four warps read their 32 accumulator lanes (rows) with tcgen05.ld, form D, write it to shared
//     memory in the 128-byte swizzled layout, and one thread stores the tile with TMA.
// Every mbarrier wait is bounded in time; a tile whose wait runs out is written as NaN and a bit is set in
// the library's distance error word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "sdtw_b200.h"
#include "sdtw_common.cuh"
#include "sdtw_tcgen05.h"

namespace sdtw {

namespace {

constexpr int kT = 128;                // tile rows (X) = tile columns (Y) = UMMA M = N
constexpr int kKC = 32;                // features per K step: one 128-byte swizzle atom of fp32
constexpr int kChunk = kT * kKC * 4;   // 16 KB: one operand's K step
constexpr uint32_t kTmemCols = 128;    // fp32 accumulator 128 x 128
// Shared memory (offsets from a 1024-byte aligned base): X head, X tail, Y head, Y tail (one K step each;
// reused as the 4 x 32-column staging of the output tile), |y|^2 of the tile's columns, two mbarriers and
// the tensor-memory address.
constexpr int kOffXh = 0, kOffXl = kChunk, kOffYh = 2 * kChunk, kOffYl = 3 * kChunk;
constexpr int kOffY2 = 4 * kChunk;
constexpr int kOffBarLoad = kOffY2 + kT * 4;
constexpr int kOffBarMma = kOffBarLoad + 8;
constexpr int kOffTmem = kOffBarMma + 8;
constexpr int kSmemUsed = kOffTmem + 16;
constexpr int kSmemBytes = kSmemUsed + 1024;  // slack for aligning the dynamic base to 1024 bytes

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

__global__ void __launch_bounds__(128) pairwise_l2_tc_kernel(const __grid_constant__ CUtensorMap mx,
                                                             const __grid_constant__ CUtensorMap my,
                                                             const __grid_constant__ CUtensorMap md, float* D,
                                                             int* clamp_flags, int N, int M, int d,
                                                             unsigned long long timeout_ns)
{
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    unsigned char* sm = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t base = smem_addr(sm);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int j0 = blockIdx.x * kT, i0 = blockIdx.y * kT, b = blockIdx.z;
    const uint32_t bar_load = base + kOffBarLoad, bar_mma = base + kOffBarMma;
    float* y2s = reinterpret_cast<float*>(sm + kOffY2);

    if (tid == 0) {
        mbar_init(bar_load, 1);
        mbar_init(bar_mma, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(base + kOffTmem),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + kOffTmem);

    // Every thread waits on each mbarrier (bounded); the outcome is made uniform with __syncthreads_and, so
    // the whole CTA leaves the loop together if a wait ran out.
    bool ok = true;
    float x2 = 0.f, y2 = 0.f;
    const int nk = (d + kKC - 1) / kKC;
    for (int kc = 0; kc < nk; ++kc) {
        if (tid == 0) {
            mbar_expect_tx(bar_load, 2 * kChunk);
            tma_load_3d(base + kOffXh, &mx, bar_load, kc * kKC, i0, b);
            tma_load_3d(base + kOffYh, &my, bar_load, kc * kKC, j0, b);
        }
        ok = __syncthreads_and(mbar_wait(bar_load, kc & 1, timeout_ns) ? 1 : 0) != 0;
        if (!ok) break;
        x2 += split_row(sm + kOffXh + 128 * tid, sm + kOffXl + 128 * tid, tid);
        y2 += split_row(sm + kOffYh + 128 * tid, sm + kOffYl + 128 * tid, tid);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint64_t xh = sw128_desc(base + kOffXh), xl = sw128_desc(base + kOffXl);
            const uint64_t yh = sw128_desc(base + kOffYh), yl = sw128_desc(base + kOffYl);
#pragma unroll
            for (int kk = 0; kk < kKC / 8; ++kk) {
                const uint64_t step = static_cast<uint64_t>((kk * 32) >> 4);  // 8 TF32 = 32 bytes along K
                umma_tf32(tmem, xh + step, yh + step, (kc > 0 || kk > 0) ? 1u : 0u);
                umma_tf32(tmem, xh + step, yl + step, 1u);
                umma_tf32(tmem, xl + step, yh + step, 1u);
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             bar_mma)
                         : "memory");
        }
        ok = __syncthreads_and(mbar_wait(bar_mma, kc & 1, timeout_ns) ? 1 : 0) != 0;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (!ok) break;
    }
    y2s[tid] = y2;
    __syncthreads();

    const int i = i0 + tid;  // this thread's row of the tile (TMEM lane = tid)
    bool clamped = false;
    if (ok) {
#pragma unroll 1
        for (int q = 0; q < kT / 32; ++q) {
            float acc[32];
            tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(q * 32), acc);
            unsigned char* row = sm + q * kChunk + 128 * tid;  // staging of columns 32q .. 32q+31
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int jl = 32 * q + 4 * u + e;
                    float v = (x2 + y2s[jl]) - 2.f * acc[4 * u + e];
                    clamped |= v < 0.f && i < N && j0 + jl < M;
                    o[e] = v < 0.f ? -0.f : v;
                }
                *reinterpret_cast<float4*>(row + 16 * (u ^ (tid & 7))) = make_float4(o[0], o[1], o[2], o[3]);
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
#pragma unroll 1
            for (int q = 0; q < kT / 32; ++q) tma_store_3d(&md, base + q * kChunk, j0 + 32 * q, i0, b);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        }
    } else {
        // A wait ran out: report it and leave NaN in this tile rather than stale data.
        if (tid == 0) atomicOr(&g_distance_err, 1u);
        if (i < N) {
            float* dst = D + (static_cast<int64_t>(b) * N + i) * M;
            for (int jl = 0; jl < kT && j0 + jl < M; ++jl) dst[j0 + jl] = __int_as_float(0x7fc00000);
        }
    }
    if (clamp_flags && __any_sync(kFull, clamped) && lane == 0) atomicOr(clamp_flags + b, 1);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
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

// 3-D tensor map of a (batch, rows, cols) fp32 array, box of 32 columns x 128 rows x 1, 128-byte swizzle.
bool make_map(PFN_cuTensorMapEncodeTiled_v12000 encode, CUtensorMap* map, const void* ptr, int64_t B,
              int64_t rows, int64_t cols)
{
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(B)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 4, static_cast<cuuint64_t>(rows * cols) * 4};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kKC), static_cast<cuuint32_t>(kT), 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

bool pairwise_tc_supported(const void* X, const void* Y, const void* D, int64_t B, int64_t N, int64_t M, int64_t d)
{
    const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return d >= 1 && d % 4 == 0 && M % 4 == 0 && al(X) && al(Y) && al(D) && N <= (1 << 30) && M <= (1 << 30) &&
           d <= (1 << 20) && B <= 65535 && (N + kT - 1) / kT <= 65535;
}

cudaError_t pairwise_tc_launch(const float* X, const float* Y, float* D, int* clamp_flags, int64_t B, int64_t N,
                               int64_t M, int64_t d, double timeout_s, cudaStream_t s)
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
            e = cudaFuncSetAttribute(pairwise_l2_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
            if (e != cudaSuccess) return e;
            g_attr_set[dev] = true;
        }
    }
    CUtensorMap mx, my, md;
    if (!make_map(encode, &mx, X, B, N, d) || !make_map(encode, &my, Y, B, M, d) || !make_map(encode, &md, D, B, N, M))
        return cudaErrorInvalidValue;
    const dim3 grid(static_cast<unsigned>((M + kT - 1) / kT), static_cast<unsigned>((N + kT - 1) / kT),
                    static_cast<unsigned>(B));
    count_launch();
    pairwise_l2_tc_kernel<<<grid, kT, kSmemBytes, s>>>(mx, my, md, D, clamp_flags, static_cast<int>(N),
                                                       static_cast<int>(M), static_cast<int>(d),
                                                       static_cast<unsigned long long>(timeout_s * 1e9));
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
