// Shared device/host helpers for the sm_100a Soft-DTW kernels.
#pragma once

#include <cfloat>
#include <cstdint>

#include <cuda_runtime.h>

namespace sdtw {

// Kernel launches made by this library in this process (all entry points; read by
// sdtw_debug_kernel_launches). Defined in sdtw_wavefront.cu.
void count_launch();
// Upper bound (seconds) of every device-side wait (sdtw_set_wait_timeout). Defined in sdtw_wavefront.cu.
double wait_timeout_s();

// Largest number of pairs one launch of the cost and gradient kernels takes (they index pairs by grid.z);
// the C-ABI entry points run larger batches in chunks of this many pairs.
constexpr int64_t kBatchChunk = 65535;

// p advanced by `elems` elements of `es` bytes (null stays null).
inline const void* at_elem(const void* p, int64_t elems, size_t es)
{
    return p ? static_cast<const void*>(static_cast<const char*>(p) + static_cast<size_t>(elems) * es) : nullptr;
}
inline void* at_elem(void* p, int64_t elems, size_t es)
{
    return p ? static_cast<void*>(static_cast<char*>(p) + static_cast<size_t>(elems) * es) : nullptr;
}

// --------------------------------------------------------------------------------------------------
// Tiling constants of the strip wavefront.
//   A strip is 32 consecutive rows of one pair, owned by one warp (lane l <-> row r0 + l).
//   Lane l processes column (tau - l) at step tau, so one step of a warp is one anti-diagonal of the
//   strip. Steps are grouped in blocks of 32 (tau in [32k, 32k+32)); columns in chunks of 32.
//   Each warp keeps a circular "ring" in shared memory: 32 (or 33) rows x kRing columns, indexed by
//   (column & kRingMask), which holds 4 chunks: the two being swept, and two being prefetched.
// --------------------------------------------------------------------------------------------------
constexpr int kRing = 128;
constexpr int kRingMask = kRing - 1;
constexpr int kSide = 64;  // per-warp side ring (boundary row values), indexed by (column & 63)
constexpr int kSideMask = kSide - 1;
constexpr int kWarpsPerCta = 4;
constexpr unsigned kFull = 0xffffffffu;

// Error bits written to the caller's sticky error word (and to the per-launch abort word).
enum : uint32_t {
    kErrTimeout = 1u,    // a wait on a neighbouring strip's progress ran out
    kErrBadLength = 2u,  // a lengths_x / lengths_y value outside [0, N] / [0, M]
    kErrBounds = 4u,     // debug builds only: a global access fell outside its buffer (and was skipped)
};

// A global buffer of `bytes` bytes at `base`: the extent the debug build checks accesses against.
struct Extent {
    const void* base;
    size_t bytes;
};

// --------------------------------------------------------------------------------------------------
// Sakoe-Chiba band (reference src/torchsoftdtw/csrc/band.h:23-38), restated as the interval of
// in-band columns of one row. The reference tests cell (i, j) with
//     2 * |l*(K-1) - k*(L-1)| <= max(2*bw*(K-1), L-1)
// (K/L = short/long length, k/l = the cell's index on the short/long axis). For a fixed row i this
// is a closed interval in j; it is intersected with [0, ny). Every row i < nx has a non-empty
// interval (the band always contains a monotone path from (0,0) to (nx-1, ny-1)), and lo/hi are
// non-decreasing in i.
// --------------------------------------------------------------------------------------------------
__host__ __device__ __forceinline__ int64_t floor_div(int64_t a, int64_t b)  // b > 0
{
    return a >= 0 ? a / b : -((-a + b - 1) / b);
}
__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return -floor_div(-a, b); }

__host__ __device__ inline void band_row_range(int64_t i, int64_t nx, int64_t ny, int64_t bw, int64_t& lo,
                                               int64_t& hi)
{
    lo = 0;
    hi = ny - 1;
    if (bw < 0) return;
    const bool x_short = nx <= ny;
    const int64_t K = x_short ? nx : ny;
    const int64_t L = x_short ? ny : nx;
    if (K <= 1) return;
    const int64_t band = 2 * bw * (K - 1);
    const int64_t W = band > L - 1 ? band : L - 1;
    const int64_t h = W / 2;  // 2*diff <= W  <=>  diff <= floor(W/2) for integer diff
    int64_t a, z;
    if (x_short) {  // rows are the short axis: |j*(K-1) - i*(L-1)| <= h
        a = ceil_div(i * (L - 1) - h, K - 1);
        z = floor_div(i * (L - 1) + h, K - 1);
    } else {  // rows are the long axis: |i*(K-1) - j*(L-1)| <= h
        a = ceil_div(i * (K - 1) - h, L - 1);
        z = floor_div(i * (K - 1) + h, L - 1);
    }
    if (a > lo) lo = a;
    if (z < hi) hi = z;
}

#ifdef __CUDACC__

// --------------------------------------------------------------------------------------------------
// Arithmetic. fp32 uses the SFU approximations (PTX ex2/lg2/rcp .approx.ftz); fp64 calls CUDA's
// double-precision exp2/log2 and an IEEE division.
// --------------------------------------------------------------------------------------------------
__device__ __forceinline__ float ex2f(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float lg2f(float x)
{
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcpf(float x)
{
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T>
struct Num;

template <>
struct Num<float> {
    static __device__ __forceinline__ float inf() { return __int_as_float(0x7f800000); }
    static __device__ __forceinline__ float big() { return FLT_MAX; }
    static __device__ __forceinline__ float nan() { return __int_as_float(0x7fc00000); }
    static __device__ __forceinline__ float exp2_(float x) { return ex2f(x); }
    static __device__ __forceinline__ float log2_(float x) { return lg2f(x); }
    static __device__ __forceinline__ float rcp_(float x) { return rcpf(x); }
    static __device__ __forceinline__ float mn(float a, float b) { return fminf(a, b); }
    static __device__ __forceinline__ float mx(float a, float b) { return fmaxf(a, b); }
};

template <>
struct Num<double> {
    static __device__ __forceinline__ double inf() { return __longlong_as_double(0x7ff0000000000000ll); }
    static __device__ __forceinline__ double big() { return DBL_MAX; }
    static __device__ __forceinline__ double nan() { return __longlong_as_double(0x7ff8000000000000ll); }
    static __device__ __forceinline__ double exp2_(double x) { return exp2(x); }
    static __device__ __forceinline__ double log2_(double x) { return log2(x); }
    static __device__ __forceinline__ double rcp_(double x) { return 1.0 / x; }
    static __device__ __forceinline__ double mn(double a, double b) { return fmin(a, b); }
    static __device__ __forceinline__ double mx(double a, double b) { return fmax(a, b); }
};

// --------------------------------------------------------------------------------------------------
// Asynchronous global->shared copies (cp.async). `src_bytes` < size zero-fills the rest.
// --------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async_16(void* dst, const void* src, int src_bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_4(void* dst, const void* src, int src_bytes)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_8(void* dst, const void* src, int src_bytes)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
template <int BYTES>
__device__ __forceinline__ void cp_async_scalar(void* dst, const void* src, int src_bytes)
{
    if constexpr (BYTES == 4)
        cp_async_4(dst, src, src_bytes);
    else
        cp_async_8(dst, src, src_bytes);
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// --------------------------------------------------------------------------------------------------
// Boundary exchange between strips (global memory, gpu scope), without flags or fences.
//   A boundary buffer is filled with an all-ones bit pattern before the launch (cudaMemset 0xFF): a NaN
//   that the kernels' arithmetic never produces (a NaN result of an FP instruction on this GPU is the
//   canonical 0x7fffffff / 0x7ff8...). Producers store finished values with st.relaxed.gpu; consumers
//   read them with ld.relaxed.gpu and treat a value as present as soon as it differs from the pattern.
//   Each element is written once and accessed single-copy-atomically, so no ordering between
//   different elements is needed: the data itself is the flag.
// --------------------------------------------------------------------------------------------------
__device__ __forceinline__ int ld_relaxed(const int* p)
{
    int v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float ld_relaxed(const float* p)
{
    float v;
    asm volatile("ld.relaxed.gpu.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ double ld_relaxed(const double* p)
{
    double v;
    asm volatile("ld.relaxed.gpu.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed(float* p, float v)
{
    asm volatile("st.relaxed.gpu.global.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed(double* p, double v)
{
    asm volatile("st.relaxed.gpu.global.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}
__device__ __forceinline__ bool is_absent(float v) { return __float_as_uint(v) == 0xffffffffu; }
__device__ __forceinline__ bool is_absent(double v) { return __double_as_longlong(v) == -1ll; }

// --------------------------------------------------------------------------------------------------
// Bounds checks of the debug build (compiled with SDTW_DEBUG_BOUNDS; the library is then built as
// libsdtw_b200_debug.so). SDTW_IN_BOUNDS(ext, p, n, err) is true when the n bytes at p lie inside the
// extent; otherwise it sets kErrBounds in the error word `err` and the caller skips the access (a load reads
// nothing, a store writes nothing): no trap, the context stays usable, the host reads the bit. In the
// release build the check is the constant true and costs nothing. It stands in for a memory checker where
// none can run.
// --------------------------------------------------------------------------------------------------
__device__ __forceinline__ bool bounds_check(const Extent& x, const void* p, size_t n, uint32_t* err)
{
    const char* c = static_cast<const char*>(p);
    const char* b0 = static_cast<const char*>(x.base);
    if (b0 != nullptr && c >= b0 && c + n <= b0 + x.bytes) return true;
    atomicOr(err, kErrBounds);
    return false;
}
#ifdef SDTW_DEBUG_BOUNDS
#define SDTW_IN_BOUNDS(ext, p, n, err) ::sdtw::bounds_check((ext), (p), (n), (err))
#else
#define SDTW_IN_BOUNDS(ext, p, n, err) true
#endif

__device__ __forceinline__ uint64_t global_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

struct Sync {
    uint32_t* err;         // caller's sticky error word (accumulates across launches)
    int* abort;            // this launch's abort word (zeroed per launch)
    uint64_t timeout_ns;   // limit of every wait on another strip
};

__device__ __forceinline__ void raise_error(const Sync& sy, uint32_t bits)
{
    atomicOr(sy.err, bits);
    atomicOr(sy.abort, static_cast<int>(bits));
}

__device__ __forceinline__ bool aborted(const Sync& sy) { return ld_relaxed(sy.abort) != 0; }

// Warp-collective. Lane `lane` needs the boundary value at `src` when `needed`; `v` holds what an
// earlier (prefetching) load returned. Re-reads the lanes whose value is still absent until every
// needed value is present. Returns false if the launch was aborted or the wait ran out (which raises
// kErrTimeout and aborts the launch).
template <typename T>
__device__ __forceinline__ bool await_boundary(T& v, const T* src, bool needed, const Sync& sy, int lane)
{
    bool ok = !needed || !is_absent(v);
    if (__all_sync(kFull, ok)) return true;
    const uint64_t t0 = global_ns();
    unsigned ns = 32;
    while (true) {
        __nanosleep(ns);
        if (!ok) {
            v = ld_relaxed(src);
            ok = !is_absent(v);
        }
        if (__all_sync(kFull, ok)) return true;
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
        ns = ns < 256 ? ns * 2 : 256;
    }
}

#endif  // __CUDACC__

}  // namespace sdtw
