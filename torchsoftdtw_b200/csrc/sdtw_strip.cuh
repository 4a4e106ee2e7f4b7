// Strip geometry and the per-cell arithmetic shared by the wavefront kernels (sm_100a).
#pragma once

#include "sdtw_common.cuh"

namespace sdtw {

// Lengths arrive as int64 or int32 device arrays (the reference converts int32 to int64 on the host,
// softdtw.cpp:67-70; here the kernel reads either directly).
struct Lengths {
    const void* px;
    const void* py;
    int is32;
    __device__ __forceinline__ int64_t x(int64_t b) const
    {
        return is32 ? static_cast<int64_t>(static_cast<const int*>(px)[b]) : static_cast<const int64_t*>(px)[b];
    }
    __device__ __forceinline__ int64_t y(int64_t b) const
    {
        return is32 ? static_cast<int64_t>(static_cast<const int*>(py)[b]) : static_cast<const int64_t*>(py)[b];
    }
};

// Per-lane geometry of one strip.
struct Strip {
    int64_t nx, ny;
    int r0, rows;          // first row, number of valid rows (<= 32)
    int lo, hi;            // this lane's in-band columns [lo, hi] (empty for lanes >= rows)
    int c_begin, c_end;    // union over the strip's rows
    int A, Z;              // this lane is valid at step tau iff A <= tau <= Z
    int Amax, Zmin;        // every lane is valid for tau in [Amax, Zmin]
    bool bad;
};

__device__ __forceinline__ int warp_max(int v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(kFull, v, o));
    return v;
}
__device__ __forceinline__ int warp_min(int v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// Returns false if the strip has no cells (empty pair, or r0 beyond the pair's length).
__device__ __forceinline__ bool make_strip(Strip& st, const Lengths& len, int64_t b, int s, int64_t N, int64_t M,
                                           int64_t bw, int lane)
{
    st.nx = len.x(b);
    st.ny = len.y(b);
    st.bad = st.nx < 0 || st.nx > N || st.ny < 0 || st.ny > M;
    if (st.bad) st.nx = st.ny = 0;
    st.r0 = 32 * s;
    if (st.nx == 0 || st.ny == 0 || st.r0 >= st.nx) return false;
    st.rows = static_cast<int>(st.nx - st.r0 < 32 ? st.nx - st.r0 : 32);
    int64_t lo = 1, hi = 0;
    if (lane < st.rows) band_row_range(st.r0 + lane, st.nx, st.ny, bw, lo, hi);
    st.lo = static_cast<int>(lo);
    st.hi = static_cast<int>(hi);
    st.c_begin = __shfl_sync(kFull, st.lo, 0);
    st.c_end = __shfl_sync(kFull, st.hi, st.rows - 1);
    st.A = lane < st.rows ? st.lo + lane : (1 << 30);
    st.Z = lane < st.rows ? st.hi + lane : -(1 << 30);
    st.Amax = warp_max(st.A);
    st.Zmin = warp_min(st.Z);
    return true;
}

// Forward cell: R = D + m - gamma*ln(1 + e^{-(x-m)/gamma} + e^{-(y-m)/gamma}) with m <= x <= y the
// three predecessors sorted (softdtw.cpp:149-163 computes the same softmin with three exponentials).
template <typename T>
__device__ __forceinline__ T fwd_cell(T d, T diag, T up, T left, T k, T gl)
{
    const T a = Num<T>::mn(up, left);
    const T y = Num<T>::mx(up, left);
    const T m = Num<T>::mn(a, diag);
    const T x = Num<T>::mx(a, diag);
    // m is +inf only when all three predecessors are: the exponents then stay -inf and R = D + inf.
    const T mc = Num<T>::mn(m, Num<T>::big());
    const T e1 = Num<T>::exp2_((mc - x) * k);
    const T e2 = Num<T>::exp2_((mc - y) * k);
    const T sum = (T(1) + e1) + e2;
    return fma(-gl, Num<T>::log2_(sum), m) + d;
}

// The same cell with every R and D value in units of gamma ln 2 (u = R log2(e) / gamma, d = D log2(e) /
// gamma): u = (m + d) - log2(1 + 2^(m - x) + 2^(m - y)). The exponents need no product with 1 / gamma and
// m + d is formed beside the exponentials, so the step's dependency chain is two operations shorter. Used
// where R stays inside the library (the R tiles between the pair-resident forward and backward).
template <typename T>
__device__ __forceinline__ T fwd_cell_scaled(T d, T diag, T up, T left)
{
    const T a = Num<T>::mn(up, left);
    const T y = Num<T>::mx(up, left);
    const T m = Num<T>::mn(a, diag);
    const T x = Num<T>::mx(a, diag);
    const T mc = Num<T>::mn(m, Num<T>::big());
    const T e1 = Num<T>::exp2_(mc - x);
    const T e2 = Num<T>::exp2_(mc - y);
    const T sum = (T(1) + e1) + e2;
    return (m + d) - Num<T>::log2_(sum);
}

}  // namespace sdtw
