// Shared device-side definitions of the sm_100a morphology kernels.
//
// Semantics follow the reference (vhrabar/serron 0.6.0, packages/serron/):
//   * op policy      csrc/gpu/morphology/ops_policy.cuh:16-54 (erode: s-w, min; dilate: s+w, max)
//   * borders        csrc/gpu/utils/boundaries.cuh:18-43 (REFLECT period 2n-2, REPLICATE clamp,
//                    CONSTANT -> the neutral element +-inf, never a user value)
//   * anchor         (kH/2, kW/2)
//   * winner         the first tap in row-major (di, dj) order that strictly improves on the running
//                    best, starting from the neutral element (csrc/cpu/morphology/backward.cpp:46-99);
//                    NaN taps and taps equal to the neutral element never win.
//   * precision      the comparison type is the reference CPU's accumulate type
//                    (csrc/compat/acc_type.h:23-53): float for half/bfloat16, double for float and
//                    double.  Float inputs are compared in float whenever that is provably the same
//                    as comparing in double (see exact_filter below).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace serron {

enum Border : int { kReflect = 0, kReplicate = 1, kConstant = 2 };
enum DType : int { kF32 = 0, kF64 = 1, kF16 = 2, kBF16 = 3 };
enum MorphOp : int { kErode = 0, kDilate = 1 };

// ------------------------------------------------------------------------------------------------
// storage <-> compute types
// ------------------------------------------------------------------------------------------------
template <typename T>
struct Storage;

template <>
struct Storage<float> {
    using acc = float;  // values: monotone rounding makes float min/max identical to the double ones
    static __device__ __forceinline__ float load(float v) { return v; }
    static __device__ __forceinline__ float store(float a) { return a; }
};
template <>
struct Storage<double> {
    using acc = double;
    static __device__ __forceinline__ double load(double v) { return v; }
    static __device__ __forceinline__ double store(double a) { return a; }
};
template <>
struct Storage<__half> {
    using acc = float;
    static __device__ __forceinline__ float load(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half store(float a) { return __float2half_rn(a); }
};
template <>
struct Storage<__nv_bfloat16> {
    using acc = float;
    static __device__ __forceinline__ float load(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 store(float a) { return __float2bfloat16_rn(a); }
};

// ------------------------------------------------------------------------------------------------
// op policies
// ------------------------------------------------------------------------------------------------
template <int OP>
struct Op;

template <>
struct Op<kErode> {
    template <typename A>
    static __device__ __forceinline__ A neutral() { return A(__int_as_float(0x7f800000)); }
    template <typename A>
    static __device__ __forceinline__ A tap(A s, A w) { return s - w; }
    // strict "a is better than b"; false whenever either is NaN
    template <typename A>
    static __device__ __forceinline__ bool better(A a, A b) { return a < b; }
    template <typename A>
    static __device__ __forceinline__ bool better_eq(A a, A b) { return a <= b; }
    static constexpr float se_sign = -1.0f;
};
template <>
struct Op<kDilate> {
    template <typename A>
    static __device__ __forceinline__ A neutral() { return A(__int_as_float(0xff800000)); }
    template <typename A>
    static __device__ __forceinline__ A tap(A s, A w) { return s + w; }
    template <typename A>
    static __device__ __forceinline__ bool better(A a, A b) { return a > b; }
    template <typename A>
    static __device__ __forceinline__ bool better_eq(A a, A b) { return a >= b; }
    static constexpr float se_sign = 1.0f;
};

// ------------------------------------------------------------------------------------------------
// borders
// ------------------------------------------------------------------------------------------------

// Maps a coordinate into [0, size).  Returns false for CONSTANT outside the image.
__device__ __forceinline__ bool resolve(int& c, int size, int border) {
    if (c >= 0 && c < size) return true;
    if (border == kReplicate) {
        c = c < 0 ? 0 : size - 1;
        return true;
    }
    if (border == kReflect) {
        if (size == 1) {
            c = 0;
            return true;
        }
        const int period = 2 * size - 2;
        int m = c % period;
        if (m < 0) m += period;
        c = m < size ? m : period - m;
        return true;
    }
    return false;
}

// Range of outputs along one axis whose window can reach pixel p through the border mapping (a
// superset: callers test each candidate exactly).  REPLICATE only maps onto the edge pixels, whose
// plain windows already hold every output that clamps onto them.  A single REFLECT fold maps the
// unresolved position -p (top) or 2(size-1)-p (bottom) onto p; for an even window the top fold
// reaches one output beyond the plain window, so a reachable fold extends the range to the edge.
// A window wider than the image under REFLECT can fold back from anywhere: the whole axis.
__device__ __forceinline__ void candidate_range(int p, int size, int k, int a, int border, int& lo, int& hi) {
    if (border == kReflect && (a > size - 1 || k - 1 - a > size - 1)) {
        lo = 0;
        hi = size - 1;
        return;
    }
    lo = max(p - (k - 1 - a), 0);
    hi = min(p + a, size - 1);
    if (border == kReflect) {
        if (p <= a) lo = 0;
        if (2 * (size - 1) - p <= size - 1 + (k - 1 - a)) hi = size - 1;
    }
}

// ------------------------------------------------------------------------------------------------
// winner encodings
//
// direct:    t = di*kW + dj, NONE = all ones of the index type (uint8 <= 254 taps, uint16 <= 65534)
// separable: (hi << B) | lo with hi = column-pass winner di of the output (NONE = all ones of the
//            hi field) and lo = row-pass winner dj of the output's own row at its column; the 2-D
//            winner of output (h, w) is row r = resolve(h + hi - aH), column dj = lo(r, w).
// ------------------------------------------------------------------------------------------------
template <typename I>
struct IndexTraits;
template <>
struct IndexTraits<uint8_t> {
    static constexpr uint32_t none = 0xffu;
    static constexpr int half_bits = 4;
};
template <>
struct IndexTraits<uint16_t> {
    static constexpr uint32_t none = 0xffffu;
    static constexpr int half_bits = 8;
};
template <>
struct IndexTraits<uint32_t> {
    static constexpr uint32_t none = 0xffffffffu;
    static constexpr int half_bits = 16;
};

template <typename I>
__device__ __forceinline__ uint32_t sep_hi(uint32_t v) {
    return v >> IndexTraits<I>::half_bits;
}
template <typename I>
__device__ __forceinline__ uint32_t sep_lo(uint32_t v) {
    return v & ((1u << IndexTraits<I>::half_bits) - 1u);
}
template <typename I>
__device__ __forceinline__ uint32_t sep_none_hi() {
    return (1u << IndexTraits<I>::half_bits) - 1u;
}

// ------------------------------------------------------------------------------------------------
// exact comparison for float inputs with a general (non 0/inf) structuring element
//
// The reference CPU compares float taps in double: d = fl64(x - w).  fl32 is monotone, and
// fl32(fl64(x - w)) == fl32(x - w) for any two floats (a double rounding of a difference can only
// differ from the direct one when fl64(v) lands on a float midpoint, which needs |w| < 2^-29 |x| or
// the reverse, and then v lies closer to x than any float midpoint).  Hence
//     s_i < s_j  =>  d_i < d_j      and      d_i == d_j  =>  s_i == s_j,
// so the first strict minimum of d is the first strict minimum of s unless two taps tie in s.
// Kernels compare in float, record whether any tie with the running best occurred, and redo the
// rare tied windows in double.  When every weight is 0 or +-inf, x - w is exact in float and no
// tie check is needed.
// ------------------------------------------------------------------------------------------------
template <typename T>
struct NeedsExactCheck {
    static constexpr bool value = false;
};
template <>
struct NeedsExactCheck<float> {
    static constexpr bool value = true;
};

__device__ __forceinline__ bool weight_is_exact(float w) { return w == 0.0f || isinf(w) || isnan(w); }

// ------------------------------------------------------------------------------------------------
// accumulation of grad_input in the storage type's arithmetic (csrc/cpu/morphology/backward.cpp:250-263)
// ------------------------------------------------------------------------------------------------
template <typename T>
struct GradAcc {
    using type = typename Storage<T>::acc;
    static __device__ __forceinline__ type add(type acc, type g) { return acc + g; }
};
template <>
struct GradAcc<__half> {
    using type = float;
    // the reference adds two halves in float and rounds the sum back to half at every step
    static __device__ __forceinline__ float add(float acc, float g) { return __half2float(__float2half_rn(acc + g)); }
};
template <>
struct GradAcc<__nv_bfloat16> {
    using type = float;
    static __device__ __forceinline__ float add(float acc, float g) {
        return __bfloat162float(__float2bfloat16_rn(acc + g));
    }
};

constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace serron
