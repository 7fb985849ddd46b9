// grad_kernel: deterministic reduction of the upstream gradient onto the winning structuring-element
// cells.  The reference scatters sign*grad_output into grad_kernel[winner] (CPU: serially in output
// order, csrc/cpu/morphology/backward.cpp:250-263; GPU: float atomicAdd in arbitrary order,
// csrc/gpu/morphology/backward_kernels.cu:97-100).  Here every thread owns private bins, threads of a
// CTA are summed in a fixed order, and CTA partials are summed in a fixed order by a second kernel, in
// double: the result is run-to-run identical and at least as accurate as either reference.
#pragma once

#include "common.cuh"

namespace serron {

// Winner tap (di*kW + dj) of output `o` at (oh, ow) of plane `plane_base`, or -1.
template <typename I, bool SEP>
__device__ __forceinline__ int winner_tap(const I* __restrict__ win, long long plane_base, int oh, int ow, int H,
                                          int W, int kH, int kW, int border) {
    const uint32_t v = win[plane_base + static_cast<long long>(oh) * W + ow];
    if (!SEP) return v == IndexTraits<I>::none ? -1 : static_cast<int>(v);
    const uint32_t hi = sep_hi<I>(v);
    if (hi == sep_none_hi<I>()) return -1;
    int r = oh + static_cast<int>(hi) - kH / 2;
    if (!resolve(r, H, border)) return -1;
    const uint32_t lo = sep_lo<I>(win[plane_base + static_cast<long long>(r) * W + ow]);
    return static_cast<int>(hi) * kW + static_cast<int>(lo);
}

// grid = (chunks, C).  Bins live in shared memory when `bins_global` is null, else in
// bins_global[(blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + tid][bins].
template <typename T, typename I, bool SEP>
__global__ void segrad_partial_kernel(const T* __restrict__ go, const I* __restrict__ win,
                                      double* __restrict__ partial, double* __restrict__ bins_global, int N, int C,
                                      int H, int W, int kH, int kW, int border, long long per_chunk) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int bins = kH * kW;
    const int nthr = blockDim.x, tid = threadIdx.x;
    const long long cta = static_cast<long long>(blockIdx.y) * gridDim.x + blockIdx.x;
    double* mine = bins_global ? bins_global + (cta * nthr + tid) * bins : reinterpret_cast<double*>(smem_raw) + tid * bins;
    for (int b = 0; b < bins; ++b) mine[b] = 0.0;

    const int c = blockIdx.y;
    const long long hw = static_cast<long long>(H) * W;
    const long long total = static_cast<long long>(N) * hw;
    const long long start = blockIdx.x * per_chunk;
    const long long end = min(start + per_chunk, total);
    for (long long e = start + tid; e < end; e += nthr) {
        const long long n = e / hw, s = e - n * hw;
        const long long plane_base = (n * C + c) * hw;
        const int oh = static_cast<int>(s / W), ow = static_cast<int>(s - static_cast<long long>(oh) * W);
        const int t = winner_tap<I, SEP>(win, plane_base, oh, ow, H, W, kH, kW, border);
        if (t >= 0) mine[t] += static_cast<double>(Storage<T>::load(go[plane_base + s]));
    }
    __syncthreads();
    if (bins_global) __threadfence_block();
    double* base = bins_global ? bins_global + cta * nthr * bins : reinterpret_cast<double*>(smem_raw);
    for (int b = tid; b < bins; b += nthr) {
        double acc = 0.0;
        for (int t = 0; t < nthr; ++t) acc += base[t * bins + b];
        partial[cta * bins + b] = acc;
    }
}

// gk[cell] = sign * sum over chunks (and over channels for a shared SE) of the partials, in order.
template <typename T>
__global__ void segrad_final_kernel(const double* __restrict__ partial, T* __restrict__ gk, int C, int chunks,
                                    int bins, int shared, double sign) {
    const int cell = blockIdx.x * blockDim.x + threadIdx.x;
    const int out_cells = shared ? bins : C * bins;
    if (cell >= out_cells) return;
    double acc = 0.0;
    if (shared) {
        for (int c = 0; c < C; ++c)
            for (int k = 0; k < chunks; ++k) acc += partial[(static_cast<long long>(c) * chunks + k) * bins + cell];
    } else {
        const int c = cell / bins, b = cell - c * bins;
        for (int k = 0; k < chunks; ++k) acc += partial[(static_cast<long long>(c) * chunks + k) * bins + b];
    }
    gk[cell] = Storage<T>::store(static_cast<typename Storage<T>::acc>(sign * acc));
}

}  // namespace serron
