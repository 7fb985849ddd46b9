// grad_kernel: deterministic reduction of the upstream gradient onto the winning structuring-element
// cells.  The reference scatters sign*grad_output into grad_kernel[winner] (CPU: serially in output
// order, csrc/cpu/morphology/backward.cpp:250-263; GPU: float atomicAdd in arbitrary order,
// csrc/gpu/morphology/backward_kernels.cu:97-100).  Here every thread owns private bins, threads of a
// CTA are summed in a fixed order, and CTA partials are summed in a fixed order by a second kernel, in
// double: the result is run-to-run identical and at least as accurate as either reference.
#pragma once

#include "common.cuh"

#include <cstring>

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
//
// With `vec` (direct records, H * W and the chunk length multiples of 16, go and win 16-byte aligned) a
// thread takes 16 consecutive outputs at a time in 16-byte loads, two groups in flight: the kernel streams
// at memory speed instead of waiting on one-byte loads.
template <typename T, typename I, bool SEP>
__global__ void segrad_partial_kernel(const T* __restrict__ go, const I* __restrict__ win,
                                      double* __restrict__ partial, double* __restrict__ bins_global, int N, int C,
                                      int H, int W, int kH, int kW, int border, long long per_chunk, int vec) {
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
    long long e = start + tid;
    if (!SEP && vec) {
        constexpr int V = 16, RW = V * int(sizeof(I)) / 16, GW = V * int(sizeof(T)) / 16;  // uint4 words per group
        auto load_group = [&](long long q, uint4 (&r)[RW], uint4 (&g)[GW]) {
            const long long e16 = q * V, n = e16 / hw, off = (n * C + c) * hw + (e16 - n * hw);
            const uint4* rp = reinterpret_cast<const uint4*>(win + off);
            const uint4* gp = reinterpret_cast<const uint4*>(go + off);
#pragma unroll
            for (int i = 0; i < RW; ++i) r[i] = __ldg(rp + i);
#pragma unroll
            for (int i = 0; i < GW; ++i) g[i] = __ldg(gp + i);
        };
        auto add_group = [&](const uint4 (&r)[RW], const uint4 (&g)[GW]) {
            I rec[V];
            T val[V];
            memcpy(rec, r, sizeof(rec));
            memcpy(val, g, sizeof(val));
#pragma unroll
            for (int i = 0; i < V; ++i)
                if (static_cast<uint32_t>(rec[i]) != IndexTraits<I>::none)
                    mine[rec[i]] += static_cast<double>(Storage<T>::load(val[i]));
        };
        const long long q1 = end / V;
        long long q = start / V + tid;
        for (; q + nthr < q1; q += 2 * static_cast<long long>(nthr)) {
            uint4 ra[RW], ga[GW], rb[RW], gb[GW];
            load_group(q, ra, ga);
            load_group(q + nthr, rb, gb);
            add_group(ra, ga);
            add_group(rb, gb);
        }
        if (q < q1) {
            uint4 ra[RW], ga[GW];
            load_group(q, ra, ga);
            add_group(ra, ga);
        }
    } else if (e < end) {
        // one division per thread; the position then advances by the block size.  Four outputs are
        // read before any is accumulated, so each thread keeps several loads in flight.
        long long n = e / hw;
        const long long s0 = e - n * hw;
        int oh = static_cast<int>(s0 / W), ow = static_cast<int>(s0 - static_cast<long long>(oh) * W);
        long long plane_base = (n * C + c) * hw;
        auto advance = [&]() {
            ow += nthr;
            while (ow >= W) {
                ow -= W;
                if (++oh == H) {
                    oh = 0;
                    ++n;
                    plane_base = (n * C + c) * hw;
                }
            }
        };
        constexpr int U = 4;
        for (; e + (U - 1) * static_cast<long long>(nthr) < end; e += U * static_cast<long long>(nthr)) {
            int t[U];
            double v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                t[u] = winner_tap<I, SEP>(win, plane_base, oh, ow, H, W, kH, kW, border);
                v[u] = static_cast<double>(Storage<T>::load(go[plane_base + static_cast<long long>(oh) * W + ow]));
                advance();
            }
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (t[u] >= 0) mine[t[u]] += v[u];
        }
        for (; e < end; e += nthr) {
            const int t = winner_tap<I, SEP>(win, plane_base, oh, ow, H, W, kH, kW, border);
            if (t >= 0)
                mine[t] += static_cast<double>(Storage<T>::load(go[plane_base + static_cast<long long>(oh) * W + ow]));
            advance();
        }
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

// gk[cell] = sign * sum over chunks (and over channels for a shared SE) of the partials.  One CTA per
// output cell: thread i sums the partials i, i + 128, ... in order, then the 128 sums are added by a
// fixed tree, so the result does not depend on scheduling.
constexpr int kSegradFinalThreads = 128;
template <typename T>
__global__ void __launch_bounds__(kSegradFinalThreads) segrad_final_kernel(const double* __restrict__ partial,
                                                                           T* __restrict__ gk, int C, int chunks,
                                                                           int bins, int shared, double sign) {
    __shared__ double red[kSegradFinalThreads];
    const int cell = blockIdx.x, tid = threadIdx.x;
    double acc = 0.0;
    if (shared) {
        const int total = C * chunks;
        for (int j = tid; j < total; j += kSegradFinalThreads) acc += partial[static_cast<long long>(j) * bins + cell];
    } else {
        const int c = cell / bins, b = cell - c * bins;
        for (int k = tid; k < chunks; k += kSegradFinalThreads)
            acc += partial[(static_cast<long long>(c) * chunks + k) * bins + b];
    }
    red[tid] = acc;
    __syncthreads();
    for (int half = kSegradFinalThreads / 2; half > 0; half >>= 1) {
        if (tid < half) red[tid] += red[tid + half];
        __syncthreads();
    }
    if (tid == 0) gk[cell] = Storage<T>::store(static_cast<typename Storage<T>::acc>(sign * red[0]));
}

}  // namespace serron
