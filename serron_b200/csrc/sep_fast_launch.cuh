// Host launchers of the compile-time-K separable sweep kernels (sep_sweep.cuh), instantiated once per
// storage type in sep_fast_<type>.cu so the type variants compile in parallel.
#pragma once

#include <type_traits>

#include "sep_sweep.cuh"

namespace serron {

// Window lengths with a compiled fast path; other flat windows take the generic kernels.
#define SERRON_SEP_FAST_KS(X) X(3) X(5) X(7) X(9) X(11) X(13) X(15) X(17) X(21) X(25) X(31)

template <int K>
using FastIndex = typename std::conditional<(K <= 15), uint8_t, uint16_t>::type;

template <typename K_>
inline cudaError_t set_smem_attr(K_ kernel, size_t bytes) {
    if (bytes > 48 * 1024) return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    return cudaSuccess;
}

// Row segments per strip: enough CTAs for ~4 waves of 148 SMs, each segment a whole number of steps.
inline void sweep_segments(long long planes, int strips, int H, int step, int& segs, int& seg_h) {
    const long long ctas = planes * strips;
    const int steps = (H + step - 1) / step;
    long long want = (592 + ctas - 1) / ctas;
    if (want > steps) want = steps;
    if (want < 1) want = 1;
    const int per = static_cast<int>((steps + want - 1) / want);
    seg_h = per * step;
    segs = (H + seg_h - 1) / seg_h;
}

template <typename T, int OP, int K, bool V, bool X>
int sep_fast_fwd_launch(const void* x, void* y, void* win, uint32_t* map, long long planes, int H, int W,
                        int border, cudaStream_t stream) {
    using G = SweepGeom<K, sizeof(T)>;
    using I = FastIndex<K>;
    const int strips = (W + kSweepTW - 1) / kSweepTW;
    int segs = 1, seg_h = H;
    sweep_segments(planes, strips, H, G::TH, segs, seg_h);
    const size_t smem = G::fwd_smem();
    auto kernel = sep_sweep_fwd_kernel<T, OP, I, V, X, K>;
    cudaError_t err = set_smem_attr(kernel, smem);
    if (err != cudaSuccess) return static_cast<int>(err);
    const long long blocks = planes * strips * segs;
    kernel<<<static_cast<unsigned>(blocks), kSweepThreads, smem, stream>>>(
        static_cast<const T*>(x), static_cast<T*>(y), static_cast<I*>(win), map, H, W, border, strips, segs, seg_h);
    return static_cast<int>(cudaGetLastError());
}

template <typename T, int OP, int K>
int sep_fast_fwd_k(bool with_value, bool with_index, const void* x, void* y, void* win, uint32_t* map, long long planes,
                   int H, int W, int border, cudaStream_t stream) {
    if (with_value && with_index)
        return sep_fast_fwd_launch<T, OP, K, true, true>(x, y, win, map, planes, H, W, border, stream);
    if (with_index) return sep_fast_fwd_launch<T, OP, K, false, true>(x, y, win, map, planes, H, W, border, stream);
    return sep_fast_fwd_launch<T, OP, K, true, false>(x, y, win, nullptr, planes, H, W, border, stream);
}

// Returns 0 on success, a cudaError_t code on a launch failure, or -1 when K has no fast path.  With
// `map` (zeroed by the caller) the winners are also set in the gather's target map.
template <typename T>
int sep_fast_fwd_t(int op, int K, bool with_value, bool with_index, const void* x, void* y, void* win, uint32_t* map,
                   long long planes, int H, int W, int border, cudaStream_t stream) {
#define SERRON_SEP_FAST_FWD_CASE(k)                                                                         \
    case k:                                                                                                 \
        return op == kErode ? sep_fast_fwd_k<T, kErode, k>(with_value, with_index, x, y, win, map, planes, H, W, \
                                                           border, stream)                                     \
                            : sep_fast_fwd_k<T, kDilate, k>(with_value, with_index, x, y, win, map, planes, H, W,\
                                                            border, stream);
    switch (K) {
        SERRON_SEP_FAST_KS(SERRON_SEP_FAST_FWD_CASE)
    default:
        return -1;
    }
#undef SERRON_SEP_FAST_FWD_CASE
}

}  // namespace serron
